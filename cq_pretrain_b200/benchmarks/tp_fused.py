"""TP collective-fused ops vs NCCL + cuBLAS at 2/4/8 GPUs (bf16).

``torchrun --nproc-per-node N -m cq_pretrain_b200.benchmarks.tp_fused`` times, with CUDA events
and the max over ranks (median of 20 after 5 warm-ups):

* column-parallel all-gather -> GEMM: ``[8192/tp, 2048] x [2048, 6144/tp]`` (each rank holds
  ``8192/tp`` rows; the output is ``[8192, 6144/tp]``);
* row-parallel GEMM -> reduce-scatter: ``[8192, 6144/tp] x [6144/tp, 2048]`` -> ``[8192/tp, 2048]``;
* row-parallel input gradient, all-gather -> GEMM with the weight as MN-major B:
  ``all_gather(dY [8192/tp, 2048]) @ W [2048, 6144/tp]``;
* the input gradient of two column-parallel projections of one gathered input (Qwen's q/gate
  over all rows plus kv over the content rows) as one GEMM -> reduce-scatter;
* Wan's QKV projection ``[32760, 1536] x [1536, 3 x 1536]`` with the full-width Q/K RMSNorm whose
  per-row sums of squares are exchanged across ranks in-kernel;
* vocabulary-parallel LM-head cross-entropy statistics: the statistics GEMM ``[8192, 2048] x
  [248320/tp, 2048]^T`` plus the in-kernel (max, sum exp, target) exchange vs the same GEMM plus
  the NCCL MAX + SUM all-reduce pair;

and reports each fused path against its roofline: the slower of FLOPs / measured bf16 peak and
bytes that must cross NVLink per GPU / 770 GB/s (measured peer-copy bandwidth).
Also checks the fused results against the NCCL path.
"""

from __future__ import annotations

import json
import os
import statistics
from pathlib import Path

import torch
import torch.distributed as dist

PEER_GBS = 770.0


def bf16_peak_tflops():
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def timed(fn, iters=20, warmup=5, reps=5):
    """Per-call device time: ``iters`` calls back to back between two CUDA events (so the host's
    launch skew between ranks after the barrier is spread over the loop, as in a training step),
    median over ``reps`` loops, max over ranks."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(reps):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / iters)
    t = torch.tensor([statistics.median(times)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def kernel_times(fn, iters=10):
    """Device time per call of each kernel ``fn`` launches (torch.profiler / CUPTI), so the time
    inside the fused kernels can be told apart from host gaps between calls."""
    from torch.profiler import ProfilerActivity, profile
    fn()
    torch.cuda.synchronize()
    dist.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(iters):
            fn()
        torch.cuda.synchronize()
    out = {}
    for e in prof.key_averages():
        if e.device_type.name == "CUDA" and e.self_device_time_total > 0:
            name = e.key.split("(")[0].replace("void cqb::(anonymous namespace)::", "")[:60]
            out[name] = round(e.self_device_time_total / 1000 / iters, 4)
    return out


def main():
    from ..parallel import fused
    from ..parallel import state as ps
    from ..parallel import symmetric
    from ..ops import gemm

    world = int(os.environ["WORLD_SIZE"])
    st = ps.initialize(world, timeout_s=300.0)
    tp = st.tp
    ws = symmetric.enable()
    torch.manual_seed(1 + st.rank)
    peak = bf16_peak_tflops()
    M, H, F = 8192, 2048, 6144
    rows = M // tp
    # all-gather -> GEMM
    x = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16)
    w1 = (torch.randn(F // tp, H, device="cuda") * 0.02).to(torch.bfloat16)
    y_f, xg = ws.gather_linear(x, w1)
    y_n = gemm.linear(fused.gather_rows_raw(x), w1)
    err1 = ((y_f.float() - y_n.float()).abs().max() / y_n.float().abs().max()).item()
    t_fused = timed(lambda: ws.gather_linear(x, w1))
    t_nccl = timed(lambda: gemm.linear(fused.gather_rows_raw(x), w1))
    flops = 2.0 * M * H * (F // tp)
    nv_bytes = (tp - 1) * rows * H * 2
    roof = max(flops / (peak * 1e12), nv_bytes / (PEER_GBS * 1e9)) * 1e3
    out = [dict(op="allgather_gemm", tp=tp, shape=[rows, H, F // tp], fused_ms=t_fused, nccl_cublas_ms=t_nccl,
                roofline_ms=roof, roofline_fraction=roof / t_fused, speedup_vs_nccl=t_nccl / t_fused, max_rel_err=err1)]
    # GEMM -> reduce-scatter
    xf = torch.randn(M, F // tp, device="cuda", dtype=torch.bfloat16)
    w2 = (torch.randn(H, F // tp, device="cuda") * 0.02).to(torch.bfloat16)
    z_f = ws.linear_scatter(xf, w2)
    z_n = fused.scatter_rows_raw(gemm.linear(xf, w2))
    err2 = ((z_f.float() - z_n.float()).abs().max() / z_n.float().abs().max()).item()
    t_fused = timed(lambda: ws.linear_scatter(xf, w2))
    t_nccl = timed(lambda: fused.scatter_rows_raw(gemm.linear(xf, w2)))
    flops = 2.0 * M * H * (F // tp)
    nv_bytes = (tp - 1) * rows * H * 2
    roof = max(flops / (peak * 1e12), nv_bytes / (PEER_GBS * 1e9)) * 1e3
    out.append(dict(op="gemm_reducescatter", tp=tp, shape=[M, F // tp, H], fused_ms=t_fused, nccl_cublas_ms=t_nccl,
                    roofline_ms=roof, roofline_fraction=roof / t_fused, speedup_vs_nccl=t_nccl / t_fused, max_rel_err=err2))
    # row-parallel input gradient: all_gather(dY) @ W, W [2048, 6144/tp] read as the MN-major B operand
    dy = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16)
    w3 = (torch.randn(H, F // tp, device="cuda") * 0.02).to(torch.bfloat16)
    g_f, _ = ws.gather_matmul(dy, w3)
    g_n = gemm.matmul_nn(fused.gather_rows_raw(dy), w3)
    err3 = ((g_f.float() - g_n.float()).abs().max() / g_n.float().abs().max()).item()
    t_fused = timed(lambda: ws.gather_matmul(dy, w3))
    t_nccl = timed(lambda: gemm.matmul_nn(fused.gather_rows_raw(dy), w3))
    flops = 2.0 * M * H * (F // tp)
    nv_bytes = (tp - 1) * rows * H * 2
    roof = max(flops / (peak * 1e12), nv_bytes / (PEER_GBS * 1e9)) * 1e3
    out.append(dict(op="allgather_gemm_mn (row-parallel dX)", tp=tp, shape=[M, H, F // tp], fused_ms=t_fused,
                    nccl_cublas_ms=t_nccl, roofline_ms=roof, roofline_fraction=roof / t_fused,
                    speedup_vs_nccl=t_nccl / t_fused, max_rel_err=err3))
    # input gradient of two column-parallel projections of one gathered input (Qwen q/gate + kv over
    # the content rows): reduce_scatter(dY1 W1 + pad(dY2) W2) in one kernel
    n1, n2, rows2 = 2 * 8 * 256 // tp, 2 * 2 * 256 // tp, M // 2
    dq = torch.randn(M, n1, device="cuda", dtype=torch.bfloat16)
    dkv = torch.randn(rows2, n2, device="cuda", dtype=torch.bfloat16)
    wq = (torch.randn(n1, H, device="cuda") * 0.02).to(torch.bfloat16)
    wkv = (torch.randn(n2, H, device="cuda") * 0.02).to(torch.bfloat16)

    def pair_nccl():
        full = gemm.matmul_nn(dq, wq)
        full[:rows2] += gemm.matmul_nn(dkv, wkv)
        return fused.scatter_rows_raw(full)

    p_f, p_n = ws.matmul_scatter(dq, wq, dkv, wkv), pair_nccl()
    err5 = ((p_f.float() - p_n.float()).abs().max() / p_n.float().abs().max()).item()
    t_fused, t_nccl = timed(lambda: ws.matmul_scatter(dq, wq, dkv, wkv)), timed(pair_nccl)
    flops = 2.0 * H * (M * n1 + rows2 * n2)
    nv_bytes = (tp - 1) * rows * H * 2
    roof = max(flops / (peak * 1e12), nv_bytes / (PEER_GBS * 1e9)) * 1e3
    out.append(dict(op="pair_input_grad_reducescatter (q/gate + kv)", tp=tp, shape=[M, n1, rows2, n2, H],
                    fused_ms=t_fused, nccl_cublas_ms=t_nccl, roofline_ms=roof, roofline_fraction=roof / t_fused,
                    speedup_vs_nccl=t_nccl / t_fused, max_rel_err=err5))
    # Wan self-attention QKV projection with the cross-rank Q/K RMSNorm and the 3D RoPE: [32760, 1536]
    # x [1536, 3 x 1536] (rows padded to 128 x tp), q and kv sharing one in-kernel all-gather, then
    # q and k normalised over the full width (per-row sums exchanged in-kernel) and rotated in one
    # kernel, as the model runs it; baseline: NCCL all-gather + GEMMs + NCCL all-reduce of the sums +
    # the normalisation + the RoPE kernel.
    from types import SimpleNamespace

    from ..config import qwen35_2b_wan
    from ..models.wan21 import Attention
    from ..ops import rope as ROPE
    wan_rows = -(-32760 // (128 * tp)) * 128 * tp
    attn = Attention(qwen35_2b_wan()).cuda().to(torch.bfloat16)
    xw = torch.randn(wan_rows // tp, 1536, device="cuda", dtype=torch.bfloat16)
    gen = torch.Generator(device="cuda").manual_seed(3)   # the same angles on every rank
    ang = torch.rand(wan_rows, attn.head_dim // 2, device="cuda", generator=gen) * 6.28
    layout = SimpleNamespace(cos_rows=ang.cos(), sin_rows=ang.sin())

    def wan_fused():
        from ..parallel import layers as PL
        q, kv = PL.column_pair(xw, attn.q, attn.kv)
        k, v = kv.chunk(2, -1)
        fused_qk = attn._fused_qk(q, k, layout)
        assert fused_qk is not None, "the fused q / k kernel does not take this shape"
        return fused_qk[0], fused_qk[1], v.reshape(-1, attn.heads, attn.head_dim)

    def wan_nccl():
        xg_ = fused.gather_rows_raw(xw)
        q = gemm.linear(xg_, attn.q.weight, attn.q.bias)
        k, v = gemm.linear(xg_, attn.kv.weight, attn.kv.bias).chunk(2, -1)
        out_ = []
        for t, norm in ((q, attn.norm_q), (k, attn.norm_k)):
            sq = t.float().square().sum(-1, keepdim=True)
            dist.all_reduce(sq, group=st.tp_group)
            y = (t.float() * torch.rsqrt(sq / 1536 + 1e-6)).to(t.dtype) * norm.weight.to(t.dtype)
            out_.append(ROPE.rotary_pairs(y.view(-1, attn.heads, attn.head_dim), layout.cos_rows, layout.sin_rows))
        return out_[0], out_[1], v.reshape(-1, attn.heads, attn.head_dim)

    with torch.no_grad():
        wf, wn = wan_fused(), wan_nccl()
        err6 = max(((a.float() - b.float()).abs().max() / b.float().abs().max()).item() for a, b in zip(wf, wn))
        t_fused, t_nccl = timed(wan_fused), timed(wan_nccl)
    flops = 2.0 * wan_rows * 1536 * (3 * 1536 // tp)
    nv_bytes = (tp - 1) * (wan_rows // tp) * 1536 * 2 + 2 * (tp - 1) * wan_rows * 4
    roof = max(flops / (peak * 1e12), nv_bytes / (PEER_GBS * 1e9)) * 1e3
    out.append(dict(op="wan_qkv_gemm + cross-rank q/k rmsnorm + rope", tp=tp, shape=[wan_rows, 1536, 3 * 1536 // tp],
                    fused_ms=t_fused, nccl_cublas_ms=t_nccl, roofline_ms=roof, roofline_fraction=roof / t_fused,
                    speedup_vs_nccl=t_nccl / t_fused, max_rel_err=err6))
    # vocabulary-parallel CE statistics: LM-head partials -> in-kernel exchange vs NCCL MAX + SUM
    from ..ops import _ext
    from ..ops.cross_entropy import _stats_combine
    vocab = 248320
    hid = torch.randn(M, H, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)).to(torch.bfloat16)
    wv = (torch.randn(vocab // tp, H, device="cuda") * 0.02).to(torch.bfloat16)
    tg = torch.randint(0, vocab, (M,), device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
    lo = st.tp_rank * (vocab // tp)
    ops = _ext.ops()

    def fused_ce():
        return ws.ce_combine(*ops.ce_partials(hid, wv, tg, lo))

    def nccl_ce():
        mx, tgt, sexp = _stats_combine(*ops.ce_stats(hid, wv, tg, lo), st.tp_group)
        return mx + torch.log(sexp), tgt

    (l_f, t_f), (l_n, t_n) = fused_ce(), nccl_ce()
    err4 = max((l_f - l_n).abs().max().item(), (t_f - t_n).abs().max().item())
    t_fused, t_nccl = timed(fused_ce), timed(nccl_ce)
    flops = 2.0 * M * H * (vocab // tp)
    nv_bytes = (tp - 1) * M * 12
    roof = max(flops / (peak * 1e12), nv_bytes / (PEER_GBS * 1e9)) * 1e3
    out.append(dict(op="lm_head_ce_stats (vocab-parallel)", tp=tp, shape=[M, H, vocab // tp], fused_ms=t_fused,
                    nccl_cublas_ms=t_nccl, roofline_ms=roof, roofline_fraction=roof / t_fused,
                    speedup_vs_nccl=t_nccl / t_fused, max_abs_err=err4))
    kernels = {
        "allgather_gemm": kernel_times(lambda: ws.gather_linear(x, w1)),
        "gemm_reducescatter": kernel_times(lambda: ws.linear_scatter(xf, w2)),
        "allgather_gemm_mn": kernel_times(lambda: ws.gather_matmul(dy, w3)),
        "pair_input_grad_reducescatter": kernel_times(lambda: ws.matmul_scatter(dq, wq, dkv, wkv)),
        "plain_gemm_reference": kernel_times(lambda: gemm.linear(torch.empty(M, H, device="cuda",
                                                                             dtype=torch.bfloat16), w1)),
    }
    status = symmetric.status()
    if st.rank == 0:
        for row in out:
            row["status"] = status
            print(json.dumps(row), flush=True)
        print(json.dumps(dict(kernel_ms_per_call=kernels)), flush=True)
    symmetric.disable()
    ps.destroy()


if __name__ == "__main__":
    main()
