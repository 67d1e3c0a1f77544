"""In-kernel TP collectives (all-gather->GEMM, GEMM->reduce-scatter, RMSNorm and cross-entropy
statistics exchanges) vs NCCL / full-precision references on 2+ GPUs."""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from cq_pretrain_b200.ops import gemm
    from cq_pretrain_b200.parallel import fused, state as ps, symmetric
    st = ps.initialize(world, timeout_s=120.0)
    ws = symmetric.enable(send_bytes=8 << 20, recv_bytes=16 << 20)
    torch.manual_seed(rank)
    errors = []
    for it in range(3):  # several epochs exercise both buffer parities
        x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
        w = (torch.randn(384, 512, device="cuda") * 0.05).to(torch.bfloat16)
        y, xg = ws.gather_linear(x, w)
        xg_ref = fused.gather_rows_raw(x)
        errors.append(("ag_rows", float((xg.float() - xg_ref.float()).abs().max())))
        ref = gemm.linear(xg_ref, w)
        errors.append(("ag_gemm", float((y.float() - ref.float()).abs().max() / ref.float().abs().max())))
        xf = torch.randn(256 * world, 256, device="cuda", dtype=torch.bfloat16)
        w2 = (torch.randn(512, 256, device="cuda") * 0.05).to(torch.bfloat16)
        z = ws.linear_scatter(xf, w2)
        zref = fused.scatter_rows_raw(gemm.linear(xf, w2))
        errors.append(("gemm_rs", float((z.float() - zref.float()).abs().max() / zref.float().abs().max())))
        # the owner adds the bias once, inside the same kernel
        bias = torch.randn(512, device="cuda", dtype=torch.bfloat16)
        zb = ws.linear_scatter(xf, w2, bias)
        errors.append(("gemm_rs_bias", float((zb.float() - zref.float() - bias.float()).abs().max() / zref.float().abs().max())))
        dy = torch.randn(256 * world, 384, device="cuda", dtype=torch.bfloat16)
        w3 = (torch.randn(384, 512, device="cuda") * 0.05).to(torch.bfloat16)
        d = ws.matmul_scatter(dy, w3)
        dref = fused.scatter_rows_raw(gemm.matmul_nn(dy, w3))
        errors.append(("matmul_rs", float((d.float() - dref.float()).abs().max() / dref.float().abs().max())))
        # two projections of one gathered input: reduce_scatter(dY1 W1 + pad(dY2) W2), dY2 over fewer rows
        dy2 = torch.randn(256 * world - 72, 160, device="cuda", dtype=torch.bfloat16)
        w5 = (torch.randn(160, 512, device="cuda") * 0.05).to(torch.bfloat16)
        d2 = ws.matmul_scatter(dy, w3, dy2, w5)
        full = gemm.matmul_nn(dy, w3).float()
        full[: dy2.shape[0]] += gemm.matmul_nn(dy2, w5).float()
        d2ref = fused.scatter_rows_raw(full)
        errors.append(("matmul_rs_pair", float((d2.float() - d2ref).abs().max() / d2ref.abs().max())))
        # row-parallel input gradient: all_gather(dY) @ W with W [K, N] (MN-major B) in one kernel
        dy_local = torch.randn(256, 384, device="cuda", dtype=torch.bfloat16)
        w4 = (torch.randn(384, 320, device="cuda") * 0.05).to(torch.bfloat16)
        g, dyg = ws.gather_matmul(dy_local, w4)
        dyg_ref = fused.gather_rows_raw(dy_local)
        errors.append(("ag_mn_rows", float((dyg.float() - dyg_ref.float()).abs().max())))
        gref = gemm.matmul_nn(dyg_ref, w4)
        errors.append(("ag_mn_gemm", float((g.float() - gref.float()).abs().max() / gref.float().abs().max())))
        # Wan full-width RMSNorm: in-kernel exchange of the per-row sums vs NCCL all-reduce
        from cq_pretrain_b200.models.wan21 import WanRMSNorm
        norm = WanRMSNorm(384 * world, 1e-6).cuda()
        with torch.no_grad():
            norm.weight.copy_(1 + 0.1 * torch.randn_like(norm.weight))
        xq = torch.randn(1000 + it, 384, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        yq = norm(xq)
        gq = torch.randn_like(yq)
        yq.backward(gq)
        xr = xq.detach().float().requires_grad_()
        wr = norm.weight.detach().float().requires_grad_()
        from torch.distributed.nn.functional import all_reduce as ar_autograd
        sq = ar_autograd(xr.square().sum(-1, keepdim=True))   # reference: NCCL all-reduce (with its backward)
        yr = xr * torch.rsqrt(sq / (384 * world) + 1e-6) * wr
        yr.backward(gq.float())
        errors.append(("wan_rms_y", float((yq.float() - yr).abs().max() / yr.abs().max())))
        errors.append(("wan_rms_dx", float((xq.grad.float() - xr.grad).norm() / xr.grad.norm())))
        errors.append(("wan_rms_dw", float((norm.weight.grad.float() - wr.grad).norm() / wr.grad.norm())))
        # vocabulary-parallel CE: in-kernel (max, sum exp, target) exchange vs full fp32 logits
        from cq_pretrain_b200.ops import cross_entropy as CE
        gen = torch.Generator(device="cuda").manual_seed(100 + it)        # same rows on every rank
        rows, vocab = 400 + 64 * it, 1024 * world
        hid = torch.randn(rows, 256, device="cuda", generator=gen).to(torch.bfloat16).requires_grad_()
        tgts = torch.randint(0, vocab, (rows,), device="cuda", generator=gen)
        w_shard = (torch.randn(vocab // world, 256, device="cuda") * 0.05).to(torch.bfloat16)
        assert CE._fused_workspace(hid, w_shard, st.tp_group, rows) is not None
        loss = CE.linear_cross_entropy(hid, w_shard, tgts, rows)
        loss.backward()
        shards = [torch.empty_like(w_shard) for _ in range(world)]
        dist.all_gather(shards, w_shard)
        href = hid.detach().float().requires_grad_()
        ref_loss = torch.nn.functional.cross_entropy(href @ torch.cat(shards).float().T, tgts)
        ref_loss.backward()
        dh = hid.grad.float().clone()
        dist.all_reduce(dh)                 # each rank holds its vocabulary shard's part of dh
        errors.append(("ce_loss", float((loss.float() - ref_loss).abs() / ref_loss.abs())))
        errors.append(("ce_dh", float((dh - href.grad).norm() / href.grad.norm())))
    # autograd pair (Qwen q/kv projection shape): forward and all gradients vs the NCCL path
    from cq_pretrain_b200.ops import linear as L
    xs = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    wa = (torch.randn(384, 512, device="cuda") * 0.05).to(torch.bfloat16)
    wb = (torch.randn(128, 512, device="cuda") * 0.05).to(torch.bfloat16)
    ba = torch.randn(384, device="cuda", dtype=torch.bfloat16)
    rows2 = 256 * world - 200
    ga = torch.randn(256 * world, 384, device="cuda", dtype=torch.bfloat16)
    gb = torch.randn(rows2, 128, device="cuda", dtype=torch.bfloat16)
    results = []
    for use_fused in (True, False):
        leaves = [t.clone().requires_grad_() for t in (xs, wa, ba, wb)]
        if use_fused:
            ya, yb = L.gather_linear_pair(leaves[0], leaves[1], leaves[2], leaves[3], None, rows2)
        else:
            xg_all = torch.cat([t for t in _all_gather(leaves[0])])
            ya = xg_all @ leaves[1].T + leaves[2]
            yb = xg_all[:rows2] @ leaves[3].T
        torch.autograd.backward([ya, yb], [ga, gb])
        results.append([ya.detach().float(), yb.detach().float()] + [t.grad.float() for t in leaves])
    for a, b in zip(*results):
        errors.append(("pair_autograd", float((a - b).norm() / b.norm().clamp_min(1e-6))))
    errors += _graph_replays(ws, world)
    errors += _qk_exchange(ws, world)
    torch.cuda.synchronize()
    status = symmetric.status()
    symmetric.disable()
    ps.destroy()
    torch.save(dict(errors=errors, status=status), f"{out}.{rank}")


def _graph_replays(ws, world):
    """Fused calls captured in a CUDA graph take fresh device epochs on every replay, interleaved
    with eager calls of the same kinds (odd counts, so replays alternate the buffer parities)."""
    from cq_pretrain_b200.ops import gemm
    from cq_pretrain_b200.parallel import fused
    errors = []
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(384, 512, device="cuda") * 0.05).to(torch.bfloat16)
    xf = torch.randn(256 * world, 256, device="cuda", dtype=torch.bfloat16)
    w2 = (torch.randn(512, 256, device="cuda") * 0.05).to(torch.bfloat16)
    xr = torch.randn(700, 384, device="cuda", dtype=torch.bfloat16)
    wr = torch.rand(384, device="cuda") + 0.5
    before = ws.device_epochs()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y, _ = ws.gather_linear(x, w)
        z = ws.linear_scatter(xf, w2)
        yr, _ = ws.rms_forward(xr, wr, 384 * world, 1e-6)
    assert ws.device_epochs() == before   # capture records work, it runs none
    for rep in range(3):
        x.copy_(torch.randn_like(x))
        xf.copy_(torch.randn_like(xf))
        xr.copy_(torch.randn_like(xr))
        graph.replay()
        ref = gemm.linear(fused.gather_rows_raw(x), w).float()
        errors.append(("graph_ag", float((y.float() - ref).abs().max() / ref.abs().max())))
        zref = fused.scatter_rows_raw(gemm.linear(xf, w2)).float()
        errors.append(("graph_rs", float((z.float() - zref).abs().max() / zref.abs().max())))
        sq = xr.float().square().sum(-1, keepdim=True)
        dist.all_reduce(sq)
        rref = xr.float() * torch.rsqrt(sq / (384 * world) + 1e-6) * wr
        errors.append(("graph_rms", float((yr.float() - rref).abs().max() / rref.abs().max())))
        ye, _ = ws.gather_linear(x, w)   # an eager call between replays shifts the parity
        errors.append(("graph_eager_ag", float((ye.float() - ref).abs().max() / ref.abs().max())))
    after = ws.device_epochs()
    assert after["all_gather"] - before["all_gather"] == 6, (before, after)
    assert after["reduce_scatter"] - before["reduce_scatter"] == 3, (before, after)
    assert after["statistics"] - before["statistics"] == 3, (before, after)
    del graph
    return errors


def _qk_exchange(ws, world):
    """Fused q / k norm + RoPE with the in-kernel row-sum exchange vs the NCCL-summed fp32 formula."""
    from cq_pretrain_b200.ops import norms as N
    from torch.distributed.nn.functional import all_reduce as ar_autograd
    dev, rows, width, hd = torch.device("cuda"), 1100, 384, 64
    gen = torch.Generator(device="cuda").manual_seed(5)   # same angles on every rank
    ang = torch.rand(rows, hd // 2, device=dev, generator=gen) * 6.28
    cos, sin = ang.cos(), ang.sin()
    q = torch.randn(rows, width, device=dev, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(rows, width, device=dev, dtype=torch.bfloat16, requires_grad=True)
    wq = (1 + 0.1 * torch.randn(width, device=dev)).requires_grad_()
    wk = (1 + 0.1 * torch.randn(width, device=dev)).requires_grad_()
    assert ws.supports_qk(q, k)
    yq, yk = N.qk_norm_rope(q, k, wq, wk, cos, sin, hd, width * world, 1e-6, ws.exchange_kwargs)
    gq, gk = torch.randn_like(yq), torch.randn_like(yk)
    torch.autograd.backward([yq, yk], [gq, gk])
    leaves = [t.detach().float().requires_grad_() for t in (q, k, wq, wk)]
    rq, rk = _qk_reference(*leaves, cos, sin, width // hd, hd, width * world, 1e-6, sum_rows=ar_autograd)
    torch.autograd.backward([rq, rk], [gq.float(), gk.float()])
    errors = []
    for got, ref in ((yq, rq), (yk, rk), (q.grad, leaves[0].grad), (k.grad, leaves[1].grad), (wq.grad, leaves[2].grad),
                     (wk.grad, leaves[3].grad)):
        errors.append(("qk", float((got.float() - ref.detach()).norm() / ref.detach().norm())))
    return errors


def _all_gather(x):
    """Differentiable row all-gather (NCCL) for the reference path."""
    from torch.distributed.nn.functional import all_gather
    return all_gather(x)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_device_epochs_advance_in_graph_replays():
    """One rank (tp = 1: the peer arrays hold this GPU's own buffers) runs the row-statistic
    exchange with device epochs: eager calls and CUDA-graph replays each advance the counter, each
    takes the buffers of its epoch's parity, and every call normalises correctly."""
    from cq_pretrain_b200.ops import _ext
    ops = _ext.ops()
    dev = torch.device("cuda")
    max_rows = 1024
    flags = torch.zeros(-(-max_rows // 64) * 8, dtype=torch.int64, device=dev)
    slabs = [torch.zeros(max_rows, dtype=torch.float32, device=dev) for _ in range(2)]
    ptr = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device=dev)
    ctr = torch.zeros(1, dtype=torch.int64, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    x = torch.randn(700, 256, device=dev, dtype=torch.bfloat16)
    w = torch.rand(256, device=dev) + 0.5
    kw = dict(peer_recv=ptr(slabs[0]), my_recv=slabs[0].data_ptr(), peer_flags=ptr(flags), my_flags=flags.data_ptr(),
              rank=0, tp=1, max_rows=max_rows, epoch=0, epoch_ctr=ctr.data_ptr(), epoch_done=done.data_ptr(),
              peer_recv_odd=ptr(slabs[1]), my_recv_odd=slabs[1].data_ptr())   # built before any capture

    def call():
        return ops.tp_rms_fwd(x, w, total_dim=256, eps=1e-6, **kw)

    def ref():
        xf = x.float()
        return xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-6) * w

    y, _ = call()
    torch.cuda.synchronize()
    assert int(ctr) == 1 and int(done) == 0
    torch.testing.assert_close(y.float(), ref(), rtol=2e-2, atol=2e-2)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yg, _ = call()
    assert int(ctr) == 1
    for rep in range(4):
        x.copy_(torch.randn_like(x))
        graph.replay()
        torch.cuda.synchronize()
        assert int(ctr) == 2 + rep and int(done) == 0
        torch.testing.assert_close(yg.float(), ref(), rtol=2e-2, atol=2e-2)
        # this epoch's partial sums went to the slab of its parity, the other one is stale
        assert slabs[(2 + rep) % 2][:700].abs().sum() > 0
    assert int(flags[:8].max()) == 5 and ops.comm_status_read(True) == 0
    # backward (eager, epoch 6): dx and dw against autograd of the fp32 formula
    y, rstd = call()
    dy = torch.randn_like(y)
    dx, dw = ops.tp_rms_bwd(dy, x, w, rstd, total_dim=256, **kw)
    xr, wr = x.float().requires_grad_(), w.clone().requires_grad_()
    (xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + 1e-6) * wr).backward(dy.float())
    torch.testing.assert_close(dx.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(dw, wr.grad, rtol=1e-2, atol=1e-1)
    torch.cuda.synchronize()
    assert int(ctr) == 7 and int(done) == 0 and ops.comm_status_read(True) == 0


def _qk_reference(q, k, wq, wk, cos, sin, heads, hd, total_dim, eps, sum_rows=None):
    """fp32 autograd reference: full-width RMSNorm (row sums through ``sum_rows`` at TP > 1) then
    the complex-pair RoPE, for q and k."""
    from cq_pretrain_b200.ops import reference as R
    outs = []
    for x, w in ((q, wq), (k, wk)):
        sq = x.square().sum(-1, keepdim=True)
        if sum_rows is not None:
            sq = sum_rows(sq)
        y = x * torch.rsqrt(sq / total_dim + eps) * w
        outs.append(R.rotary_pairs(y.view(-1, heads, hd), cos, sin).flatten(1))
    return outs


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("width,hd", [(1536, 128), (768, 128), (256, 64)])
def test_qk_norm_rope_single_rank(width, hd):
    """The fused q / k RMSNorm + RoPE kernel (no exchange) against the fp32 formula, forward and
    backward, with k a row-strided view of a wider projection (the kv output's first half)."""
    from cq_pretrain_b200.ops import norms as N
    torch.manual_seed(0)
    rows, dev = 1000, torch.device("cuda")
    q = torch.randn(rows, width, device=dev, dtype=torch.bfloat16, requires_grad=True)
    kv = torch.randn(rows, 2 * width, device=dev, dtype=torch.bfloat16, requires_grad=True)
    k = kv[:, :width]
    wq = (1 + 0.1 * torch.randn(width, device=dev)).requires_grad_()
    wk = (1 + 0.1 * torch.randn(width, device=dev)).requires_grad_()
    ang = torch.rand(rows, hd // 2, device=dev) * 6.28
    cos, sin = ang.cos(), ang.sin()
    assert N.qk_norm_rope_supported(q, k)
    yq, yk = N.qk_norm_rope(q, k, wq, wk, cos, sin, hd, width, 1e-6)
    gq, gk = torch.randn_like(yq), torch.randn_like(yk)
    torch.autograd.backward([yq, yk], [gq, gk])
    leaves = [t.detach().float().requires_grad_() for t in (q, kv, wq, wk)]
    rq, rk = _qk_reference(leaves[0], leaves[1][:, :width], leaves[2], leaves[3], cos, sin, width // hd, hd, width,
                           1e-6)
    torch.autograd.backward([rq, rk], [gq.float(), gk.float()])
    for got, ref in ((yq, rq), (yk, rk), (q.grad, leaves[0].grad), (kv.grad, leaves[1].grad)):
        err = float((got.float() - ref.detach()).norm() / ref.detach().norm())
        assert err < 1e-2, err
    for got, ref in ((wq.grad, leaves[2].grad), (wk.grad, leaves[3].grad)):
        torch.testing.assert_close(got, ref, rtol=1e-2, atol=1e-1)
    assert float(kv.grad[:, width:].abs().max()) == 0.0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_qk_exchange_slabs_of_partial_blocks():
    """q and k exchanged in one call with a row count that is not a multiple of the 64-row block:
    tensor 0's last (partial) block must not store over tensor 1's first rows in the slab. One
    rank (tp = 1, this GPU's own slabs as the peer arrays) gives the same bits as no exchange."""
    from cq_pretrain_b200.ops import _ext
    ops = _ext.ops()
    dev = torch.device("cuda")
    max_rows = 4096
    flags = torch.zeros(-(-max_rows // 64) * 8, dtype=torch.int64, device=dev)
    slabs = [torch.zeros(max_rows, dtype=torch.float32, device=dev) for _ in range(2)]
    ptr = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device=dev)
    ctr = torch.zeros(1, dtype=torch.int64, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    kw = dict(peer_recv=ptr(slabs[0]), my_recv=slabs[0].data_ptr(), peer_flags=ptr(flags), my_flags=flags.data_ptr(),
              rank=0, tp=1, max_rows=max_rows, epoch_ctr=ctr.data_ptr(), epoch_done=done.data_ptr(),
              peer_recv_odd=ptr(slabs[1]), my_recv_odd=slabs[1].data_ptr())
    torch.manual_seed(3)
    rows, width = 1100, 512
    q = torch.randn(rows, width, device=dev, dtype=torch.bfloat16)
    k = torch.randn(rows, width, device=dev, dtype=torch.bfloat16) * 3
    wq, wk = torch.rand(width, device=dev) + 0.5, torch.rand(width, device=dev) + 0.5
    want = ops.qk_norm_rope_fwd(q, k, wq, wk, total_dim=width, eps=1e-6)
    dyq, dyk = torch.randn_like(q), torch.randn_like(k)
    want_b = ops.qk_norm_rope_bwd(dyq, dyk, q, k, wq, wk, want[2], total_dim=width)
    for _ in range(6):
        got = ops.qk_norm_rope_fwd(q, k, wq, wk, total_dim=width, eps=1e-6, **kw)
        got_b = ops.qk_norm_rope_bwd(dyq, dyk, q, k, wq, wk, got[2], total_dim=width, **kw)
        for a, b in zip(got + got_b, want + want_b):
            assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert int(ctr) == 12 and ops.comm_status_read(True) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
def test_fused_tp_collectives_match_nccl():
    world = min(torch.cuda.device_count(), 4)
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "res")
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
        for r in range(world):
            res = torch.load(f"{out}.{r}")
            assert res["status"] == dict(gemm=0, comm=0), res["status"]
            bad = [(name, err) for name, err in res["errors"] if not err < 2e-2]
            assert not bad, bad
