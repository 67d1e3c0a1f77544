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
        errors.append(float((xg.float() - xg_ref.float()).abs().max()))
        ref = gemm.linear(xg_ref, w)
        errors.append(float((y.float() - ref.float()).abs().max() / ref.float().abs().max()))
        xf = torch.randn(256 * world, 256, device="cuda", dtype=torch.bfloat16)
        w2 = (torch.randn(512, 256, device="cuda") * 0.05).to(torch.bfloat16)
        z = ws.linear_scatter(xf, w2)
        zref = fused.scatter_rows_raw(gemm.linear(xf, w2))
        errors.append(float((z.float() - zref.float()).abs().max() / zref.float().abs().max()))
        # the owner adds the bias once, inside the same kernel
        bias = torch.randn(512, device="cuda", dtype=torch.bfloat16)
        zb = ws.linear_scatter(xf, w2, bias)
        errors.append(float((zb.float() - zref.float() - bias.float()).abs().max() / zref.float().abs().max()))
        dy = torch.randn(256 * world, 384, device="cuda", dtype=torch.bfloat16)
        w3 = (torch.randn(384, 512, device="cuda") * 0.05).to(torch.bfloat16)
        d = ws.matmul_scatter(dy, w3)
        dref = fused.scatter_rows_raw(gemm.matmul_nn(dy, w3))
        errors.append(float((d.float() - dref.float()).abs().max() / dref.float().abs().max()))
        # two projections of one gathered input: reduce_scatter(dY1 W1 + pad(dY2) W2), dY2 over fewer rows
        dy2 = torch.randn(256 * world - 72, 160, device="cuda", dtype=torch.bfloat16)
        w5 = (torch.randn(160, 512, device="cuda") * 0.05).to(torch.bfloat16)
        d2 = ws.matmul_scatter(dy, w3, dy2, w5)
        full = gemm.matmul_nn(dy, w3).float()
        full[: dy2.shape[0]] += gemm.matmul_nn(dy2, w5).float()
        d2ref = fused.scatter_rows_raw(full)
        errors.append(float((d2.float() - d2ref).abs().max() / d2ref.abs().max()))
        # row-parallel input gradient: all_gather(dY) @ W with W [K, N] (MN-major B) in one kernel
        dy_local = torch.randn(256, 384, device="cuda", dtype=torch.bfloat16)
        w4 = (torch.randn(384, 320, device="cuda") * 0.05).to(torch.bfloat16)
        g, dyg = ws.gather_matmul(dy_local, w4)
        dyg_ref = fused.gather_rows_raw(dy_local)
        errors.append(float((dyg.float() - dyg_ref.float()).abs().max()))
        gref = gemm.matmul_nn(dyg_ref, w4)
        errors.append(float((g.float() - gref.float()).abs().max() / gref.float().abs().max()))
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
        errors.append(float((yq.float() - yr).abs().max() / yr.abs().max()))
        errors.append(float((xq.grad.float() - xr.grad).norm() / xr.grad.norm()))
        errors.append(float((norm.weight.grad.float() - wr.grad).norm() / wr.grad.norm()))
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
        errors.append(float((loss.float() - ref_loss).abs() / ref_loss.abs()))
        errors.append(float((dh - href.grad).norm() / href.grad.norm()))
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
        errors.append(float((a - b).norm() / b.norm().clamp_min(1e-6)))
    torch.cuda.synchronize()
    status = symmetric.status()
    symmetric.disable()
    ps.destroy()
    torch.save(dict(errors=errors, status=status), f"{out}.{rank}")


def _all_gather(x):
    """Differentiable row all-gather (NCCL) for the reference path."""
    from torch.distributed.nn.functional import all_gather
    return all_gather(x)


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
            assert max(res["errors"]) < 2e-2, res["errors"]
