"""Range-masked attention kernels on the flagship CQ layout and the Wan self-attention shape.

``python -m cq_pretrain_b200.benchmarks.attention [--iters 20] [--only cq256]`` times the tcgen05
``attn_fwd`` and ``attn_bwd`` of ``csrc/attention.cu`` with CUDA events (median after 3 warm-ups)
and reports TFLOP/s over the VISIBLE (row, key) pairs: forward 4 * H * D * pairs, backward
10 * H * D * pairs (the S and dP recomputations of the backward are not counted). The unmasked
``wan128`` case also times ``torch.nn.functional.scaled_dot_product_attention`` (flash backend)
on the same tensors.

* ``cq256``: the joint 8K pack of ``bench.py`` (rows 14848, 8192 content keys, Hq 8, Hkv 2, D 256).
* ``wan128``: Wan2.1-1.3B self-attention, one 1024-token sample, 12 heads of 128.
"""

from __future__ import annotations

import argparse
import json
import statistics


def _time(fn, iters):
    import torch
    for _ in range(3):
        fn()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times)


def cases():
    from ..config import qwen35_2b_wan
    from ..data.synthetic import synthetic_batch
    from ..ops.attention import ranges_from_ends
    cfg = qwen35_2b_wan(visual_query_mode="fixed", image_condition_queries=256)
    host, _ = synthetic_batch(cfg, 8192, seed=42, kind="joint", images=2, grid=(1, 64, 64),
                              latent_shape=(16, 1, 64, 64), understanding=False, pad_multiple=128)
    p = host.mainline
    yield "cq256", p.rows, p.content_length, 8, 2, 256, p.attn_kstart.int(), p.attn_kend.int()
    ks, ke = ranges_from_ends((1024,), (1024,), "cpu")
    yield "wan128", 1024, 1024, 12, 12, 128, ks.int(), ke.int()


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--iters", type=int, default=20)
    parser.add_argument("--only", default=None)
    args = parser.parse_args()
    import torch
    import torch.nn.functional as F
    from ..ops import _ext
    ops = _ext.ops()
    for name, rows, keys, hq, hkv, d, ks, ke in cases():
        if args.only and name != args.only:
            continue
        torch.manual_seed(0)
        q = torch.randn(rows, hq, d, device="cuda", dtype=torch.bfloat16)
        k = torch.randn(keys, hkv, d, device="cuda", dtype=torch.bfloat16)
        v = torch.randn(keys, hkv, d, device="cuda", dtype=torch.bfloat16)
        ks, ke = ks.cuda(), ke.cuda()
        pairs = float((ke.long() - ks.long()).clamp_min(0).sum())
        scale = d ** -0.5
        o, lse = ops.attn_fwd(q, k, v, ks, ke, scale)
        do = torch.randn_like(o)
        row = dict(case=name, rows=rows, keys=keys, hq=hq, hkv=hkv, d=d, pairs=int(pairs))
        ms = _time(lambda: ops.attn_fwd(q, k, v, ks, ke, scale), args.iters)
        row["fwd_ms"], row["fwd_tflops"] = round(ms, 4), round(4 * hq * d * pairs / ms / 1e9, 1)
        ms = _time(lambda: ops.attn_bwd(do, q, k, v, o, lse, ks, ke, scale), args.iters)
        row["bwd_ms"], row["bwd_tflops"] = round(ms, 4), round(10 * hq * d * pairs / ms / 1e9, 1)
        row["status"] = ops.attn_status()
        if name == "wan128":
            qt, kt, vt = (t.transpose(0, 1)[None].detach().requires_grad_() for t in (q, k, v))
            with torch.nn.attention.sdpa_kernel(torch.nn.attention.SDPBackend.FLASH_ATTENTION):
                out = F.scaled_dot_product_attention(qt, kt, vt)
                g = torch.randn_like(out)
                ms = _time(lambda: F.scaled_dot_product_attention(qt, kt, vt), args.iters)
                row["sdpa_fwd_ms"] = round(ms, 4)
                ms = _time(lambda: torch.autograd.grad(F.scaled_dot_product_attention(qt, kt, vt), (qt, kt, vt), g),
                           args.iters)
                row["sdpa_fwd_bwd_ms"] = round(ms, 4)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
