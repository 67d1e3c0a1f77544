"""CQ cached text-decode latency (reference ``evaluations/benchmarks/main_infra_refactor_20261105.json:169-170``:
34.64 / 36.87 ms per token at prefixes of 323 / 2115 tokens on 910B).

``python -m cq_pretrain_b200.benchmarks.decode [--prefixes 323 2115] [--tokens 64]`` builds the
Qwen3.5-2B backbone (random init, bf16, TP 1), prefills one text document of each prefix length
with the CUDA kernels (the GDN prefill returns each layer's final state from the forward recurrence
kernel), then decodes greedily with ``GraphedCQDecoder``: every step is one CUDA-graph replay of
all 24 layers (the fused recurrent GDN step, KV-cache attention, MLPs) plus the LM-head argmax read
back to the host, exactly as a caption loop runs. Reported per prefix: the median wall ms per
token over the timed tokens (after 4 warm-up tokens) and the median device ms of the graph replay
alone (CUDA events).
"""

from __future__ import annotations

import argparse
import json
import statistics
import time


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--prefixes", type=int, nargs="+", default=[323, 2115])
    parser.add_argument("--tokens", type=int, default=64)
    parser.add_argument("--warmup", type=int, default=4)
    args = parser.parse_args()
    import numpy as np
    import torch
    from ..config import qwen35_2b_wan
    from ..data.synthetic import decode_prompt
    from ..eval.sampling import greedy_token
    from ..models.decoding import GraphedCQDecoder
    from ..parallel import state as ps
    from ..train.trainer import build_model

    ps.initialize(1)
    cfg = qwen35_2b_wan()
    model = build_model(cfg, torch.device("cuda"), seed=3).eval()
    rng = np.random.default_rng(0)
    for prefix in args.prefixes:
        ids = rng.integers(16, cfg.vocab_size, size=prefix)
        batch = decode_prompt(cfg, ids)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        decoder = GraphedCQDecoder(model, batch, args.tokens + args.warmup + 2)
        torch.cuda.synchronize()
        prefill_ms = (time.perf_counter() - t0) * 1e3
        wall, device = [], []
        for step in range(args.tokens + args.warmup):
            start = time.perf_counter()
            token = greedy_token(model, decoder.hidden)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            decoder.advance(token)
            b.record()
            torch.cuda.synchronize()
            if step >= args.warmup:
                wall.append((time.perf_counter() - start) * 1e3)
                device.append(a.elapsed_time(b))
        print(json.dumps(dict(prefix_tokens=prefix, decoded_tokens=len(wall), prefill_ms=round(prefill_ms, 2),
                              ms_per_token=round(statistics.median(wall), 3),
                              device_ms_per_step=round(statistics.median(device), 3),
                              reference_910b_ms_per_token={323: 34.64, 2115: 36.87}.get(prefix),
                              graphed=decoder.graph is not None)), flush=True)


if __name__ == "__main__":
    main()
