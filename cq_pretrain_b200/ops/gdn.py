"""Gated DeltaNet ops: chunked gated delta rule over CQ event streams and the causal short conv.

``gated_delta`` takes event-ordered q, k ``[E, H, Dk]``, v ``[E, H, Dv]``, log-decay g and
beta ``[E, H]`` (fp32) and per-document event boundaries; q/k are L2-normalised inside
(``use_qk_l2norm_in_kernel``). Read-only query events carry k = v = 0, beta = 0, g = 0, so they
read the state without changing it (reference ``ops/gated_delta_net.py:143-214``).

CUDA runs ``csrc/gdn.cu``: a chunk-parallel kernel builds the WY factors (T = (I+A)^-1, W, U)
for every 64-event chunk, a per-(document, head) kernel carries the 128x128 fp32 state across
chunks, and the backward mirrors both passes in reverse. CPU runs the chunked reference.
"""

from __future__ import annotations

import torch

from . import _ext
from . import reference as R


def _kernel(q):
    return q.is_cuda and _ext.cuda_kernels_enabled() and hasattr(_ext.ops(), "gdn_fwd")


def gated_delta(q, k, v, g, beta, bounds, chunk=64):
    if _kernel(q):
        from .gdn_cuda import gated_delta_cuda
        return gated_delta_cuda(q, k, v, g, beta, bounds, chunk)
    return R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk).to(v.dtype)


def causal_conv_silu(x, weight, bounds):
    """Causal depthwise conv + SiLU per document over content order; x ``[n, C]``, weight ``[C, K]``."""
    if x.is_cuda and _ext.cuda_kernels_enabled() and hasattr(_ext.ops(), "conv_fwd") and x.dtype == torch.bfloat16:
        from .gdn_cuda import causal_conv_cuda
        return causal_conv_cuda(x, weight, bounds)
    return R.causal_conv_silu(x, weight, bounds)
