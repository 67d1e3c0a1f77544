"""Symmetric-memory workspace for in-kernel TP collectives over NVLink peer memory.

Filled in with the fused GEMM/collective kernels; until a workspace is created, the fused
entry points use NCCL + GEMM.
"""

from __future__ import annotations

_WORKSPACE = None


def workspace():
    return _WORKSPACE
