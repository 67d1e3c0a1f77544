"""Loader for the in-tree sm_100a extension (``cq_pretrain_b200/_build/cqb_kernels*.so``).

The extension is compiled by :func:`cq_pretrain_b200.build.build` (``nvcc -gencode
arch=compute_100a,code=sm_100a``). CUDA tensors always take the kernel path: if the library
is missing on a machine with a GPU, :func:`ops` raises instead of silently falling back.
``CQB_EAGER=1`` deliberately selects the plain-PyTorch path on CUDA (used only to measure the
unfused NCCL + cuBLAS baseline).
"""

from __future__ import annotations

import glob
import importlib.util
import os
import sys
from pathlib import Path

import torch

_DEBUG = os.environ.get("CQB_DEBUG_BOUNDS", "0") == "1"
# CQB_DEBUG_BOUNDS=1 selects the bounds-checked build (``python -m cq_pretrain_b200.build --debug``):
# out-of-range indices in the checked kernels are recorded (``debug_bounds_status``) and skipped.
BUILD_DIR = Path(__file__).resolve().parents[1] / ("_build_debug" if _DEBUG else "_build")
NAME = "cqb_kernels_debug" if _DEBUG else "cqb_kernels"
_MODULE = None
_ERROR = None


def library_path():
    hits = sorted(glob.glob(str(BUILD_DIR / f"{NAME}*.so")))
    return Path(hits[0]) if hits else None


def _load():
    global _MODULE, _ERROR
    if _MODULE is not None or _ERROR is not None:
        return _MODULE
    path = library_path()
    if path is None:
        _ERROR = f"{NAME} is not built (run `python -m cq_pretrain_b200.build`)"
        return None
    spec = importlib.util.spec_from_file_location(NAME, path)
    module = importlib.util.module_from_spec(spec)
    try:
        spec.loader.exec_module(module)
    except Exception as error:  # pragma: no cover - surfaced by ops()
        _ERROR = f"failed to load {path}: {error}"
        return None
    sys.modules[NAME] = module
    _MODULE = module
    return module


def eager_requested() -> bool:
    return os.environ.get("CQB_EAGER", "0") == "1"


def cuda_kernels_enabled() -> bool:
    """True when CUDA ops should run the sm_100a kernels (raises if they are required but missing)."""
    if eager_requested() or not torch.cuda.is_available():
        return False
    if _load() is None:
        raise RuntimeError(f"sm_100a kernels required on this GPU machine: {_ERROR}")
    return True


def has(name: str) -> bool:
    """True when CUDA ops should run and the library exports ``name``."""
    return cuda_kernels_enabled() and hasattr(_MODULE, name)


_GRAPH_LAUNCHES = 0


def add_graph_launches(n: int) -> None:
    """Adjust the count by kernels that CUDA-graph replays run (or a capture recorded without running)."""
    global _GRAPH_LAUNCHES
    _GRAPH_LAUNCHES += int(n)


def launches() -> int:
    """Kernel launches of this library so far, graph replays included (0 when it is not loaded)."""
    if _MODULE is None or not hasattr(_MODULE, "launch_count"):
        return 0
    return int(_MODULE.launch_count()) + _GRAPH_LAUNCHES


def ops():
    module = _load()
    if module is None:
        raise RuntimeError(f"sm_100a kernels unavailable: {_ERROR}")
    return module


def loaded() -> bool:
    return _MODULE is not None
