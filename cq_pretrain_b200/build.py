"""Build the in-tree sm_100a extension (``python -m cq_pretrain_b200.build``).

Compiles every ``csrc/*.cu`` / ``*.cpp`` with nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) into ``cq_pretrain_b200/_build``,
so the shared library travels with the source tree. Rebuilds are incremental (ninja).
``--debug`` builds the bounds-checked variant into ``_build_debug`` instead (see ``csrc/common.cuh``).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
DEBUG_BUILD = ROOT / "_build_debug"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cutlass_include():
    import site
    for base in site.getsitepackages():
        path = Path(base) / "flashinfer" / "data" / "cutlass" / "include"
        if path.is_dir():
            return str(path)
    return None


def build(verbose=False, debug=False):
    """``debug``: the bounds-checked variant (``-DCQB_DEBUG_BOUNDS``) in ``_build_debug`` as
    ``cqb_kernels_debug``; ``ops._ext`` loads it when ``CQB_DEBUG_BOUNDS=1``."""
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    from torch.utils import cpp_extension

    out = DEBUG_BUILD if debug else BUILD
    out.mkdir(exist_ok=True)
    sources = sorted(str(p) for p in CSRC.glob("*.cu")) + sorted(str(p) for p in CSRC.glob("*.cpp"))
    cuda_flags = ARCH + ["-lineinfo", "-O3", "--use_fast_math", "-std=c++17", "--expt-relaxed-constexpr",
                         "-Xptxas", "-v" if verbose else "-O3", "-DNDEBUG"]
    cflags = ["-O3", "-std=c++17"]
    if debug:
        cuda_flags.append("-DCQB_DEBUG_BOUNDS")
        cflags.append("-DCQB_DEBUG_BOUNDS")
    inc = [str(CSRC)]
    cut = cutlass_include()
    if cut:
        inc.append(cut)
    module = cpp_extension.load(
        name="cqb_kernels_debug" if debug else "cqb_kernels", sources=sources, build_directory=str(out),
        extra_cflags=cflags,
        extra_cuda_cflags=cuda_flags, extra_include_paths=inc, extra_ldflags=["-lcuda"], verbose=verbose,
        with_cuda=True)
    return module


def build_all(verbose=False):
    """The sm_100a kernel library plus the host C++ libraries (SSCD graph)."""
    module = build(verbose)
    from .corpus.sscd import build_library
    build_library()
    return module


if __name__ == "__main__":
    if "--debug" in sys.argv:
        build(verbose="-v" in sys.argv, debug=True)
        print("built", next(DEBUG_BUILD.glob("cqb_kernels_debug*.so")))
        sys.exit(0)
    build_all(verbose="-v" in sys.argv)
    print("built", next(BUILD.glob("cqb_kernels*.so")), BUILD / "sscd_graph.so")
