"""SSCD near-duplicate graph and exact all-pairs search (corpus side, off the training path).

* ``build_library()`` compiles ``sscd_graph.cpp`` (host C++17, ``-O3``) into
  ``cq_pretrain_b200/_build/sscd_graph.so``; ``Graph`` drives it through ctypes on NumPy arrays:
  components, CSR adjacency and greedy one-hop representatives over thresholded edges
  (reference ``corpus_pipeline/dedup/_sscd_graph.cpp:1-92``, ``sscd_graph.py:229-253``).
* ``exact_pairs(left, right, threshold)`` finds every pair with cosine >= threshold: tiled
  ``left @ right^T`` on the tcgen05 GEMM in bf16 with a safety margin, threshold compaction on
  the GPU, then an fp32 rerank of the candidates (reference
  ``corpus_pipeline/postprocess/sscd_exact_npu.py:250-277``). ``left is right`` searches one set
  against itself (pairs i < j only).

Edge records are ``EDGE_DTYPE`` = {uint32 a, uint32 b, float32 score} with ``a < b``.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

SOURCE = Path(__file__).resolve().with_name("sscd_graph.cpp")
LIBRARY = Path(__file__).resolve().parents[1] / "_build" / "sscd_graph.so"
EDGE_DTYPE = np.dtype([("a", "<u4"), ("b", "<u4"), ("score", "<f4")])
ERRORS = {1: "too many vertices", 2: "malformed edge or score below threshold", 3: "malformed edge",
          4: "adjacency row overflow", 5: "priority order out of range", 6: "bad neighbour or score",
          7: "inconsistent representatives"}


def build_library(force=False) -> Path:
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < SOURCE.stat().st_mtime:
        LIBRARY.parent.mkdir(parents=True, exist_ok=True)
        tmp = LIBRARY.with_suffix(".tmp.so")
        subprocess.run(["g++", "-O3", "-std=c++17", "-fPIC", "-shared", str(SOURCE), "-o", str(tmp)], check=True)
        tmp.replace(LIBRARY)
    return LIBRARY


_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(str(build_library()))
    return _LIB


def _call(name, *args):
    conv = []
    for a in args:
        if isinstance(a, np.ndarray):
            if not a.flags.c_contiguous:
                raise ValueError(f"{name}: arrays must be C-contiguous")
            conv.append(ctypes.c_void_p(a.ctypes.data))
        elif isinstance(a, float):
            conv.append(ctypes.c_float(a))
        else:
            conv.append(ctypes.c_uint64(int(a)))
    rc = getattr(_lib(), name)(*conv)
    if rc != 0:
        raise ValueError(f"{name} failed ({rc}): {ERRORS.get(rc, 'unknown error')}")


class Graph:
    """Thresholded similarity graph over ``n`` vertices."""

    def __init__(self, n, edges, threshold):
        edges = np.ascontiguousarray(edges, dtype=EDGE_DTYPE)
        self.n, self.threshold, self.edges = int(n), float(threshold), edges
        self.parent = np.empty(n, np.uint32)
        self.size = np.empty(n, np.uint32)
        self.degree = np.empty(n, np.uint64)
        _call("sscd_init", n, self.parent, self.size, self.degree)
        _call("sscd_union", n, len(edges), edges, self.parent, self.size, self.degree, self.threshold)
        self.label = np.empty(n, np.uint32)
        self.component_size = np.empty(n, np.uint32)
        self.offsets = np.empty(n + 1, np.uint64)
        summary = np.empty(6, np.uint64)
        self.histogram = np.empty(32, np.uint64)
        _call("sscd_components", n, self.parent, self.size, self.degree, self.label, self.component_size,
              self.offsets, summary, self.histogram)
        self.summary = dict(zip(("components", "nontrivial_components", "largest_component", "vertices_with_edges",
                                 "isolated_vertices", "max_degree"), summary.tolist()))
        self.neighbors = np.empty(int(self.offsets[-1]), np.uint32)
        self.scores = np.empty(int(self.offsets[-1]), np.float32)
        cursor = self.offsets[:-1].copy()
        _call("sscd_fill", n, len(edges), edges, self.offsets, cursor, self.neighbors, self.scores)

    def representatives(self, order=None, eligible=None, protect=None):
        """Greedy one-hop selection in ``order`` (default: vertex id). Returns
        ``(representative, direct_score, group_size, summary)``."""
        n = self.n
        order = np.arange(n, dtype=np.uint32) if order is None else np.ascontiguousarray(order, np.uint32)
        eligible = np.ones(n, np.uint8) if eligible is None else np.ascontiguousarray(eligible, np.uint8)
        protect = np.zeros(n, np.uint8) if protect is None else np.ascontiguousarray(protect, np.uint8)
        rep = np.empty(n, np.uint32)
        direct = np.empty(n, np.float32)
        group = np.empty(n, np.uint32)
        summary = np.empty(5, np.uint64)
        _call("sscd_representatives", n, self.offsets, self.neighbors, self.scores, order, eligible, protect, rep,
              direct, group, summary, self.threshold)
        return rep, direct, group, dict(zip(("eligible", "representatives", "suppressed", "ineligible", "protected"),
                                             summary.tolist()))


def exact_pairs(left, right, threshold, tile=8192, margin=0.02, device=None):
    """All (i, j, score) with ``left[i] . right[j] >= threshold`` (rows L2-normalised), as edges.

    With ``right is left`` only pairs i < j are returned. bf16 products find candidates with
    ``score >= threshold - margin``; each candidate is rescored in fp32 before the final cut.
    """
    import torch
    same = right is left
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    lt = torch.as_tensor(np.asarray(left, np.float32), device=dev)
    rt = lt if same else torch.as_tensor(np.asarray(right, np.float32), device=dev)
    lb, rb = (lt.to(torch.bfloat16), rt.to(torch.bfloat16)) if dev.type == "cuda" else (lt, rt)
    from ..ops import gemm
    out = []
    for i0 in range(0, lt.shape[0], tile):
        for j0 in range(i0 if same else 0, rt.shape[0], tile):
            a, b = lb[i0:i0 + tile], rb[j0:j0 + tile]
            scores = gemm.linear(a, b) if dev.type == "cuda" else a @ b.T
            keep = scores.float() >= threshold - margin
            if same and j0 == i0:
                keep &= torch.ones_like(keep).triu(1)
            ii, jj = keep.nonzero(as_tuple=True)
            if not ii.numel():
                continue
            exact = (lt[i0 + ii] * rt[j0 + jj]).sum(-1)   # fp32 rerank
            ok = exact >= threshold
            out.append(torch.stack(((ii[ok] + i0).double(), (jj[ok] + j0).double(), exact[ok].double()), 1).cpu())
    if not out:
        return np.zeros(0, EDGE_DTYPE)
    rows = torch.cat(out).numpy()
    edges = np.zeros(len(rows), EDGE_DTYPE)
    edges["a"], edges["b"], edges["score"] = rows[:, 0], rows[:, 1], rows[:, 2]
    if not same:
        return edges
    return edges[np.lexsort((edges["b"], edges["a"]))]
