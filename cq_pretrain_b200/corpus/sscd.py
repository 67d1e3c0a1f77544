"""SSCD near-duplicate graph and exact all-pairs search (corpus side, off the training path).

* ``build_library()`` compiles ``sscd_graph.cpp`` (host C++17, ``-O3``) into
  ``cq_pretrain_b200/_build/sscd_graph.so``; ``Graph`` owns one native graph object (CSR
  adjacency by counting sort, BFS components) and copies components, adjacency, statistics and
  greedy one-hop representatives out into NumPy arrays (the behaviour of the reference's
  ``corpus_pipeline/dedup/_sscd_graph.cpp:1-92`` / ``sscd_graph.py:229-253``).
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
NO_REPRESENTATIVE = np.iinfo(np.uint32).max


class _Stats(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint64) for name in ("components", "nontrivial_components", "largest_component",
                                                     "vertices_with_edges", "isolated_vertices", "max_degree")] \
        + [("size_histogram", ctypes.c_uint64 * 32)]


class _Selection(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint64) for name in ("eligible", "representatives", "suppressed", "ineligible",
                                                     "protected_vertices")]


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
        lib = ctypes.CDLL(str(build_library()))
        vp, u64 = ctypes.c_void_p, ctypes.c_uint64
        lib.sscd_last_error.restype = ctypes.c_char_p
        lib.sscd_graph_build.argtypes = [u64, vp, u64, ctypes.c_float, ctypes.POINTER(vp)]
        lib.sscd_graph_free.argtypes = [vp]
        lib.sscd_graph_free.restype = None
        lib.sscd_graph_edges.argtypes = [vp]
        lib.sscd_graph_edges.restype = u64
        lib.sscd_graph_components.argtypes = [vp, vp, vp]
        lib.sscd_graph_adjacency.argtypes = [vp, vp, vp, vp]
        lib.sscd_graph_stats.argtypes = [vp, ctypes.POINTER(_Stats)]
        lib.sscd_graph_select.argtypes = [vp, vp, vp, vp, vp, vp, vp, ctypes.POINTER(_Selection)]
        _LIB = lib
    return _LIB


def _ptr(array):
    if array is None:
        return None
    if not array.flags.c_contiguous:
        raise ValueError("arrays passed to the graph library must be C-contiguous")
    return ctypes.c_void_p(array.ctypes.data)


def _check(rc):
    if rc != 0:
        raise ValueError(f"SSCD graph library: {_lib().sscd_last_error().decode()} (status {rc})")


class Graph:
    """Thresholded similarity graph over ``n`` vertices, held by the native library.

    Attributes copied out at construction: ``label`` (smallest vertex id of each vertex's
    component), ``component_size``, the CSR adjacency ``offsets`` / ``neighbors`` / ``scores``
    (neighbours in edge order), ``summary`` and the log2 component-size ``histogram``.
    """

    def __init__(self, n, edges, threshold):
        edges = np.ascontiguousarray(edges, dtype=EDGE_DTYPE)
        self.n, self.threshold = int(n), float(threshold)
        lib = _lib()
        handle = ctypes.c_void_p()
        _check(lib.sscd_graph_build(self.n, _ptr(edges) if len(edges) else None, len(edges), self.threshold,
                                    ctypes.byref(handle)))
        self._handle = handle
        self.label = np.empty(self.n, np.uint32)
        self.component_size = np.empty(self.n, np.uint32)
        _check(lib.sscd_graph_components(handle, _ptr(self.label), _ptr(self.component_size)))
        m = int(lib.sscd_graph_edges(handle))
        self.offsets = np.empty(self.n + 1, np.uint64)
        self.neighbors = np.empty(2 * m, np.uint32)
        self.scores = np.empty(2 * m, np.float32)
        _check(lib.sscd_graph_adjacency(handle, _ptr(self.offsets), _ptr(self.neighbors), _ptr(self.scores)))
        stats = _Stats()
        _check(lib.sscd_graph_stats(handle, ctypes.byref(stats)))
        self.summary = {name: int(getattr(stats, name)) for name, _ in _Stats._fields_[:6]}
        self.histogram = np.array(list(stats.size_histogram), np.uint64)

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and _LIB is not None:
            _LIB.sscd_graph_free(handle)
            self._handle = None

    def representatives(self, order=None, eligible=None, protect=None):
        """Greedy one-hop selection in ``order`` (default: vertex id). Returns
        ``(representative, direct_score, group_size, summary)``; ineligible vertices get
        ``NO_REPRESENTATIVE``."""
        n = self.n
        order = np.arange(n, dtype=np.uint32) if order is None else np.ascontiguousarray(order, np.uint32)
        if order.shape != (n,):
            raise ValueError("the priority order must list n vertices")
        eligible = None if eligible is None else np.ascontiguousarray(eligible, np.uint8)
        protect = None if protect is None else np.ascontiguousarray(protect, np.uint8)
        rep = np.empty(n, np.uint32)
        direct = np.empty(n, np.float32)
        group = np.empty(n, np.uint32)
        sel = _Selection()
        _check(_lib().sscd_graph_select(self._handle, _ptr(order), _ptr(eligible), _ptr(protect), _ptr(rep),
                                        _ptr(direct), _ptr(group), ctypes.byref(sel)))
        summary = dict(eligible=sel.eligible, representatives=sel.representatives, suppressed=sel.suppressed,
                       ineligible=sel.ineligible, protected=sel.protected_vertices)
        return rep, direct, group, summary


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
