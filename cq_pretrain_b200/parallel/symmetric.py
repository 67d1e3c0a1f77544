"""Symmetric peer-memory workspace for the in-kernel TP collectives (one process per GPU).

Every rank of a TP group allocates one buffer with the same layout, exchanges CUDA IPC
handles, and opens every peer's buffer (NVLink P2P). Layout::

    [0, 512)        all-gather flags: slot s = last epoch rank s published its shard
    [512, 1024)     (unused) reduce-scatter flags of the former three-kernel path
    [2048, 2052)    all-gather staging counter (own sub-chunks staged in the running call)
    send[0], send[1]   this rank's staged shard for all-gather (double-buffered by epoch parity)
    recv[0], recv[1]   [tp, rows/tp, N] partial slabs written by peers for reduce-scatter
    stat flags         [row blocks][8] epoch flags of the row-statistic exchange (TP RMSNorm)
    stat[0], stat[1]   [tp, max_rows] fp32 per-row partials written by peers (parity buffered)
    rs stamps          [tiles][8 sources][4 warps] int64 epoch stamps of GEMM -> reduce-scatter tiles

Protocol (epochs count calls of each kind; every rank issues the same sequence):

* all-gather -> GEMM (epoch e): one kernel. The tensor cores read this rank's rows straight from
  the caller's shard; the copy warps stage that shard into ``send[e % 2]``, publish flag e to every
  peer once the whole shard is staged, pull each peer's shard into the gather buffer sub-chunk by
  sub-chunk (after acquiring that peer's flag) while the tensor cores consume the blocks already
  present, and finally copy the own rows into the gather buffer (the gathered output).
* GEMM -> reduce-scatter (epoch e): one kernel. Tiles of rows owned by another rank are stored
  into the owner's ``recv[e % 2][src]`` and stamped with e in the owner's (tile, src, warp) slot;
  this rank's own tiles come last, wait for the peers' stamps of the same tile, and add the
  peers' bf16 partials to their fp32 accumulator (and the bias) before storing the result.
* row statistics (epoch e, Wan's full-width Q/K RMSNorm (q and k in one call, with the RoPE of the
  self-attention fused), and the vocabulary-parallel cross-entropy's
  (max, sum exp, target logit) triples): one kernel per call; each 64-row block
  stores its partial sums into ``stat[e % 2][rank]`` of every peer, publishes a per-block flag and
  acquires the peers' flags of the same block before normalising its rows.

Double buffering plus the flag order makes buffer reuse safe: a rank can only overwrite a slot
of parity p at epoch e after every peer has signalled epoch e-1, which each peer does only after
its own epoch e-2 work (the last reader/writer of that slot) completed in stream order.
All waits are bounded in the kernels and report a status code instead of hanging.

Epochs live on the device: each kind (all-gather, reduce-scatter, statistics) has an int64 counter
in local memory that a call's kernel reads at its start (epoch = counter + 1) and its last CTA
advances at its end, and the kernel picks the parity buffers from the epoch it read. A CUDA graph
that captured fused TP calls therefore takes fresh epochs on every replay, interleaved correctly
with eager calls of the same kind. The host passes both parities' buffers and counts calls only
for reporting.
"""

from __future__ import annotations

from contextlib import contextmanager

import torch
import torch.distributed as dist

from ..ops import _ext
from . import state as ps

FLAG_BYTES = 1024
_WORKSPACE = None


def _align(n, a=4096):
    return -(-n // a) * a


class SymmetricWorkspace:
    def __init__(self, send_bytes=192 << 20, recv_bytes=384 << 20, max_subchunks=8192, stat_rows=131072,
                 rs_tiles=8192):
        st = ps.state()
        if st.tp < 2:
            raise ValueError("symmetric workspace needs TP >= 2")
        ops = _ext.ops()
        self.tp, self.rank, self.group = st.tp, st.tp_rank, st.tp_group
        self.send_bytes, self.recv_bytes = _align(send_bytes), _align(recv_bytes)
        self.off_send = [FLAG_BYTES * 4, FLAG_BYTES * 4 + self.send_bytes]
        self.off_recv = [self.off_send[1] + self.send_bytes, self.off_send[1] + self.send_bytes + self.recv_bytes]
        self.stat_rows = stat_rows
        stat_blocks = -(-stat_rows // 64)
        self.off_stat_flags = self.off_recv[1] + self.recv_bytes
        stat_bytes = _align(self.tp * stat_rows * 4)
        self.off_stat = [self.off_stat_flags + _align(stat_blocks * 8 * 8), 0]
        self.off_stat[1] = self.off_stat[0] + stat_bytes
        self.rs_slots = rs_tiles * 8 * 4
        self.off_rs_flags = self.off_stat[1] + stat_bytes
        total = self.off_rs_flags + _align(self.rs_slots * 8)
        ptr, handle = ops.symm_alloc(total)
        self.base = int(ptr[0])
        handles = [None] * self.tp
        dist.all_gather_object(handles, handle.numpy().tobytes(), group=self.group)
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self.base)
            else:
                bases.append(ops.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
        self.bases = bases
        dev = torch.device("cuda", torch.cuda.current_device())
        as_dev = lambda xs: torch.tensor(xs, dtype=torch.int64, device=dev)
        self.flag_ag = as_dev([b for b in bases])                       # slot array base of each peer
        self.flag_rs = as_dev([b + 512 for b in bases])
        self.send = [as_dev([b + self.off_send[p] for b in bases]) for p in range(2)]
        self.recv = [as_dev([b + self.off_recv[p] for b in bases]) for p in range(2)]
        self.stat_flags = as_dev([b + self.off_stat_flags for b in bases])
        self.stat = [as_dev([b + self.off_stat[p] for b in bases]) for p in range(2)]
        self.rs_flags = as_dev([b + self.off_rs_flags for b in bases])
        # one publication flag per 16 gathered rows (the all-gather copy unit)
        self.chunk_flags = torch.zeros(max_subchunks, dtype=torch.int64, device=dev)
        # device epoch counters and finished-CTA counts of the three kinds (all-gather, RS, statistics)
        self.ectr = torch.zeros(3, dtype=torch.int64, device=dev)
        self.edone = torch.zeros(3, dtype=torch.int32, device=dev)
        self._ctr = [self.ectr.data_ptr() + 8 * k for k in range(3)]
        self._done = [self.edone.data_ptr() + 4 * k for k in range(3)]
        self.epoch_ag = self.epoch_rs = self.epoch_stat = 0   # host-issued calls (reporting only)
        dist.barrier(group=self.group)

    def device_epochs(self):
        """The device counters (all_gather, reduce_scatter, statistics): calls completed on the
        device, CUDA-graph replays included (reads the counters, so it synchronises)."""
        ag, rs, stat = self.ectr.tolist()
        return dict(all_gather=ag, reduce_scatter=rs, statistics=stat)

    # ---- eligibility --------------------------------------------------------------------------
    def supports(self, x, w, transposed=False):
        if not (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2):
            return False
        rows = x.shape[0]
        n_out = w.shape[1] if transposed else w.shape[0]   # dY @ W (transposed) or x @ W^T
        return (rows % (128 * self.tp) == 0 and n_out % 16 == 0 and x.shape[1] % 16 == 0
                and rows * n_out * 2 <= self.recv_bytes and x.data_ptr() % 16 == 0)

    def supports_gather(self, x, w, transposed=False):
        n_out = w.shape[1] if transposed else w.shape[0]   # all_gather(x) @ W (transposed) or @ W^T
        return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
                and x.shape[1] % 16 == 0 and n_out % 16 == 0 and self._gather_ok(x))

    def _gather_ok(self, x):
        rows = x.shape[0] * self.tp
        return (x.shape[0] % 128 == 0 and x.numel() * 2 <= self.send_bytes and rows // 16 <= self.chunk_flags.numel()
                and x.shape[1] % 8 == 0 and (not x.is_contiguous() or x.data_ptr() % 16 == 0))

    # ---- fused ops --------------------------------------------------------------------------------
    def gather_linear(self, x, weight, bias=None):
        """``(all_gather(x) @ W^T + b, all_gather(x))`` in one all-gather->GEMM kernel."""
        return self._gather(x, weight, bias, False)

    def gather_matmul(self, dy, weight):
        """``(all_gather(dY) @ W, all_gather(dY))`` for ``W [K, N]``: the input gradient of a
        row-parallel linear, gathered inside the GEMM (the gathered rows feed the weight gradient)."""
        return self._gather(dy, weight, None, True)

    def _gather(self, x, weight, bias, mn_major):
        ops = _ext.ops()
        if not self._gather_ok(x):
            from .fused import gather_rows_raw
            from ..ops import gemm
            xg = gather_rows_raw(x)
            return (gemm.matmul_nn(xg, weight) if mn_major else gemm.linear(xg, weight, bias)), xg
        self.epoch_ag += 1
        rows = x.shape[0]
        xg = torch.empty(rows * self.tp, x.shape[1], dtype=x.dtype, device=x.device)
        y = ops.gather_gemm(xg, weight.contiguous(), bias, self.send[0], self.base, self.chunk_flags, 0, rows,
                            self.rank, self.tp, mn_major, x_local=x.contiguous(),
                            send_mine=self.base + self.off_send[0], peer_ready=self.flag_ag,
                            own_done=self.base + 2 * FLAG_BYTES, epoch_ctr=self._ctr[0], epoch_done=self._done[0],
                            peer_in_odd=self.send[1], send_mine_odd=self.base + self.off_send[1])
        return y, xg

    def _scatter(self, x, weight, mn_major, x2=None, w2=None, bias=None):
        self.epoch_rs += 1
        rows = x.shape[0] // self.tp
        if x2 is not None:
            x2, w2 = x2.contiguous(), w2.contiguous()
        return _ext.ops().gemm_scatter_reduce(
            x.contiguous(), weight.contiguous(), mn_major, x2, w2, bias, self.recv[0], self.base + self.off_recv[0],
            self.rs_flags, self.base + self.off_rs_flags, self.rs_slots, 0, rows, self.rank, self.tp,
            epoch_ctr=self._ctr[1], epoch_done=self._done[1], peer_recv_odd=self.recv[1],
            my_recv_odd=self.base + self.off_recv[1])

    def supports_scatter(self, x, w, transposed=False, x2=None, w2=None):
        """Eligibility of the one-kernel GEMM -> reduce-scatter (optionally with a second operand pair)."""
        if not self.supports(x, w, transposed):
            return False
        n_out = w.shape[1] if transposed else w.shape[0]
        tiles = (x.shape[0] // self.tp // 128) * -(-n_out // 256)
        if tiles * 32 > self.rs_slots or self.tp > 8:
            return False
        if x2 is None:
            return True
        return (x2.is_cuda and x2.dtype == torch.bfloat16 and w2.dtype == torch.bfloat16 and x2.dim() == 2
                and 0 < x2.shape[0] <= x.shape[0] and x2.shape[1] % 16 == 0 and x2.data_ptr() % 16 == 0
                and (w2.shape[1] if transposed else w2.shape[0]) == n_out)

    # ---- row statistics ----------------------------------------------------------------------
    def supports_rms(self, x):
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
                and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0 and x.shape[1] % 8 == 0
                and x.shape[1] <= 2048 and -(-x.shape[0] // 64) * 64 <= self.stat_rows)

    def supports_qk(self, q, k):
        """Eligibility of the fused q / k norm (+ RoPE): both tensors in one exchange."""
        return (self.supports_rms(q) and self.supports_rms(k) and q.shape == k.shape
                and 2 * (-(-q.shape[0] // 64) * 64) <= self.stat_rows and _ext.has("qk_norm_rope_fwd"))

    def exchange_kwargs(self):
        """Keyword arguments of one row-statistic exchange call (the statistics kind's slabs,
        flags and device epoch counter); every rank must make the same sequence of such calls."""
        self.epoch_stat += 1
        return dict(peer_recv=self.stat[0], my_recv=self.base + self.off_stat[0], peer_flags=self.stat_flags,
                    my_flags=self.base + self.off_stat_flags, rank=self.rank, tp=self.tp, max_rows=self.stat_rows,
                    epoch_ctr=self._ctr[2], epoch_done=self._done[2], peer_recv_odd=self.stat[1],
                    my_recv_odd=self.base + self.off_stat[1])

    def _stat_kwargs(self):
        return dict(self.exchange_kwargs(), epoch=0)

    def rms_forward(self, x, weight, total_dim, eps):
        return _ext.ops().tp_rms_fwd(x, weight, total_dim=total_dim, eps=eps, **self._stat_kwargs())

    def rms_backward(self, dy, x, weight, rstd, total_dim):
        return _ext.ops().tp_rms_bwd(dy, x, weight, rstd, total_dim=total_dim, **self._stat_kwargs())

    def supports_ce(self, rows):
        return 3 * (-(-rows // 64) * 64) <= self.stat_rows and _ext.has("ce_combine_tp")

    def ce_combine(self, part, tgt_local):
        """Full-vocabulary (lse, target logit) per row from this rank's LM-head partials: the
        (max, sum exp, target) triples cross NVLink inside one kernel (no NCCL call)."""
        return _ext.ops().ce_combine_tp(part, tgt_local, **self._stat_kwargs())

    def linear_scatter(self, x, weight, bias=None):
        """``reduce_scatter_rows(x @ W^T) + b`` in one GEMM -> reduce-scatter kernel."""
        return self._scatter(x, weight, False, bias=bias)

    def matmul_scatter(self, dy, weight, dy2=None, weight2=None):
        """``reduce_scatter_rows(dY @ W [+ dY2 @ W2])`` (input gradient of one or two column-parallel
        projections of the same gathered input; ``dY2`` may cover only its first rows)."""
        return self._scatter(dy, weight, True, dy2, weight2)

    def close(self):
        ops = _ext.ops()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for r, b in enumerate(self.bases):
            if r != self.rank:
                ops.symm_close(b)
        dist.barrier(group=self.group)
        ops.symm_free(self.base)


_SUSPENDED = 0


def workspace():
    return None if _SUSPENDED else _WORKSPACE


@contextmanager
def suspended():
    """Route the TP linears through NCCL + the plain GEMM inside this block (for comparisons
    and for work that one rank runs without its peers)."""
    global _SUSPENDED
    _SUSPENDED += 1
    try:
        yield
    finally:
        _SUSPENDED -= 1


def enable(**kwargs):
    """Create the TP workspace (collective over the TP group); fused linears use it from now on."""
    global _WORKSPACE
    if _WORKSPACE is None and ps.tp_size() > 1 and _ext.has("gather_gemm"):
        _WORKSPACE = SymmetricWorkspace(**kwargs)
    return _WORKSPACE


def disable():
    global _WORKSPACE
    if _WORKSPACE is not None:
        _WORKSPACE.close()
    _WORKSPACE = None


def status(reset=True):
    ops = _ext.ops()
    return dict(gemm=ops.gemm_status(reset), comm=ops.comm_status_read(reset))
