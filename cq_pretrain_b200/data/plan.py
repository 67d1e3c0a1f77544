"""CPU planning of CQ (content/query) execution: visibility, GDN event streams and MRoPE.

Semantics (reference ``ops/attention_layout.py:69-102``, ``ops/gated_delta_layout.py:54-186``,
``data/batch_layout.py:325-386``):

* Content row ``i`` of document ``d`` reads content ``j`` of the same document iff
  ``sigma[j] <= sigma[i]``. Tokens of one image (or one video time block) share a rank, so
  they read each other; everything else is causal.
* A query row (one per supervised text position and one per visual generation query)
  anchored at content position ``p`` reads content ``j`` of its document iff
  ``sigma[j] < sigma[p]``: strictly earlier content, never itself or its own visual block.
  Queries never write attention keys, recurrent state or convolution state.
* Unconditional (non-CFG) visual queries read nothing.

The B200 design never builds a dense ``[S+Q, S]`` mask. Ranks are nondecreasing inside a
document (checked), so every row's visible keys form one contiguous range
``[kstart, kend)``; attention kernels consume these two int32 vectors and skip key tiles
outside the union of a row tile's ranges exactly.

For the Gated DeltaNet layers each document becomes an event stream: content writes in rank
order; the read-only query events of a rank group come right before that group's writes;
a multi-token group (image block) is written in full and then re-read by each member.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, fields

import numpy as np
import torch

from .batch import Batch, Movable


# ----------------------------------------------------------------------------------------
# plan containers
# ----------------------------------------------------------------------------------------
@dataclass
class DeltaPlan(Movable):
    """Per-document GDN event stream (write events and read-only query events)."""

    content_order: torch.Tensor     # [nc] hidden row of each content write, in write order
    content_cu: torch.Tensor        # [docs+1] int32 write boundaries per document
    event_q: torch.Tensor           # [E] row in cat(content conv q [nc], query conv q [nq])
    event_write: torch.Tensor       # [E] content write index, or nc for a read-only event
    event_cu: torch.Tensor          # [docs+1] int32 event boundaries per document
    hidden_event: torch.Tensor      # [rows] event whose output feeds each hidden row
    padding_hidden: torch.Tensor    # [*] hidden rows that receive no GDN output (zeroed)
    query_source: torch.Tensor      # [nq] hidden row of each query event's own projection
    query_history: torch.Tensor     # [nq, K-1] conv history (content index or nc = zero)
    # The same history as CSR keyed by content row (for the query-conv backward, no atomics):
    # rows read by some query, entry offsets per row, entries = query * (K-1) + tap.
    query_hist_rows: torch.Tensor = None
    query_hist_offsets: torch.Tensor = None
    query_hist_entries: torch.Tensor = None
    content_bounds: tuple = ()      # host copy of content_cu
    event_bounds: tuple = ()        # host copy of event_cu
    rows: int = 0
    # Inverse gather maps (see ops/gather.py): backward of each gather is a gather too.
    content_order_inv: tuple = ()
    query_source_inv: tuple = ()
    event_q_inv: tuple = ()
    event_write_inv: tuple = ()
    hidden_event_inv: tuple = ()

    @property
    def events(self) -> int:
        return int(self.event_bounds[-1]) if self.event_bounds else int(self.event_q.numel())


@dataclass
class CQPlan(Movable):
    method: str
    content_length: int                    # S: content rows; query rows follow
    rows: int                              # padded row count of the backbone hidden state
    query_positions: torch.Tensor          # [Q] content anchor of each query
    query_image: torch.Tensor              # [Q] bool: visual (vs text) query
    query_rope: torch.Tensor               # [3, Q] MRoPE coordinates of queries
    query_unconditional: torch.Tensor      # [Q] bool
    output_positions: torch.Tensor         # [Q] slot of each query in the output buffer
    output_size: int
    condition_indices: torch.Tensor        # [n_visual, max_q] output slots of visual queries, -1 pad
    attn_kstart: torch.Tensor              # [rows] int32 first visible key
    attn_kend: torch.Tensor                # [rows] int32 one past the last visible key
    attn_valid: torch.Tensor               # [rows] bool
    rope_cos: torch.Tensor                 # [rows, rotary_dim] float32 (rotate-half layout)
    rope_sin: torch.Tensor
    delta: DeltaPlan = None
    key_tiles: tuple = ()                  # host (row_start, row_end, kmin, kmax) per 128-row tile

    @property
    def queries(self) -> int:
        return int(self.query_positions.numel())

    def dense_mask(self) -> torch.Tensor:
        """[rows, S] bool, True = visible. Oracle / debugging only; the device path never builds it."""
        keys = torch.arange(self.content_length, device=self.attn_kstart.device)
        return (keys[None] >= self.attn_kstart[:, None].long()) & (keys[None] < self.attn_kend[:, None].long())


# ----------------------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------------------
def _documents(segments: np.ndarray):
    """[(doc_id, start, stop)] for contiguous documents with segment >= 0, in position order."""
    docs = []
    seen = set()
    s = len(segments)
    i = 0
    while i < s:
        seg = int(segments[i])
        if seg < 0:
            i += 1
            continue
        j = i
        while j < s and segments[j] == seg:
            j += 1
        if seg in seen:
            raise ValueError("a packed document must occupy contiguous content positions")
        seen.add(seg)
        docs.append((seg, i, j))
        i = j
    return docs


def visual_query_coordinates(grid, count, mode):
    """(t, h, w) offsets of a visual's queries on its merged grid (reference ``data/batch_layout.py:302-322``)."""
    t, h, w = grid
    h //= 2
    w //= 2
    if mode == "native":
        tt, hh, ww = np.meshgrid(np.arange(t), np.arange(h), np.arange(w), indexing="ij")
        return np.stack((tt.ravel(), hh.ravel(), ww.ravel())).astype(np.float64)
    nt = min(t, count)
    nh = max(1, math.ceil(math.sqrt(count / nt * h / w)))
    nw = math.ceil(count / (nt * nh))
    axes = [(np.arange(n) + 0.5) * (size / n) - 0.5 for n, size in zip((nt, nh, nw), (t, h, w))]
    grid3 = np.stack([a.ravel() for a in np.meshgrid(*axes, indexing="ij")])
    chosen = ((np.arange(count) + 0.5) * grid3.shape[1] / count).astype(np.int64)
    return grid3[:, chosen].astype(np.float64)


def visual_query_count(grid, cfg) -> int:
    return math.prod(grid) // 4 if cfg.visual_query_mode == "native" else cfg.image_condition_queries


def mrope_tables(positions: torch.Tensor, cfg):
    """Interleaved (t, h, w) MRoPE over the partial rotary dims, computed in float64.

    Frequency index ``i`` uses the h coordinate when ``i % 3 == 1`` and ``i < 3*sections[1]``,
    the w coordinate when ``i % 3 == 2`` and ``i < 3*sections[2]``, else t
    (reference ``ops/gated_delta_layout.py:209-219``). Returns cos/sin ``[rows, rotary_dim]``.
    """
    dim = cfg.rotary_dim
    pos = positions.double()
    inv = cfg.rope_theta ** (-torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    axis = torch.zeros(dim // 2, dtype=torch.long)
    idx = torch.arange(dim // 2)
    for a in (1, 2):
        axis[(idx % 3 == a) & (idx < 3 * cfg.mrope_section[a])] = a
    chosen = pos.index_select(0, axis.clone()) if pos.shape[0] == 3 else pos[:1].expand(dim // 2, -1)
    # chosen[i, r] = coordinate of row r on the axis that frequency i uses
    angles = (chosen.T * inv[None])
    angles = torch.cat((angles, angles), -1)
    return angles.cos().float(), angles.sin().float()


# ----------------------------------------------------------------------------------------
# planner
# ----------------------------------------------------------------------------------------
def build_plan(batch: Batch, cfg, pad_multiple: int = 1) -> CQPlan:
    """Plan one packed sequence for the CQ_IT method (queries for text and visual targets)."""
    if batch.ids.device.type != "cpu" or batch.ids.shape[0] != 1:
        raise ValueError("plan CQ batches on CPU with micro-batch 1")
    if cfg.method != "CQ_IT":
        raise ValueError("the Wan renderer trains with the CQ_IT method")
    s = batch.ids.shape[1]
    segments = batch.segments[0].numpy()
    sigma = batch.sigma[0].numpy().astype(np.int64)
    if cfg.content_visibility == "causal":
        sigma = np.arange(s, dtype=np.int64)
    positions = batch.positions.double()
    if positions.shape[0] == 2:  # legacy (h, w) layouts: temporal axis follows the row axis
        positions = torch.cat((positions[:1], positions))
    spans = [row[row >= 0] for row in batch.image_indices]
    grids = batch.vision.grid_thw if (spans and batch.vision is not None) else ()
    if spans and len(grids) != len(spans):
        raise ValueError("visual spans need matching vision grids")
    selected = (list(range(len(spans))) if batch.generation_image_indices is None
                else batch.generation_image_indices.tolist())
    counts = [visual_query_count(g, cfg) for g in grids]
    text = batch.text_indices.numpy().astype(np.int64)
    maxq = max((counts[i] for i in selected), default=0)
    conditions = np.full((len(spans), maxq), -1, dtype=np.int64)
    offset = s
    for i in selected:
        conditions[i, : counts[i]] = np.arange(offset, offset + counts[i])
        offset += counts[i]
    q_pos = [text]
    q_rope = [positions[:, torch.from_numpy(text)]]
    q_uncond = [np.zeros(len(text), dtype=bool)]
    outputs = [text]
    for i in selected:
        span = spans[i].numpy()
        grid = grids[i]
        n = counts[i]
        if len(span) != math.prod(grid) // 4:
            raise ValueError("visual span length differs from its merged grid")
        coords = visual_query_coordinates(grid, n, cfg.visual_query_mode)
        blocks = span.reshape(grid[0], -1)[:, 0]
        bases = positions[:, torch.from_numpy(blocks)].numpy()
        ti = np.clip(coords[0], 0, grid[0] - 1)
        lo = np.floor(ti).astype(np.int64)
        hi = np.minimum(lo + 1, grid[0] - 1)
        interp = bases[:, lo] + (bases[:, hi] - bases[:, lo]) * (ti - lo)
        coords = coords.copy()
        coords[0] = interp[0]
        coords[1:] += interp[1:]
        q_pos.append(np.full(n, span[0], dtype=np.int64))
        q_rope.append(torch.from_numpy(coords))
        unc = bool(batch.generation_unconditional[i]) if batch.generation_unconditional is not None else False
        q_uncond.append(np.full(n, unc, dtype=bool))
        outputs.append(conditions[i, :n])
    query_positions = np.concatenate(q_pos) if q_pos else np.zeros(0, np.int64)
    query_unconditional = np.concatenate(q_uncond)
    query_image = np.concatenate([np.zeros(len(text), bool)] + [np.ones(counts[i], bool) for i in selected])
    query_rope = torch.cat(q_rope, dim=1) if q_rope else torch.zeros(3, 0, dtype=torch.float64)
    nq = len(query_positions)
    rows = s + nq
    rows_padded = -(-rows // pad_multiple) * pad_multiple if pad_multiple > 1 else rows

    # ---- attention key ranges ------------------------------------------------------------
    kstart = np.zeros(rows_padded, dtype=np.int32)
    kend = np.zeros(rows_padded, dtype=np.int32)
    docs = _documents(segments)
    doc_of = {}
    for seg, a, b in docs:
        sig = sigma[a:b]
        if np.any(np.diff(sig) < 0):
            raise ValueError("visibility ranks must be nondecreasing inside a document")
        doc_of[seg] = (a, b)
        kstart[a:b] = a
        kend[a:b] = a + np.searchsorted(sig, sig, side="right")
    for j in range(nq):
        p = int(query_positions[j])
        seg = int(segments[p])
        if seg < 0 or query_unconditional[j]:
            continue
        a, b = doc_of[seg]
        end = a + int(np.searchsorted(sigma[a:b], sigma[p], side="left"))
        if end > a:
            kstart[s + j] = a
            kend[s + j] = end
    valid = kend > kstart

    # ---- rope --------------------------------------------------------------------------
    all_pos = torch.cat((positions, query_rope, torch.zeros(3, rows_padded - rows, dtype=torch.float64)), dim=1)
    cos, sin = mrope_tables(all_pos, cfg)

    delta = build_delta_plan(segments, sigma, query_positions, query_unconditional, s, rows_padded,
                             cfg.linear_conv_kernel)
    tiles = []
    for r0 in range(0, rows_padded, 128):
        r1 = min(r0 + 128, rows_padded)
        v = valid[r0:r1]
        if v.any():
            tiles.append((r0, r1, int(kstart[r0:r1][v].min()), int(kend[r0:r1][v].max())))
        else:
            tiles.append((r0, r1, 0, 0))
    return CQPlan(
        method=cfg.method, content_length=s, rows=rows_padded,
        query_positions=torch.from_numpy(query_positions), query_image=torch.from_numpy(query_image),
        query_rope=query_rope.float(), query_unconditional=torch.from_numpy(query_unconditional),
        output_positions=torch.from_numpy(np.concatenate(outputs) if outputs else np.zeros(0, np.int64)),
        output_size=offset, condition_indices=torch.from_numpy(conditions),
        attn_kstart=torch.from_numpy(kstart), attn_kend=torch.from_numpy(kend), attn_valid=torch.from_numpy(valid),
        rope_cos=cos, rope_sin=sin, delta=delta, key_tiles=tuple(tiles))


def build_delta_plan(segments, sigma, query_positions, query_unconditional, s, rows, conv_kernel) -> DeltaPlan:
    docs = _documents(segments)
    if not docs:  # an all-padding pack still runs a one-write graph so every parameter sees a gradient
        docs = [(0, 0, 1)]
        segments = segments.copy()
        segments[0] = 0
    queries_by_doc: dict = {}
    for j, p in enumerate(query_positions.tolist()):
        seg = int(segments[p])
        if seg < 0:
            continue
        key = None if query_unconditional[j] else int(sigma[p])
        queries_by_doc.setdefault(seg, {}).setdefault(key, []).append(j)
    order, event_q, event_write, out_event, out_hidden = [], [], [], [], []
    q_source, q_history = [], []
    content_cu, event_cu = [0], [0]
    hist_len = conv_kernel - 1
    READ = -1
    for seg, a, b in docs:
        groups: dict = {}
        for i in range(a, b):
            groups.setdefault(int(sigma[i]), []).append(i)
        queries = dict(queries_by_doc.get(seg, {}))
        if None in queries:  # non-CFG queries read first: zero state, empty conv history
            first = next(iter(groups))
            queries[first] = queries.pop(None) + queries.get(first, [])
        history: list = []
        for rank, members in groups.items():
            for j in queries.get(rank, []):
                qi = len(q_source)
                q_source.append(s + j)
                prev = history[-hist_len:] if hist_len else []
                q_history.append([READ] * (hist_len - len(prev)) + prev)
                event_q.append(("q", qi))
                event_write.append(READ)
                out_event.append(len(event_q) - 1)
                out_hidden.append(s + j)
            written = []
            for i in members:
                ci = len(order)
                order.append(i)
                written.append((ci, i))
                event_q.append(("c", ci))
                event_write.append(ci)
                history.append(ci)
                if len(members) == 1:
                    out_event.append(len(event_q) - 1)
                    out_hidden.append(i)
            if len(members) > 1:  # bidirectional block: re-read after the whole group is written
                for ci, i in written:
                    event_q.append(("c", ci))
                    event_write.append(READ)
                    out_event.append(len(event_q) - 1)
                    out_hidden.append(i)
        content_cu.append(len(order))
        event_cu.append(len(event_q))
    nc = len(order)
    eq = np.array([i if kind == "c" else nc + i for kind, i in event_q], dtype=np.int64)
    ew = np.array([nc if w == READ else w for w in event_write], dtype=np.int64)
    n_events = len(event_q)
    hidden_event = np.full(rows, n_events, dtype=np.int64)   # rows without output read a zero row
    has = np.zeros(rows, dtype=bool)
    if out_hidden:
        hidden_event[np.array(out_hidden)] = np.array(out_event)
        has[np.array(out_hidden)] = True
    qh = np.array([[nc if x == READ else x for x in row] for row in q_history], dtype=np.int64).reshape(-1, hist_len)
    from ..ops.gather import inverse_levels
    order_np = np.array(order, dtype=np.int64)
    qsrc_np = np.array(q_source, dtype=np.int64)
    inverses = dict(content_order_inv=inverse_levels(order_np, rows), query_source_inv=inverse_levels(qsrc_np, rows),
                    event_q_inv=inverse_levels(eq, nc + len(q_source)), event_write_inv=inverse_levels(ew, nc + 1, ignore=nc),
                    hidden_event_inv=inverse_levels(hidden_event, n_events + 1, ignore=n_events))
    flat = qh.reshape(-1)
    used = np.nonzero(flat != nc)[0]
    order_h = used[np.argsort(flat[used], kind="stable")]
    hist_rows, counts = np.unique(flat[order_h], return_counts=True)
    hist_offsets = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
    return DeltaPlan(**inverses,
        query_hist_rows=torch.from_numpy(hist_rows.astype(np.int32)),
        query_hist_offsets=torch.from_numpy(hist_offsets),
        query_hist_entries=torch.from_numpy(order_h.astype(np.int32)),
        content_order=torch.from_numpy(np.array(order, dtype=np.int64)),
        content_cu=torch.tensor(content_cu, dtype=torch.int32),
        event_q=torch.from_numpy(eq), event_write=torch.from_numpy(ew),
        event_cu=torch.tensor(event_cu, dtype=torch.int32),
        hidden_event=torch.from_numpy(hidden_event),
        padding_hidden=torch.from_numpy(np.nonzero(~has)[0].astype(np.int64)),
        query_source=torch.from_numpy(np.array(q_source, dtype=np.int64)),
        query_history=torch.from_numpy(qh),
        content_bounds=tuple(content_cu), event_bounds=tuple(event_cu), rows=rows)
