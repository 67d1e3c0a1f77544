"""Exact model-only conversion of saved TP shards to another TP size.

Approach: rebuild each full (unsharded) tensor from the saved shards, then cut the destination
rank's slice out of it with the same rule that loads official full checkpoints
(``parallel.layers.checkpoint_shard``). Both directions go through one description of how a
parameter is laid out across TP (``Layout``): the partition dimension and the list of logical
blocks along it (the ``_checkpoint_splits`` of a fused projection, or ``partition_stride`` equal
blocks, or one block). Each rank holds the same fraction of every block, so the full tensor is,
block by block, the concatenation of the ranks' pieces. Only copies happen: values and dtypes
are preserved bit for bit. Tensors that are not TP-sharded must be identical in every saved
shard. (Behaviour of the reference ``utils/checkpoint_reshard.py:5-64``.)
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Layout:
    dim: int
    blocks: tuple          # logical block widths along ``dim`` in the FULL tensor

    @classmethod
    def of(cls, parameter, full_width):
        splits = getattr(parameter, "_checkpoint_splits", None)
        if splits is not None:
            return cls(parameter.partition_dim, tuple(int(s) for s in splits))
        stride = int(getattr(parameter, "partition_stride", 1))
        if full_width % stride:
            raise ValueError(f"width {full_width} is not a multiple of the projection stride {stride}")
        return cls(parameter.partition_dim, (full_width // stride,) * stride)

    def check(self, *tp_sizes):
        for tp in tp_sizes:
            bad = [b for b in self.blocks if b % tp]
            if bad:
                raise ValueError(f"logical blocks {bad} do not split evenly over TP={tp}")

    def unshard(self, shards):
        """Full tensor from the shards of every TP rank (rank order)."""
        tp = len(shards)
        pieces = [s.split([b // tp for b in self.blocks], dim=self.dim) for s in shards]
        return torch.cat([torch.cat([pieces[r][i] for r in range(tp)], dim=self.dim)
                          for i in range(len(self.blocks))], dim=self.dim)

    def shard(self, full, tp, rank):
        """Rank ``rank``'s slice of a full tensor at TP ``tp``."""
        return torch.cat([block.chunk(tp, dim=self.dim)[rank] for block in full.split(list(self.blocks), dim=self.dim)],
                         dim=self.dim)


def reshard_tensor(values, target, target_tp, target_rank):
    """Destination slice for ``target`` (a parameter of the destination model) from the saved
    per-TP-rank ``values`` (rank order)."""
    if not values:
        raise ValueError("no saved shards")
    if not 0 <= target_rank < target_tp:
        raise ValueError(f"rank {target_rank} is outside TP={target_tp}")
    dtypes = {v.dtype for v in values}
    if dtypes != {target.dtype}:
        raise ValueError(f"saved dtype {sorted(map(str, dtypes))} differs from the model's {target.dtype}")
    if not getattr(target, "tensor_model_parallel", False):
        first = values[0]
        if first.shape != target.shape:
            raise ValueError(f"replicated tensor has shape {tuple(first.shape)}, the model wants {tuple(target.shape)}")
        if any(not torch.equal(v, first) for v in values[1:]):
            raise ValueError("replicated tensor differs between the saved TP ranks")
        return first
    source_tp = len(values)
    dim = target.partition_dim
    full_width = target.shape[dim] * target_tp
    expected = list(target.shape)
    expected[dim] = full_width // source_tp
    if full_width % source_tp or any(list(v.shape) != expected for v in values):
        raise ValueError(f"saved shard shapes {[tuple(v.shape) for v in values]} do not fit the model's "
                         f"{tuple(target.shape)} at TP {target_tp}")
    layout = Layout.of(target, full_width)
    if sum(layout.blocks) != full_width:
        raise ValueError(f"logical blocks {layout.blocks} do not add up to width {full_width}")
    layout.check(source_tp, target_tp)
    result = layout.shard(layout.unshard(values), target_tp, target_rank)
    if result.shape != target.shape:
        raise ValueError(f"resharded shape {tuple(result.shape)} differs from {tuple(target.shape)}")
    return result.contiguous()


def reshard_state(states, model, target_tp, target_rank):
    """The destination rank's model state dict from the saved per-TP-rank state dicts."""
    wanted = model.state_dict(keep_vars=True)
    for tp_rank, state in enumerate(states):
        missing, extra = wanted.keys() - state.keys(), state.keys() - wanted.keys()
        if missing or extra:
            raise ValueError(f"saved TP rank {tp_rank} does not match the model: missing {sorted(missing)[:5]}, "
                             f"unexpected {sorted(extra)[:5]}")
    out = {}
    for name, parameter in wanted.items():
        if not isinstance(parameter, torch.Tensor):
            raise TypeError(f"{name}: only tensors can be resharded")
        try:
            out[name] = reshard_tensor([s[name] for s in states], parameter, target_tp, target_rank)
        except (ValueError, TypeError) as error:
            raise ValueError(f"{name}: {error}") from error
    return out
