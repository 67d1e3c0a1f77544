"""Exact model-only TP -> TP' conversion of saved model shards.

Each destination tensor is assembled from the saved TP slices of every logical part of a
fused projection (``_checkpoint_splits``) or stride group (``partition_stride``), using the
metadata of the constructed destination parameter; no arithmetic or dtype change happens.
Replicated tensors must agree across the saved TP ranks (reference
``utils/checkpoint_reshard.py:5-64``).
"""

from __future__ import annotations

import torch


def reshard_tensor(values, target, target_tp, target_rank):
    source_tp = len(values)
    if not source_tp or not 0 <= target_rank < target_tp:
        raise ValueError("invalid source/destination TP topology")
    if any(v.dtype != target.dtype for v in values):
        raise ValueError("resharding must preserve parameter dtype")
    if not getattr(target, "tensor_model_parallel", False):
        if any(v.shape != target.shape or not torch.equal(v, values[0]) for v in values):
            raise ValueError("replicated checkpoint tensors differ across TP ranks")
        return values[0]
    dim = target.partition_dim
    width = target.shape[dim] * target_tp
    splits = getattr(target, "_checkpoint_splits", None)
    if splits is None:
        stride = getattr(target, "partition_stride", 1)
        if width % stride:
            raise ValueError("invalid projection stride")
        splits = (width // stride,) * stride
    if sum(splits) != width or any(n % source_tp or n % target_tp for n in splits):
        raise ValueError("logical projection widths do not divide both TP sizes")
    shape = list(target.shape)
    shape[dim] = width // source_tp
    if any(list(v.shape) != shape for v in values):
        raise ValueError("saved TP shape does not match destination metadata")
    parts = [v.split([n // source_tp for n in splits], dim=dim) for v in values]
    out = []
    for index, n in enumerate(splits):
        lo, hi = target_rank * (n // target_tp), (target_rank + 1) * (n // target_tp)
        pieces = []
        for rank in range(source_tp):
            origin = rank * (n // source_tp)
            a, b = max(lo, origin), min(hi, origin + n // source_tp)
            if a < b:
                pieces.append(parts[rank][index].narrow(dim, a - origin, b - a))
        out.append(pieces[0] if len(pieces) == 1 else torch.cat(pieces, dim=dim))
    result = out[0] if len(out) == 1 else torch.cat(out, dim=dim)
    if result.shape != target.shape:
        raise ValueError("unexpected resharded tensor shape")
    return result


def reshard_state(states, model, target_tp, target_rank):
    target = model.state_dict(keep_vars=True)
    if any(s.keys() != target.keys() for s in states):
        raise ValueError("initialization checkpoint keys differ from the model")
    out = {}
    for name, param in target.items():
        values = [s[name] for s in states]
        if not isinstance(param, torch.Tensor):
            raise TypeError(f"unsupported checkpoint entry: {name}")
        try:
            out[name] = reshard_tensor(values, param, target_tp, target_rank)
        except (ValueError, TypeError) as error:
            raise ValueError(f"{name}: {error}") from error
    return out
