"""Sharding across the GPUs of one node (one process per GPU, torch.distributed).

The reference is single-process; these helpers are the multi-GPU form of its
hot path. Weights are split along N (the output dimension): each rank holds
``W^T[n0:n1, :]`` (rows of the nn.Linear-oriented weight), casts it, and
computes ``C[:, n0:n1] = A @ W^T[n0:n1, :]^T``. Block recipes need no
communication (their blocks run along K, inside one rank's rows). Per-tensor
recipes (DelayedScaling / Float8CurrentScaling) need the amax of the whole
weight: each rank reduces its shard into a 32-bit word holding the float's bit
pattern, one all-reduce(MAX) of that word runs over NCCL (an int32 MAX over
non-negative float bit patterns is a float MAX, NaN included), and every rank
then encodes with the same scale -- bit-identical to casting the full tensor
(``src/breccia/kernels/reference/cast.py:364-373``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .api import _input, _classes, _stream, _IN_DT, _FMT, _TORCH_FP8

__all__ = ["shard_rows", "allreduce_amax_word", "cast_per_tensor_sharded", "cast_sharded"]


def shard_rows(n: int, world: int, rank: int, align: int = 128):
    """[lo, hi) row range of ``rank`` when ``n`` rows are split into ``world``
    contiguous, ``align``-aligned pieces (the last may be shorter)."""
    per = -(-n // world)
    per = -(-per // align) * align
    lo = min(n, rank * per)
    return lo, min(n, lo + per)


def allreduce_amax_word(word: torch.Tensor, group=None) -> torch.Tensor:
    """In-place all-reduce(MAX) of a one-element int32 tensor holding the
    float32 bit pattern of a non-negative amax (or NaN). Non-negative float
    bit patterns order like integers and NaN's pattern is above +inf's, so the
    integer maximum is the float maximum with NaN propagating. A no-op outside
    an initialised process group of more than one rank."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(word, op=dist.ReduceOp.MAX, group=group)
    return word


def cast_per_tensor_sharded(x_shard, recipe, group=None):
    """Per-tensor FP8 cast of this rank's shard with the global amax of all
    ranks' shards (one NCCL all-reduce of 4 bytes)."""
    x = _input(x_shard)
    ST, L = _classes(recipe)
    dev = x.device
    fmt = recipe.fp8_format
    codes = torch.empty(x.shape, dtype=torch.uint8, device=dev)
    scale = torch.empty((), dtype=torch.float32, device=dev)
    word = torch.empty(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = _stream(dev)
        _lib.call("brc_amax_reset", word.data_ptr(), st)
        _lib.call("brc_amax_accumulate", x.data_ptr(), _IN_DT[x.dtype], x.numel(),
                  word.data_ptr(), st)
        allreduce_amax_word(word, group)
        _lib.call("brc_cast_pertensor_fp8_apply", x.data_ptr(), _IN_DT[x.dtype], x.numel(),
                  _FMT[fmt], word.data_ptr(), codes.data_ptr(), scale.data_ptr(), st)
    return ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe,
              layout=L.PerTensor())


def cast_sharded(x_shard, recipe, group=None, **kw):
    """Cast of one rank's row shard: per-tensor recipes reduce the amax across
    ranks; block recipes are shard-local."""
    from .api import cast
    if getattr(recipe, "name", None) in ("delayed", "current"):
        return cast_per_tensor_sharded(x_shard, recipe, group)
    return cast(x_shard, recipe, **kw)
