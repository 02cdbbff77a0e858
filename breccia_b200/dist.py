"""Sharding across the GPUs of one node (one process per GPU, torch.distributed).

The reference is single-process; these helpers are the multi-GPU form of its
hot path. Two layouts use them.

Data parallel (bench.py --shard batch): each rank holds its own batch of
activation rows and the whole weight. The activations' per-tensor scale is the
one of the concatenated batch, so the local amax words are all-reduced; the
weight's cast is local. ``cast_per_tensor_async`` lets that all-reduce overlap
the weight's cast.

Weight split (bench.py's default for N > 1, ``cast_weight_split``): weights are
split along N (the output dimension): each rank holds
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

__all__ = ["shard_rows", "allreduce_amax_word", "cast_per_tensor_sharded", "cast_sharded",
           "cast_per_tensor_async", "PendingCast", "cast_weight_split",
           "cast_matmul_weight_split"]


def shard_rows(n: int, world: int, rank: int, align: int = 128):
    """[lo, hi) row range of ``rank`` when ``n`` rows are split into ``world``
    contiguous, ``align``-aligned pieces (the last may be shorter)."""
    per = -(-n // world)
    per = -(-per // align) * align
    lo = min(n, rank * per)
    return lo, min(n, lo + per)


def _world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def allreduce_amax_word(word: torch.Tensor, group=None) -> torch.Tensor:
    """In-place all-reduce(MAX) of a one-element int32 tensor holding the
    float32 bit pattern of a non-negative amax (or NaN). Non-negative float
    bit patterns order like integers and NaN's pattern is above +inf's, so the
    integer maximum is the float maximum with NaN propagating. A no-op outside
    an initialised process group of more than one rank."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(word, op=dist.ReduceOp.MAX, group=group)
    return word


class PendingCast:
    """A per-tensor FP8 cast whose amax all-reduce is in flight.

    ``cast_per_tensor_async`` reduces the local shard's amax and starts the
    all-reduce without making the current stream wait for it, so independent
    work issued next (the weight's cast, say) overlaps the collective.
    ``wait()`` makes the current stream wait for the reduced amax, encodes the
    shard and returns its ScaledTensor."""

    def __init__(self, x, recipe, word, work):
        self._x, self._recipe, self._word, self._work = x, recipe, word, work

    def wait(self):
        if self._work is not None:
            self._work.wait()
            self._work = None
        x, recipe = self._x, self._recipe
        ST, L = _classes(recipe)
        dev = x.device
        fmt = recipe.fp8_format
        codes = torch.empty(x.shape, dtype=torch.uint8, device=dev)
        scale = torch.empty((), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("brc_cast_pertensor_fp8_apply", x.data_ptr(), _IN_DT[x.dtype], x.numel(),
                      _FMT[fmt], self._word.data_ptr(), codes.data_ptr(), scale.data_ptr(),
                      _stream(dev))
        return ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe,
                  layout=L.PerTensor())


def cast_per_tensor_async(x_shard, recipe, group=None) -> PendingCast:
    """Start a per-tensor FP8 cast of this rank's shard with the global amax
    of all ranks' shards: the local amax is reduced on the current stream and
    its 4-byte all-reduce(MAX) is launched asynchronously (no collective
    outside an initialised process group of more than one rank)."""
    x = _input(x_shard)
    if getattr(recipe, "name", None) not in ("delayed", "current"):
        raise ValueError("cast_per_tensor_async takes a per-tensor recipe "
                         "(DelayedScaling or Float8CurrentScaling)")
    dev = x.device
    word = torch.empty(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = _stream(dev)
        _lib.call("brc_amax_reset", word.data_ptr(), st)
        _lib.call("brc_amax_accumulate", x.data_ptr(), _IN_DT[x.dtype], x.numel(),
                  word.data_ptr(), st)
    work = None
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        work = dist.all_reduce(word, op=dist.ReduceOp.MAX, group=group, async_op=True)
    return PendingCast(x, recipe, word, work)


def cast_per_tensor_sharded(x_shard, recipe, group=None):
    """Per-tensor FP8 cast of this rank's shard with the global amax of all
    ranks' shards (one NCCL all-reduce of 4 bytes)."""
    return cast_per_tensor_async(x_shard, recipe, group).wait()


def cast_sharded(x_shard, recipe, group=None, **kw):
    """Cast of one rank's row shard: per-tensor recipes reduce the amax across
    ranks; block recipes are shard-local."""
    from .api import cast
    if getattr(recipe, "name", None) in ("delayed", "current"):
        return cast_per_tensor_sharded(x_shard, recipe, group)
    return cast(x_shard, recipe, **kw)


def cast_weight_split(a, w_shard, recipe, group=None, **kw):
    """Operands of one layer in the weight-split layout: ``a`` is the whole
    activation (replicated: every rank holds all of it), ``w_shard`` this
    rank's rows ``[n0, n1)`` of ``W^T``. Returns ``(cast(a), cast(w_shard))``
    equal, bit for bit, to the single-GPU casts of ``a`` and of the rows
    ``[n0, n1)`` of the whole weight.

    Per-tensor recipes need two global amaxes: the activation's (over all its
    rows) and the weight's (over every rank's shard). Each rank reduces only
    its ``1/world`` share of the activation's rows (``shard_rows``) and its
    weight shard into two 32-bit words, ONE all-reduce(MAX) of those 8 bytes
    gives both global amaxes, and each rank then encodes the whole activation
    and its shard. The activation's amax pass thus shrinks with the number of
    ranks; its encode pass does not (every rank needs all of its codes).
    Block recipes are rank-local (their blocks run along K)."""
    from .api import cast
    if getattr(recipe, "name", None) not in ("delayed", "current"):
        return cast(a, recipe, **kw), cast(w_shard, recipe, **kw)
    x, w = _input(a), _input(w_shard)
    world, rank = _world(group)
    K = x.shape[-1] if x.ndim else 1
    rows = x.numel() // K if K else 0
    lo, hi = shard_rows(rows, world, rank)
    dev = x.device
    words = torch.empty(2, dtype=torch.int32, device=dev)
    fmt = recipe.fp8_format
    ST, L = _classes(recipe)
    with torch.cuda.device(dev):
        st = _stream(dev)
        _lib.call("brc_amax_reset", words.data_ptr(), st)
        _lib.call("brc_amax_reset", words.data_ptr() + 4, st)
        _lib.call("brc_amax_accumulate", x.data_ptr() + lo * K * x.element_size(),
                  _IN_DT[x.dtype], (hi - lo) * K, words.data_ptr(), st)
        _lib.call("brc_amax_accumulate", w.data_ptr(), _IN_DT[w.dtype], w.numel(),
                  words.data_ptr() + 4, st)
    if world > 1:
        dist.all_reduce(words, op=dist.ReduceOp.MAX, group=group)
    out = []
    with torch.cuda.device(dev):
        st = _stream(dev)
        for t, off in ((x, 0), (w, 4)):
            codes = torch.empty(t.shape, dtype=torch.uint8, device=dev)
            scale = torch.empty((), dtype=torch.float32, device=dev)
            _lib.call("brc_cast_pertensor_fp8_apply", t.data_ptr(), _IN_DT[t.dtype], t.numel(),
                      _FMT[fmt], words.data_ptr() + off, codes.data_ptr(), scale.data_ptr(), st)
            out.append(ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe,
                          layout=L.PerTensor()))
    return out[0], out[1]


def cast_matmul_weight_split(a, w_shard, recipe, group=None, out_dtype=torch.bfloat16,
                             fused=None):
    """One layer's step in the weight-split layout with the activation's cast
    fused into the GEMM (``cast_matmul``): the two amax words of
    ``cast_weight_split`` (a ``1/world`` share of the activation's rows and
    this rank's weight shard, one all-reduce(MAX) of 8 bytes), the weight
    shard's cast, then one launch that encodes the whole activation with the
    global amax while the tensor cores compute ``a @ w_shard^T``. Returns
    ``(out, cast(a), cast(w_shard))``, bit-identical to ``cast_weight_split``
    followed by ``linear``.

    Every rank encodes the whole (replicated) activation while its GEMM
    covers only ``1/world`` of the output columns. On B200 the fused launch
    measured slower than the apply pass + GEMM at every shard width (N = 1024:
    0.441 vs 0.169 ms; N = 8192: 0.819 vs 0.809 ms), so ``fused=None`` runs the
    apply pass first; ``fused=True`` takes the fused launch. Per-tensor
    recipes only (others: ``cast_weight_split`` + ``linear``)."""
    from .api import _fused_cast_gemm, _torch_out_dtype, linear
    if getattr(recipe, "name", None) not in ("delayed", "current"):
        sa, sw = cast_weight_split(a, w_shard, recipe, group)
        return linear(sa, sw, out_dtype), sa, sw
    x, w = _input(a), _input(w_shard)
    world, rank = _world(group)
    K = x.shape[-1] if x.ndim else 1
    rows = x.numel() // K if K else 0
    N = w.shape[0]
    if fused is None:
        fused = False  # the current-amax step measured no faster fused (cast_matmul)
    if not (fused and K > 0 and K % 128 == 0 and N % 16 == 0 and w.ndim == 2 and x.ndim >= 1):
        sa, sw = cast_weight_split(a, w_shard, recipe, group)
        return linear(sa, sw, out_dtype), sa, sw
    lo, hi = shard_rows(rows, world, rank)
    dev = x.device
    words = torch.empty(2, dtype=torch.int32, device=dev)
    fmt = recipe.fp8_format
    ST, L = _classes(recipe)
    with torch.cuda.device(dev):
        st = _stream(dev)
        _lib.call("brc_amax_reset", words.data_ptr(), st)
        _lib.call("brc_amax_reset", words.data_ptr() + 4, st)
        _lib.call("brc_amax_accumulate", x.data_ptr() + lo * K * x.element_size(),
                  _IN_DT[x.dtype], (hi - lo) * K, words.data_ptr(), st)
        _lib.call("brc_amax_accumulate", w.data_ptr(), _IN_DT[w.dtype], w.numel(),
                  words.data_ptr() + 4, st)
    if world > 1:
        dist.all_reduce(words, op=dist.ReduceOp.MAX, group=group)
    with torch.cuda.device(dev):
        st = _stream(dev)
        wc = torch.empty(w.shape, dtype=torch.uint8, device=dev)
        wsc = torch.empty((), dtype=torch.float32, device=dev)
        _lib.call("brc_cast_pertensor_fp8_apply", w.data_ptr(), _IN_DT[w.dtype], w.numel(),
                  _FMT[fmt], words.data_ptr() + 4, wc.data_ptr(), wsc.data_ptr(), st)
    sw = ST(data=wc.view(_TORCH_FP8[fmt]), scale=wsc, recipe=recipe, layout=L.PerTensor())
    out, sa = _fused_cast_gemm(x, recipe, wc, sw, N, _torch_out_dtype(out_dtype), None,
                               words[0:1], -1)
    return out, sa, sw
