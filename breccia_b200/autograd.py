"""``cast_ste`` / ``cast_ste_clipped`` for CUDA tensors: quantization-aware
casts with straight-through gradients, the forward value computed by one
fused kernel per recipe.

Reference: ``src/breccia/autograd.py:50-87`` (``cast_ste``: forward
``x + (dequantize(cast(x, recipe)) - x).detach()``, gradient the identity)
and ``autograd.py:124-190`` (``cast_ste_clipped``: the same value, gradient
zeroed where ``x`` lies outside ``[clip_min, clip_max]``; the defaults are
the recipe format's saturation bound, ``autograd.py:161-177``).

The fused kernels (``brc_cast_ste_pertensor_fp8``, ``brc_cast_ste_block``)
encode each element exactly as ``cast`` does, decode the code with the scale
``cast`` would store, and write ``x + (y - x)`` in float32: the reference's
value bit for bit, without writing codes or scales and without the separate
dequantize and elementwise passes. Inputs the fused kernels do not cover
(block sizes other than 16/32/64/128/256, float64 or integer inputs) take
``dequantize(cast(x))`` and the same expression in torch, on the GPU.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from . import _lib
from .api import _input, _stream, _IN_DT, _FMT, _require_cuda, cast, dequantize

__all__ = ["cast_ste", "cast_ste_clipped"]

_FP_MAX = {"E4M3": 448.0, "E5M2": 57344.0}


def _fused_forward(x: torch.Tensor, recipe: Any) -> Optional[torch.Tensor]:
    """x + (dequantize(cast(x, recipe)) - x) as float32 through the fused
    kernels, or None when they do not cover this input."""
    if x.dtype not in _IN_DT:
        return None
    name = getattr(recipe, "name", None)
    x = _input(x)
    dev = x.device
    out = torch.empty(x.shape, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = _stream(dev)
        if name in ("delayed", "current"):
            word = torch.empty(1, dtype=torch.int32, device=dev)
            _lib.call("brc_cast_ste_pertensor_fp8", x.data_ptr(), _IN_DT[x.dtype], x.numel(),
                      _FMT[recipe.fp8_format], word.data_ptr(), out.data_ptr(), st)
            return out
        if x.ndim < 2:
            return None  # the reference's own error message comes from cast()
        K = x.shape[-1]
        rows = x.numel() // K if K else 0
        if name == "block":
            kind, block, fmt = _lib.STE_BLOCK_FP8, recipe.block_k, _FMT[recipe.fp8_format]
            signed = symmetric = 0
            sdt = _lib.SCALE_F32
        elif name == "mxfp8":
            kind, block, fmt = _lib.STE_MXFP8, recipe.block_size, _FMT[recipe.fp8_format]
            signed = symmetric = 0
            sdt = _lib.SCALE_F32
        elif name == "nvfp4":
            kind, block, fmt = _lib.STE_NVFP4, recipe.block_size, 0
            signed = symmetric = 0
            sdt = _lib.SCALE_F32
        elif name == "int4":
            kind, block, fmt = _lib.STE_INT4, recipe.group_size, 0
            signed, symmetric = int(bool(recipe.signed)), int(bool(recipe.symmetric))
            sdt = _lib.SCALE_F16 if recipe.scale_dtype == "fp16" else _lib.SCALE_F32
        else:
            return None
        if block not in (16, 32, 64, 128, 256) or K % block:
            return None
        _lib.call("brc_cast_ste_block", x.data_ptr(), _IN_DT[x.dtype], rows, K, kind, block,
                  fmt, signed, symmetric, sdt, out.data_ptr(), st)
        return out


def _forward_value(x: torch.Tensor, recipe: Any) -> torch.Tensor:
    out = _fused_forward(x, recipe)
    if out is None:
        y = dequantize(cast(x, recipe))
        out = x + (y - x)
    return out


class _Ste(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, recipe, lo, hi):
        ctx.clip = lo is not None
        if ctx.clip:
            ctx.save_for_backward(x)
            ctx.lo, ctx.hi = lo, hi
        ctx.x_dtype = x.dtype
        return _forward_value(x.detach(), recipe)

    @staticmethod
    def backward(ctx, g):
        if ctx.clip:
            (x,) = ctx.saved_tensors
            g = torch.where((x >= ctx.lo) & (x <= ctx.hi), g, torch.zeros_like(g))
        return g.to(ctx.x_dtype), None, None, None


def cast_ste(x: Any, recipe: Any) -> torch.Tensor:
    """Quantization-aware cast, straight-through gradient
    (``autograd.py:50-87``). The value is ``dequantize(cast(x, recipe))``
    evaluated as ``x + (y - x)``; ``d out / d x`` is the identity."""
    _require_cuda(x)
    return _Ste.apply(x, recipe, None, None)


def cast_ste_clipped(x: Any, recipe: Any, clip_min: Optional[float] = None,
                     clip_max: Optional[float] = None) -> torch.Tensor:
    """``cast_ste`` whose gradient is zero where ``x`` is outside
    ``[clip_min, clip_max]`` (``autograd.py:124-190``). Defaults: the
    format's saturation bound (448 / 57344 for FP8, 6 for NVFP4, 7 or 15
    for INT4) and its negation."""
    _require_cuda(x)
    if clip_max is None:
        name = getattr(recipe, "name", None)
        if name in ("delayed", "current", "block", "mxfp8"):
            clip_max = _FP_MAX[recipe.fp8_format]
        elif name == "nvfp4":
            clip_max = 6.0
        elif name == "int4":
            clip_max = 7.0 if recipe.signed else 15.0
        else:
            clip_max = float("inf")
        clip_max = float(clip_max)
    if clip_min is None:
        clip_min = -clip_max
    return _Ste.apply(x, recipe, clip_min, clip_max)
