"""CPU restatement of breccia's cast / dequantize / requantize (TEST
INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module. The product path (``breccia_b200``) never does.

Each function restates the NumPy path of the reference (jvoltci/breccia
v0.1.3, ``src/breccia/kernels/reference/cast.py``) expression by expression,
so that float32 rounding happens at the same places. Recipes are read by
their ``name`` class attribute (``"delayed"``, ``"current"``, ``"block"``,
``"mxfp8"``, ``"nvfp4"``, ``"int4"``), which the reference's recipe classes
and ``breccia_b200``'s mirror classes share.

Results are :class:`Q` records of NumPy arrays. ``layout`` is
``("per_tensor",)``, ``("per_block_k", B)`` or ``("per_block_mn", bm, bn)``.

``cast_block_fp8_2d`` (128x128 weight tiles) has no producer in the
reference: it is a restated oracle that applies ``_cast_block_fp8``'s
arithmetic (``cast.py:384-404``) to 2-D tiles.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional, Tuple

import numpy as np

from . import codec

_E4M3_MIN_SUBNORMAL = np.float32(2.0 ** -9)  # cast.py:465


@dataclass
class Q:
    data: np.ndarray
    scale: np.ndarray
    layout: Tuple
    recipe: Any
    zero_point: Optional[np.ndarray] = None


def _fmt_max(fmt: str) -> float:  # cast.py:352-353
    return codec.E4M3_MAX if fmt == "E4M3" else codec.E5M2_MAX


def _encode_fp8(x, fmt: str, literal=False):  # cast.py:356-357
    return codec.encode_e4m3(x, literal) if fmt == "E4M3" else codec.encode_e5m2(x, literal)


def _decode_fp8(b, fmt: str):  # cast.py:360-361
    return codec.decode_e4m3(b) if fmt == "E4M3" else codec.decode_e5m2(b)


def _chunked_encode(values_fn, n_rows: int, fmt_encode, chunk_rows: int):
    """Encode row chunks (valid: every recipe is elementwise once its scale is
    known, so row slices of the result equal the full result)."""
    parts = []
    for lo in range(0, n_rows, chunk_rows):
        parts.append(fmt_encode(values_fn(lo, min(n_rows, lo + chunk_rows))))
    return np.concatenate(parts, axis=0) if parts else fmt_encode(values_fn(0, 0))


# ------------------------------------------------------------------ cast


def cast(x, recipe, literal=False, chunk_rows: int = 4096) -> Q:
    """``cast.py:64-92`` NumPy path: ``np.asarray(x, float32)`` then dispatch."""
    x = np.asarray(x, dtype=np.float32)
    name = recipe.name
    if name in ("delayed", "current"):
        return cast_per_tensor_fp8(x, recipe, literal, chunk_rows)
    if name == "block":
        return cast_block_fp8(x, recipe, literal, chunk_rows)
    if name == "mxfp8":
        return cast_mxfp8(x, recipe, literal, chunk_rows)
    if name == "nvfp4":
        return cast_nvfp4(x, recipe, literal)
    if name == "int4":
        return cast_int4(x, recipe)
    raise TypeError(f"unsupported recipe: {type(recipe).__name__}")


def _rows2d(x):
    """View ``x`` as (rows, K) so row chunks can be encoded separately."""
    return x.reshape(-1, x.shape[-1]) if x.ndim >= 1 else x.reshape(1, 1)


def cast_per_tensor_fp8(x, recipe, literal=False, chunk_rows=4096, amax=None) -> Q:
    """``cast.py:364-373``: float64 tensor amax -> float32 scale -> encode.

    ``amax`` (test helper): the ``tensor_amax`` of a larger tensor of which
    ``x`` is a row subset, so sampled rows of a full-size tensor encode with
    the full tensor's scale, as they do inside it."""
    fmt = recipe.fp8_format
    amax = codec.tensor_amax(x) if amax is None else amax
    scale_dequant = np.float32(amax / _fmt_max(fmt))
    x2 = _rows2d(x)
    data = _chunked_encode(lambda a, b: x2[a:b] / scale_dequant, x2.shape[0],
                           lambda v: _encode_fp8(v, fmt, literal), chunk_rows)
    return Q(data.reshape(x.shape), np.asarray(scale_dequant, dtype=np.float32),
             ("per_tensor",), recipe)


def cast_block_fp8(x, recipe, literal=False, chunk_rows=4096) -> Q:
    """``cast.py:384-404``: 1 x block_k amax -> float32 scale -> encode."""
    if x.ndim < 2:
        raise ValueError(f"Float8BlockScaling requires x.ndim >= 2, got {x.ndim}")
    B = recipe.block_k
    fmt = recipe.fp8_format
    amax = codec.block_amax(x, B)
    scale_dequant = (amax / _fmt_max(fmt)).astype(np.float32)
    K = x.shape[-1]
    blocks = x.reshape(-1, K // B, B)
    s2 = scale_dequant.reshape(-1, K // B)
    data = _chunked_encode(lambda a, b: (blocks[a:b] / s2[a:b, :, None]).reshape(b - a, K),
                           blocks.shape[0], lambda v: _encode_fp8(v, fmt, literal), chunk_rows)
    return Q(data.reshape(x.shape), scale_dequant, ("per_block_k", B), recipe)


def cast_block_fp8_2d(x, recipe, block_m: int = 128, literal=False) -> Q:
    """Restated oracle (no reference producer): ``cast.py:384-404`` arithmetic
    over ``block_m x block_k`` tiles of the last two axes. Scale shape is
    ``(..., M // block_m, K // block_k)``; layout ``PerBlockMN(block_m, block_k)``."""
    if x.ndim < 2:
        raise ValueError(f"Float8BlockScaling requires x.ndim >= 2, got {x.ndim}")
    B = recipe.block_k
    fmt = recipe.fp8_format
    M, K = x.shape[-2], x.shape[-1]
    if M % block_m or K % B:
        raise ValueError(
            f"2-D block cast needs M % {block_m} == 0 and K % {B} == 0, got {(M, K)}")
    lead = x.shape[:-2]
    t = x.reshape(lead + (M // block_m, block_m, K // B, B))
    amax = np.max(np.abs(t), axis=(-3, -1))
    amax = np.maximum(amax, codec.AMAX_EPS).astype(np.float32)
    scale = (amax / _fmt_max(fmt)).astype(np.float32)
    v = t / scale[..., :, None, :, None]
    data = _encode_fp8(v.reshape(x.shape), fmt, literal)
    return Q(data, scale, ("per_block_mn", block_m, B), recipe)


def cast_mxfp8(x, recipe, literal=False, chunk_rows=4096) -> Q:
    """``cast.py:420-446``: 1 x 32 amax -> E8M0 (numpy log2 rounding) -> encode."""
    if x.ndim < 2:
        raise ValueError(f"MXFP8BlockScaling requires x.ndim >= 2, got {x.ndim}")
    B = recipe.block_size
    fmt = recipe.fp8_format
    amax = codec.block_amax(x, B)
    scale_dequant_fp32 = (amax / _fmt_max(fmt)).astype(np.float32)
    scale_e8m0 = codec.quantize_e8m0_scale(scale_dequant_fp32)
    actual_scale = codec.dequantize_e8m0_scale(scale_e8m0)
    K = x.shape[-1]
    blocks = x.reshape(-1, K // B, B)
    s2 = actual_scale.reshape(-1, K // B)
    data = _chunked_encode(lambda a, b: (blocks[a:b] / s2[a:b, :, None]).reshape(b - a, K),
                           blocks.shape[0], lambda v: _encode_fp8(v, fmt, literal), chunk_rows)
    return Q(data.reshape(x.shape), scale_e8m0, ("per_block_mn", 1, B), recipe)


def cast_nvfp4(x, recipe, literal=False) -> Q:
    """``cast.py:468-496``: 1 x 16 amax / 6 -> E4M3 scale code (division uses
    ``max(decode, 2^-9)``) -> E2M1 codes, one per byte."""
    if x.ndim < 2:
        raise ValueError(f"NVFP4BlockScaling requires x.ndim >= 2, got {x.ndim}")
    B = recipe.block_size
    amax = codec.block_amax(x, B)
    scale_dequant_fp32 = (amax / codec.E2M1_MAX).astype(np.float32)
    scale_e4m3 = codec.encode_e4m3(scale_dequant_fp32, literal)
    actual_scale = codec.decode_e4m3(scale_e4m3)
    actual_scale = np.where(actual_scale > 0, actual_scale, _E4M3_MIN_SUBNORMAL)
    K = x.shape[-1]
    blocks = x.reshape(x.shape[:-1] + (K // B, B))
    scaled = blocks / actual_scale[..., None]
    data = codec.encode_e2m1(scaled.reshape(x.shape), literal)
    return Q(data, scale_e4m3, ("per_block_mn", 1, B), recipe)


def _int4_dtype(name: str):  # cast.py:512-513
    return {"fp16": np.float16, "bf16": np.float32, "fp32": np.float32}[name]


def cast_int4(x, recipe) -> Q:
    """``cast.py:516-571``: group-wise symmetric or asymmetric INT4."""
    if x.ndim < 2:
        raise ValueError(f"INT4Scaling requires x.ndim >= 2, got {x.ndim}")
    G = recipe.group_size
    K = x.shape[-1]
    if K % G != 0:
        raise ValueError(f"K={K} must be divisible by group_size={G}")
    blocks = x.reshape(x.shape[:-1] + (K // G, G))
    scale_dtype = _int4_dtype(recipe.scale_dtype)
    if recipe.symmetric:
        max_int = 7 if recipe.signed else 15
        amax = np.maximum(np.max(np.abs(blocks), axis=-1), 1e-10).astype(np.float32)
        s = (amax / max_int).astype(np.float32)
        scaled = blocks / s[..., None]
        data = codec.encode_int4(scaled.reshape(x.shape), signed=recipe.signed)
        return Q(data, s.astype(scale_dtype), ("per_block_k", G), recipe)
    bmin = np.min(blocks, axis=-1).astype(np.float32)
    bmax = np.max(blocks, axis=-1).astype(np.float32)
    brange = np.maximum(bmax - bmin, 1e-10)
    s = (brange / 15.0).astype(np.float32)
    zp_fp32 = (-bmin / s).astype(np.float32)
    zp = np.clip(np.round(zp_fp32), 0, 15).astype(np.float32)
    q = np.clip(np.round(blocks / s[..., None] + zp[..., None]), 0, 15).astype(np.uint8)
    data = q.reshape(x.shape) & 0x0F
    return Q(data, s.astype(scale_dtype), ("per_block_k", G), recipe,
             zero_point=zp.astype(scale_dtype))


# ------------------------------------------------------------ dequantize


def dequantize(q: Q) -> np.ndarray:
    """``cast.py:106-118`` dispatch; output is always float32."""
    name = q.recipe.name
    data = np.asarray(q.data)
    scale = np.asarray(q.scale)
    if name in ("delayed", "current"):
        # cast.py:376-378
        return _decode_fp8(data, q.recipe.fp8_format) * np.float32(scale)
    if name == "block":
        if q.layout[0] == "per_block_mn":
            return _dequantize_2d(data, scale, q)
        # cast.py:407-414
        B = q.recipe.block_k
        dec = _decode_fp8(data, q.recipe.fp8_format)
        K = dec.shape[-1]
        out = dec.reshape(dec.shape[:-1] + (K // B, B)) * scale[..., None]
        return out.reshape(dec.shape).astype(np.float32)
    if name == "mxfp8":
        # cast.py:449-459
        B = q.recipe.block_size
        dec = _decode_fp8(data, q.recipe.fp8_format)
        s = codec.dequantize_e8m0_scale(scale)
        K = dec.shape[-1]
        out = dec.reshape(dec.shape[:-1] + (K // B, B)) * s[..., None]
        return out.reshape(dec.shape).astype(np.float32)
    if name == "nvfp4":
        # cast.py:499-506
        B = q.recipe.block_size
        dec = codec.decode_e2m1(data)
        s = codec.decode_e4m3(scale)
        K = dec.shape[-1]
        out = dec.reshape(dec.shape[:-1] + (K // B, B)) * s[..., None]
        return out.reshape(dec.shape).astype(np.float32)
    if name == "int4":
        # cast.py:574-586
        G = q.recipe.group_size
        dec = codec.decode_int4(data, signed=q.recipe.signed)
        s = np.asarray(scale, dtype=np.float32)
        K = dec.shape[-1]
        blocks = dec.reshape(dec.shape[:-1] + (K // G, G))
        if q.zero_point is None:
            out = blocks * s[..., None]
        else:
            zp = np.asarray(q.zero_point, dtype=np.float32)
            out = (blocks - zp[..., None]) * s[..., None]
        return out.reshape(dec.shape).astype(np.float32)
    raise TypeError(f"unsupported recipe: {type(q.recipe).__name__}")


def _dequantize_2d(data, scale, q):
    _, bm, bk = q.layout
    dec = _decode_fp8(data, q.recipe.fp8_format)
    M, K = dec.shape[-2], dec.shape[-1]
    lead = dec.shape[:-2]
    t = dec.reshape(lead + (M // bm, bm, K // bk, bk))
    out = t * scale[..., :, None, :, None]
    return out.reshape(dec.shape).astype(np.float32)


def cast_delayed_fp8(x, recipe, history, recorded, literal=False):
    """DelayedScaling with an amax history: a restated oracle for an extension
    with no reference producer (the reference keeps ``amax_history_len`` and
    ``margin`` on the recipe, ``recipes.py:43-77``, but its cast uses the
    current amax, ``cast.py:364-373``).

    ``history``: float32 array, most recent amax first; ``recorded``: how many
    casts wrote into it. Returns ``(Q, new_history)``. With nothing recorded
    the result is ``cast_per_tensor_fp8`` (the reference's cast). Otherwise
    ``s = float32(max(max(history), 1e-10) / fmt_max) * float32(2**margin)``
    and the codes are ``encode(x / s)`` (float32 division; the encoder clips).
    The tensor's raw amax is pushed into the history either way."""
    x = np.asarray(x, dtype=np.float32)
    history = np.asarray(history, dtype=np.float32)
    fmt = recipe.fp8_format
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0.0)
    if recorded == 0:
        q = cast_per_tensor_fp8(x, recipe, literal)
    else:
        m = np.max(np.abs(history))
        if np.isnan(m):
            s = np.float32(np.nan)
        elif float(m) < 1e-10:
            s = np.float32(1e-10 / _fmt_max(fmt))
        else:
            s = np.float32(np.float32(m) / np.float32(_fmt_max(fmt)))
        with np.errstate(over="ignore", invalid="ignore"):
            s = np.float32(s * np.float32(2.0 ** recipe.margin))
        with np.errstate(divide="ignore", invalid="ignore"):
            data = _encode_fp8(x / s, fmt, literal)
        q = Q(data.reshape(x.shape), np.asarray(s, dtype=np.float32), ("per_tensor",), recipe)
    new_history = np.concatenate([[amax], history[:-1]]).astype(np.float32)
    return q, new_history


def requantize(q: Q, recipe, literal=False) -> Q:
    """``cast.py:339-346``: ``cast(dequantize(st), recipe)``."""
    return cast(dequantize(q), recipe, literal)


# ---------------------------------------------------------------- matmul


def matmul(a, b, out_dtype=np.float32) -> np.ndarray:
    """``matmul.py:123-133`` NumPy branch: dequantize both sides to float32,
    ``a @ b`` (float32 BLAS), then ``astype(out_dtype)``."""
    a_fp = dequantize(a) if isinstance(a, Q) else np.asarray(a, dtype=np.float32)
    b_fp = dequantize(b) if isinstance(b, Q) else np.asarray(b, dtype=np.float32)
    if a_fp.shape[-1] != b_fp.shape[-2]:
        raise ValueError(
            f"matmul shape mismatch: a.shape[-1]={a_fp.shape[-1]} != "
            f"b.shape[-2]={b_fp.shape[-2]}")
    return (a_fp @ b_fp).astype(out_dtype)
