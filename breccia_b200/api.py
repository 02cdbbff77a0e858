"""breccia's hot path on B200: ``cast``, ``dequantize``, ``requantize``,
``matmul`` (and the K-major ``linear``) for CUDA torch tensors.

Signatures, result conventions and error messages follow the reference
(jvoltci/breccia v0.1.3):

* ``cast(x, recipe)`` -- ``src/breccia/kernels/reference/cast.py:64-92``
* ``dequantize(st)`` -- ``cast.py:95-118``
* ``requantize(st, recipe)`` -- ``cast.py:339-346``
* ``matmul(a, b, out_dtype)`` -- ``src/breccia/kernels/reference/matmul.py:42-133``

Result conventions (``cast.py:170-217`` for per-tensor/block FP8, ``cast.py:124-161``
for the others): per-tensor and block FP8 data are ``torch.float8_e4m3fn`` /
``float8_e5m2``; MXFP8, NVFP4 and INT4 data are ``uint8`` with one code per
byte; scales and zero points have the reference's dtypes and shapes; the
result's ``recipe`` is the object passed in; everything stays on the input's
device. Codes and scales equal the reference NumPy path's bit for bit (the
reference's own torch path rounds FP8 ties to even through ATen and so
differs from its NumPy path; this backend follows the NumPy path).

Only CUDA tensors are accepted: there is no CPU fallback. ``install()``
routes CUDA inputs of the real ``breccia`` package here and leaves every
other input on breccia's own code.
"""

from __future__ import annotations

import weakref
from typing import Any, Optional

import numpy as np
import torch

from . import _lib
from . import types as T

__all__ = ["cast", "dequantize", "requantize", "matmul", "linear", "gemm_operands",
           "attach_gemm_operands", "AmaxHistory", "cast_matmul"]

_TORCH_FP8 = {"E4M3": torch.float8_e4m3fn, "E5M2": torch.float8_e5m2}
_FMT = {"E4M3": _lib.FP8_E4M3, "E5M2": _lib.FP8_E5M2}
_IN_DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
          torch.float16: _lib.DTYPE_F16}
_OUT_DT = _IN_DT


# ----------------------------------------------------------------- plumbing


def _classes(recipe):
    """ScaledTensor and layout classes of the recipe's own package, so that a
    recipe from the real breccia gets a breccia.ScaledTensor back."""
    mod = type(recipe).__module__
    if mod == "breccia" or mod.startswith("breccia."):
        import breccia
        return breccia.ScaledTensor, breccia
    return T.ScaledTensor, T


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(x, what="x"):
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise TypeError(
            f"breccia_b200 operates on CUDA torch tensors; {what} is "
            f"{type(x).__name__}{'' if not isinstance(x, torch.Tensor) else ' on ' + str(x.device)}")


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _input(x) -> torch.Tensor:
    _require_cuda(x)
    if x.dtype not in _IN_DT:
        x = x.to(torch.float32)  # np.asarray(x, dtype=np.float32), cast.py:77
    return _aligned(x)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


# Side data the tensor-core GEMMs consume (scales in the tcgen05 layout,
# packed FP4/INT4 nibbles), keyed by the identity of a ScaledTensor's data
# tensor and dropped when that tensor is freed. Each entry carries a tag of
# the data, scale and zero-point tensors' addresses and version counters
# (torch bumps a tensor's version on every in-place write: copy_, index
# assignment, out= ops), so codes or scales rewritten in place after the
# cast make the entry stale; stale entries are never returned, and
# ``_side_of`` rebuilds them from the current codes and scales on the GPU.
_SIDE: dict = {}


def _tag(data: torch.Tensor, companions=()) -> tuple:
    tag = [data.data_ptr(), data._version]
    for t in companions:
        if isinstance(t, torch.Tensor):
            tag += [t.data_ptr(), t._version]
        else:
            tag += [None, None]
    return tuple(tag)


def _remember(data: torch.Tensor, companions=(), **side) -> None:
    key = id(data)
    ent = _SIDE.get(key)
    if ent is None:
        weakref.finalize(data, _SIDE.pop, key, None)
        ent = _SIDE[key] = {}
    tag = _tag(data, companions)
    if ent.get("_tag") != tag:
        ent.clear()
    ent.update(side)
    ent["_tag"] = tag


def _side(data: torch.Tensor, companions=()) -> dict:
    ent = _SIDE.get(id(data))
    if not ent or ent.get("_tag") != _tag(data, companions):
        return {}
    return ent


def _companions(scaled) -> tuple:
    return (scaled.scale, getattr(scaled, "zero_point", None))


def _side_of(scaled, rebuild: bool = True) -> dict:
    """Current side data of a CUDA ScaledTensor; rebuilt from its codes and
    scales when missing or stale (``attach_gemm_operands``)."""
    side = _side(scaled.data, _companions(scaled))
    if not side and rebuild:
        attach_gemm_operands(scaled)
        side = _side(scaled.data, _companions(scaled))
    return side


def _mma_scale_shape(rows: int, scale_cols: int):
    return (((rows + 127) // 128) * ((scale_cols + 3) // 4) * 512,)


def _mma_scale_buffer(rows: int, scale_cols: int, dev):
    """Scale atoms for the tcgen05 GEMMs (128 rows x 4 scale columns per
    512-byte atom). The cast writes one byte per (row, scale column); atom
    bytes past the last row or column must read as zero, so only a ragged
    shape needs the buffer cleared first (a separate fill kernel)."""
    shape = _mma_scale_shape(rows, scale_cols)
    if rows % 128 == 0 and scale_cols % 4 == 0:
        return torch.empty(shape, dtype=torch.uint8, device=dev)
    return torch.zeros(shape, dtype=torch.uint8, device=dev)


# ------------------------------------------------------------------- cast


class AmaxHistory:
    """DelayedScaling state of one tensor across steps (extension).

    breccia's ``DelayedScaling`` carries ``amax_history_len`` and ``margin``
    (``recipes.py:43-77``) but its cast uses the current amax (``cast.py:
    364-373``). Passed to ``cast(x, DelayedScaling(...), amax_history=h)``,
    this object makes the cast use them, as TransformerEngine's delayed
    scaling does: ``history`` is a float32 ring of the last amaxes on the
    device (most recent first) and ``recorded`` counts the casts that wrote
    into it (kept on the host, so no device read is needed to choose).

    * While nothing is recorded the cast is the reference's current-amax cast,
      bit for bit, and records that amax.
    * Afterwards the scale comes from the ring before the tensor is read,
      ``float32(max(max(history), 1e-10) / fmt_max) * 2**margin``, and the
      cast is one pass (each element read once instead of twice); values
      beyond the scaled range saturate; the tensor's amax is recorded.
    """

    def __init__(self, length: int = 16, device: Any = None):
        if length < 1:
            raise ValueError(f"amax history length must be >= 1, got {length}")
        self.history = torch.zeros(length, dtype=torch.float32,
                                   device=device if device is not None else "cuda")
        self.recorded = 0

    def reset(self) -> None:
        self.history.zero_()
        self.recorded = 0


def cast(x: Any, recipe: Any, *, block_m: Optional[int] = None,
         amax_history: Optional[AmaxHistory] = None):
    """Quantize a CUDA tensor with ``recipe`` (``cast.py:64-92``).

    ``block_m`` (extension, ``Float8BlockScaling`` only): scale
    ``block_m x block_k`` tiles of the last two axes instead of ``1 x block_k``
    runs -- the DeepSeek-v3 128x128 weight layout, ``PerBlockMN(block_m,
    block_k)``. The reference can describe but not produce it.

    ``amax_history`` (extension, ``DelayedScaling`` only): an
    :class:`AmaxHistory` that carries the recipe's amax history and margin
    across calls (one-pass casts once it holds an amax).
    """
    x = _input(x)
    ST, L = _classes(recipe)
    name = getattr(recipe, "name", None)
    dev = x.device
    with torch.cuda.device(dev):
        st = _stream(dev)
        if amax_history is not None:
            if name != "delayed":
                raise ValueError("amax_history applies to DelayedScaling only")
            return _cast_delayed(x, recipe, ST, L, st, amax_history)
        if name in ("delayed", "current"):
            return _cast_per_tensor(x, recipe, ST, L, st)
        if name == "block":
            return _cast_block(x, recipe, ST, L, st, block_m)
        if name == "mxfp8":
            return _cast_mxfp8(x, recipe, ST, L, st)
        if name == "nvfp4":
            return _cast_nvfp4(x, recipe, ST, L, st)
        if name == "int4":
            return _cast_int4(x, recipe, ST, L, st)
    raise TypeError(f"unsupported recipe: {type(recipe).__name__}")


def _cast_per_tensor(x, recipe, ST, L, st):
    fmt = recipe.fp8_format
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    ws = torch.empty(1, dtype=torch.int32, device=x.device)
    _lib.call("brc_cast_pertensor_fp8", x.data_ptr(), _IN_DT[x.dtype], x.numel(), _FMT[fmt],
              codes.data_ptr(), scale.data_ptr(), ws.data_ptr(), st)
    return ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe, layout=L.PerTensor())


def _cast_delayed(x, recipe, ST, L, st, h):
    fmt = recipe.fp8_format
    hist = h.history
    if not (isinstance(hist, torch.Tensor) and hist.is_cuda and hist.dtype == torch.float32 and
            hist.is_contiguous() and hist.device == x.device):
        raise TypeError("AmaxHistory.history must be a contiguous float32 tensor on x's device")
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    ws = torch.empty(1, dtype=torch.int32, device=x.device)
    _lib.call("brc_cast_pertensor_fp8_delayed", x.data_ptr(), _IN_DT[x.dtype], x.numel(),
              _FMT[fmt], hist.data_ptr(), hist.numel(), int(recipe.margin),
              1 if h.recorded > 0 else 0, codes.data_ptr(), scale.data_ptr(), ws.data_ptr(), st)
    h.recorded += 1
    return ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe, layout=L.PerTensor())


def _last_axis_checks(x, recipe_cls_name, block, msg_kind):
    if x.ndim < 2:
        raise ValueError(f"{recipe_cls_name} requires x.ndim >= 2, got {x.ndim}")
    K = x.shape[-1]
    if K % block != 0:
        if msg_kind == "block_k":  # cast.py:203-204
            raise ValueError(f"K={K} must be divisible by block_k={block}")
        if msg_kind == "group_size":  # cast.py:521-522
            raise ValueError(f"K={K} must be divisible by group_size={block}")
        # _utils.py:25-28 (block_amax)
        raise ValueError(f"last-axis size {K} must be divisible by block_size {block}")
    return K


def _cast_block(x, recipe, ST, L, st, block_m):
    B = recipe.block_k
    fmt = recipe.fp8_format
    K = _last_axis_checks(x, "Float8BlockScaling", B, "block_k")
    rows = x.numel() // K if K else 0
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    if block_m is None:
        scale = torch.empty(x.shape[:-1] + (K // B,), dtype=torch.float32, device=x.device)
        _lib.call("brc_cast_block_fp8", x.data_ptr(), _IN_DT[x.dtype], rows, K, B, _FMT[fmt],
                  codes.data_ptr(), scale.data_ptr(), st)
        layout = L.PerBlockK(block_size=B)
    else:
        M = x.shape[-2]
        if M % block_m:
            raise ValueError(f"M={M} must be divisible by block_m={block_m}")
        scale = torch.empty(x.shape[:-2] + (M // block_m, K // B), dtype=torch.float32,
                            device=x.device)
        _lib.call("brc_cast_block_fp8_2d", x.data_ptr(), _IN_DT[x.dtype], rows, K, block_m, B,
                  _FMT[fmt], codes.data_ptr(), scale.data_ptr(), st)
        layout = L.PerBlockMN(block_m=block_m, block_n=B)
    return ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe, layout=layout)


def _cast_mxfp8(x, recipe, ST, L, st):
    fmt = recipe.fp8_format
    K = _last_axis_checks(x, "MXFP8BlockScaling", 32, "block_size")
    rows = x.numel() // K if K else 0
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty(x.shape[:-1] + (K // 32,), dtype=torch.uint8, device=x.device)
    sf_mma = _mma_scale_buffer(rows, K // 32, x.device)
    _lib.call("brc_cast_mxfp8", x.data_ptr(), _IN_DT[x.dtype], rows, K, _FMT[fmt],
              codes.data_ptr(), scale.data_ptr(), sf_mma.data_ptr(), st)
    _remember(codes, (scale, None), sf_mma=sf_mma)
    return ST(data=codes, scale=scale, recipe=recipe, layout=L.PerBlockMN(block_m=1, block_n=32))


def _cast_nvfp4(x, recipe, ST, L, st):
    K = _last_axis_checks(x, "NVFP4BlockScaling", 16, "block_size")
    rows = x.numel() // K if K else 0
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    packed = torch.empty(x.shape[:-1] + (K // 2,), dtype=torch.uint8, device=x.device)
    scale = torch.empty(x.shape[:-1] + (K // 16,), dtype=torch.uint8, device=x.device)
    sf_mma = _mma_scale_buffer(rows, K // 16, x.device)
    _lib.call("brc_cast_nvfp4", x.data_ptr(), _IN_DT[x.dtype], rows, K, codes.data_ptr(),
              packed.data_ptr(), scale.data_ptr(), sf_mma.data_ptr(), st)
    _remember(codes, (scale, None), packed=packed, sf_mma=sf_mma)
    return ST(data=codes, scale=scale, recipe=recipe, layout=L.PerBlockMN(block_m=1, block_n=16))


def _cast_int4(x, recipe, ST, L, st):
    G = recipe.group_size
    K = _last_axis_checks(x, "INT4Scaling", G, "group_size")
    rows = x.numel() // K if K else 0
    sdt = torch.float16 if recipe.scale_dtype == "fp16" else torch.float32  # cast.py:512-513
    dev = x.device
    codes = torch.empty(x.shape, dtype=torch.uint8, device=dev)
    scale = torch.empty(x.shape[:-1] + (K // G,), dtype=sdt, device=dev)
    zp = None if recipe.symmetric else torch.empty_like(scale)
    # the skinny-GEMM tile layout, when the weight shape allows it
    tiles = stiles = ztiles = None
    if G == 128 and rows % 16 == 0 and rows > 0:
        tiles = torch.empty(rows * K // 2, dtype=torch.uint8, device=dev)
        stiles = torch.empty(rows * (K // G), dtype=torch.float32, device=dev)
        ztiles = None if recipe.symmetric else torch.empty_like(stiles)
    _lib.call("brc_cast_int4", x.data_ptr(), _IN_DT[x.dtype], rows, K, G,
              int(bool(recipe.signed)), int(bool(recipe.symmetric)),
              _lib.SCALE_F16 if sdt == torch.float16 else _lib.SCALE_F32,
              codes.data_ptr(), None, scale.data_ptr(), _ptr(zp), _ptr(tiles), _ptr(stiles),
              _ptr(ztiles), st)
    if tiles is not None:
        _remember(codes, (scale, zp), int4_tiles=tiles, int4_scale_tiles=stiles,
                  int4_zp_tiles=ztiles)
    return ST(data=codes, scale=scale, recipe=recipe, layout=L.PerBlockK(block_size=G),
              zero_point=zp)


# ------------------------------------------------------------- dequantize


def _codes_u8(data: torch.Tensor) -> torch.Tensor:
    _require_cuda(data, "ScaledTensor.data")
    if data.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        data = data.view(torch.uint8)
    if data.dtype != torch.uint8:
        raise TypeError(f"unsupported data dtype {data.dtype}")
    return _aligned(data)


def dequantize(scaled, out_dtype=torch.float32):
    """``decode(data) * scale`` as float32 (``cast.py:95-118``).

    ``out_dtype`` (extension): ``torch.bfloat16`` / ``torch.float16`` write
    the same products rounded to that type.
    """
    r = scaled.recipe
    name = getattr(r, "name", None)
    codes = _codes_u8(scaled.data)
    dev = codes.device
    if out_dtype not in _OUT_DT:
        raise TypeError(f"out_dtype must be float32, bfloat16 or float16, got {out_dtype}")
    out = torch.empty(codes.shape, dtype=out_dtype, device=dev)
    odt = _OUT_DT[out_dtype]
    scale = _aligned(scaled.scale)
    K = codes.shape[-1] if codes.ndim else 1
    rows = codes.numel() // K if K else 0
    with torch.cuda.device(dev):
        st = _stream(dev)
        if name in ("delayed", "current"):
            _lib.call("brc_dequant_pertensor_fp8", codes.data_ptr(), codes.numel(),
                      _FMT[r.fp8_format], scale.to(torch.float32).data_ptr(), out.data_ptr(),
                      odt, st)
        elif name == "block":
            lay = scaled.layout
            bm = getattr(lay, "block_m", 1) if getattr(lay, "name", "") == "per_block_mn" else 1
            _lib.call("brc_dequant_block_fp8", codes.data_ptr(), rows, K, bm, r.block_k,
                      _FMT[r.fp8_format], scale.data_ptr(), out.data_ptr(), odt, st)
        elif name == "mxfp8":
            _lib.call("brc_dequant_mxfp8", codes.data_ptr(), rows, K, _FMT[r.fp8_format],
                      scale.data_ptr(), out.data_ptr(), odt, st)
        elif name == "nvfp4":
            _lib.call("brc_dequant_nvfp4", codes.data_ptr(), rows, K, scale.data_ptr(),
                      out.data_ptr(), odt, st)
        elif name == "int4":
            zp = scaled.zero_point
            sdt = _lib.SCALE_F16 if scale.dtype == torch.float16 else _lib.SCALE_F32
            if zp is not None:
                zp = _aligned(zp.to(scale.dtype))
            _lib.call("brc_dequant_int4", codes.data_ptr(), rows, K, r.group_size,
                      int(bool(r.signed)), sdt, scale.data_ptr(), _ptr(zp), out.data_ptr(),
                      odt, st)
        else:
            raise TypeError(f"unsupported recipe: {type(r).__name__}")
    return out


# -------------------------------------------------------------- requantize


def requantize(scaled, recipe):
    """``cast(dequantize(st), recipe)`` (``cast.py:339-346``). NVFP4 -> MXFP8
    runs as one fused kernel; other pairs dequantize to float32 first."""
    src = getattr(scaled.recipe, "name", None)
    if src == "nvfp4" and getattr(recipe, "name", None) == "mxfp8":
        codes = _codes_u8(scaled.data)
        K = codes.shape[-1]
        if codes.ndim < 2 or K % 32:
            return cast(dequantize(scaled), recipe)
        rows = codes.numel() // K
        ST, L = _classes(recipe)
        dev = codes.device
        out = torch.empty(codes.shape, dtype=torch.uint8, device=dev)
        scale = torch.empty(codes.shape[:-1] + (K // 32,), dtype=torch.uint8, device=dev)
        sf_mma = _mma_scale_buffer(rows, K // 32, dev)
        with torch.cuda.device(dev):
            _lib.call("brc_requant_nvfp4_to_mxfp8", codes.data_ptr(),
                      _aligned(scaled.scale).data_ptr(), rows, K, _FMT[recipe.fp8_format],
                      out.data_ptr(), scale.data_ptr(), sf_mma.data_ptr(), _stream(dev))
        _remember(out, (scale, None), sf_mma=sf_mma)
        return ST(data=out, scale=scale, recipe=recipe,
                  layout=L.PerBlockMN(block_m=1, block_n=32))
    return cast(dequantize(scaled), recipe)


# ------------------------------------------------------------------ matmul


def _torch_out_dtype(out_dtype):
    """``matmul.py:136-147``, extended to accept torch dtypes (incl. bfloat16)."""
    if isinstance(out_dtype, torch.dtype):
        return out_dtype
    key = np.dtype(out_dtype).type
    return {np.float32: torch.float32, np.float64: torch.float64,
            np.float16: torch.float16}.get(key, torch.float32)


def _is_scaled(t) -> bool:
    return hasattr(t, "recipe") and hasattr(t, "scale") and hasattr(t, "data")


def matmul(a, b, out_dtype=np.float32, *, b_kmajor=False):
    """Scaled matmul with the reference's semantics (``matmul.py:42-133``):
    ``a (..., M, K) @ b (..., K, N)`` of the dequantized operands with
    float32 accumulation, then ``out_dtype`` (a NumPy dtype as in the
    reference, or a torch dtype such as ``torch.bfloat16``).

    ``b_kmajor`` (extension): ``b`` is an ``(N, K)`` operand cast with its
    blocks along K (a weight in nn.Linear orientation); the result is
    ``a @ b^T``, the layout the block-scaled tensor-core GEMMs consume."""
    from . import gemm
    return gemm.matmul(a, b, _torch_out_dtype(out_dtype), b_kmajor=b_kmajor)


# cast_matmul picks the fused kernel by itself only for a history-scaled cast
# (one pass, no amax pass before the GEMM) and N >= _FUSED_MIN_N. At C2
# (16384 x 8192 x 8192) it measured 0.809-0.811 against 0.817-0.825 ms for the
# cast then the GEMM; with the current amax 0.847-0.854 against 0.851-0.859 ms
# (level: the amax pass still runs first); at N = 4096 it took 0.52-0.58 ms
# against 0.44-0.47 ms.
_FUSED_MIN_N = 8192


def cast_matmul(x, b, recipe, *, amax_history: Optional[AmaxHistory] = None,
                out_dtype=np.float32, b_kmajor: bool = False, fused: Optional[bool] = None,
                prologue_rows: int = -1):
    """``matmul(cast(x, recipe), b)`` with the cast fused into the GEMM
    (extension; the reference casts, then multiplies: ``cast.py:64-92``,
    ``matmul.py:42-133``). Returns ``(out, a)``: ``a`` is the ScaledTensor
    ``cast(x, recipe, amax_history=amax_history)`` returns and ``out`` the
    product ``matmul(a, b, out_dtype, b_kmajor=b_kmajor)`` returns, both bit
    for bit, whichever way it runs.

    The fused kernel takes a per-tensor recipe (``DelayedScaling`` /
    ``Float8CurrentScaling``) and a 2-D per-tensor ``b`` with ``K % 128 == 0``
    and ``N % 16 == 0``: one GEMM launch whose extra warps encode ``x`` while
    the tensor cores work (only the first ``prologue_rows`` rows, ``-1`` = one
    tile group of 4096, are encoded before it). ``fused=None`` uses it where
    it measured no slower than the separate cast on B200: a DelayedScaling
    cast from a recorded amax history with ``N >= 8192`` (each activation tile
    feeds at least 32 output tiles). Otherwise ``cast`` then ``matmul`` runs:
    with the current amax the separate passes measured as fast or faster, and
    below ``N = 8192`` the in-kernel encode cannot keep up. ``True`` /
    ``False`` force either way (``True`` still needs the shape conditions)."""
    from . import gemm
    x = _input(x)
    name = getattr(recipe, "name", None)
    if amax_history is not None and name != "delayed":
        raise ValueError("amax_history applies to DelayedScaling only")
    odt = _torch_out_dtype(out_dtype)
    K = x.shape[-1] if x.ndim else 0
    ok = (name in ("delayed", "current") and _is_scaled(b) and
             getattr(getattr(b, "recipe", None), "name", None) in ("delayed", "current") and
             b.data.ndim == 2 and b.data.is_cuda and b.data.device == x.device and x.ndim >= 1)
    if ok:
        N, Kb = b.data.shape if b_kmajor else tuple(reversed(b.data.shape))
        ok = Kb == K and K > 0 and K % 128 == 0 and N % 16 == 0
        if ok and fused is None:
            ok = (N >= _FUSED_MIN_N and amax_history is not None and
                  amax_history.recorded > 0)
    if not ok or fused is False:
        a = cast(x, recipe, amax_history=amax_history)
        return matmul(a, b, out_dtype, b_kmajor=b_kmajor), a
    with torch.cuda.device(x.device):
        w_codes = _codes_u8(b.data) if b_kmajor else gemm._transposed_codes(b)
    return _fused_cast_gemm(x, recipe, w_codes, b, N, odt, amax_history, None, prologue_rows)


def _fused_cast_gemm(x, recipe, w_codes, b, N, odt, amax_history, amax_word, prologue_rows):
    """brc_cast_gemm_pertensor_fp8 on ``x`` and the (N, K) codes of the
    per-tensor ScaledTensor ``b``; ``amax_word`` (a device int32 word holding
    the float bits of an amax already reduced by the caller) replaces the
    amax pass. Returns (out, cast(x))."""
    ST, L = _classes(recipe)
    fmt = recipe.fp8_format
    dev = x.device
    K = x.shape[-1]
    M = x.numel() // K
    cdt = odt if odt in _OUT_DT else torch.float32
    with torch.cuda.device(dev):
        st = _stream(dev)
        codes = torch.empty(x.shape, dtype=torch.uint8, device=dev)
        scale = torch.empty((), dtype=torch.float32, device=dev)
        out = torch.empty(x.shape[:-1] + (N,), dtype=cdt, device=dev)
        ws_bytes = int(_lib.lib().brc_cast_gemm_workspace_bytes(M, K))
        ws = torch.empty((ws_bytes + 3) // 4, dtype=torch.int32, device=dev)
        hist, hlen, margin, use = None, 0, 0, 0
        if amax_history is not None:
            h = amax_history.history
            if not (isinstance(h, torch.Tensor) and h.is_cuda and h.dtype == torch.float32 and
                    h.is_contiguous() and h.device == dev):
                raise TypeError(
                    "AmaxHistory.history must be a contiguous float32 tensor on x's device")
            hist, hlen, margin = h.data_ptr(), h.numel(), int(recipe.margin)
            use = 1 if amax_history.recorded > 0 else 0
        _lib.call("brc_cast_gemm_pertensor_fp8", x.data_ptr(), _IN_DT[x.dtype], _FMT[fmt],
                  w_codes.data_ptr(), _FMT[b.recipe.fp8_format],
                  b.scale.to(torch.float32).data_ptr(), M, N, K, hist, hlen, margin, use,
                  None if amax_word is None else amax_word.data_ptr(),
                  codes.data_ptr(), scale.data_ptr(), out.data_ptr(), _OUT_DT[cdt],
                  ws.data_ptr(), ws_bytes, int(prologue_rows), st)
    if amax_history is not None:
        amax_history.recorded += 1
    a = ST(data=codes.view(_TORCH_FP8[fmt]), scale=scale, recipe=recipe, layout=L.PerTensor())
    return (out if cdt == odt else out.to(odt)), a


def linear(a, w, out_dtype=torch.bfloat16):
    """``a @ w.T`` with ``w`` an ``(N, K)`` ScaledTensor whose blocks run
    along K (a weight cast in nn.Linear orientation). This is the layout the
    block-scaled tensor-core GEMMs consume directly."""
    from . import gemm
    return gemm.linear(a, w, _torch_out_dtype(out_dtype))


def attach_gemm_operands(scaled):
    """Rebuild, on the GPU, the side operands ``cast`` records for the
    tensor-core GEMMs, for a CUDA ``ScaledTensor`` that was not cast here
    (loaded from a file, or produced by another implementation): for NVFP4
    the packed codes (tensor-core nibble order) and the tcgen05 scale atoms,
    for MXFP8 the scale atoms, for INT4 of group 128 with a multiple of 16
    rows the skinny-GEMM tiles. They equal what ``cast`` writes byte for
    byte, so ``matmul`` / ``linear`` take the same kernels. Other recipes
    need none. Returns ``scaled``."""
    name = getattr(getattr(scaled, "recipe", None), "name", None)
    data = scaled.data
    if name not in ("nvfp4", "mxfp8", "int4") or not isinstance(data, torch.Tensor) \
            or not data.is_cuda or data.ndim < 1:
        return scaled
    comp = _companions(scaled)
    side = _side(data, comp)
    dev = data.device
    codes = _aligned(data.contiguous().view(torch.uint8))
    K = codes.shape[-1]
    rows = codes.numel() // K if K else 0
    if rows == 0:
        return scaled
    with torch.cuda.device(dev):
        st = _stream(dev)
        if name in ("nvfp4", "mxfp8"):
            add = {}
            bs = 16 if name == "nvfp4" else 32
            if "sf_mma" not in side:
                sc = _aligned(scaled.scale.contiguous().view(torch.uint8))
                sf = torch.empty(_mma_scale_shape(rows, K // bs), dtype=torch.uint8, device=dev)
                _lib.call("brc_scale_atoms", sc.data_ptr(), rows, K // bs, sf.data_ptr(), st)
                add["sf_mma"] = sf
            if name == "nvfp4" and "packed" not in side and K % 2 == 0:
                packed = torch.empty(codes.shape[:-1] + (K // 2,), dtype=torch.uint8, device=dev)
                _lib.call("brc_pack_codes_lo", codes.data_ptr(), codes.numel(),
                          packed.data_ptr(), st)
                add["packed"] = packed
            if add:
                _remember(data, comp, **add)
        elif "int4_tiles" not in side and scaled.recipe.group_size == 128 and \
                rows % 16 == 0 and K % 128 == 0:
            sc = _aligned(scaled.scale.contiguous())
            if sc.dtype not in (torch.float16, torch.float32):
                return scaled
            sdt = _lib.SCALE_F16 if sc.dtype == torch.float16 else _lib.SCALE_F32
            zp = None if scaled.zero_point is None else \
                _aligned(scaled.zero_point.contiguous().to(sc.dtype))
            tiles = torch.empty(rows * K // 2, dtype=torch.uint8, device=dev)
            stiles = torch.empty(rows * (K // 128), dtype=torch.float32, device=dev)
            ztiles = None if zp is None else torch.empty_like(stiles)
            _lib.call("brc_int4_tiles", codes.data_ptr(), rows, K, sc.data_ptr(), _ptr(zp),
                      sdt, tiles.data_ptr(), stiles.data_ptr(), _ptr(ztiles), st)
            _remember(data, comp, int4_tiles=tiles, int4_scale_tiles=stiles,
                      int4_zp_tiles=ztiles)
    return scaled


def gemm_operands(scaled) -> dict:
    """Side data recorded by ``cast`` for ``scaled``: ``sf_mma`` (scales in
    the tcgen05 layout), ``packed`` (two 4-bit codes per byte, element 2i in
    the low nibble), or the INT4 skinny-GEMM tiles (``int4_tiles``,
    ``int4_scale_tiles``, ``int4_zp_tiles``)."""
    side = _side(scaled.data, _companions(scaled))
    return {k: v for k, v in side.items() if not k.startswith("_")}
