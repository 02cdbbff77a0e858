"""Scaled matmul dispatch onto this library's tensor-core GEMMs.

Reference: ``src/breccia/kernels/reference/matmul.py:42-133`` (jvoltci/breccia
v0.1.3): dequantize both operands, ``a.float() @ b.float()``, cast to
``out_dtype``.

Block-scaled tensor-core kinds (both operands K-major, i.e. ``linear(a, w)``
with ``w`` an ``(N, K)`` weight cast in nn.Linear orientation, or
``matmul(a, w, b_kmajor=True)``):

* per-tensor FP8 x per-tensor FP8 -> ``brc_gemm_fp8_pertensor``
  (``matmul`` also reaches it in breccia's ``(K, N)`` orientation:
  per-tensor codes do not depend on orientation, so ``brc_transpose_u8``
  moves them as plain bytes)
* MXFP8 x MXFP8 -> ``brc_gemm_mxfp8``
* NVFP4 x NVFP4 -> ``brc_gemm_nvfp4``
* Float8BlockScaling 1 x 128 activations x 128 x 128 weights (DeepSeek-v3
  layout, ``cast(w, Float8BlockScaling(), block_m=128)``) -> ``brc_gemm_block_fp8``
* raw bfloat16 activations (at most 16 rows) x INT4 weight (group 128) ->
  ``brc_gemm_int4`` (dequantization fused, weight read once)

Every other recipe pair, and block-scaled weights in breccia's own ``(K, N)``
orientation (scale blocks along N, which a K-blocked MMA cannot consume),
follow the reference literally -- dequantize both, then one float32-
accumulated GEMM -- on this library's kernels: the operands are dequantized
to bf16 (``brc_dequant_*``; a ``(K, N)`` operand through
``brc_dequant_transposed``, which writes it K-major) and multiplied by the
tcgen05 ``kind::f16`` GEMM ``brc_gemm_bf16``. MXFP8 and NVFP4 values are
exact in bf16, so those products equal the reference's; per-tensor FP8,
block FP8 and INT4 values take one bf16 rounding (relative error <= 2^-9 per
element, inside the 1e-2 / 0.9999 matmul tolerance). Shapes that kernel
cannot take (K % 8, N % 16, batched ``b``) use torch's float32 matmul on the
GPU.
"""

from __future__ import annotations

import torch

from . import _lib
from .api import (dequantize, _is_scaled, _require_cuda, _side_of, _codes_u8, _stream, _FMT,
                  _OUT_DT, _aligned)

_PER_TENSOR = ("delayed", "current")


def _dense(t):
    if _is_scaled(t):
        return dequantize(t)
    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t, dtype=torch.float32)
    return t


def _general(a_t, b_t, out_dtype):
    """matmul.py:75-89: float32 matmul of dequantized operands."""
    if a_t.shape[-1] != b_t.shape[-2]:
        raise ValueError(
            f"matmul shape mismatch: a.shape[-1]={a_t.shape[-1]} != "
            f"b.shape[-2]={b_t.shape[-2]}")
    dev = a_t.device if a_t.is_cuda else b_t.device
    return (a_t.to(dev).float() @ b_t.to(dev).float()).to(out_dtype)


def _name(t):
    return getattr(getattr(t, "recipe", None), "name", None) if _is_scaled(t) else None


def _tc_pair(a, w):
    """Kind of tensor-core GEMM usable for a (..., K) x w (N, K), or None."""
    na, nw = _name(a), _name(w)
    if na is None or nw is None or w.data.ndim != 2 or a.data.ndim < 2:
        return None
    if not (a.data.is_cuda and w.data.is_cuda) or a.data.device != w.data.device:
        return None
    K = a.data.shape[-1]
    N = w.data.shape[0]
    if w.data.shape[-1] != K or N % 16 or K == 0:
        return None
    if na in _PER_TENSOR and nw in _PER_TENSOR and K % 128 == 0:
        if a.scale.ndim == 0 and w.scale.ndim == 0:
            return "fp8"
    if na == "mxfp8" and nw == "mxfp8" and K % 128 == 0:
        if "sf_mma" in _side_of(a) and "sf_mma" in _side_of(w):
            return "mxfp8"
    if na == "block" and nw == "block" and K % 128 == 0 and \
            a.recipe.block_k == 128 and w.recipe.block_k == 128:
        la, lw = getattr(a.layout, "name", ""), getattr(w.layout, "name", "")
        if la == "per_block_k" and lw == "per_block_mn" and w.layout.block_m == 128 and \
                w.layout.block_n == 128:
            return "block"
    if na == "nvfp4" and nw == "nvfp4" and K % 256 == 0:
        sa, sw = _side_of(a), _side_of(w)
        if "sf_mma" in sa and "packed" in sa and "sf_mma" in sw and "packed" in sw:
            return "nvfp4"
    return None


def _int4_pair(a, w):
    """Raw bf16 activations (<= 16 rows) x packed INT4 weight (N, K)."""
    if _is_scaled(a) or not isinstance(a, torch.Tensor) or _name(w) != "int4":
        return False
    if not (a.is_cuda and w.data.is_cuda) or a.device != w.data.device:
        return False
    if a.dtype != torch.bfloat16 or a.ndim < 1 or w.data.ndim != 2:
        return False
    K = a.shape[-1]
    M = a.numel() // K if K else 0
    N = w.data.shape[0]
    return (w.data.shape[1] == K and 0 < M <= 16 and K % 1024 == 0 and N % 16 == 0 and
            w.recipe.group_size == 128 and "int4_tiles" in _side_of(w))


def _run_int4(a, w, out_dtype):
    K = a.shape[-1]
    M = a.numel() // K
    N = w.data.shape[0]
    dev = a.device
    cdt = out_dtype if out_dtype in _OUT_DT else torch.float32
    out = torch.empty(a.shape[:-1] + (N,), dtype=cdt, device=dev)
    a2 = a.contiguous()
    if a2.data_ptr() % 16:
        a2 = a2.clone()
    r = w.recipe
    side = _side_of(w)
    zt = side["int4_zp_tiles"]
    with torch.cuda.device(dev):
        _lib.call("brc_gemm_int4", a2.data_ptr(), M, K, side["int4_tiles"].data_ptr(), N,
                  int(bool(r.signed)), int(bool(r.symmetric)),
                  side["int4_scale_tiles"].data_ptr(), None if zt is None else zt.data_ptr(),
                  out.data_ptr(), _OUT_DT[cdt], _stream(dev))
    return out if cdt == out_dtype else out.to(out_dtype)


def _run_tc(kind, a, w, out_dtype, w_codes=None):
    K = a.data.shape[-1]
    M = a.data.numel() // K
    N = w.data.shape[0]
    dev = a.data.device
    cdt = out_dtype if out_dtype in _OUT_DT else torch.float32
    out = torch.empty(a.data.shape[:-1] + (N,), dtype=cdt, device=dev)
    with torch.cuda.device(dev):
        st = _stream(dev)
        if kind == "fp8":
            ac = _codes_u8(a.data)
            wc = _codes_u8(w.data) if w_codes is None else w_codes
            _lib.call("brc_gemm_fp8_pertensor", ac.data_ptr(), wc.data_ptr(), M, N, K,
                      _FMT[a.recipe.fp8_format], _FMT[w.recipe.fp8_format],
                      a.scale.to(torch.float32).data_ptr(), w.scale.to(torch.float32).data_ptr(),
                      out.data_ptr(), _OUT_DT[cdt], st)
        elif kind == "block":
            _lib.call("brc_gemm_block_fp8", _codes_u8(a.data).data_ptr(),
                      _codes_u8(w.data).data_ptr(), M, N, K, _FMT[a.recipe.fp8_format],
                      _FMT[w.recipe.fp8_format], a.scale.contiguous().data_ptr(),
                      w.scale.contiguous().data_ptr(), out.data_ptr(), _OUT_DT[cdt], st)
        elif kind == "mxfp8":
            sa, sw = _side_of(a), _side_of(w)
            _lib.call("brc_gemm_mxfp8", _codes_u8(a.data).data_ptr(), _codes_u8(w.data).data_ptr(),
                      M, N, K, _FMT[a.recipe.fp8_format], _FMT[w.recipe.fp8_format],
                      sa["sf_mma"].data_ptr(), sw["sf_mma"].data_ptr(), out.data_ptr(),
                      _OUT_DT[cdt], st)
        else:
            sa, sw = _side_of(a), _side_of(w)
            _lib.call("brc_gemm_nvfp4", sa["packed"].data_ptr(), sw["packed"].data_ptr(), M, N, K,
                      sa["sf_mma"].data_ptr(), sw["sf_mma"].data_ptr(), out.data_ptr(),
                      _OUT_DT[cdt], st)
    return out if cdt == out_dtype else out.to(out_dtype)


def _transposed_codes(b):
    """(K, N) per-tensor codes -> (N, K) bytes (brc_transpose_u8)."""
    codes = _codes_u8(b.data)
    K, N = codes.shape
    out = torch.empty((N, K), dtype=torch.uint8, device=codes.device)
    with torch.cuda.device(codes.device):
        _lib.call("brc_transpose_u8", codes.data_ptr(), K, N, out.data_ptr(),
                  _stream(codes.device))
    return out


def _dq_kind(t):
    """brc_dequant_transposed arguments for a ScaledTensor, or None."""
    r = t.recipe
    name = getattr(r, "name", None)
    fmt = _FMT.get(getattr(r, "fp8_format", "E4M3"), _lib.FP8_E4M3)
    if name in _PER_TENSOR:
        return _lib.KIND_PERTENSOR_FP8, fmt, 16, 0, _lib.SCALE_F32
    if name == "block":
        if getattr(t.layout, "name", "") != "per_block_k":
            return None  # 2-D weight tiles: no transposed form
        return _lib.STE_BLOCK_FP8, fmt, r.block_k, 0, _lib.SCALE_F32
    if name == "mxfp8":
        return _lib.STE_MXFP8, fmt, 32, 0, _lib.SCALE_F32
    if name == "nvfp4":
        return _lib.STE_NVFP4, fmt, 16, 0, _lib.SCALE_F32
    if name == "int4":
        sdt = _lib.SCALE_F16 if t.scale.dtype == torch.float16 else _lib.SCALE_F32
        return _lib.STE_INT4, fmt, r.group_size, int(bool(r.signed)), sdt
    return None


def _bf16_nk(b):
    """breccia-orientation operand b (K, N) as a K-major (N, K) bf16 tensor, or
    None when it cannot be produced here."""
    if _is_scaled(b):
        if b.data.ndim != 2 or not b.data.is_cuda:
            return None
        args = _dq_kind(b)
        K, N = b.data.shape
        if args is None or K % 8 or N % 16 or N % args[2]:
            return None
        kind, fmt, block, signed, sdt = args
        codes = _codes_u8(b.data)
        scale = _aligned(b.scale)
        if kind == _lib.STE_INT4 and scale.dtype not in (torch.float16, torch.float32):
            scale = scale.to(torch.float32)
            sdt = _lib.SCALE_F32
        zp = getattr(b, "zero_point", None)
        if zp is not None:
            zp = _aligned(zp.to(scale.dtype))
        out = torch.empty((N, K), dtype=torch.bfloat16, device=codes.device)
        with torch.cuda.device(codes.device):
            _lib.call("brc_dequant_transposed", codes.data_ptr(), K, N, kind, fmt, block, signed,
                      sdt, scale.to(torch.float32).data_ptr() if kind in (
                          _lib.KIND_PERTENSOR_FP8, _lib.STE_BLOCK_FP8) else scale.data_ptr(),
                      None if zp is None else zp.data_ptr(), out.data_ptr(),
                      _lib.DTYPE_BF16, _stream(codes.device))
        return out
    if isinstance(b, torch.Tensor) and b.is_cuda and b.ndim == 2:
        return b.to(torch.bfloat16).t().contiguous()
    return None


def _bf16_kmajor(t):
    """K-major operand (..., K) as bf16: a ScaledTensor dequantized by this
    library (bf16 output), a raw CUDA tensor converted."""
    if _is_scaled(t):
        if not t.data.is_cuda:
            return None
        return dequantize(t, out_dtype=torch.bfloat16)
    if isinstance(t, torch.Tensor) and t.is_cuda:
        return t.to(torch.bfloat16)
    return None


def _run_bf16(a_bf, b_nk, out_dtype):
    """a_bf (..., K) x b_nk (N, K) on brc_gemm_bf16, or None if the shape or
    placement is outside what the kernel takes."""
    if a_bf is None or b_nk is None or a_bf.device != b_nk.device or b_nk.ndim != 2:
        return None
    K = a_bf.shape[-1]
    N = b_nk.shape[0]
    if b_nk.shape[1] != K or K == 0 or K % 8 or N % 16:
        return None
    M = a_bf.numel() // K
    a2 = _aligned(a_bf.reshape(M, K))
    b2 = _aligned(b_nk)
    dev = a2.device
    cdt = out_dtype if out_dtype in _OUT_DT else torch.float32
    out = torch.empty(a_bf.shape[:-1] + (N,), dtype=cdt, device=dev)
    if M:
        with torch.cuda.device(dev):
            _lib.call("brc_gemm_bf16", a2.data_ptr(), b2.data_ptr(), M, N, K, out.data_ptr(),
                      _OUT_DT[cdt], _stream(dev))
    return out if cdt == out_dtype else out.to(out_dtype)


def _shape_check(a_shape, b_shape):
    """matmul.py:127-131 message."""
    if a_shape[-1] != b_shape[-2]:
        raise ValueError(
            f"matmul shape mismatch: a.shape[-1]={a_shape[-1]} != "
            f"b.shape[-2]={b_shape[-2]}")


def _shape_of(t):
    return tuple(t.data.shape) if _is_scaled(t) else tuple(getattr(t, "shape", ()))


def matmul(a, b, out_dtype, b_kmajor=False):
    """Reference semantics: ``a (..., M, K) @ b (..., K, N)``. With
    ``b_kmajor`` (extension) ``b`` is an ``(N, K)`` operand whose blocks run
    along K (nn.Linear orientation) and the result is ``a @ b^T``."""
    if b_kmajor:
        return linear(a, b, out_dtype)
    sa, sb = _shape_of(a), _shape_of(b)
    if len(sa) >= 1 and len(sb) >= 2:
        _shape_check(sa, sb)
    if _name(a) in _PER_TENSOR and _name(b) in _PER_TENSOR and b.data.ndim == 2:
        kind = _tc_pair(a, _Transposed(b))
        if kind == "fp8" and b.data.shape[0] % 16 == 0:
            return _run_tc(kind, a, _Transposed(b), out_dtype, w_codes=_transposed_codes(b))
    if len(sb) == 2:
        out = _run_bf16(_bf16_kmajor(a), _bf16_nk(b), out_dtype)
        if out is not None:
            return out
    a_t, b_t = _dense(a), _dense(b)
    if not (a_t.is_cuda or b_t.is_cuda):
        _require_cuda(a_t, "a")
    return _general(a_t, b_t, out_dtype)


class _Transposed:
    """View of a 2-D per-tensor ScaledTensor as its transpose (shape only:
    per-tensor codes are elementwise, so only the byte order changes)."""

    def __init__(self, st):
        self.recipe = st.recipe
        self.scale = st.scale
        self.layout = st.layout
        self.data = _ShapeOnly(st.data)


class _ShapeOnly:
    def __init__(self, t):
        self._t = t
        self.shape = tuple(reversed(t.shape))
        self.ndim = t.ndim
        self.is_cuda = t.is_cuda
        self.device = t.device
        self.dtype = t.dtype


def linear(a, w, out_dtype):
    """``a @ w.T`` with ``w`` an ``(N, K)`` operand."""
    if _int4_pair(a, w):
        return _run_int4(a, w, out_dtype)
    kind = _tc_pair(a, w)
    if kind is not None:
        return _run_tc(kind, a, w, out_dtype)
    sa, sw = _shape_of(a), _shape_of(w)
    if len(sa) >= 1 and len(sw) >= 1 and sa[-1] != sw[-1]:
        raise ValueError(
            f"linear shape mismatch: a.shape[-1]={sa[-1]} != w.shape[-1]={sw[-1]}")
    if len(sw) == 2:
        w_bf = _bf16_kmajor(w)
        out = _run_bf16(_bf16_kmajor(a), None if w_bf is None else _aligned(w_bf), out_dtype)
        if out is not None:
            return out
    a_t, w_t = _dense(a), _dense(w)
    return _general(a_t, w_t.transpose(-1, -2), out_dtype)
