"""Scaled matmul dispatch: tcgen05 tensor-core GEMMs for the recipe pairs
that have one, the reference's dequantize-then-float32-matmul semantics for
the rest.

Reference: ``src/breccia/kernels/reference/matmul.py:42-133`` (jvoltci/breccia
v0.1.3): dequantize both operands, ``a.float() @ b.float()``, cast to
``out_dtype``.

Tensor-core paths (both operands K-major, i.e. ``linear(a, w)`` with ``w`` an
``(N, K)`` weight cast in nn.Linear orientation):

* per-tensor FP8 x per-tensor FP8 -> ``brc_gemm_fp8_pertensor``
  (``matmul`` also reaches it: per-tensor codes do not depend on orientation,
  so a ``(K, N)`` operand is transposed as plain bytes)
* MXFP8 x MXFP8 -> ``brc_gemm_mxfp8``
* NVFP4 x NVFP4 -> ``brc_gemm_nvfp4``
* Float8BlockScaling 1 x 128 activations x 128 x 128 weights (DeepSeek-v3
  layout, ``cast(w, Float8BlockScaling(), block_m=128)``) -> ``brc_gemm_block_fp8``
* raw bfloat16 activations (at most 16 rows) x INT4 weight (group 128) ->
  ``brc_gemm_int4`` (dequantization fused, weight read once)
"""

from __future__ import annotations

import torch

from . import _lib
from .api import (dequantize, _is_scaled, _require_cuda, _side_of, _codes_u8, _stream, _FMT,
                  _OUT_DT)

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


def matmul(a, b, out_dtype):
    """Reference semantics: ``a (..., M, K) @ b (..., K, N)``."""
    if _name(a) in _PER_TENSOR and _name(b) in _PER_TENSOR and b.data.ndim == 2:
        kind = _tc_pair(a, _Transposed(b))
        if kind == "fp8":
            wc = _codes_u8(b.data).t().contiguous()
            return _run_tc(kind, a, _Transposed(b), out_dtype, w_codes=wc)
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
    a_t, w_t = _dense(a), _dense(w)
    if a_t.shape[-1] != w_t.shape[-1]:
        raise ValueError(
            f"linear shape mismatch: a.shape[-1]={a_t.shape[-1]} != "
            f"w.shape[-1]={w_t.shape[-1]}")
    return _general(a_t, w_t.transpose(-1, -2), out_dtype)
