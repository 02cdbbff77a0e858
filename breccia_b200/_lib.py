"""ctypes binding of the C ABI in ``include/breccia_b200.h``.

The shared library ``libbreccia_b200.so`` is built in-tree by
``python -m breccia_b200.build``. There is no fallback: if the library is
missing, every operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbreccia_b200.so")

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64

# name -> argument types (every function returns int status unless noted)
# brc_cast_ste_block kinds
STE_BLOCK_FP8, STE_MXFP8, STE_NVFP4, STE_INT4 = 0, 1, 2, 3
KIND_PERTENSOR_FP8 = 4

PROTOTYPES = {
    "brc_status_string": ([_i], ctypes.c_char_p),
    "brc_last_cuda_error": ([], _i),
    "brc_version": ([], _i),
    "brc_amax_reset": ([_p, _p], _i),
    "brc_amax_accumulate": ([_p, _i, _i64, _p, _p], _i),
    "brc_cast_pertensor_fp8_apply": ([_p, _i, _i64, _i, _p, _p, _p, _p], _i),
    "brc_cast_pertensor_fp8": ([_p, _i, _i64, _i, _p, _p, _p, _p], _i),
    "brc_cast_pertensor_fp8_noalloc": ([_p, _i, _i64, _i, _p, _p, _p], _i),
    "brc_cast_pertensor_fp8_delayed": ([_p, _i, _i64, _i, _p, _i, _i, _i, _p, _p, _p, _p], _i),
    "brc_cast_block_fp8": ([_p, _i, _i64, _i64, _i, _i, _p, _p, _p], _i),
    "brc_cast_block_fp8_2d": ([_p, _i, _i64, _i64, _i, _i, _i, _p, _p, _p], _i),
    "brc_cast_mxfp8": ([_p, _i, _i64, _i64, _i, _p, _p, _p, _p], _i),
    "brc_cast_nvfp4": ([_p, _i, _i64, _i64, _p, _p, _p, _p, _p], _i),
    "brc_cast_int4": ([_p, _i, _i64, _i64, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p], _i),
    "brc_cast_ste_pertensor_fp8": ([_p, _i, _i64, _i, _p, _p, _p], _i),
    "brc_cast_ste_block": ([_p, _i, _i64, _i64, _i, _i, _i, _i, _i, _i, _p, _p], _i),
    "brc_pack_nibbles_hi": ([_p, _i64, _p, _p], _i),
    "brc_unpack_nibbles_hi": ([_p, _i64, _p, _p, _p], _i),
    "brc_pack_codes_lo": ([_p, _i64, _p, _p], _i),
    "brc_scale_atoms": ([_p, _i64, _i64, _p, _p], _i),
    "brc_int4_tiles": ([_p, _i64, _i64, _p, _p, _i, _p, _p, _p, _p], _i),
    "brc_dequant_pertensor_fp8": ([_p, _i64, _i, _p, _p, _i, _p], _i),
    "brc_dequant_block_fp8": ([_p, _i64, _i64, _i, _i, _i, _p, _p, _i, _p], _i),
    "brc_dequant_mxfp8": ([_p, _i64, _i64, _i, _p, _p, _i, _p], _i),
    "brc_dequant_nvfp4": ([_p, _i64, _i64, _p, _p, _i, _p], _i),
    "brc_dequant_int4": ([_p, _i64, _i64, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_requant_nvfp4_to_mxfp8": ([_p, _p, _i64, _i64, _i, _p, _p, _p, _p], _i),
    "brc_selftest_division": ([_p, _p, _i64, _p, _p, _p], _i),
    "brc_gemm_fp8_pertensor": ([_p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_cast_gemm_workspace_bytes": ([_i, _i], _i64),
    "brc_cast_gemm_pertensor_fp8": ([_p, _i, _i, _p, _i, _p, _i, _i, _i, _p, _i, _i, _i, _p, _p,
                                     _p, _p, _i, _p, _i64, _i, _p], _i),
    "brc_gemm_mxfp8": ([_p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_gemm_nvfp4": ([_p, _p, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_gemm_block_fp8": ([_p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_gemm_int4": ([_p, _i, _i, _p, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_gemm_status": ([_i], _i),
    "brc_selftest_wait_timeout": ([_i, _p, _p], _i),
    "brc_gemm_bf16": ([_p, _p, _i, _i, _i, _p, _i, _p], _i),
    "brc_dequant_transposed": ([_p, _i64, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _i, _p], _i),
    "brc_transpose_u8": ([_p, _i64, _i64, _p, _p], _i),
}

# status codes (include/breccia_b200.h)
BRC_OK = 0
BRC_ERR_NULL = -1
BRC_ERR_SHAPE = -2
BRC_ERR_ALIGN = -3
BRC_ERR_DTYPE = -4
BRC_ERR_UNSUPPORTED = -5
BRC_ERR_CUDA = -6
BRC_ERR_TIMEOUT = -7
BRC_ERR_RANGE = -8

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
FP8_E4M3, FP8_E5M2 = 0, 1
SCALE_F16, SCALE_F32 = 0, 1

_lock = threading.Lock()
_lib = None


class BrecciaB200Error(RuntimeError):
    """A C ABI call returned a non-zero status."""

    def __init__(self, name: str, status: int, detail: str):
        super().__init__(f"{name}: {detail} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the shared library once (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"breccia_b200 CUDA library not found at {LIB_PATH}; "
                        "build it with `python -m breccia_b200.build`")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (argtypes, restype) in PROTOTYPES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = argtypes
                    fn.restype = restype
                _lib = handle
    return _lib


def call(name: str, *args) -> None:
    """Call ``name`` and raise on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    if rc != BRC_OK:
        detail = lib().brc_status_string(rc).decode()
        if rc == BRC_ERR_CUDA:
            detail += f" (cudaError {lib().brc_last_cuda_error()})"
        if rc in (BRC_ERR_SHAPE, BRC_ERR_RANGE, BRC_ERR_ALIGN):
            raise ValueError(f"{name}: {detail} (status {rc})")
        if rc == BRC_ERR_DTYPE:
            raise TypeError(f"{name}: {detail} (status {rc})")
        raise BrecciaB200Error(name, rc, detail)
