"""C ABI: the library loads without a GPU, exports exactly what the header
declares, and rejects bad arguments on the host before touching CUDA."""

import ctypes
import os
import re

import pytest

from breccia_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fn in os.listdir(inc):
        if fn.endswith(".h"):
            text = open(os.path.join(inc, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(brc_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    declared = _declared()
    assert declared, "no declarations found"
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    assert _declared() == set(_lib.PROTOTYPES)


def test_status_strings():
    L = _lib.lib()
    assert L.brc_status_string(0) == b"ok"
    assert L.brc_status_string(-2) == b"inconsistent sizes"
    assert L.brc_version() >= 100


def _buf(n=64):
    # host memory, 16-byte aligned: the checks below fail before any CUDA call
    raw = (ctypes.c_uint8 * (n + 16))()
    addr = ctypes.addressof(raw)
    return raw, addr + (-addr % 16)


def test_null_pointers_rejected():
    L = _lib.lib()
    _, p = _buf()
    assert L.brc_cast_block_fp8(None, 0, 4, 128, 128, 0, p, p, None) == _lib.BRC_ERR_NULL
    assert L.brc_cast_mxfp8(p, 0, 4, 64, 0, None, p, None, None) == _lib.BRC_ERR_NULL
    assert L.brc_cast_nvfp4(p, 0, 4, 64, None, None, p, None, None) == _lib.BRC_ERR_NULL
    # asymmetric INT4 needs a zero-point buffer
    assert L.brc_cast_int4(p, 0, 4, 128, 128, 0, 0, 0, p, None, p, None, None, None, None,
                           None) == _lib.BRC_ERR_NULL


def test_shapes_dtypes_alignment_rejected():
    L = _lib.lib()
    _, p = _buf()
    assert L.brc_cast_block_fp8(p, 0, 4, 100, 128, 0, p, p, None) == _lib.BRC_ERR_SHAPE
    assert L.brc_cast_mxfp8(p, 0, 4, 48, 0, p, p, None, None) == _lib.BRC_ERR_SHAPE
    assert L.brc_cast_block_fp8(p, 7, 4, 128, 128, 0, p, p, None) == _lib.BRC_ERR_DTYPE
    assert L.brc_cast_block_fp8(p, 0, 4, 128, 128, 9, p, p, None) == _lib.BRC_ERR_DTYPE
    assert L.brc_cast_block_fp8(p + 4, 0, 4, 128, 128, 0, p, p, None) == _lib.BRC_ERR_ALIGN
    assert L.brc_cast_int4(p, 0, 4, 128, 128, 1, 0, 0, p, None, p, p, None, None, None,
                           None) == _lib.BRC_ERR_UNSUPPORTED  # asymmetric + signed is invalid
    assert L.brc_dequant_nvfp4(p, 4, 24, p, p, 0, None) == _lib.BRC_ERR_SHAPE
    assert L.brc_dequant_mxfp8(p, 4, 64, 0, p, p, 5, None) == _lib.BRC_ERR_DTYPE


def test_empty_inputs_are_noops():
    L = _lib.lib()
    _, p = _buf()
    assert L.brc_cast_block_fp8(p, 0, 0, 128, 128, 0, p, p, None) == _lib.BRC_OK
    assert L.brc_cast_mxfp8(p, 1, 0, 64, 0, p, p, None, None) == _lib.BRC_OK
    assert L.brc_amax_accumulate(None, 0, 0, p, None) == _lib.BRC_OK


def test_call_raises_python_exceptions():
    _, p = _buf()
    with pytest.raises(ValueError):
        _lib.call("brc_cast_block_fp8", p, 0, 4, 100, 128, 0, p, p, None)
    with pytest.raises(TypeError):
        _lib.call("brc_cast_block_fp8", p, 5, 4, 128, 128, 0, p, p, None)
    with pytest.raises(_lib.BrecciaB200Error):
        _lib.call("brc_cast_block_fp8", None, 0, 4, 128, 128, 0, p, p, None)


def test_bridge_entry_points_reject_bad_arguments():
    """Stored-4-bit / operand-rebuild entry points: shape, null, alignment and
    dtype checks happen on the host, before any CUDA call."""
    L = _lib.lib()
    _, p = _buf(256)
    # odd code counts, negative sizes
    assert L.brc_pack_nibbles_hi(p, 3, p, None) == _lib.BRC_ERR_SHAPE
    assert L.brc_unpack_nibbles_hi(p, -2, p, None, None) == _lib.BRC_ERR_SHAPE
    assert L.brc_pack_codes_lo(p, 5, p, None) == _lib.BRC_ERR_SHAPE
    # empty inputs are a no-op
    assert L.brc_pack_nibbles_hi(None, 0, None, None) == _lib.BRC_OK
    assert L.brc_scale_atoms(None, 0, 8, None, None) == _lib.BRC_OK
    assert L.brc_int4_tiles(None, 0, 128, None, None, 0, None, None, None, None) == _lib.BRC_OK
    # null buffers
    assert L.brc_pack_nibbles_hi(None, 4, p, None) == _lib.BRC_ERR_NULL
    assert L.brc_unpack_nibbles_hi(p, 4, None, None, None) == _lib.BRC_ERR_NULL
    assert L.brc_scale_atoms(None, 4, 4, p, None) == _lib.BRC_ERR_NULL
    assert L.brc_int4_tiles(p, 16, 128, None, None, 0, p, p, None, None) == _lib.BRC_ERR_NULL
    # zero points and their tiles come together
    assert L.brc_int4_tiles(p, 16, 128, p, p, 0, p, p, None, None) == _lib.BRC_ERR_NULL
    # alignment
    assert L.brc_pack_nibbles_hi(p + 1, 4, p, None) == _lib.BRC_ERR_ALIGN
    assert L.brc_unpack_nibbles_hi(p + 8, 4, p, None, None) == _lib.BRC_ERR_ALIGN
    assert L.brc_scale_atoms(p, 4, 4, p + 2, None) == _lib.BRC_ERR_ALIGN
    # shapes the INT4 tile layout cannot hold, and scale dtypes it does not take
    assert L.brc_int4_tiles(p, 15, 128, p, None, 0, p, p, None, None) == _lib.BRC_ERR_UNSUPPORTED
    assert L.brc_int4_tiles(p, 16, 96, p, None, 0, p, p, None, None) == _lib.BRC_ERR_UNSUPPORTED
    assert L.brc_int4_tiles(p, 16, 128, p, None, 7, p, p, None, None) == _lib.BRC_ERR_DTYPE


def test_layout_entry_points_reject_bad_arguments():
    """breccia-orientation layout entry points (transposing dequantize, byte
    transpose): every rejection happens on the host, before any CUDA call."""
    L = _lib.lib()
    raw, p = _buf(256)
    F32, BF16, E4M3 = _lib.DTYPE_F32, _lib.DTYPE_BF16, _lib.FP8_E4M3
    MX, NV, I4, PT = _lib.STE_MXFP8, _lib.STE_NVFP4, _lib.STE_INT4, _lib.KIND_PERTENSOR_FP8
    S32 = _lib.SCALE_F32

    def dqt(codes=p, rows=8, cols=32, kind=MX, fmt=E4M3, block=32, signed=0, sdt=S32,
            scales=p, zp=None, out=p, odt=BF16):
        return L.brc_dequant_transposed(codes, rows, cols, kind, fmt, block, signed, sdt, scales,
                                        zp, out, odt, None)
    assert dqt(rows=-8) == _lib.BRC_ERR_SHAPE
    assert dqt(codes=None) == _lib.BRC_ERR_NULL
    assert dqt(scales=None) == _lib.BRC_ERR_NULL
    assert dqt(out=None) == _lib.BRC_ERR_NULL
    assert dqt(odt=9) == _lib.BRC_ERR_DTYPE
    assert dqt(fmt=5) == _lib.BRC_ERR_DTYPE
    assert dqt(kind=7) == _lib.BRC_ERR_UNSUPPORTED
    assert dqt(rows=12) == _lib.BRC_ERR_SHAPE            # rows % 8
    assert dqt(cols=48) == _lib.BRC_ERR_SHAPE            # cols % 32 for MXFP8
    assert dqt(kind=NV, cols=24) == _lib.BRC_ERR_SHAPE   # cols % 16
    assert dqt(kind=I4, block=40, cols=80) == _lib.BRC_ERR_SHAPE  # block % 16
    assert dqt(kind=I4, block=32, sdt=7) == _lib.BRC_ERR_DTYPE
    assert dqt(codes=None, scales=None, out=None, rows=0) == _lib.BRC_OK  # empty: no launch
    assert dqt(kind=PT, codes=p + 4) == _lib.BRC_ERR_ALIGN
    assert dqt(out=p + 2, odt=F32) == _lib.BRC_ERR_ALIGN

    assert L.brc_transpose_u8(p, -16, 16, p, None) == _lib.BRC_ERR_SHAPE
    assert L.brc_transpose_u8(p, 24, 16, p, None) == _lib.BRC_ERR_SHAPE   # rows % 16
    assert L.brc_transpose_u8(p, 16, 8, p, None) == _lib.BRC_ERR_SHAPE    # cols % 16
    assert L.brc_transpose_u8(None, 16, 16, p, None) == _lib.BRC_ERR_NULL
    assert L.brc_transpose_u8(p, 16, 16, None, None) == _lib.BRC_ERR_NULL
    assert L.brc_transpose_u8(None, 0, 16, None, None) == _lib.BRC_OK
    assert L.brc_transpose_u8(p + 8, 16, 16, p, None) == _lib.BRC_ERR_ALIGN
    del raw


def test_fused_cast_gemm_rejects_bad_arguments():
    """brc_cast_gemm_pertensor_fp8 / brc_cast_pertensor_fp8_delayed check
    everything on the host before the first CUDA call."""
    L = _lib.lib()
    _, p = _buf(4096)
    ws = L.brc_cast_gemm_workspace_bytes(256, 2048)
    assert ws == 16 + 4 * 1 * 2  # one 256-row block, two 1024-wide K chunks
    assert L.brc_cast_gemm_workspace_bytes(-1, 128) == -1

    def call(**kw):
        a = dict(x=p, x_dtype=_lib.DTYPE_BF16, a_fmt=_lib.FP8_E4M3, b=p, b_fmt=_lib.FP8_E4M3,
                 b_scale=p, M=256, N=256, K=2048, history=None, history_len=0, margin=0,
                 use_history=0, amax_in=None, a_codes=p, a_scale=p, d=p,
                 d_dtype=_lib.DTYPE_BF16, ws=p, ws_bytes=ws, prologue=-1)
        a.update(kw)
        return L.brc_cast_gemm_pertensor_fp8(
            a["x"], a["x_dtype"], a["a_fmt"], a["b"], a["b_fmt"], a["b_scale"], a["M"], a["N"],
            a["K"], a["history"], a["history_len"], a["margin"], a["use_history"], a["amax_in"],
            a["a_codes"], a["a_scale"], a["d"], a["d_dtype"], a["ws"], a["ws_bytes"],
            a["prologue"], None)

    assert call(a_codes=None) == _lib.BRC_ERR_NULL
    assert call(ws=None) == _lib.BRC_ERR_NULL
    assert call(b_scale=None) == _lib.BRC_ERR_NULL
    assert call(x_dtype=7) == _lib.BRC_ERR_DTYPE
    assert call(a_fmt=5) == _lib.BRC_ERR_DTYPE
    assert call(d_dtype=9) == _lib.BRC_ERR_DTYPE
    assert call(K=2000) == _lib.BRC_ERR_UNSUPPORTED     # K % 128
    assert call(N=250) == _lib.BRC_ERR_UNSUPPORTED      # N % 16
    assert call(x=p + 8) == _lib.BRC_ERR_ALIGN
    assert call(a_codes=p + 4) == _lib.BRC_ERR_ALIGN
    assert call(history=p, history_len=0) == _lib.BRC_ERR_SHAPE
    assert call(history=p, history_len=4, amax_in=p) == _lib.BRC_ERR_UNSUPPORTED
    assert call(margin=200) == _lib.BRC_ERR_RANGE
    assert call(ws_bytes=ws - 4) == _lib.BRC_ERR_SHAPE
    assert call(M=-1) == _lib.BRC_ERR_SHAPE
    # the delayed cast's own checks
    assert L.brc_cast_pertensor_fp8_delayed(p, 1, 64, 0, None, 4, 0, 1, p, p, p,
                                            None) == _lib.BRC_ERR_NULL
    assert L.brc_cast_pertensor_fp8_delayed(p, 1, 64, 0, p, 0, 0, 1, p, p, p,
                                            None) == _lib.BRC_ERR_SHAPE
    assert L.brc_cast_pertensor_fp8_delayed(p, 1, 64, 0, p, 4, -127, 1, p, p, p,
                                            None) == _lib.BRC_ERR_RANGE
    assert L.brc_cast_pertensor_fp8_delayed(p, 9, 64, 0, p, 4, 0, 1, p, p, p,
                                            None) == _lib.BRC_ERR_DTYPE
