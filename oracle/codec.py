"""CPU restatement of breccia's bit codecs (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module. The product path (``breccia_b200``) never does.

Every function restates the corresponding function of the reference
(jvoltci/breccia v0.1.3, ``src/breccia/_formats.py`` and
``src/breccia/kernels/reference/_utils.py``), citing ``file:line``.

Two encoders are provided for each float format:

* ``encode_*_lut`` follows the reference algorithm literally: an
  ``(n, lut_size)`` float32 distance matrix and ``argmin`` (first index wins),
  chunked so memory stays bounded (``_formats.py:117-130``). It is the
  faithful CPU baseline.
* ``encode_*`` is an equivalent O(n log 256) search over the same LUT with the
  same float32 distances and the same first-index tie rule. The test suite
  checks it against ``encode_*_lut`` and against golden vectors produced by the
  reference itself.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------- LUTs
# _formats.py:41-61 (E4M3 "FN": bias 7, no inf, NaN at 0x7F/0xFF)


def _e4m3_table() -> np.ndarray:
    out = np.zeros(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 3) & 0xF
        man = code & 0x7
        if exp == 15 and man == 7:
            out[code] = np.nan
        elif exp == 0:
            out[code] = sign * (man / 8.0) * 2.0 ** -6
        else:
            out[code] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return out


# _formats.py:64-79 (E5M2: IEEE-like, bias 15, inf at e=31 m=0, NaN otherwise)
def _e5m2_table() -> np.ndarray:
    out = np.zeros(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 2) & 0x1F
        man = code & 0x3
        if exp == 31:
            out[code] = np.nan if man else sign * np.inf
        elif exp == 0:
            out[code] = sign * (man / 4.0) * 2.0 ** -14
        else:
            out[code] = sign * (1.0 + man / 4.0) * 2.0 ** (exp - 15)
    return out


# _formats.py:82-99 (E2M1: bias 1, values {0, .5, 1, 1.5, 2, 3, 4, 6} and negatives)
def _e2m1_table() -> np.ndarray:
    out = np.zeros(16, dtype=np.float32)
    for code in range(16):
        sign = -1.0 if code & 0x8 else 1.0
        exp = (code >> 1) & 0x3
        man = code & 0x1
        if exp == 0:
            out[code] = sign * (man / 2.0)
        else:
            out[code] = sign * (1.0 + man / 2.0) * 2.0 ** (exp - 1)
    return out


E4M3_LUT = _e4m3_table()
E5M2_LUT = _e5m2_table()
E2M1_LUT = _e2m1_table()

# _formats.py:109-111
E4M3_MAX = 448.0
E5M2_MAX = 57344.0
E2M1_MAX = 6.0

E4M3_NAN_CODE = 0x7F  # _formats.py:145
E5M2_NAN_CODE = 0x7D  # _formats.py:159
E2M1_NAN_CODE = 0x00  # _formats.py:173

# ------------------------------------------------------- literal LUT encode


def encode_via_lut_literal(x: np.ndarray, lut: np.ndarray, lut_size: int,
                           chunk: int = 1 << 16) -> np.ndarray:
    """``_formats.py:117-130``: argmin of a float32 |x - lut| matrix, chunked."""
    flat = np.asarray(x, dtype=np.float32).ravel()
    finite = np.isfinite(lut[:lut_size])
    out = np.empty(flat.size, dtype=np.uint8)
    for lo in range(0, flat.size, chunk):
        part = flat[lo:lo + chunk]
        diffs = np.abs(part[:, None] - lut[None, :lut_size])
        diffs = np.where(finite[None, :], diffs, np.inf)
        out[lo:lo + chunk] = np.argmin(diffs, axis=1).astype(np.uint8)
    return out


# ------------------------------------------------------- fast equivalent


class _Nearest:
    """Nearest-LUT-entry search equal to ``argmin(|x - lut|)`` with ties to the
    lowest code, using the same float32 distances as the reference."""

    def __init__(self, lut: np.ndarray, lut_size: int):
        vals = lut[:lut_size]
        codes = np.arange(lut_size)
        keep = np.isfinite(vals)
        vals, codes = vals[keep], codes[keep]
        # one entry per distinct value, keeping the lowest code (e.g. +0 over -0)
        order = np.lexsort((codes, vals))
        vals, codes = vals[order], codes[order]
        first = np.ones(vals.size, dtype=bool)
        first[1:] = vals[1:] != vals[:-1]
        self.vals = vals[first].astype(np.float32)
        self.codes = codes[first].astype(np.int64)

    def __call__(self, v: np.ndarray) -> np.ndarray:
        v = np.asarray(v, dtype=np.float32)
        n = self.vals.size
        hi = np.searchsorted(self.vals, v, side="left")
        hi = np.clip(hi, 1, n - 1)
        lo = hi - 1
        d_lo = np.abs(v - self.vals[lo])  # float32, as _formats.py:125
        d_hi = np.abs(v - self.vals[hi])
        c_lo, c_hi = self.codes[lo], self.codes[hi]
        pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (c_hi < c_lo))
        return np.where(pick_hi, c_hi, c_lo).astype(np.uint8)


_NEAREST_E4M3 = _Nearest(E4M3_LUT, 256)
_NEAREST_E5M2 = _Nearest(E5M2_LUT, 256)
_NEAREST_E2M1 = _Nearest(E2M1_LUT, 16)


def _encode(x, fmt_max, nan_code, nearest, lut=None, lut_size=None, literal=False):
    x_arr = np.asarray(x, dtype=np.float32)
    is_nan = np.isnan(x_arr)
    sat = np.clip(x_arr, -fmt_max, fmt_max)
    if literal:
        codes = encode_via_lut_literal(sat, lut, lut_size).reshape(x_arr.shape)
    else:
        # NaN entries are overwritten below; feed 0 so the search is defined.
        codes = nearest(np.where(is_nan, np.float32(0), sat)).reshape(x_arr.shape)
    codes[is_nan] = nan_code
    return codes


def encode_e4m3(x, literal=False):
    """``_formats.py:133-146``: clip to +-448, nearest code, NaN -> 0x7F."""
    return _encode(x, E4M3_MAX, E4M3_NAN_CODE, _NEAREST_E4M3, E4M3_LUT, 256, literal)


def encode_e5m2(x, literal=False):
    """``_formats.py:149-160``: clip to +-57344, nearest code, NaN -> 0x7D."""
    return _encode(x, E5M2_MAX, E5M2_NAN_CODE, _NEAREST_E5M2, E5M2_LUT, 256, literal)


def encode_e2m1(x, literal=False):
    """``_formats.py:163-174``: clip to +-6, nearest code, NaN -> 0."""
    return _encode(x, E2M1_MAX, E2M1_NAN_CODE, _NEAREST_E2M1, E2M1_LUT, 16, literal)


def encode_int4(x, signed=True):
    """``_formats.py:177-189``: ``round(clip(x))`` (half to even), low nibble."""
    x_arr = np.asarray(x, dtype=np.float32)
    if signed:
        rounded = np.round(np.clip(x_arr, -8, 7)).astype(np.int8)
        return rounded.astype(np.uint8) & 0x0F
    rounded = np.round(np.clip(x_arr, 0, 15)).astype(np.uint8)
    return rounded & 0x0F


def decode_e4m3(b):
    """``_formats.py:195-197``."""
    return E4M3_LUT[np.asarray(b, dtype=np.uint8)]


def decode_e5m2(b):
    """``_formats.py:200-202``."""
    return E5M2_LUT[np.asarray(b, dtype=np.uint8)]


def decode_e2m1(b):
    """``_formats.py:205-207``: low nibble only."""
    return E2M1_LUT[np.asarray(b, dtype=np.uint8) & 0x0F]


def decode_int4(b, signed=True):
    """``_formats.py:210-221``: two's-complement low nibble when signed."""
    low = np.asarray(b, dtype=np.uint8) & 0x0F
    if signed:
        return np.where(low >= 8, low.astype(np.int16) - 16,
                        low.astype(np.int16)).astype(np.float32)
    return low.astype(np.float32)


def pack_nibbles(codes):
    """``_formats.py:227-243``: byte i = codes[2i] << 4 | codes[2i+1]."""
    flat = np.asarray(codes, dtype=np.uint8).ravel()
    if flat.size % 2 != 0:
        raise ValueError(
            f"pack_nibbles requires an even number of elements, got {flat.size}")
    return (((flat[0::2] & 0x0F) << 4) | (flat[1::2] & 0x0F)).astype(np.uint8)


def unpack_nibbles(packed, n_values):
    """``_formats.py:246-260``."""
    flat = np.asarray(packed, dtype=np.uint8).ravel()
    if n_values > 2 * flat.size:
        raise ValueError(
            f"unpack_nibbles: requested {n_values} values but buffer has "
            f"capacity for at most {2 * flat.size}")
    out = np.empty(2 * flat.size, dtype=np.uint8)
    out[0::2] = (flat >> 4) & 0x0F
    out[1::2] = flat & 0x0F
    return out[:n_values]


# ------------------------------------------------------------ amax / E8M0
AMAX_EPS = 1e-10  # _utils.py:8


def block_amax(x, block_size):
    """``_utils.py:11-31``: last-axis block abs-max, floored at float32(1e-10)."""
    K = x.shape[-1]
    if K % block_size != 0:
        raise ValueError(
            f"last-axis size {K} must be divisible by block_size {block_size}")
    reshaped = x.reshape(x.shape[:-1] + (K // block_size, block_size))
    amax = np.max(np.abs(reshaped), axis=-1)
    return np.maximum(amax, AMAX_EPS).astype(np.float32)


def tensor_amax(x) -> float:
    """``_utils.py:34-37``: whole-tensor abs-max as a Python float (float64)."""
    v = float(np.max(np.abs(x))) if x.size else 0.0
    return max(v, AMAX_EPS)


def quantize_e8m0_scale(scale_fp32):
    """``_utils.py:40-50``: ``round(log2(max(s, 1e-10)))`` + 127, clipped."""
    s = np.maximum(scale_fp32, AMAX_EPS)
    e_raw = np.round(np.log2(s)).astype(np.int32) + 127
    return np.clip(e_raw, 0, 255).astype(np.uint8)


def dequantize_e8m0_scale(scale_uint8):
    """``_utils.py:53-56``: ``2 ** (e - 127)`` in float32."""
    e = np.asarray(scale_uint8).astype(np.int32) - 127
    return np.float32(2.0) ** e.astype(np.float32)


def e8m0_thresholds(k_lo: int = -33, k_hi: int = 127, window: int = 1 << 16):
    """Per binade ``k`` (scale in ``[2^k, 2^(k+1))``), the first float32
    mantissa ``m`` at which :func:`quantize_e8m0_scale` steps from ``127+k`` to
    ``128+k``. Scans a window around the exact sqrt(2) point and checks that
    the code is a single monotone step inside it."""
    centre = int(round((np.sqrt(2.0) - 1.0) * (1 << 23)))
    out = []
    for k in range(k_lo, k_hi + 1):
        base = np.array(np.float32(2.0 ** k)).view(np.uint32)
        m = np.arange(centre - window, centre + window, dtype=np.int64)
        bits = (np.uint32(base) + m.astype(np.uint32)).astype(np.uint32)
        codes = quantize_e8m0_scale(bits.view(np.float32)).astype(np.int32)
        lo_code = 127 + k
        if k == k_lo:
            # values below 1e-10 floor to code 94; 2^-33 binade starts at 94
            lo_code = max(lo_code, 94)
        step = np.nonzero(codes != codes[0])[0]
        if codes[0] != lo_code or step.size == 0:
            raise RuntimeError(f"E8M0 binade {k}: no step inside the scan window")
        i = int(step[0])
        if not (np.all(codes[i:] == codes[0] + 1) and np.all(codes[:i] == codes[0])):
            raise RuntimeError(f"E8M0 binade {k}: code is not one monotone step")
        out.append(int(m[i]))
    return np.array(out, dtype=np.int64)
