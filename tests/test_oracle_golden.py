"""The CPU oracle, checked bit for bit against vectors produced by the
reference implementation itself (tests/golden/make_golden.py)."""

import numpy as np
import pytest

from conftest import load_golden, golden_recipes, golden_requant_pairs, golden_cases, same_bits
from oracle import codec, cast as ocast

CODEC = load_golden("codec.npz")
CASTS = load_golden("casts.npz")
REQ = load_golden("requant.npz")
MM = load_golden("matmul.npz")


def test_luts_match_reference():
    assert same_bits(codec.E4M3_LUT, CODEC["e4m3_lut"])
    assert same_bits(codec.E5M2_LUT, CODEC["e5m2_lut"])
    assert same_bits(codec.E2M1_LUT, CODEC["e2m1_lut"])


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m1"])
@pytest.mark.parametrize("literal", [False, True])
def test_float_encoders(fmt, literal):
    enc = getattr(codec, f"encode_{fmt}")
    p = CODEC[f"p_{fmt}"]
    with np.errstate(all="ignore"):
        got = enc(p, literal=literal)
    np.testing.assert_array_equal(got, CODEC[f"c_{fmt}"])


def test_int4_codec_and_nibbles():
    np.testing.assert_array_equal(codec.encode_int4(CODEC["p_int4"], True), CODEC["c_int4_s"])
    np.testing.assert_array_equal(codec.encode_int4(CODEC["p_int4"], False), CODEC["c_int4_u"])
    np.testing.assert_array_equal(codec.decode_int4(np.arange(16, dtype=np.uint8)),
                                  CODEC["d_int4_s"])
    np.testing.assert_array_equal(codec.pack_nibbles(CODEC["pack_src"]), CODEC["pack_out"])
    # tests/test_formats.py:209-219 of the reference pins these bytes
    np.testing.assert_array_equal(CODEC["pack_out"], [0x01, 0x23, 0xFA, 0x57])
    np.testing.assert_array_equal(codec.unpack_nibbles(CODEC["pack_out"], 8), CODEC["pack_src"])


def test_e8m0_codec():
    with np.errstate(all="ignore"):
        np.testing.assert_array_equal(codec.quantize_e8m0_scale(CODEC["e8m0_probe"]),
                                      CODEC["e8m0_codes"])
    assert same_bits(codec.dequantize_e8m0_scale(np.arange(256, dtype=np.uint8)),
                     CODEC["e8m0_decode"])


def test_e8m0_threshold_table():
    np.testing.assert_array_equal(codec.e8m0_thresholds(), CODEC["e8m0_thresholds"])


@pytest.mark.parametrize("case", golden_cases(CASTS), ids=lambda c: "__".join(c))
def test_cast_and_dequantize(case):
    rname, iname = case
    key = f"{rname}__{iname}"
    r = golden_recipes()[rname]
    with np.errstate(all="ignore"):
        q = ocast.cast(CASTS[key + "__x"], r)
        deq = ocast.dequantize(q)
    assert same_bits(q.data, CASTS[key + "__data"])
    assert q.scale.dtype == CASTS[key + "__scale"].dtype
    assert same_bits(q.scale, CASTS[key + "__scale"])
    if key + "__zp" in CASTS:
        assert same_bits(q.zero_point, CASTS[key + "__zp"])
    else:
        assert q.zero_point is None
    assert same_bits(deq, CASTS[key + "__deq"])


@pytest.mark.parametrize("case", golden_cases(REQ), ids=lambda c: "__".join(c))
def test_requantize(case):
    pname, iname = case
    key = f"{pname}__{iname}"
    r1, r2 = golden_requant_pairs()[pname]
    with np.errstate(all="ignore"):
        q = ocast.requantize(ocast.cast(REQ[key + "__x"], r1), r2)
    assert same_bits(q.data, REQ[key + "__data"])
    assert same_bits(q.scale, REQ[key + "__scale"])


def test_literal_cast_matches_fast_cast():
    r = golden_recipes()["mxfp8_e4m3"]
    x = CASTS["mxfp8_e4m3__binades__x"]
    a = ocast.cast(x, r, literal=False)
    b = ocast.cast(x, r, literal=True)
    assert same_bits(a.data, b.data) and same_bits(a.scale, b.scale)


def test_matmul_oracle_matches_reference():
    from breccia_b200.types import (Float8CurrentScaling, Float8BlockScaling,
                                    MXFP8BlockScaling, NVFP4BlockScaling)
    A, W = MM["A"], MM["W"]
    cases = {"current": Float8CurrentScaling(), "block128": Float8BlockScaling(block_k=128),
             "mxfp8": MXFP8BlockScaling(), "nvfp4": NVFP4BlockScaling()}
    for name, r in cases.items():
        qa = ocast.cast(A, r)
        kn = ocast.matmul(qa, ocast.cast(W, r))
        nk = ocast.matmul(qa, ocast.dequantize(ocast.cast(np.ascontiguousarray(W.T), r)).T)
        # same float32 operands; BLAS summation order may differ between runs
        np.testing.assert_allclose(kn, MM[f"{name}__kn"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(nk, MM[f"{name}__nk"], rtol=1e-5, atol=1e-5)
