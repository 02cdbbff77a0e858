"""Generate golden vectors by running the reference implementation itself.

Usage::

    python tests/golden/make_golden.py <path-to-breccia-src>

``<path-to-breccia-src>`` is the ``src/`` directory of jvoltci/breccia v0.1.3
(it must contain the ``breccia`` package). The script imports the reference,
runs its NumPy path (``breccia.cast`` / ``dequantize`` / ``requantize`` /
``matmul`` and the ``_formats`` / ``_utils`` codecs) on seeded inputs chosen
to hit the numerically delicate cases (exact midpoints, subnormals,
saturation, zero blocks, NaN/inf, many E8M0 binades), and writes the inputs
and outputs to ``tests/golden/*.npz``. Nothing here is used at run time: the
tests read the ``.npz`` files only.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _f32_neighbours(v: np.ndarray, k: int) -> np.ndarray:
    """v and its k float32 neighbours on each side."""
    v = np.asarray(v, dtype=np.float32)
    out = [v]
    up, dn = v.copy(), v.copy()
    for _ in range(k):
        up = np.nextafter(up, np.float32(np.inf))
        dn = np.nextafter(dn, np.float32(-np.inf))
        out += [up, dn]
    return np.concatenate(out)


def _grid_probe(lut: np.ndarray) -> np.ndarray:
    finite = np.unique(lut[np.isfinite(lut)].astype(np.float64))
    mids = ((finite[1:] + finite[:-1]) / 2).astype(np.float32)
    return np.concatenate([_f32_neighbours(mids, 3), _f32_neighbours(finite.astype(np.float32), 2)])


def codec_golden(br):
    from breccia import _formats as F
    from breccia.kernels.reference import _utils as U

    rng = np.random.default_rng(1234)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, -np.nan, 1e30, -1e30,
                         1e-30, -1e-30, 1e-45, -1e-45, 3e-39, -3e-39], dtype=np.float32)
    randoms = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * s
        for s in (1e-4, 1e-2, 1.0, 10.0, 300.0, 5e4)])
    p8 = np.concatenate([_grid_probe(F._E4M3_LUT), specials, randoms])
    p5 = np.concatenate([_grid_probe(F._E5M2_LUT), specials, randoms])
    p2 = np.concatenate([_grid_probe(F._E2M1_LUT), specials, randoms / 50])
    pi = np.concatenate([
        _f32_neighbours(np.arange(-10, 17, dtype=np.float32) + np.float32(0.5), 2),
        np.arange(-10, 17, dtype=np.float32), rng.uniform(-12, 20, 2000).astype(np.float32)])

    # E8M0: the step point of every binade, found with the reference's own function
    ths = []
    e8_probe = [np.array([0.0, 1e-12, 1e-10, 9.9999e-11, 2.0 ** -34, 2.0 ** -33,
                          1e-5, 1.0, 3e38, np.inf, np.nan], dtype=np.float32)]
    centre = int(round((np.sqrt(2.0) - 1.0) * (1 << 23)))
    for k in range(-33, 128):
        base = np.array(np.float32(2.0 ** k)).view(np.uint32)
        m = np.arange(centre - (1 << 16), centre + (1 << 16), dtype=np.int64)
        vals = (np.uint32(base) + m.astype(np.uint32)).view(np.float32)
        codes = U.quantize_e8m0_scale(vals).astype(np.int32)
        i = int(np.nonzero(codes != codes[0])[0][0])
        ths.append(int(m[i]))
        e8_probe.append(vals[max(0, i - 4): i + 4])
        e8_probe.append(np.array([np.float32(2.0 ** k)], dtype=np.float32))
    e8_probe = np.concatenate(e8_probe).astype(np.float32)

    packed_src = np.array([0x0, 0x1, 0x2, 0x3, 0xF, 0xA, 0x5, 0x7], dtype=np.uint8)
    np.savez_compressed(
        os.path.join(HERE, "codec.npz"),
        e4m3_lut=F._E4M3_LUT, e5m2_lut=F._E5M2_LUT, e2m1_lut=F._E2M1_LUT,
        p_e4m3=p8, c_e4m3=F.encode_e4m3(p8),
        p_e5m2=p5, c_e5m2=F.encode_e5m2(p5),
        p_e2m1=p2, c_e2m1=F.encode_e2m1(p2),
        p_int4=pi, c_int4_s=F.encode_int4(pi, True), c_int4_u=F.encode_int4(pi, False),
        d_int4_s=F.decode_int4(np.arange(16, dtype=np.uint8), True),
        pack_src=packed_src, pack_out=F.pack_nibbles(packed_src),
        e8m0_thresholds=np.array(ths, dtype=np.int64),
        e8m0_probe=e8_probe, e8m0_codes=U.quantize_e8m0_scale(e8_probe),
        e8m0_decode=U.dequantize_e8m0_scale(np.arange(256, dtype=np.uint8)),
    )


def _bf16(x):
    """Round float32 values to bfloat16 (RNE) and return them as float32."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return (b.astype(np.uint32) << 16).view(np.float32)


def _inputs():
    rng = np.random.default_rng(20260101)
    X = {}
    a = rng.standard_normal((32, 256)).astype(np.float32)
    mask = rng.random(a.shape) < 0.01
    a[mask] = rng.standard_normal(mask.sum()).astype(np.float32) * 50
    X["gauss_outliers"] = a
    X["gauss_bf16"] = _bf16(rng.standard_normal((32, 256)).astype(np.float32))
    # many binades per row (E8M0 / E4M3-scale coverage), including tiny rows
    mag = (2.0 ** rng.integers(-45, 40, size=(32, 1))).astype(np.float32)
    X["binades"] = (rng.standard_normal((32, 256)) * mag).astype(np.float32)
    # rows of zeros, tiny values (below the 1e-10 amax floor), constants, heavy tails
    e = rng.standard_normal((32, 256)).astype(np.float32)
    e[0] = 0.0
    e[1] = 1e-12
    e[2, :128] = 0.0
    e[3] = 0.375
    e[4] = -2.0
    e[5] = rng.standard_t(4, 256).astype(np.float32) * 0.02
    e[6] = np.abs(e[6])
    e[7] = -np.abs(e[7])
    e[8] = 448.0 * (np.arange(256, dtype=np.float32) / 255.0)
    e[9, ::7] = 1e-30
    X["edges"] = e
    # exact E4M3 midpoints once divided by a block scale of 1.0 (amax 448)
    lut = np.unique(np.abs(_lut("e4m3")[np.isfinite(_lut("e4m3"))]))
    mids = ((lut[1:] + lut[:-1]) / 2).astype(np.float32)
    t = np.resize(np.concatenate([mids, -mids]), (32, 256)).astype(np.float32)
    t[:, ::128] = 448.0  # every 128-block has amax 448 -> scale exactly 1
    X["e4m3_ties"] = t
    # exact E2M1 midpoints for NVFP4: amax 6 -> scale 1.0 (E4M3 code of 1.0)
    m2 = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    t2 = np.resize(np.concatenate([m2, -m2, [6.0]]), (32, 256)).astype(np.float32)
    t2[:, ::16] = 6.0
    X["e2m1_ties"] = t2
    # INT4 ties: symmetric amax 7 -> scale 1; values k + 0.5
    t4 = np.resize(np.arange(-7, 7, dtype=np.float32) + 0.5, (32, 256)).astype(np.float32)
    t4[:, ::64] = 7.0
    X["int4_ties"] = t4
    X["nan_inf"] = rng.standard_normal((8, 256)).astype(np.float32)
    X["nan_inf"][1, 5] = np.nan
    X["nan_inf"][3, 200] = np.inf
    X["nan_inf"][5, 17] = -np.inf
    X["rank3"] = rng.standard_normal((2, 8, 128)).astype(np.float32)
    return X


_LUTS = {}


def _lut(name):
    return _LUTS[name]


def cast_golden(br):
    from breccia import _formats as F
    from breccia.recipes import (DelayedScaling, Float8CurrentScaling, Float8BlockScaling,
                                 MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling)

    X = _inputs()
    recipes = {
        "delayed_e4m3": DelayedScaling(fp8_format="E4M3"),
        "current_e4m3": Float8CurrentScaling(fp8_format="E4M3"),
        "current_e5m2": Float8CurrentScaling(fp8_format="E5M2"),
        "block128_e4m3": Float8BlockScaling(fp8_format="E4M3", block_k=128),
        "block64_e5m2": Float8BlockScaling(fp8_format="E5M2", block_k=64),
        "block32_e4m3": Float8BlockScaling(fp8_format="E4M3", block_k=32),
        "mxfp8_e4m3": MXFP8BlockScaling(fp8_format="E4M3"),
        "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
        "nvfp4": NVFP4BlockScaling(),
        "int4_sym_s_fp16_g128": INT4Scaling(group_size=128),
        "int4_sym_u_fp32_g64": INT4Scaling(group_size=64, signed=False, scale_dtype="fp32"),
        "int4_sym_s_bf16_g32": INT4Scaling(group_size=32, scale_dtype="bf16"),
        "int4_asym_fp16_g128": INT4Scaling(group_size=128, signed=False, symmetric=False),
        "int4_asym_fp32_g64": INT4Scaling(group_size=64, signed=False, symmetric=False,
                                          scale_dtype="fp32"),
    }
    inputs_for = {
        "int4_sym_s_fp16_g128": ["gauss_outliers", "gauss_bf16", "binades", "edges",
                                 "int4_ties", "rank3"],
        "int4_sym_u_fp32_g64": ["gauss_bf16", "edges", "binades"],
        "int4_sym_s_bf16_g32": ["gauss_bf16", "edges"],
        "int4_asym_fp16_g128": ["gauss_outliers", "gauss_bf16", "binades", "edges", "rank3"],
        "int4_asym_fp32_g64": ["gauss_bf16", "edges"],
        "nvfp4": ["gauss_outliers", "gauss_bf16", "binades", "edges", "e2m1_ties",
                  "nan_inf", "rank3"],
    }
    default_inputs = ["gauss_outliers", "gauss_bf16", "binades", "edges", "e4m3_ties",
                      "nan_inf", "rank3"]
    out = {}
    for rname, r in recipes.items():
        for iname in inputs_for.get(rname, default_inputs):
            x = X[iname]
            st = br.cast(x, r)
            key = f"{rname}__{iname}"
            out[key + "__x"] = x
            out[key + "__data"] = np.asarray(st.data)
            out[key + "__scale"] = np.asarray(st.scale)
            if st.zero_point is not None:
                out[key + "__zp"] = np.asarray(st.zero_point)
            with np.errstate(all="ignore"):
                out[key + "__deq"] = np.asarray(br.dequantize(st))
    np.savez_compressed(os.path.join(HERE, "casts.npz"), **out)


def requant_golden(br):
    from breccia.recipes import (Float8CurrentScaling, Float8BlockScaling, MXFP8BlockScaling,
                                 NVFP4BlockScaling, INT4Scaling)
    X = _inputs()
    pairs = {
        "nvfp4_to_mxfp8": (NVFP4BlockScaling(), MXFP8BlockScaling()),
        "mxfp8_to_nvfp4": (MXFP8BlockScaling(), NVFP4BlockScaling()),
        "block128_to_current": (Float8BlockScaling(block_k=128), Float8CurrentScaling()),
        "current_to_int4": (Float8CurrentScaling(), INT4Scaling(group_size=128)),
        "int4asym_to_block": (INT4Scaling(group_size=64, signed=False, symmetric=False),
                              Float8BlockScaling(block_k=64)),
    }
    out = {}
    for name, (r1, r2) in pairs.items():
        for iname in ("gauss_outliers", "binades", "edges"):
            x = X[iname]
            st2 = br.requantize(br.cast(x, r1), r2)
            key = f"{name}__{iname}"
            out[key + "__x"] = x
            out[key + "__data"] = np.asarray(st2.data)
            out[key + "__scale"] = np.asarray(st2.scale)
            if st2.zero_point is not None:
                out[key + "__zp"] = np.asarray(st2.zero_point)
    np.savez_compressed(os.path.join(HERE, "requant.npz"), **out)


def matmul_golden(br):
    from breccia.recipes import (Float8CurrentScaling, Float8BlockScaling, MXFP8BlockScaling,
                                 NVFP4BlockScaling, INT4Scaling)
    rng = np.random.default_rng(77)
    M, K, N = 64, 512, 256
    A = _bf16(rng.standard_normal((M, K)).astype(np.float32))
    W = _bf16((rng.standard_normal((K, N)) * 0.02).astype(np.float32))
    out = {"A": A, "W": W}
    cases = {
        "current": (Float8CurrentScaling(), Float8CurrentScaling()),
        "block128": (Float8BlockScaling(block_k=128), Float8BlockScaling(block_k=128)),
        "mxfp8": (MXFP8BlockScaling(), MXFP8BlockScaling()),
        "nvfp4": (NVFP4BlockScaling(), NVFP4BlockScaling()),
    }
    for name, (ra, rw) in cases.items():
        sa = br.cast(A, ra)
        # reference-layout B: cast W (K, N) directly (scales along N)
        out[f"{name}__kn"] = br.matmul(sa, br.cast(W, rw))
        # K-major B: cast W^T (N, K) (scales along K), dequantize, transpose back
        out[f"{name}__nk"] = br.matmul(sa, br.dequantize(br.cast(np.ascontiguousarray(W.T), rw)).T)
    # INT4 weight-only: raw activations x dequantized K-major INT4 weight
    for name, r in {"int4_asym": INT4Scaling(group_size=128, signed=False, symmetric=False),
                    "int4_sym": INT4Scaling(group_size=128)}.items():
        wq = br.cast(np.ascontiguousarray(W.T), r)
        out[f"{name}__nk"] = br.matmul(A, br.dequantize(wq).T)
    np.savez_compressed(os.path.join(HERE, "matmul.npz"), **out)


def main():
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    sys.path.insert(0, sys.argv[1])
    import breccia as br
    from breccia import _formats as F
    _LUTS["e4m3"] = F._E4M3_LUT
    print("reference breccia", br.__version__, "numpy", np.__version__)
    codec_golden(br)
    cast_golden(br)
    requant_golden(br)
    matmul_golden(br)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
