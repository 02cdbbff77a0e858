"""GPU parity of the cast / dequantize / requantize kernels with the
reference's NumPy path: bit-exact codes, scales and zero points, bit-exact
dequantized values (NaN positions must match; NaN payloads may differ).

Sources of truth: golden vectors produced by the reference itself
(tests/golden/), and the CPU oracle (oracle/, pinned to those vectors) for
random and full-size inputs. Full-size casts are checked on sampled rows:
every block recipe is row-independent, and the per-tensor recipe is
elementwise once its scale is known.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden, golden_recipes, golden_requant_pairs, golden_cases, same_bits

pytestmark = pytest.mark.gpu

CASTS = load_golden("casts.npz")
REQ = load_golden("requant.npz")


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def bb():
    import breccia_b200
    return breccia_b200


def _np(t):
    if t is None:
        return None
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        t = t.view(torch.uint8)
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.detach().cpu().numpy()


def assert_deq_equal(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn), "NaN positions differ"
    assert same_bits(np.where(gn, 0, got), np.where(wn, 0, want))


def assert_cast_equal(st, q, check_deq=True):
    assert same_bits(_np(st.data), q.data), _first_diff(_np(st.data), q.data)
    s = _np(st.scale)
    assert s.dtype == q.scale.dtype, (s.dtype, q.scale.dtype)
    assert same_bits(s, q.scale), _first_diff(s, q.scale)
    if q.zero_point is None:
        assert st.zero_point is None
    else:
        assert same_bits(_np(st.zero_point), q.zero_point)


def _first_diff(a, b):
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape:
        return f"shape {a.shape} vs {b.shape}"
    u = {1: np.uint8, 2: np.uint16, 4: np.uint32}[a.dtype.itemsize]
    idx = np.argwhere(a.view(u) != b.view(u))
    if not len(idx):
        return "equal"
    i = tuple(idx[0])
    return f"{len(idx)} differences; first at {i}: got {a[i]!r} want {b[i]!r}"


# ------------------------------------------------------------- golden cases


@pytest.mark.parametrize("case", golden_cases(CASTS), ids=lambda c: "__".join(c))
def test_golden_cast(case):
    rname, iname = case
    key = f"{rname}__{iname}"
    r = golden_recipes()[rname]
    x = torch.from_numpy(CASTS[key + "__x"]).cuda()
    st = bb().cast(x, r)
    assert st.recipe is r
    assert same_bits(_np(st.data), CASTS[key + "__data"]), \
        _first_diff(_np(st.data), CASTS[key + "__data"])
    assert same_bits(_np(st.scale), CASTS[key + "__scale"]), \
        _first_diff(_np(st.scale), CASTS[key + "__scale"])
    if key + "__zp" in CASTS:
        assert same_bits(_np(st.zero_point), CASTS[key + "__zp"])
    assert_deq_equal(_np(bb().dequantize(st)), CASTS[key + "__deq"])


@pytest.mark.parametrize("case", [c for c in golden_cases(CASTS) if c[1] == "gauss_bf16"],
                         ids=lambda c: "__".join(c))
def test_golden_cast_bf16_input(case):
    """bf16 inputs are read directly; their float32 values equal the golden x."""
    rname, iname = case
    key = f"{rname}__{iname}"
    x = torch.from_numpy(CASTS[key + "__x"]).cuda().to(torch.bfloat16)
    st = bb().cast(x, golden_recipes()[rname])
    assert same_bits(_np(st.data), CASTS[key + "__data"])
    assert same_bits(_np(st.scale), CASTS[key + "__scale"])


@pytest.mark.parametrize("case", golden_cases(REQ), ids=lambda c: "__".join(c))
def test_golden_requantize(case):
    pname, iname = case
    key = f"{pname}__{iname}"
    r1, r2 = golden_requant_pairs()[pname]
    x = torch.from_numpy(REQ[key + "__x"]).cuda()
    st = bb().requantize(bb().cast(x, r1), r2)
    assert same_bits(_np(st.data), REQ[key + "__data"]), _first_diff(_np(st.data), REQ[key + "__data"])
    assert same_bits(_np(st.scale), REQ[key + "__scale"])


# ------------------------------------------------------------- random inputs

def _recipes():
    from breccia_b200.types import (DelayedScaling, Float8CurrentScaling, Float8BlockScaling,
                                    MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling)
    return {
        "current_e4m3": Float8CurrentScaling(),
        "delayed_e5m2": DelayedScaling(fp8_format="E5M2"),
        "block128": Float8BlockScaling(block_k=128),
        "block64_e5m2": Float8BlockScaling(block_k=64, fp8_format="E5M2"),
        "block256": Float8BlockScaling(block_k=256),
        "block16": Float8BlockScaling(block_k=16),
        "block96_generic": Float8BlockScaling(block_k=96),
        "mxfp8": MXFP8BlockScaling(),
        "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
        "nvfp4": NVFP4BlockScaling(),
        "int4_sym": INT4Scaling(group_size=128),
        "int4_sym_u_g64": INT4Scaling(group_size=64, signed=False, scale_dtype="fp32"),
        "int4_asym": INT4Scaling(group_size=128, signed=False, symmetric=False),
        "int4_asym_g32_bf16scale": INT4Scaling(group_size=32, signed=False, symmetric=False,
                                               scale_dtype="bf16"),
        "int4_g48_generic": INT4Scaling(group_size=48),
    }


def _random_input(rows, cols, seed, spread=30):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g)
    # per-row magnitudes over many binades, some outliers, some exact zeros
    x *= torch.exp2(torch.randint(-spread, spread, (rows, 1), generator=g).float())
    mask = torch.rand(rows, cols, generator=g) < 0.002
    x[mask] *= 300.0
    x[torch.rand(rows, cols, generator=g) < 0.01] = 0.0
    return x


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rname", list(_recipes()))
def test_random_vs_oracle(rname, dtype):
    from oracle import cast as ocast
    r = _recipes()[rname]
    cols = 1152 if "generic" in rname else 1024
    seed = sum(map(ord, rname))
    if dtype == torch.float16:
        x = _random_input(192, cols, seed, spread=6).clamp(-6e4, 6e4)  # float16 range
    else:
        x = _random_input(192, cols, seed)
    xd = x.to(dtype)
    st = bb().cast(xd.cuda(), r)
    q = ocast.cast(xd.float().numpy(), r)
    assert_cast_equal(st, q)
    assert_deq_equal(_np(bb().dequantize(st)), ocast.dequantize(q))


def test_rank3_and_views():
    from oracle import cast as ocast
    from breccia_b200.types import MXFP8BlockScaling, Float8BlockScaling
    x = torch.randn(3, 40, 256)
    for r in (MXFP8BlockScaling(), Float8BlockScaling(block_k=128)):
        st = bb().cast(x.cuda(), r)
        assert tuple(st.scale.shape) == (3, 40, 256 // (32 if r.name == "mxfp8" else 128))
        assert_cast_equal(st, ocast.cast(x.numpy(), r))
    # a non-contiguous, offset view is copied to an aligned buffer first
    big = torch.randn(64, 300).cuda()
    view = big[3:, 12:268]
    st = bb().cast(view, MXFP8BlockScaling())
    assert_cast_equal(st, ocast.cast(view.cpu().numpy(), MXFP8BlockScaling()))


def test_empty_and_errors():
    from breccia_b200.types import (Float8CurrentScaling, Float8BlockScaling, MXFP8BlockScaling,
                                    INT4Scaling)
    st = bb().cast(torch.empty(0, 64).cuda(), MXFP8BlockScaling())
    assert tuple(st.data.shape) == (0, 64) and tuple(st.scale.shape) == (0, 2)
    st = bb().cast(torch.empty(0).cuda(), Float8CurrentScaling())
    # tensor_amax of an empty tensor is 0 -> floored to 1e-10 (float64)
    assert st.scale.item() == np.float32(1e-10 / 448.0)
    with pytest.raises(ValueError, match="K=100 must be divisible by block_k=128"):
        bb().cast(torch.zeros(2, 100).cuda(), Float8BlockScaling())
    with pytest.raises(ValueError, match="last-axis size 48 must be divisible by block_size 32"):
        bb().cast(torch.zeros(2, 48).cuda(), MXFP8BlockScaling())
    with pytest.raises(ValueError, match="requires x.ndim >= 2"):
        bb().cast(torch.zeros(64).cuda(), MXFP8BlockScaling())
    with pytest.raises(ValueError, match="K=64 must be divisible by group_size=128"):
        bb().cast(torch.zeros(2, 64).cuda(), INT4Scaling())


def test_float64_and_int_inputs_convert_like_numpy():
    from oracle import cast as ocast
    from breccia_b200.types import MXFP8BlockScaling
    x = torch.randn(8, 64, dtype=torch.float64) * 3
    st = bb().cast(x.cuda(), MXFP8BlockScaling())
    assert_cast_equal(st, ocast.cast(x.numpy().astype(np.float32), MXFP8BlockScaling()))


def test_packed_side_outputs():
    """Packed nibbles (element 2i low) and tcgen05-layout scales match the
    unpacked codes / reference-layout scales."""
    from breccia_b200.types import NVFP4BlockScaling, MXFP8BlockScaling
    x = torch.randn(256, 512).cuda()
    st = bb().cast(x, NVFP4BlockScaling())
    side = bb().gemm_operands(st)
    codes = st.data.cpu().numpy()
    packed = side["packed"].cpu().numpy()
    np.testing.assert_array_equal(packed & 0xF, codes[:, 0::2])
    np.testing.assert_array_equal(packed >> 4, codes[:, 1::2])
    for r, nsf in ((NVFP4BlockScaling(), 512 // 16), (MXFP8BlockScaling(), 512 // 32)):
        st = bb().cast(x, r)
        sf = st.scale.cpu().numpy()
        mma = bb().gemm_operands(st)["sf_mma"].cpu().numpy()
        rows = np.arange(256)[:, None]
        cols = np.arange(nsf)[None, :]
        off = ((rows // 128) * ((nsf + 3) // 4) + cols // 4) * 512 + (rows % 32) * 16 + \
            ((rows // 32) % 4) * 4 + cols % 4
        np.testing.assert_array_equal(mma[off], sf)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("block_m,rows,cols", [(128, 384, 640), (64, 192, 384), (32, 96, 256),
                                              (128, 128 * 20, 128 * 9)])
def test_block2d_vs_oracle(dtype, fmt, block_m, rows, cols):
    """128 x 128 (and 64 / 32 x 128) weight-tile cast, bit-exact against the
    restated oracle; one tile holds a NaN, one an inf, one is all zeros and
    one sits below the 1e-10 amax floor. The last shape has more tiles than
    SMs (the persistent form's grid-stride loop)."""
    from oracle import cast as ocast
    from breccia_b200.types import Float8BlockScaling
    r = Float8BlockScaling(fp8_format=fmt)
    g = torch.Generator().manual_seed(rows + cols + block_m)
    x = torch.randn(rows, cols, generator=g) * torch.exp2(torch.randint(-6, 6, (rows, 1),
                                                                         generator=g).float())
    x[1, 3] = float("nan")
    x[block_m + 2, 128 + 5] = float("inf")
    x[:block_m, 256:384] = 0.0
    x[block_m:2 * block_m, 0:128] *= 1e-30
    x = x.to(dtype)
    st = bb().cast(x.cuda(), r, block_m=block_m)
    torch.cuda.synchronize()
    q = ocast.cast_block_fp8_2d(x.float().numpy(), r, block_m=block_m)
    np.testing.assert_array_equal(st.data.view(torch.uint8).cpu().numpy(), q.data)
    assert same_bits(st.scale.cpu().numpy(), q.scale)


@pytest.mark.parametrize("symmetric", [False, True])
def test_int4_gemm_tile_layout(symmetric):
    """INT4 skinny-GEMM tiles: tile T = (r // 16) * (cols // 128) + g of 1 KB,
    row r % 16 at 64 * (r % 16); in each run of 8 elements 8j..8j+7 byte
    4j + i holds element 8j + i (low nibble) and 8j + i + 4 (high nibble);
    scale / 128 + zero point at T * 16 + 2 * (r % 8) + (r % 16) // 8."""
    from breccia_b200.types import INT4Scaling
    rows, cols = 48, 384
    r = INT4Scaling(group_size=128, signed=False, symmetric=symmetric)
    x = (torch.randn(rows, cols) * 0.02).cuda()
    st = bb().cast(x, r)
    side = bb().gemm_operands(st)
    codes = st.data.cpu().numpy().astype(np.uint8)
    groups = cols // 128
    rr, cc = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    g, e = cc // 128, cc % 128
    tile = (rr // 16) * groups + g
    byte = tile * 1024 + (rr % 16) * 64 + (e // 8) * 4 + (e % 4)
    high = (e % 8) >= 4
    tiles = side["int4_tiles"].cpu().numpy()
    got = np.where(high, tiles[byte] >> 4, tiles[byte] & 0xF)
    np.testing.assert_array_equal(got, codes)
    rrs, gs = np.meshgrid(np.arange(rows), np.arange(groups), indexing="ij")
    q = ((rrs // 16) * groups + gs) * 16 + 2 * (rrs % 8) + (rrs % 16) // 8
    np.testing.assert_array_equal(side["int4_scale_tiles"].cpu().numpy()[q],
                                  st.scale.float().cpu().numpy())
    if not symmetric:
        np.testing.assert_array_equal(side["int4_zp_tiles"].cpu().numpy()[q],
                                      128.0 + st.zero_point.float().cpu().numpy())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_nvfp4_quotients_near_midpoints(dtype):
    """NVFP4 blocks whose quotients x / s sit on and within a few ulps of every
    E2M1 midpoint, for non-power-of-two E4M3 scales (in about a third of them
    x * RN(1/s) differs from RN(x / s)): the codes must follow the IEEE
    quotient, as the oracle's division does, bit for bit."""
    from oracle import cast as ocast
    from breccia_b200.types import NVFP4BlockScaling
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    rows = []
    for k in range(-12, 7):
        for mant in (1.125, 1.25, 1.375, 1.625, 1.875, 1.0):
            s = np.float32(mant * 2.0 ** k)
            for d in range(-6, 7):
                # one element 6 s fixes the block scale at s; 15 elements near midpoints
                vals = [np.float32(6.0) * s]
                for i in range(15):
                    x = mids[i % 7] * s
                    x = np.float32(x)
                    step = np.inf if d > 0 else -np.inf
                    for _ in range(abs(d) + (i // 7)):
                        x = np.nextafter(x, np.float32(step))
                    vals.append(x if i % 2 == 0 else -x)
                rows.append(vals)
    x = np.array(rows, np.float32).reshape(-1, 48)  # 1482 blocks, three per row
    if dtype == torch.bfloat16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    r = NVFP4BlockScaling()
    st = bb().cast(torch.from_numpy(x).to(dtype).cuda(), r)
    q = ocast.cast(x, r)
    assert_cast_equal(st, q)


@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_requant_nvfp4_to_mxfp8_adversarial(fmt):
    """The fused NVFP4 -> MXFP8 requantize on hand-built NVFP4 tensors: random
    E2M1 codes under every finite E4M3 scale code (subnormals included), MXFP8
    blocks whose two NVFP4 halves have extreme scale ratios, all-zero blocks,
    zero scales, and NaN scales (the non-finite path). Codes and E8M0 scales
    bit-exact against the oracle's cast(dequantize(st))."""
    from oracle import cast as ocast
    from breccia_b200.types import NVFP4BlockScaling, MXFP8BlockScaling, PerBlockMN
    rng = np.random.default_rng(3 if fmt == "E4M3" else 4)
    rows, K = 512, 256
    codes = rng.integers(0, 16, (rows, K), dtype=np.uint8)
    sc = rng.integers(0, 0x7F, (rows, K // 16), dtype=np.uint8)  # finite E4M3 codes
    sc[0, :] = np.arange(K // 16, dtype=np.uint8) * 7              # a sweep of codes
    sc[1, 0::2], sc[1, 1::2] = 1, 0x7E                             # 2^-9 next to 448
    sc[2, 0::2], sc[2, 1::2] = 0x7E, 1
    sc[3, :] = 0                                                    # zero scales
    codes[4, :] = 0                                                 # all-zero codes
    codes[5, :] = 8                                                 # negative zeros
    sc[6, 3] = 0x7F                                                 # NaN scale
    sc[7, :] = np.arange(1, 1 + K // 16, dtype=np.uint8)            # subnormal scales
    r_src, r_dst = NVFP4BlockScaling(), MXFP8BlockScaling(fp8_format=fmt)
    st = bb().ScaledTensor(data=torch.from_numpy(codes).cuda(), scale=torch.from_numpy(sc).cuda(),
                           recipe=r_src, layout=PerBlockMN(block_m=1, block_n=16))
    got = bb().requantize(st, r_dst)
    q = ocast.Q(codes, sc, ("per_block_mn", 1, 16), r_src)
    want = ocast.cast(ocast.dequantize(q), r_dst)
    assert same_bits(_np(got.data), want.data), _first_diff(_np(got.data), want.data)
    assert same_bits(_np(got.scale), want.scale), _first_diff(_np(got.scale), want.scale)


def test_division_matches_ieee():
    from breccia_b200 import _lib
    g = torch.Generator().manual_seed(5)
    n = 1 << 24
    # quotients across 2^-40..2^40 with random scales over many binades
    x = torch.exp2(torch.empty(n).uniform_(-60, 60, generator=g)) * torch.sign(torch.randn(n, generator=g))
    s = torch.exp2(torch.empty(n).uniform_(-40, 40, generator=g))
    x, s = x.cuda(), s.cuda()
    qf, qi = torch.empty_like(x), torch.empty_like(x)
    _lib.call("brc_selftest_division", x.data_ptr(), s.data_ptr(), n, qf.data_ptr(),
              qi.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert torch.equal(qf.view(torch.int32), qi.view(torch.int32))
    assert torch.equal(qi, x / s)


# ------------------------------------------------------------- full sizes


def _sample_rows(n, k, seed=0):
    g = np.random.default_rng(seed)
    return np.sort(g.choice(n, size=min(k, n), replace=False))


def _config_inputs(name):
    """BASELINE.json configs, generated as seeded torch tensors on the CPU."""
    g = torch.Generator().manual_seed(0)
    if name == "c1_A":
        return torch.randn(2048, 7168, generator=g)
    if name == "c2_A":
        a = torch.randn(16384, 8192, generator=g)
        m = torch.rand(16384, 8192, generator=g) < 0.001
        a[m] = torch.randn(int(m.sum()), generator=g) * 50
        return a.to(torch.bfloat16)
    if name == "c1_Wt":
        torch.randn(2048, 7168, generator=g)  # A comes first in the config
        return torch.randn(4096, 7168, generator=g) * 0.02
    if name == "c2_Wt":
        return (torch.randn(8192, 8192, generator=g) * 0.02).to(torch.bfloat16)
    if name == "c3_A":
        return torch.randn(8192, 8192, generator=g).to(torch.bfloat16)
    if name == "c3_Wt":
        return (torch.randn(28672, 8192, generator=g) * 0.02).to(torch.bfloat16)
    if name == "c4_A":
        return torch.randn(4096, 8192, generator=g).to(torch.bfloat16)
    if name == "c4_Wt":
        w = torch.distributions.StudentT(4.0).sample((28672, 8192)) * 0.02
        return w.to(torch.bfloat16)
    if name == "c5_Wt":
        return torch.randn(28672, 8192, generator=g) * 0.02
    raise KeyError(name)


@pytest.mark.parametrize("cfg,rname", [
    ("c1_A", "block128"), ("c2_A", "current_e4m3"), ("c2_Wt", "current_e4m3"),
    ("c3_A", "mxfp8"), ("c3_Wt", "mxfp8"), ("c4_A", "nvfp4"), ("c4_Wt", "nvfp4"),
    ("c5_Wt", "int4_asym"),
])
def test_full_size_sampled_rows(cfg, rname):
    from oracle import cast as ocast, codec
    r = _recipes()[rname]
    x = _config_inputs(cfg)
    xd = x.cuda()
    st = bb().cast(xd, r)
    rows = _sample_rows(x.shape[0], 48)
    xs = x[rows].float().numpy()
    data = _np(st.data[rows])
    if rname == "current_e4m3":
        amax = float(x.float().abs().max())
        scale = np.float32(max(amax, 1e-10) / 448.0)
        assert _np(st.scale) == scale
        want = codec.encode_e4m3(xs / scale)
        assert same_bits(data, want), _first_diff(data, want)
        return
    q = ocast.cast(xs, r)
    assert same_bits(data, q.data), _first_diff(data, q.data)
    assert same_bits(_np(st.scale[rows]), q.scale)
    if q.zero_point is not None:
        assert same_bits(_np(st.zero_point[rows]), q.zero_point)


def test_full_size_block128x128_weight():
    """C1 W^T f32 (4096, 7168) with 128 x 128 tiles (the DeepSeek-v3 weight
    layout, restated oracle): sampled 128-row bands, codes and tile scales."""
    from oracle import cast as ocast
    r = _recipes()["block128"]
    x = _config_inputs("c1_Wt")
    st = bb().cast(x.cuda(), r, block_m=128)
    assert tuple(st.scale.shape) == (4096 // 128, 7168 // 128)
    for band in (0, 13, 31):
        xs = x[128 * band: 128 * (band + 1)].numpy()
        q = ocast.cast_block_fp8_2d(xs, r, block_m=128)
        data = _np(st.data[128 * band: 128 * (band + 1)])
        assert same_bits(data, q.data), _first_diff(data, q.data)
        assert same_bits(_np(st.scale[band: band + 1]), q.scale)
