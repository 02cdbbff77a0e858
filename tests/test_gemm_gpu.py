"""GPU parity of the tcgen05 scaled GEMMs with the reference's matmul
(dequantize both operands, float32 matmul: src/breccia/kernels/reference/
matmul.py:123-133).

Tolerance: max |gpu - ref| / max |ref| <= 1e-2 and
cosine similarity >= 0.9999. The operands are exactly representable, so the
only differences are float32 summation order and the output rounding; the
tests also check the much tighter bound that this implies for float32 output.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MIN_COS = 0.9999


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def bb():
    import breccia_b200
    return breccia_b200


def _metrics(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    cos = float((got.ravel() @ ref.ravel()) /
                (np.linalg.norm(got) * np.linalg.norm(ref) + 1e-300))
    return rel, cos


def _check(got, ref, tight=None):
    rel, cos = _metrics(got, ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    if tight is not None:
        assert rel <= tight, rel


def _recipe(kind):
    from breccia_b200.types import (Float8CurrentScaling, DelayedScaling, MXFP8BlockScaling,
                                    NVFP4BlockScaling)
    return {"current": Float8CurrentScaling(), "delayed_e5m2": DelayedScaling(fp8_format="E5M2"),
            "mxfp8": MXFP8BlockScaling(), "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
            "nvfp4": NVFP4BlockScaling()}[kind]


def _gemm_status():
    from breccia_b200 import _lib
    return _lib.lib().brc_gemm_status(1)


def _operands(M, N, K, seed, heavy=False):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    if heavy:
        W = (torch.distributions.StudentT(4.0).sample((N, K)) * 0.02).to(torch.bfloat16)
    else:
        W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    return A, W


@pytest.mark.parametrize("kind", ["current", "mxfp8", "nvfp4"])
def test_single_tile(kind):
    """Smallest case: one 128 x 256 tile, one or two K stages."""
    from oracle import cast as ocast
    r = _recipe(kind)
    K = 256
    A, W = _operands(128, 256, K, seed=1)
    sa, sw = bb().cast(A.cuda(), r), bb().cast(W.cuda(), r)
    out = bb().linear(sa, sw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _gemm_status() == 0
    qa, qw = ocast.cast(A.float().numpy(), r), ocast.cast(W.float().numpy(), r)
    ref = ocast.matmul(qa, ocast.dequantize(qw).T)
    _check(out.cpu().numpy(), ref, tight=1e-5)


@pytest.mark.parametrize("kind", ["current", "delayed_e5m2", "mxfp8", "mxfp8_e5m2", "nvfp4"])
@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (200, 384, 512), (1, 256, 512),
                                   (384, 1040, 768)])
def test_linear_vs_oracle(kind, M, N, K):
    from oracle import cast as ocast
    if kind == "nvfp4" and K % 256:
        pytest.skip("NVFP4 GEMM needs K % 256 == 0")
    r = _recipe(kind)
    A, W = _operands(M, N, K, seed=M + N + K, heavy=(kind == "nvfp4"))
    sa, sw = bb().cast(A.cuda(), r), bb().cast(W.cuda(), r)
    out = bb().linear(sa, sw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _gemm_status() == 0
    qa, qw = ocast.cast(A.float().numpy(), r), ocast.cast(W.float().numpy(), r)
    ref = ocast.matmul(qa, ocast.dequantize(qw).T)
    _check(out.cpu().numpy(), ref, tight=1e-5)


@pytest.mark.parametrize("kind", ["current", "delayed_e5m2", "mxfp8", "mxfp8_e5m2", "nvfp4"])
@pytest.mark.parametrize("M,N,K", [(2048, 2560, 512), (2000, 2576, 384), (4096, 4864, 256)])
def test_cta_pair_path(kind, M, N, K):
    """Shapes large enough for the CTA-pair GEMMs (256 x 256 tiles, at least
    one per SM pair): ragged M and N (scale atoms past the operand's end),
    several tiles per pair."""
    from oracle import cast as ocast
    if kind == "nvfp4" and K % 256:
        pytest.skip("NVFP4 GEMM needs K % 256 == 0")
    r = _recipe(kind)
    A, W = _operands(M, N, K, seed=M + N + K + 7, heavy=(kind == "nvfp4"))
    sa, sw = bb().cast(A.cuda(), r), bb().cast(W.cuda(), r)
    out = bb().linear(sa, sw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _gemm_status() == 0
    qa, qw = ocast.cast(A.float().numpy(), r), ocast.cast(W.float().numpy(), r)
    ref = ocast.matmul(qa, ocast.dequantize(qw).T)
    _check(out.cpu().numpy(), ref, tight=1e-5)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("kind", ["current", "mxfp8", "nvfp4"])
def test_output_dtypes(kind, out_dtype):
    from oracle import cast as ocast
    r = _recipe(kind)
    A, W = _operands(256, 512, 512, seed=3)
    out = bb().linear(bb().cast(A.cuda(), r), bb().cast(W.cuda(), r), out_dtype=out_dtype)
    assert out.dtype == out_dtype
    qa, qw = ocast.cast(A.float().numpy(), r), ocast.cast(W.float().numpy(), r)
    ref = ocast.matmul(qa, ocast.dequantize(qw).T)
    _check(out.float().cpu().numpy(), ref)


def test_tensor_core_path_is_taken():
    """The fast path must not silently fall back to the float32 reference
    semantics for the supported recipe pairs."""
    from breccia_b200 import gemm
    A, W = _operands(128, 256, 256, seed=4)
    for kind in ("current", "mxfp8", "nvfp4"):
        r = _recipe(kind)
        sa, sw = bb().cast(A.cuda(), r), bb().cast(W.cuda(), r)
        assert gemm._tc_pair(sa, sw) is not None, kind


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (256, 512, 1024), (200, 384, 768),
                                   (2048, 4096, 7168), (384, 512, 128), (1000, 1280, 384)])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_block_fp8_deepseek(M, N, K, fmt):
    """Float8BlockScaling: 1 x 128 activation scales, 128 x 128 weight scales
    (restated oracle for the weight layout; the reference cannot produce it).
    Includes a single K block (K = 128) and an odd number of K blocks, so the
    two partial buffers are used unevenly."""
    from oracle import cast as ocast
    from breccia_b200 import gemm
    from breccia_b200.types import Float8BlockScaling
    r = Float8BlockScaling(block_k=128, fp8_format=fmt)
    g = torch.Generator().manual_seed(M + K)
    A = torch.randn(M, K, generator=g)
    Wt = torch.randn(N, K, generator=g) * 0.02
    Wt[: min(N, 128), :128] *= 40.0  # one tile with a very different scale
    sa = bb().cast(A.cuda(), r)
    sw = bb().cast(Wt.cuda(), r, block_m=128)
    assert gemm._tc_pair(sa, sw) == "block"
    out = bb().linear(sa, sw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _gemm_status() == 0
    qa = ocast.cast(A.numpy(), r)
    qw = ocast.cast_block_fp8_2d(Wt.numpy(), r, block_m=128)
    ref = ocast.matmul(qa, ocast.dequantize(qw).T)
    _check(out.cpu().numpy(), ref, tight=1e-5)


def test_golden_matmul_kmajor():
    """Reference matmul outputs (tests/golden/matmul.npz, K-major weight)."""
    MM = load_golden("matmul.npz")
    A, W = MM["A"], MM["W"]  # (64, 512), (512, 256)
    for name in ("current", "mxfp8", "nvfp4"):
        r = _recipe(name)
        sa = bb().cast(torch.from_numpy(A).cuda(), r)
        sw = bb().cast(torch.from_numpy(np.ascontiguousarray(W.T)).cuda(), r)
        out = bb().linear(sa, sw, out_dtype=torch.float32).cpu().numpy()
        _check(out, MM[f"{name}__nk"], tight=1e-5)


def test_reference_semantics_matmul():
    """matmul(a, b) with b (K, N) as in the reference; per-tensor goes to the
    tensor cores, block recipes in the reference layout use float32."""
    import numpy as np
    MM = load_golden("matmul.npz")
    A, W = MM["A"], MM["W"]
    for name in ("current", "mxfp8", "nvfp4"):
        r = _recipe(name)
        sa = bb().cast(torch.from_numpy(A).cuda(), r)
        sb = bb().cast(torch.from_numpy(W).cuda(), r)
        out = bb().matmul(sa, sb)
        assert out.dtype == torch.float32
        _check(out.cpu().numpy(), MM[f"{name}__kn"], tight=1e-5)
    out = bb().matmul(bb().cast(torch.from_numpy(A).cuda(), _recipe("current")),
                      bb().cast(torch.from_numpy(W).cuda(), _recipe("current")),
                      out_dtype=np.float16)
    assert out.dtype == torch.float16


def test_shape_mismatch_raises():
    r = _recipe("current")
    a = bb().cast(torch.randn(4, 128).cuda(), r)
    b = bb().cast(torch.randn(64, 16).cuda(), r)
    with pytest.raises(ValueError, match="shape mismatch"):
        bb().matmul(a, b)


@pytest.mark.parametrize("M", [1, 4, 16, 11])
@pytest.mark.parametrize("variant", ["asym_fp16", "sym_signed_fp16", "sym_unsigned_fp32",
                                     "asym_bf16scale"])
def test_int4_weight_only(M, variant):
    """Raw bf16 activations x INT4 weight (group 128): the dequant-fused
    skinny GEMM against the reference's dequantize-then-float32 matmul."""
    from oracle import cast as ocast
    from breccia_b200 import gemm
    from breccia_b200.types import INT4Scaling
    r = {"asym_fp16": INT4Scaling(group_size=128, signed=False, symmetric=False),
         "sym_signed_fp16": INT4Scaling(group_size=128),
         "sym_unsigned_fp32": INT4Scaling(group_size=128, signed=False, scale_dtype="fp32"),
         "asym_bf16scale": INT4Scaling(group_size=128, signed=False, symmetric=False,
                                       scale_dtype="bf16")}[variant]
    N, K = 512, 2048
    g = torch.Generator().manual_seed(M)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Wt = torch.randn(N, K, generator=g) * 0.02
    if variant == "sym_unsigned_fp32":
        Wt = Wt.abs()
    sw = bb().cast(Wt.cuda(), r)
    assert gemm._int4_pair(A.cuda(), sw)
    out = bb().linear(A.cuda(), sw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    qw = ocast.cast(Wt.numpy(), r)
    ref = ocast.matmul(A.float().numpy(), ocast.dequantize(qw).T)
    _check(out.cpu().numpy(), ref, tight=1e-4)


@pytest.mark.parametrize("M,N,K", [(16, 16 * 149, 5120), (3, 16 * 300, 3072), (9, 16 * 7, 1024),
                                   (1, 16, 1024), (16, 16 * 2, 8192)])
def test_int4_weight_only_shapes(M, N, K):
    """Ragged work splits of the skinny GEMM: more row blocks than SMs, fewer
    row blocks than warps, one row block, activations streamed in an odd
    number of double-buffered chunks (M = 16, K = 5120), asymmetric g128."""
    from oracle import cast as ocast
    from breccia_b200.types import INT4Scaling
    r = INT4Scaling(group_size=128, signed=False, symmetric=False)
    g = torch.Generator().manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Wt = torch.randn(N, K, generator=g) * 0.02
    sw = bb().cast(Wt.cuda(), r)
    out = bb().linear(A.cuda(), sw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    qw = ocast.cast(Wt.numpy(), r)
    ref = ocast.matmul(A.float().numpy(), ocast.dequantize(qw).T)
    _check(out.cpu().numpy(), ref, tight=1e-4)


def test_int4_weight_only_config5_shape():
    """W^T (28672, 8192) f32 ~ N(0, 0.02), asymmetric g128,
    activations (16, 8192) bf16; checked on a column sample of the output."""
    from oracle import cast as ocast
    from breccia_b200.types import INT4Scaling
    r = INT4Scaling(group_size=128, signed=False, symmetric=False)
    g = torch.Generator().manual_seed(5)
    Wt = torch.randn(28672, 8192, generator=g) * 0.02
    A = torch.randn(16, 8192, generator=g).to(torch.bfloat16)
    sw = bb().cast(Wt.cuda(), r)
    out = bb().linear(A.cuda(), sw, out_dtype=torch.bfloat16).float().cpu().numpy()
    cols = np.arange(0, 28672, 97)
    qw = ocast.cast(Wt[cols].numpy(), r)
    ref = ocast.matmul(A.float().numpy(), ocast.dequantize(qw).T)
    _check(out[:, cols], ref)


# ------------------------------------------------ shapes the benchmark times
# The CTA-pair kernels stream K through a 5-7 stage shared-memory ring and a
# cluster walks several 256 x 256 tiles; these cases wrap the ring many times
# (K = 2048: 16 K blocks, K = 8192: 64) with several tiles per cluster, at
# the BASELINE config shapes themselves. The output is checked on a sample of
# rows and columns (the first and last, tile edges, random ones) against the
# reference's matmul of the oracle's casts of those rows.


def _pick(n, k, seed):
    g = np.random.default_rng(seed)
    edges = [i for i in (0, 127, 128, 255, 256, n // 2, n - 129, n - 128, n - 1) if 0 <= i < n]
    return np.unique(np.concatenate([edges, g.choice(n, size=min(k, n), replace=False)]))


def _oracle_sample(A, W, r, rows, cols):
    """Reference matmul of A[rows] @ W[cols]^T (W given as (N, K)). Block
    recipes are row-independent, so the sampled rows cast alone equal their
    rows of the full cast; per-tensor recipes encode them with the amax of
    the whole tensor (``cast.py:364-373``)."""
    from oracle import cast as ocast, codec
    a, w = A[rows].float().numpy(), W[cols].float().numpy()
    if r.name in ("delayed", "current"):
        qa = ocast.cast_per_tensor_fp8(a, r, amax=codec.tensor_amax(A.abs().max().float().numpy()))
        qw = ocast.cast_per_tensor_fp8(w, r, amax=codec.tensor_amax(W.abs().max().float().numpy()))
    else:
        qa, qw = ocast.cast(a, r), ocast.cast(w, r)
    return ocast.matmul(qa, ocast.dequantize(qw).T)


def _gemm_sampled(A, W, r, rows, cols, out_dtype=torch.bfloat16):
    from breccia_b200 import gemm
    sa, sw = bb().cast(A.cuda(), r), bb().cast(W.cuda(), r)
    assert gemm._tc_pair(sa, sw) is not None
    out = bb().linear(sa, sw, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert _gemm_status() == 0
    got = out[torch.as_tensor(rows).cuda()][:, torch.as_tensor(cols).cuda()].float().cpu().numpy()
    del sa, sw, out
    return got


@pytest.mark.parametrize("kind", ["current", "delayed_e5m2", "mxfp8", "mxfp8_e5m2", "nvfp4"])
@pytest.mark.parametrize("M,N,K", [(2048, 2560, 8192), (4096, 4864, 2048), (2304, 2320, 8192)])
def test_cta_pair_long_k(kind, M, N, K):
    """CTA-pair path (at least 74 tiles of 256 x 256) with 16 or 64 K blocks,
    ragged M and N, float32 output."""
    from breccia_b200 import _lib
    assert _lib.lib() is not None
    assert ((M + 255) // 256) * ((N + 255) // 256) >= torch.cuda.get_device_properties(
        0).multi_processor_count // 2
    r = _recipe(kind)
    A, W = _operands(M, N, K, seed=M + N + K + 11, heavy=(kind == "nvfp4"))
    rows, cols = _pick(M, 80, 1), _pick(N, 200, 2)
    got = _gemm_sampled(A, W, r, rows, cols, out_dtype=torch.float32)
    _check(got, _oracle_sample(A, W, r, rows, cols), tight=1e-5)


def _config_operands(cfg):
    """BASELINE.json configs[1..3] as seeded CPU tensors: A (M, K), W^T (N, K)."""
    g = torch.Generator().manual_seed(0)
    if cfg == "c2":
        A = torch.randn(16384, 8192, generator=g)
        m = torch.rand(16384, 8192, generator=g) < 0.001
        A[m] = torch.randn(int(m.sum()), generator=g) * 50
        W = torch.randn(8192, 8192, generator=g) * 0.02
        return A.to(torch.bfloat16), W.to(torch.bfloat16), "current"
    if cfg == "c3":
        A = torch.randn(8192, 8192, generator=g).to(torch.bfloat16)
        W = (torch.randn(28672, 8192, generator=g) * 0.02).to(torch.bfloat16)
        return A, W, "mxfp8"
    A = torch.randn(4096, 8192, generator=g).to(torch.bfloat16)
    torch.manual_seed(4)
    W = (torch.distributions.StudentT(4.0).sample((28672, 8192)) * 0.02).to(torch.bfloat16)
    return A, W, "nvfp4"


@pytest.mark.parametrize("cfg", ["c2", "c3", "c4"])
def test_config_shape_gemm(cfg):
    """The GEMMs bench.py times, at full size with bf16 output: C2 per-tensor
    E4M3 16384 x 8192 x 8192, C3 MXFP8 8192 x 28672 x 8192, C4 NVFP4
    4096 x 28672 x 8192 (Student-t weights)."""
    A, W, kind = _config_operands(cfg)
    r = _recipe(kind)
    rows, cols = _pick(A.shape[0], 64, 3), _pick(W.shape[0], 400, 4)
    got = _gemm_sampled(A, W, r, rows, cols)
    _check(got, _oracle_sample(A, W, r, rows, cols))


@pytest.mark.parametrize("kind", ["mxfp8", "nvfp4"])
def test_in_place_rewrite_of_operands(kind):
    """Codes and scales written into an existing ScaledTensor in place (a
    reused weight buffer) must reach the tensor-core GEMM: the packed codes
    and scale atoms recorded at cast time are stale then and are rebuilt."""
    from breccia_b200 import gemm
    r = _recipe(kind)
    A, W1 = _operands(256, 512, 512, seed=21)
    _, W2 = _operands(256, 512, 512, seed=22)
    sa = bb().cast(A.cuda(), r)
    sw = bb().cast(W1.cuda(), r)
    first = bb().linear(sa, sw, out_dtype=torch.float32)
    other = bb().cast(W2.cuda(), r)
    sw.data.copy_(other.data)
    sw.scale.copy_(other.scale)
    assert gemm._tc_pair(sa, sw) == kind
    got = bb().linear(sa, sw, out_dtype=torch.float32)
    want = bb().linear(sa, other, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert not torch.equal(got, first)
