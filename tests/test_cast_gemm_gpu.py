"""Fused activation cast + per-tensor FP8 GEMM (``cast_matmul``, extension)
against the unfused path and the oracle.

``cast_matmul(x, w, recipe)`` must return exactly what ``cast(x, recipe)``
followed by ``matmul(a, w)`` returns (``cast.py:64-92`` then
``matmul.py:42-133``): the activation codes and scale bit for bit (so the
oracle's codes, ``oracle/cast.py``), and the product bit for bit (the fused
kernel runs the same MMAs on the same codes in the same order). With an
AmaxHistory the scale, codes and history follow the restated DelayedScaling
oracle call after call.

Cases: rows cast by the in-kernel casters from the first row
(``prologue_rows=0``), by the cast kernel before the GEMM, or split between
them; ragged M, N and K (a K chunk shorter than 1024, a partial last row
block); float32 / bfloat16 / float16 activations; E4M3 and E5M2 on either
side; every output dtype; NaN and all-zero activations; weights in breccia's
``(K, N)`` orientation and in K-major form.
"""

import numpy as np
import pytest
import torch

from conftest import same_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _u8(t):
    return t.view(torch.uint8).cpu().numpy()


def _weight(N, K, fmt="E4M3", seed=1, kmajor=True):
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.05
    if not kmajor:
        w = w.T.contiguous()
    return bb.cast(w.cuda(), bb.Float8CurrentScaling(fp8_format=fmt))


def _check_against_unfused(x, w, recipe, out_dtype=torch.float32, kmajor=True, **kw):
    import breccia_b200 as bb
    kw.setdefault("fused", True)
    out, a = bb.cast_matmul(x, w, recipe, out_dtype=out_dtype, b_kmajor=kmajor, **kw)
    a_ref = bb.cast(x, recipe)
    out_ref = bb.matmul(a_ref, w, out_dtype, b_kmajor=kmajor)
    torch.cuda.synchronize()
    assert a.data.dtype == a_ref.data.dtype and tuple(a.data.shape) == tuple(x.shape)
    assert same_bits(_u8(a.data), _u8(a_ref.data))
    assert same_bits(np.atleast_1d(a.scale.cpu().numpy()), np.atleast_1d(a_ref.scale.cpu().numpy()))
    assert out.dtype == out_ref.dtype and out.shape == out_ref.shape
    assert torch.equal(out.view(torch.uint8) if out.dtype != torch.float32 else out.view(torch.int32),
                       out_ref.view(torch.uint8) if out.dtype != torch.float32
                       else out_ref.view(torch.int32))
    return out, a


@pytest.mark.parametrize("prologue_rows", [0, 256, 1024, -1])
def test_fused_equals_unfused_rows_split(prologue_rows):
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(7)
    M, N, K = 2304, 2560, 2048   # 9 row blocks, 2 K chunks
    x = (torch.randn(M, K, generator=g) * 3).to(torch.bfloat16).cuda()
    w = _weight(N, K)
    _check_against_unfused(x, w, bb.Float8CurrentScaling(), prologue_rows=prologue_rows)


@pytest.mark.parametrize("M,N,K", [(1000, 272, 1152), (300, 2048, 128), (2100, 512, 3200),
                                   (256, 16, 1024), (33, 4096, 896)])
def test_fused_ragged_shapes(M, N, K):
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(M + N + K)
    x = (torch.randn(M, K, generator=g) * 0.7).to(torch.bfloat16).cuda()
    w = _weight(N, K, seed=K)
    _check_against_unfused(x, w, bb.Float8CurrentScaling(), fused=True, prologue_rows=0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("afmt,wfmt", [("E4M3", "E4M3"), ("E5M2", "E4M3"), ("E4M3", "E5M2"),
                                       ("E5M2", "E5M2")])
def test_fused_dtypes_formats(dtype, afmt, wfmt):
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(3)
    M, N, K = 640, 768, 1280
    x = (torch.randn(M, K, generator=g) * 5).to(dtype).cuda()
    w = _weight(N, K, fmt=wfmt)
    _check_against_unfused(x, w, bb.Float8CurrentScaling(fp8_format=afmt), fused=True, prologue_rows=0)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fused_out_dtypes_and_orientation(out_dtype):
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(11)
    M, N, K = 512, 1024, 1024
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    _check_against_unfused(x, _weight(N, K), bb.Float8CurrentScaling(), out_dtype=out_dtype,
                           fused=True, prologue_rows=0)
    _check_against_unfused(x, _weight(N, K, kmajor=False), bb.Float8CurrentScaling(),
                           out_dtype=out_dtype, kmajor=False, fused=True, prologue_rows=0)


def test_fused_codes_match_oracle():
    import breccia_b200 as bb
    from oracle import cast as ocast
    g = torch.Generator().manual_seed(5)
    M, N, K = 384, 256, 1024
    x = torch.randn(M, K, generator=g) * 2
    x[3, 5] = 0.0
    x[7, 9] = -0.0
    x[10, :8] = 1e-12            # below every code: codes 0
    xb = x.to(torch.bfloat16)
    w = _weight(N, K)
    r = bb.Float8CurrentScaling()
    out, a = bb.cast_matmul(xb.cuda(), w, r, b_kmajor=True, fused=True, prologue_rows=0)
    q = ocast.cast_per_tensor_fp8(xb.float().numpy(), r)
    torch.cuda.synchronize()
    assert same_bits(_u8(a.data), q.data)
    assert same_bits(np.atleast_1d(a.scale.cpu().numpy()), np.atleast_1d(q.scale))
    # the product of the oracle's operands, float32-accumulated (1e-3 relative
    # to the output's scale: the accumulation order differs from float64)
    av = ocast.dequantize(q).astype(np.float64)
    wv = bb.dequantize(w).cpu().numpy().astype(np.float64)
    ref = av @ wv.T
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref).max()
    assert err <= 1e-3 * np.abs(ref).max()


def test_fused_special_values():
    import breccia_b200 as bb
    M, N, K = 512, 256, 1024
    w = _weight(N, K)
    r = bb.Float8CurrentScaling()
    zeros = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    _check_against_unfused(zeros, w, r, fused=True, prologue_rows=0)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    x[300, 17] = float("nan")    # current scaling: the scale becomes NaN
    out, a = bb.cast_matmul(x, w, r, b_kmajor=True, fused=True, prologue_rows=0)
    a_ref = bb.cast(x, r)
    torch.cuda.synchronize()
    assert same_bits(_u8(a.data), _u8(a_ref.data))
    assert torch.isnan(a.scale).item()
    x[300, 17] = float("inf")
    _, a = bb.cast_matmul(x, w, r, b_kmajor=True, fused=True, prologue_rows=0)
    assert same_bits(_u8(a.data), _u8(bb.cast(x, r).data))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("fmt,margin", [("E4M3", 0), ("E4M3", 1), ("E5M2", -2)])
def test_fused_history_sequence(dtype, fmt, margin):
    """Call after call the fused cast's codes, scale and history follow the
    restated DelayedScaling oracle; the first call is the current-amax cast."""
    import breccia_b200 as bb
    from oracle import cast as ocast
    r = bb.DelayedScaling(fp8_format=fmt, amax_history_len=3, margin=margin)
    g = torch.Generator().manual_seed(9 + margin)
    M, N, K = 1280, 512, 1024
    w = _weight(N, K)
    h, h2 = bb.AmaxHistory(3), bb.AmaxHistory(3)
    hist, recorded = np.zeros(3, np.float32), 0
    for mag in (2.0, 8.0, 0.25, 1.0, 30.0):
        x = (torch.randn(M, K, generator=g) * mag).to(dtype)
        if mag == 0.25:
            # encoded by the in-kernel casters with a finite scale (the NaN
            # code), then pushed: the following calls' scale is NaN
            x[1000, 3] = float("nan")
        out, a = bb.cast_matmul(x.cuda(), w, r, amax_history=h, b_kmajor=True, fused=True,
                                prologue_rows=256)
        a2 = bb.cast(x.cuda(), r, amax_history=h2)
        out2 = bb.matmul(a2, w, np.float32, b_kmajor=True)
        q, hist = ocast.cast_delayed_fp8(x.float().numpy(), r, hist, recorded)
        recorded += 1
        torch.cuda.synchronize()
        assert same_bits(_u8(a.data), q.data)
        assert same_bits(np.atleast_1d(a.scale.cpu().numpy()), np.atleast_1d(q.scale))
        assert same_bits(h.history.cpu().numpy(), hist)
        assert same_bits(h.history.cpu().numpy(), h2.history.cpu().numpy())
        assert torch.equal(out.view(torch.int32), out2.view(torch.int32))
    assert h.recorded == 5


def test_fused_falls_back_for_unsupported_shapes():
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(2)
    x = torch.randn(64, 200, generator=g).cuda()        # K % 128 != 0
    w = bb.cast(torch.randn(96, 200, generator=g).cuda(), bb.Float8CurrentScaling())
    out, a = bb.cast_matmul(x, w, bb.Float8CurrentScaling(), b_kmajor=True)
    a_ref = bb.cast(x, bb.Float8CurrentScaling())
    assert same_bits(_u8(a.data), _u8(a_ref.data))
    assert torch.equal(out, bb.matmul(a_ref, w, np.float32, b_kmajor=True))


def test_fused_large_many_units():
    """4096 x 4096 x 4096 with every row cast in the kernel: 16 row blocks x 4
    K chunks of ready counters, 512 cast units."""
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(13)
    M = N = K = 4096
    x = (torch.randn(M, K, generator=g) * 4).to(torch.bfloat16).cuda()
    w = _weight(N, K)
    _check_against_unfused(x, w, bb.Float8CurrentScaling(), out_dtype=torch.bfloat16,
                           fused=True, prologue_rows=0)


def test_fused_arguments():
    import breccia_b200 as bb
    w = _weight(256, 1024)
    x = torch.randn(256, 1024, device="cuda")
    with pytest.raises(ValueError):
        bb.cast_matmul(x, w, bb.Float8CurrentScaling(), amax_history=bb.AmaxHistory(4))
    with pytest.raises(ValueError):
        bb.cast_matmul(torch.randn(256, 512, device="cuda"), w, bb.Float8CurrentScaling(),
                       b_kmajor=True)


@pytest.mark.parametrize("M,N,K", [(4096, 1024, 4096), (2048, 256, 2048), (8192, 512, 1024)])
def test_fused_narrow_n(M, N, K):
    """Weight-split shapes (a rank's few output columns): the GEMM is short, so
    most of A is encoded while few tiles are left to overlap with."""
    import breccia_b200 as bb
    g = torch.Generator().manual_seed(M + N)
    x = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16).cuda()
    w = _weight(N, K)
    _check_against_unfused(x, w, bb.Float8CurrentScaling(), out_dtype=torch.bfloat16,
                           fused=True, prologue_rows=0)


def test_fused_with_reduced_amax():
    """An amax reduced elsewhere (another rank's larger values): the codes equal
    the apply pass with that amax word, the product the GEMM on those codes."""
    import breccia_b200 as bb
    from breccia_b200 import _lib
    from breccia_b200.api import _fused_cast_gemm
    g = torch.Generator().manual_seed(21)
    M, N, K = 1536, 1024, 2048
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = _weight(N, K)
    r = bb.Float8CurrentScaling()
    st = torch.cuda.current_stream().cuda_stream
    for amax in (float(x.float().abs().max()), 37.5):
        word = torch.tensor([np.float32(amax).view(np.int32)], dtype=torch.int32, device="cuda")
        out, a = _fused_cast_gemm(x, r, w.data.view(torch.uint8), w, N, torch.bfloat16, None,
                                  word, 0)
        codes = torch.empty(M, K, dtype=torch.uint8, device="cuda")
        scale = torch.empty((), dtype=torch.float32, device="cuda")
        _lib.call("brc_cast_pertensor_fp8_apply", x.data_ptr(), _lib.DTYPE_BF16, x.numel(),
                  _lib.FP8_E4M3, word.data_ptr(), codes.data_ptr(), scale.data_ptr(), st)
        torch.cuda.synchronize()
        assert torch.equal(a.data.view(torch.uint8), codes)
        assert same_bits(np.atleast_1d(a.scale.cpu().numpy()), np.atleast_1d(scale.cpu().numpy()))
        ref = bb.linear(bb.ScaledTensor(data=codes.view(torch.float8_e4m3fn), scale=scale,
                                        recipe=r, layout=bb.PerTensor()),
                        w, out_dtype=torch.bfloat16)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_fused_weight_split_single_rank():
    """cast_matmul_weight_split without a process group equals
    cast_weight_split followed by linear, bit for bit."""
    import breccia_b200 as bb
    from breccia_b200.dist import cast_matmul_weight_split, cast_weight_split
    g = torch.Generator().manual_seed(17)
    x = torch.randn(2048, 2048, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(768, 2048, generator=g) * 0.05).to(torch.bfloat16).cuda()
    r = bb.Float8CurrentScaling()
    out, sa, sw = cast_matmul_weight_split(x, w, r, fused=True)
    sa2, sw2 = cast_weight_split(x, w, r)
    out2 = bb.linear(sa2, sw2, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(sa.data.view(torch.uint8), sa2.data.view(torch.uint8))
    assert torch.equal(sw.data.view(torch.uint8), sw2.data.view(torch.uint8))
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
