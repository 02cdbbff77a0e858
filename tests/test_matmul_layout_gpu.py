"""breccia's own matmul orientation on this library's kernels.

``matmul(a, b)`` takes ``b`` as ``(K, N)`` with its scale blocks along N
(src/breccia/kernels/reference/matmul.py:123-133; cast.py blocks the last
axis). Block-scaled MMAs need blocks along K, so such a ``b`` is dequantized
to bf16 by ``brc_dequant_transposed`` (written K-major) and multiplied by the
tcgen05 bf16 GEMM ``brc_gemm_bf16``; per-tensor codes move as bytes
(``brc_transpose_u8``) into the FP8 GEMM. Checked here:

* the transposing dequantize equals the oracle's dequantize, transposed, bit
  for bit (float32 output) and rounded once (bf16 output);
* the byte transpose and the bf16 GEMM on their own;
* ``matmul`` for every recipe (and mixed pairs) against the oracle's matmul,
  with torch's float32 matmul disabled, so the path under test is this
  library's. Tolerance: max|gpu - ref| / max|ref| <= 1e-2,
  cosine >= 0.9999; MXFP8 and NVFP4 values are exact in bf16, so those
  products are the reference's and the bound tightens to 1e-5 (float32 out).
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


def bb():
    import breccia_b200
    return breccia_b200


def _metrics(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    cos = float((got.ravel() @ ref.ravel()) / (np.linalg.norm(got) * np.linalg.norm(ref) + 1e-300))
    return rel, cos


def _check(got, ref, tight=None):
    rel, cos = _metrics(got, ref)
    assert rel <= 1e-2 and cos >= 0.9999, (rel, cos)
    if tight is not None:
        assert rel <= tight, rel


def _recipes():
    from breccia_b200.types import (Float8CurrentScaling, DelayedScaling, Float8BlockScaling,
                                    MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling)
    return {
        "current": Float8CurrentScaling(),
        "delayed_e5m2": DelayedScaling(fp8_format="E5M2"),
        "block128": Float8BlockScaling(block_k=128),
        "block32_e5m2": Float8BlockScaling(block_k=32, fp8_format="E5M2"),
        "mxfp8": MXFP8BlockScaling(),
        "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
        "nvfp4": NVFP4BlockScaling(),
        "int4_sym": INT4Scaling(group_size=128),
        "int4_asym_f32": INT4Scaling(group_size=64, signed=False, symmetric=False,
                                     scale_dtype="fp32"),
        "int4_asym_bf16": INT4Scaling(group_size=32, signed=False, symmetric=False,
                                      scale_dtype="bf16"),
    }


@pytest.fixture
def no_torch_fallback(monkeypatch):
    from breccia_b200 import gemm

    def refuse(*a, **k):
        raise AssertionError("torch float32 matmul fallback used")
    monkeypatch.setattr(gemm, "_general", refuse)


def _check_dequant_transposed(r, rows, cols, out, seed):
    from oracle import cast as ocast
    from breccia_b200 import _lib, gemm
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * 0.3
    x[3, :40] = 0.0
    x[7, 5] = 80.0
    st = bb().cast(x.cuda(), r)
    q = ocast.cast(x.numpy(), r)
    want = np.ascontiguousarray(ocast.dequantize(q).T)
    kind, fmt, block, signed, sdt = gemm._dq_kind(st)
    scale = st.scale.contiguous()
    if scale.dtype == torch.bfloat16:
        scale = scale.float()
        sdt = _lib.SCALE_F32
    zp = None if st.zero_point is None else st.zero_point.to(scale.dtype).contiguous()
    odt = torch.float32 if out == "f32" else torch.bfloat16
    got = torch.empty((cols, rows), dtype=odt, device="cuda")
    _lib.call("brc_dequant_transposed", st.data.view(torch.uint8).data_ptr(), rows, cols, kind,
              fmt, block, signed, sdt, scale.data_ptr(), None if zp is None else zp.data_ptr(),
              got.data_ptr(), _lib.DTYPE_F32 if out == "f32" else _lib.DTYPE_BF16,
              torch.cuda.current_stream().cuda_stream)
    g_np = got.float().cpu().numpy()
    if out == "f32":
        assert same_bits(np.nan_to_num(g_np, nan=1234.5), np.nan_to_num(want, nan=1234.5))
    else:
        ref_bf = torch.from_numpy(want).to(torch.bfloat16).float().numpy()
        assert same_bits(np.nan_to_num(g_np, nan=1234.5), np.nan_to_num(ref_bf, nan=1234.5))


@pytest.mark.parametrize("rname", list(_recipes()))
@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_dequant_transposed_vs_oracle(rname, out):
    _check_dequant_transposed(_recipes()[rname], 200, 384, out, len(rname))


@pytest.mark.parametrize("rname,rows,cols", [
    ("block48", 136, 480),    # 48-wide blocks straddle the 128-column tiles
    ("int4_g48", 264, 384),
    ("mxfp8", 392, 640),      # several tiles each way, a partial last row tile
    ("nvfp4", 8, 1040),
    ("pertensor", 520, 144),
])
def test_dequant_transposed_tiles(rname, rows, cols):
    from breccia_b200.types import (Float8CurrentScaling, Float8BlockScaling, MXFP8BlockScaling,
                                    NVFP4BlockScaling, INT4Scaling)
    r = {"block48": Float8BlockScaling(block_k=48),
         "int4_g48": INT4Scaling(group_size=48, signed=False, symmetric=False),
         "mxfp8": MXFP8BlockScaling(), "nvfp4": NVFP4BlockScaling(),
         "pertensor": Float8CurrentScaling()}[rname]
    for out in ("f32", "bf16"):
        _check_dequant_transposed(r, rows, cols, out, rows + cols)


def test_transpose_u8():
    from breccia_b200 import _lib
    g = torch.Generator().manual_seed(1)
    for rows, cols in ((16, 16), (272, 48), (1024, 4112)):
        x = torch.randint(0, 256, (rows, cols), generator=g, dtype=torch.uint8)
        xd = x.cuda()  # kept alive across the launch
        out = torch.empty((cols, rows), dtype=torch.uint8, device="cuda")
        _lib.call("brc_transpose_u8", xd.data_ptr(), rows, cols, out.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        assert torch.equal(out.cpu(), x.t().contiguous())


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 400, 520), (1, 16, 8),
                                   (2048, 2560, 4096), (4096, 4864, 1000)])
def test_gemm_bf16(M, N, K):
    """Single-CTA and CTA-pair paths, K not a multiple of the 64-element stage
    (the last stage reads zeros past the row end), one-row and one-tile cases."""
    from breccia_b200 import _lib
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, generator=g).to(torch.bfloat16)
    ad, bd = a.cuda(), b.cuda()  # kept alive across the launch
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    _lib.call("brc_gemm_bf16", ad.data_ptr(), bd.data_ptr(), M, N, K, out.data_ptr(),
              _lib.DTYPE_F32, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.lib().brc_gemm_status(1) == 0
    ref = a.double() @ b.double().t()
    _check(out.cpu().numpy(), ref.numpy(), tight=1e-5)


@pytest.mark.parametrize("rname", list(_recipes()))
@pytest.mark.parametrize("M,N,K", [(64, 256, 512), (300, 1152, 384)])
def test_matmul_reference_orientation(rname, M, N, K, no_torch_fallback):
    """matmul(cast(A), cast(W)) with W (K, N) blocked along N, as breccia
    callers write it, against the oracle's matmul of the same casts."""
    from oracle import cast as ocast
    r = _recipes()[rname]
    g = torch.Generator().manual_seed(M * 3 + N + K)
    A = torch.randn(M, K, generator=g)
    W = torch.randn(K, N, generator=g) * 0.02
    sa, sw = bb().cast(A.cuda(), r), bb().cast(W.cuda(), r)
    out = bb().matmul(sa, sw)
    assert out.dtype == torch.float32 and tuple(out.shape) == (M, N)
    ref = ocast.matmul(ocast.cast(A.numpy(), r), ocast.cast(W.numpy(), r))
    exact = rname.startswith(("mxfp8", "nvfp4"))
    _check(out.cpu().numpy(), ref, tight=1e-5 if exact else None)


@pytest.mark.parametrize("ra,rb", [("mxfp8", "nvfp4"), ("current", "mxfp8"),
                                   ("block128", "int4_sym"), ("nvfp4", "current")])
def test_matmul_mixed_recipes(ra, rb, no_torch_fallback):
    """Operands cast with different recipes (the reference dequantizes each
    with its own recipe), in both orientations."""
    from oracle import cast as ocast
    R = _recipes()
    g = torch.Generator().manual_seed(7)
    A = torch.randn(96, 256, generator=g)
    W = torch.randn(256, 512, generator=g) * 0.02
    sa, sw = bb().cast(A.cuda(), R[ra]), bb().cast(W.cuda(), R[rb])
    ref = ocast.matmul(ocast.cast(A.numpy(), R[ra]), ocast.cast(W.numpy(), R[rb]))
    _check(bb().matmul(sa, sw).cpu().numpy(), ref)
    swt = bb().cast(W.t().contiguous().cuda(), R[rb])
    ref_t = ocast.matmul(ocast.cast(A.numpy(), R[ra]),
                         ocast.dequantize(ocast.cast(np.ascontiguousarray(W.numpy().T), R[rb])).T)
    _check(bb().matmul(sa, swt, b_kmajor=True).cpu().numpy(), ref_t)


def test_matmul_raw_activations_int4_weight(no_torch_fallback):
    """Weight-only INT4 in breccia's orientation: raw bf16 activations x an
    INT4 (K, N) weight, more rows than the skinny GEMM takes."""
    from oracle import cast as ocast
    r = _recipes()["int4_asym_f32"]
    g = torch.Generator().manual_seed(8)
    A = torch.randn(64, 512, generator=g).to(torch.bfloat16)
    W = torch.randn(512, 256, generator=g) * 0.02
    sw = bb().cast(W.cuda(), r)
    ref = ocast.matmul(A.float().numpy(), ocast.cast(W.numpy(), r))
    _check(bb().matmul(A.cuda(), sw).cpu().numpy(), ref)


def test_b_kmajor_flag_takes_block_scaled_gemm(no_torch_fallback):
    from breccia_b200 import gemm
    from oracle import cast as ocast
    r = _recipes()["mxfp8"]
    g = torch.Generator().manual_seed(9)
    A = torch.randn(256, 1024, generator=g).to(torch.bfloat16)
    Wt = (torch.randn(512, 1024, generator=g) * 0.02).to(torch.bfloat16)
    sa, sw = bb().cast(A.cuda(), r), bb().cast(Wt.cuda(), r)
    assert gemm._tc_pair(sa, sw) == "mxfp8"
    out = bb().matmul(sa, sw, b_kmajor=True)
    ref = ocast.matmul(ocast.cast(A.float().numpy(), r),
                       ocast.dequantize(ocast.cast(Wt.float().numpy(), r)).T)
    _check(out.cpu().numpy(), ref, tight=1e-5)
