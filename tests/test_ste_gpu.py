"""cast_ste / cast_ste_clipped on the GPU: the fused forward equals the
reference's x + (dequantize(cast(x)) - x) in float32 bit for bit (NaN
positions), gradients are the identity / the clipped identity
(src/breccia/autograd.py:50-87, 124-190; the reference's
tests/test_autograd.py checks the same two properties)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _recipes():
    from breccia_b200.types import (Float8CurrentScaling, DelayedScaling, Float8BlockScaling,
                                    MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling)
    return {
        "current_e4m3": Float8CurrentScaling(),
        "delayed_e5m2": DelayedScaling(fp8_format="E5M2"),
        "block128": Float8BlockScaling(),
        "block32_e5m2": Float8BlockScaling(block_k=32, fp8_format="E5M2"),
        "mxfp8": MXFP8BlockScaling(),
        "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
        "nvfp4": NVFP4BlockScaling(),
        "int4_sym": INT4Scaling(group_size=128),
        "int4_sym_u_g64_f32": INT4Scaling(group_size=64, signed=False, scale_dtype="fp32"),
        "int4_asym": INT4Scaling(group_size=128, signed=False, symmetric=False),
        "int4_asym_g32_bf16": INT4Scaling(group_size=32, signed=False, symmetric=False,
                                          scale_dtype="bf16"),
        "block96_generic": Float8BlockScaling(block_k=96),
    }


def _oracle_ste(x32: np.ndarray, recipe) -> np.ndarray:
    from oracle import cast as ocast
    y = ocast.dequantize(ocast.cast(x32, recipe)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        return (x32 + (y - x32)).astype(np.float32)


def _same(got: np.ndarray, ref: np.ndarray):
    gn, rn = np.isnan(got), np.isnan(ref)
    np.testing.assert_array_equal(gn, rn)
    np.testing.assert_array_equal(got[~gn].view(np.uint32), ref[~rn].view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rname", list(_recipes()))
def test_ste_forward_vs_oracle(rname, dtype):
    from breccia_b200 import cast_ste
    r = _recipes()[rname]
    g = torch.Generator().manual_seed(hash(rname) % 1000)
    x = torch.randn(48, 384, generator=g) * torch.exp2(
        torch.randint(-8, 8, (48, 1), generator=g).float())
    x[3, 7] = float("nan")
    x[5, 100] = float("inf")
    x[7, :] = 0.0
    x[9, 0:96] *= 1e-30
    x = x.to(dtype)
    out = cast_ste(x.cuda(), r)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == x.shape
    _same(out.cpu().numpy(), _oracle_ste(x.float().numpy(), r))


def test_ste_full_size_rows():
    """C3-shaped activations (bf16 8192 x 8192, MXFP8), checked on sampled
    rows (the recipe is row-independent)."""
    from breccia_b200 import cast_ste
    from breccia_b200.types import MXFP8BlockScaling
    r = MXFP8BlockScaling()
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(8192, 8192, generator=g, device="cuda").to(torch.bfloat16)
    out = cast_ste(x, r)
    rows = np.arange(0, 8192, 331)
    _same(out[rows].cpu().numpy(), _oracle_ste(x[rows].float().cpu().numpy(), r))


def test_ste_gradient_is_identity():
    from breccia_b200 import cast_ste
    from breccia_b200.types import Float8CurrentScaling, NVFP4BlockScaling
    for r, dtype in ((Float8CurrentScaling(), torch.float32), (NVFP4BlockScaling(), torch.bfloat16)):
        x = torch.randn(4, 64, device="cuda").to(dtype).requires_grad_(True)
        y = cast_ste(x, r)
        (y * torch.arange(64, device="cuda")).sum().backward()
        assert x.grad.dtype == dtype
        torch.testing.assert_close(x.grad.float(),
                                   torch.arange(64, device="cuda").float().expand(4, 64))


def test_ste_clipped_gradient():
    from breccia_b200 import cast_ste, cast_ste_clipped
    from breccia_b200.types import Float8CurrentScaling, INT4Scaling
    x = (torch.randn(4, 64, device="cuda") * 20).requires_grad_(True)
    y = cast_ste_clipped(x, Float8CurrentScaling(), clip_min=-10, clip_max=10)
    y.sum().backward()
    inside = (x.detach() >= -10) & (x.detach() <= 10)
    torch.testing.assert_close(x.grad, inside.float())
    torch.testing.assert_close(y.detach(), cast_ste(x.detach(), Float8CurrentScaling()))
    # default bound: the format's saturation (INT4 unsigned: +-15)
    x2 = (torch.randn(2, 128, device="cuda") * 30).requires_grad_(True)
    cast_ste_clipped(x2, INT4Scaling(group_size=128, signed=False)).sum().backward()
    torch.testing.assert_close(x2.grad, (x2.detach().abs() <= 15).float())


def test_ste_float64_input_keeps_reference_dtype():
    """float64 inputs: y is float32 (dequantize), x + (y - x) promotes to
    float64 as in the reference's torch expression."""
    from breccia_b200 import cast_ste
    from breccia_b200.types import MXFP8BlockScaling
    x = torch.randn(8, 64, dtype=torch.float64, device="cuda")
    out = cast_ste(x, MXFP8BlockScaling())
    assert out.dtype == torch.float64
    ref = _oracle_ste(x.float().cpu().numpy(), MXFP8BlockScaling())
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-6, atol=0)
