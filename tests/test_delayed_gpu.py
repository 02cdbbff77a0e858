"""DelayedScaling with an amax history (extension) against the restated
oracle, bit for bit: codes, the scale used and the history after every call.

The reference keeps amax_history_len and margin on DelayedScaling
(src/breccia/recipes.py:43-77) but casts with the current amax
(cast.py:364-373). With an AmaxHistory the first cast is that reference cast
and records its amax; later casts take their scale from the history (max,
margin as a power of two) in one pass over the tensor and record the
tensor's own amax. Cases: growing and shrinking amaxes (saturation when the
tensor exceeds the history's range), margins, E5M2, float32 / bf16 / f16
inputs, ragged lengths, a NaN that reaches the history.
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


def _np(t):
    return t.view(torch.uint8).cpu().numpy() if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2) \
        else t.cpu().numpy()


def _run_sequence(recipe, xs, dtype, length=4):
    import breccia_b200 as bb
    from oracle import cast as ocast
    h = bb.AmaxHistory(length)
    hist, recorded = np.zeros(length, np.float32), 0
    for x in xs:
        xd = x.to(dtype)
        st = bb.cast(xd.cuda(), recipe, amax_history=h)
        q, hist = ocast.cast_delayed_fp8(xd.float().numpy(), recipe, hist, recorded)
        recorded += 1
        torch.cuda.synchronize()
        assert same_bits(_np(st.data), q.data)
        assert same_bits(np.atleast_1d(_np(st.scale)), np.atleast_1d(q.scale))
        assert same_bits(h.history.cpu().numpy(), hist), (h.history.cpu().numpy(), hist)
    assert h.recorded == len(xs)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fmt,margin", [("E4M3", 0), ("E4M3", 2), ("E5M2", 0), ("E4M3", -1)])
def test_history_sequence(dtype, fmt, margin):
    from breccia_b200.types import DelayedScaling
    r = DelayedScaling(fp8_format=fmt, amax_history_len=4, margin=margin)
    g = torch.Generator().manual_seed(len(fmt) + margin)
    mags = (3.0, 9.0, 0.5, 2.0, 40.0, 1.0)  # the ring wraps; growth saturates
    xs = [torch.randn(257, 515, generator=g) * m for m in mags]
    _run_sequence(r, xs, dtype)


def test_history_edge_cases():
    from breccia_b200.types import DelayedScaling
    r = DelayedScaling(amax_history_len=3)
    g = torch.Generator().manual_seed(1)
    zeros = torch.zeros(64, 64)
    tiny = torch.full((7,), 1e-12)           # below the 1e-10 floor
    ragged = torch.randn(3 * 1024 + 5, generator=g)
    _run_sequence(r, [zeros, tiny, ragged, torch.randn(8, 8, generator=g)], torch.float32, 3)
    nan = torch.randn(16, 32, generator=g)
    nan[3, 4] = float("nan")
    _run_sequence(r, [torch.randn(16, 32, generator=g), nan, torch.randn(16, 32, generator=g)],
                  torch.bfloat16, 3)


def test_history_argument_checks():
    import breccia_b200 as bb
    from breccia_b200.types import Float8CurrentScaling, DelayedScaling
    x = torch.randn(16, 32).cuda()
    with pytest.raises(ValueError, match="DelayedScaling only"):
        bb.cast(x, Float8CurrentScaling(), amax_history=bb.AmaxHistory(4))
    with pytest.raises(ValueError):
        bb.AmaxHistory(0)
    with pytest.raises(ValueError):
        bb.cast(x, DelayedScaling(margin=300), amax_history=bb.AmaxHistory(4))
