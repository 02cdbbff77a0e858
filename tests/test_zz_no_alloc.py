"""The allocation-free per-tensor cast gives the same result as the regular one.

brc_cast_pertensor_fp8_noalloc exists for callers that cannot allocate device
memory -- a host runtime that passes only its own input and output buffers,
or an op slot without a workspace argument -- so it keeps its scratch (the
per-chunk amax partials and the final amax) in a fixed array inside the
library instead of a caller-provided workspace. This test calls it through the
C ABI twice in a row and compares each result with brc_cast_pertensor_fp8 on
the same input. The second input is smaller and has a smaller amax than the
first, so stale scratch from the first call would change its scale. Codes and
scales must match bit for bit (the tolerance the cast tests use).

This file is named to be collected last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _input(rows, cols, seed, mag):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * mag
    x[torch.rand(rows, cols, generator=g) < 0.001] *= 50.0
    return x.to(torch.bfloat16).cuda()


_DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _cast(fn_name, x, lib, with_workspace, fmt=0):
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    stream = torch.cuda.current_stream().cuda_stream
    xp = x.data_ptr() if x.numel() else 0
    cp = codes.data_ptr() if x.numel() else 0
    if with_workspace:
        ws = torch.empty(1, dtype=torch.int32, device=x.device)
        rc = getattr(lib, fn_name)(xp, _DT[x.dtype], x.numel(), fmt, cp,
                                   scale.data_ptr(), ws.data_ptr(), stream)
    else:
        rc = getattr(lib, fn_name)(xp, _DT[x.dtype], x.numel(), fmt, cp,
                                   scale.data_ptr(), stream)
    assert rc == 0, lib.brc_status_string(rc)
    return codes, scale


def _same(x, lib, fmt=0):
    want_codes, want_scale = _cast("brc_cast_pertensor_fp8", x, lib, True, fmt)
    got_codes, got_scale = _cast("brc_cast_pertensor_fp8_noalloc", x, lib, False, fmt)
    torch.cuda.synchronize()
    assert got_scale.view(torch.int32).item() == want_scale.view(torch.int32).item()
    assert torch.equal(got_codes, want_codes)


def test_noalloc_matches_allocating_cast_twice():
    from breccia_b200 import _lib
    lib = _lib.lib()
    for rows, cols, seed, mag in ((4099, 4096, 1, 3.0), (1000, 512, 2, 0.25)):
        x = _input(rows, cols, seed, mag)
        want_codes, want_scale = _cast("brc_cast_pertensor_fp8", x, lib, True)
        got_codes, got_scale = _cast("brc_cast_pertensor_fp8_noalloc", x, lib, False)
        torch.cuda.synchronize()
        assert got_scale.view(torch.int32).item() == want_scale.view(torch.int32).item()
        assert torch.equal(got_codes, want_codes)


def test_noalloc_rejects_inputs_beyond_its_scratch():
    from breccia_b200 import _lib
    lib = _lib.lib()
    x = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(16, dtype=torch.uint8, device="cuda")
    scale = torch.empty((), dtype=torch.float32, device="cuda")
    too_big = 16384 * 32768 + 1  # checked before any launch or memory access
    rc = lib.brc_cast_pertensor_fp8_noalloc(x.data_ptr(), 1, too_big, 0, out.data_ptr(),
                                            scale.data_ptr(), ctypes.c_void_p(None))
    assert rc == _lib.BRC_ERR_RANGE


def test_noalloc_special_inputs():
    """Edge cases with their own handling in the scratch kernels, each
    compared bit for bit with the allocating cast: an empty input (no chunk
    runs; the final amax word is written as 0 and the 1e-10 floor gives the
    scale), a NaN (the per-chunk max propagates it, the reduction over float
    bits keeps it), an infinity, all zeros, and lengths that are not a
    multiple of the 16-byte vector (the last chunk takes the scalar loop),
    in all three input dtypes and both FP8 formats. Runs after a large call,
    so every slot read here was last written by another input."""
    from breccia_b200 import _lib
    lib = _lib.lib()
    _same(_input(2048, 4096, 7, 100.0), lib)  # leaves large partials behind
    _same(torch.empty(0, dtype=torch.bfloat16, device="cuda"), lib)
    for dt in (torch.float32, torch.bfloat16, torch.float16):
        for fmt in (0, 1):
            g = torch.Generator().manual_seed(11)
            base = torch.randn(3 * 32768 + 5, generator=g)
            _same(base.to(dt).cuda(), lib, fmt)  # ragged tail chunk
            x = base.clone()
            x[40000] = float("nan")
            _same(x.to(dt).cuda(), lib, fmt)
            x = base.clone()
            x[70001] = float("-inf")
            _same(x.to(dt).cuda(), lib, fmt)
            _same(torch.zeros(1000, dtype=dt, device="cuda"), lib, fmt)
            _same(base[:7].to(dt).cuda(), lib, fmt)  # shorter than one vector
