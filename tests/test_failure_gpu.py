"""The GEMMs' failure path, exercised on the GPU without a fault.

Every wait in the tensor-core GEMMs is bounded: on a timeout the waiting role
records a sticky status bit, raises its CTA's abort flag, the other roles
leave their own waits on that flag, TMEM is freed and the kernel returns, so
the context stays usable. ``brc_selftest_wait_timeout`` runs that code in one
CTA against a barrier nothing arrives at (a short, bounded limit; no trap, no
bad address, no endless loop). This test checks the status it reports, that
the second role left on the abort flag rather than on its own 2 s bound, and
that a GEMM launched afterwards runs clean and correct.
"""

import ctypes
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_bounded_wait_times_out_and_context_survives():
    import breccia_b200 as bb
    from breccia_b200 import _lib
    from oracle import cast as ocast
    lib = _lib.lib()
    torch.cuda.synchronize()
    assert lib.brc_gemm_status(1) == 0  # nothing timed out before
    roles = ctypes.c_int(-1)
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = lib.brc_selftest_wait_timeout(1000, ctypes.byref(roles), stream)  # 1 ms bound
    elapsed = time.perf_counter() - t0
    assert rc == _lib.BRC_ERR_TIMEOUT, lib.brc_status_string(rc)
    assert roles.value == 3          # both roles left without the barrier completing
    assert elapsed < 1.0             # the 2 s role left on the abort flag
    assert lib.brc_gemm_status(1) == 1  # sticky bit 0, cleared here
    assert lib.brc_gemm_status(0) == 0
    assert lib.brc_selftest_wait_timeout(0, None, stream) == _lib.BRC_ERR_RANGE

    # the context is intact: a GEMM afterwards is clean and matches the oracle
    g = torch.Generator().manual_seed(9)
    A = torch.randn(256, 512, generator=g).to(torch.bfloat16)
    W = (torch.randn(512, 512, generator=g) * 0.02).to(torch.bfloat16)
    r = bb.MXFP8BlockScaling()
    out = bb.linear(bb.cast(A.cuda(), r), bb.cast(W.cuda(), r), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert lib.brc_gemm_status(0) == 0
    ref = ocast.matmul(ocast.cast(A.float().numpy(), r),
                       ocast.dequantize(ocast.cast(W.float().numpy(), r)).T)
    got = out.cpu().numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 1e-5
