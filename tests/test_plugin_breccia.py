"""install() against the real breccia package (CPU; skipped where the
reference package is not available, e.g. on a GPU box).

breccia is pure Python and cannot travel with this repository, so this test
runs where the reference source tree is present, with the location taken
from BRECCIA_REFERENCE_SRC. It checks what the stand-in modules of
test_plugin.py cannot:

* every function install() rebinds exists in breccia's real modules and is
  rebound, and uninstall() restores the originals;
* NumPy and CPU torch inputs still take breccia's own path (same results as
  its original functions), including breccia.autograd.cast_ste, which calls
  the rebound module-level cast/dequantize;
* inputs on the GPU reach this backend with breccia's own recipe objects
  (a recording stand-in replaces the backend function: no GPU here);
* the results this backend builds are breccia.ScaledTensor objects with
  breccia's layouts: this backend's own cast code runs on CPU tensors with
  only the kernel launch stubbed, so breccia's __post_init__ and
  layout.validate check exactly the tensors the backend returns, and their
  shapes and dtypes match breccia's torch conventions.
"""

import contextlib
import importlib
import os

import numpy as np
import pytest
import torch

# the reference checkout next to this repository's, unless the variable names one
_BESIDE = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                       "reference", "src")
REFERENCE_SRC = os.environ.get("BRECCIA_REFERENCE_SRC", _BESIDE)


@pytest.fixture
def breccia_mod(monkeypatch):
    if not os.path.isdir(os.path.join(REFERENCE_SRC, "breccia")):
        pytest.skip("the reference breccia package is not available here")
    monkeypatch.syspath_prepend(REFERENCE_SRC)
    import breccia
    if not hasattr(breccia, "MXFP8BlockScaling"):
        pytest.skip("a stand-in breccia module is loaded")
    from breccia_b200 import plugin
    yield breccia
    plugin.uninstall()


def test_install_rebinds_every_site_and_uninstall_restores(breccia_mod):
    from breccia_b200 import plugin
    originals = {}
    for modname, names in plugin._SITES:
        mod = importlib.import_module(modname)
        for name in names:
            assert hasattr(mod, name), f"{modname}.{name} missing in breccia"
            originals[(modname, name)] = getattr(mod, name)
    plugin.install()
    for (modname, name), fn in originals.items():
        bound = getattr(importlib.import_module(modname), name)
        assert getattr(bound, "__breccia_b200__", False), (modname, name)
        assert bound.__wrapped__ is fn
    plugin.uninstall()
    for (modname, name), fn in originals.items():
        assert getattr(importlib.import_module(modname), name) is fn


def test_host_inputs_keep_breccias_path(breccia_mod):
    from breccia_b200 import plugin
    br = breccia_mod
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 64)).astype(np.float32)
    want = {r: br.cast(x, r) for r in (br.MXFP8BlockScaling(), br.Float8CurrentScaling())}
    want_mm = br.matmul(want[next(iter(want))], want[next(iter(want))].data.T.astype(np.float32))
    xt = torch.from_numpy(x)
    want_ste = br.cast_ste(xt, br.NVFP4BlockScaling())
    plugin.install()
    for r, w in want.items():
        got = br.cast(x, r)
        assert type(got) is br.ScaledTensor
        assert np.array_equal(np.asarray(got.data).view(np.uint8), np.asarray(w.data).view(np.uint8))
        assert np.array_equal(np.asarray(got.scale), np.asarray(w.scale))
    r0 = next(iter(want))
    got_mm = br.matmul(want[r0], want[r0].data.T.astype(np.float32))
    assert np.array_equal(np.asarray(got_mm), np.asarray(want_mm))
    got_ste = br.cast_ste(xt, br.NVFP4BlockScaling())  # CPU torch: breccia's autograd path
    assert torch.equal(got_ste, want_ste)


class _OnGpu:
    """Stands for a CUDA tensor in a host-only test."""
    shape = (4, 32)


def test_gpu_inputs_reach_the_backend_with_breccias_recipes(breccia_mod, monkeypatch):
    from breccia_b200 import api, autograd, plugin
    br = breccia_mod
    calls = []

    def recorder(name):
        def f(*args, **kwargs):
            calls.append((name, args, kwargs))
            return name
        return f

    for name in ("cast", "dequantize", "requantize", "matmul"):
        monkeypatch.setattr(api, name, recorder(name))
    for name in ("cast_ste", "cast_ste_clipped"):
        monkeypatch.setattr(autograd, name, recorder(name))
    monkeypatch.setattr(plugin, "_on_cuda", lambda obj: isinstance(obj, _OnGpu))
    plugin.install()
    x = _OnGpu()
    r = br.MXFP8BlockScaling()
    assert br.cast(x, r) == "cast"
    assert calls[-1][1][1] is r  # breccia's recipe object, passed through
    # the module breccia.kernels.reference.cast (its package re-exports a
    # function of the same name)
    assert importlib.import_module("breccia.kernels.reference.cast").cast(x, r) == "cast"
    assert br.dequantize(x) == "dequantize"
    assert br.requantize(x, br.NVFP4BlockScaling()) == "requantize"
    assert br.matmul(np.zeros((2, 2)), x) == "matmul"
    assert br.cast_ste(x, r) == "cast_ste"
    assert br.cast_ste_clipped(x, r) == "cast_ste_clipped"
    assert br.autograd.cast_ste(x, r) == "cast_ste"


def _stub_kernels(monkeypatch):
    """Run this backend's host code on CPU tensors: no kernel is launched,
    outputs keep their (uninitialised) contents."""
    from breccia_b200 import _lib, api
    monkeypatch.setattr(_lib, "call", lambda *a, **k: None)
    monkeypatch.setattr(api, "_require_cuda", lambda *a, **k: None)
    monkeypatch.setattr(api, "_stream", lambda dev: 0)
    monkeypatch.setattr(torch.cuda, "device", lambda dev: contextlib.nullcontext())


def test_backend_results_are_valid_breccia_scaled_tensors(breccia_mod, monkeypatch):
    import breccia_b200 as bb
    br = breccia_mod
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 64, 256)).astype(np.float32)
    recipes = [br.DelayedScaling(), br.Float8CurrentScaling(fp8_format="E5M2"),
               br.Float8BlockScaling(block_k=64), br.MXFP8BlockScaling(), br.NVFP4BlockScaling(),
               br.INT4Scaling(group_size=128), br.INT4Scaling(group_size=64, signed=False,
                                                              symmetric=False, scale_dtype="bf16")]
    want = {id(r): br.cast(x, r) for r in recipes}  # breccia's NumPy path, before stubbing
    want_t = {id(r): br.cast(torch.from_numpy(x), r) for r in recipes}  # its torch path
    _stub_kernels(monkeypatch)
    for r in recipes:
        st = bb.cast(torch.from_numpy(x), r)  # validated by breccia's own classes
        w, wt = want[id(r)], want_t[id(r)]
        assert type(st) is br.ScaledTensor and st.recipe is r
        assert type(st.layout) is type(w.layout) and st.layout == w.layout
        assert tuple(st.data.shape) == tuple(w.data.shape)
        assert tuple(st.scale.shape) == tuple(np.shape(w.scale))
        assert st.data.dtype == wt.data.dtype, (r, st.data.dtype, wt.data.dtype)
        assert st.scale.dtype == torch.from_numpy(np.asarray(w.scale)).dtype
        assert (st.zero_point is None) == (w.zero_point is None)
        deq = bb.dequantize(st)
        assert deq.dtype == torch.float32 and tuple(deq.shape) == x.shape
    st = bb.cast(torch.from_numpy(x[0]), br.Float8BlockScaling(block_k=128), block_m=64)
    assert type(st.layout) is br.PerBlockMN and st.layout == br.PerBlockMN(block_m=64, block_n=128)
