"""install() rebinds breccia's public functions so CUDA inputs reach this
backend and everything else keeps breccia's own path. Exercised on stand-in
modules with breccia's module layout (no GPU, no reference needed)."""

import sys
import types

import numpy as np
import pytest
import torch

import breccia_b200
from breccia_b200 import plugin


@pytest.fixture
def fake_breccia(monkeypatch):
    calls = []

    def mk(name):
        def f(*a, **k):
            calls.append(name)
            return name
        return f

    mods = {}
    for modname in ("breccia", "breccia.kernels", "breccia.kernels.reference",
                    "breccia.kernels.reference.cast", "breccia.kernels.reference.matmul",
                    "breccia.autograd"):
        m = types.ModuleType(modname)
        for fn in ("cast", "dequantize", "requantize", "matmul"):
            setattr(m, fn, mk(f"{modname}.{fn}"))
        if modname in ("breccia", "breccia.autograd"):
            for fn in ("cast_ste", "cast_ste_clipped"):
                setattr(m, fn, mk(f"{modname}.{fn}"))
        mods[modname] = m
        monkeypatch.setitem(sys.modules, modname, m)
    yield mods, calls
    plugin.uninstall()


def test_install_routes_cpu_inputs_to_breccia(fake_breccia):
    mods, calls = fake_breccia
    breccia_b200.install()
    breccia_b200.install()  # idempotent
    x = np.zeros((2, 32), np.float32)
    assert mods["breccia"].cast(x, None) == "breccia.cast"
    assert mods["breccia.autograd"].dequantize(torch.zeros(2)) == "breccia.autograd.dequantize"
    assert mods["breccia"].matmul(x, x) == "breccia.matmul"
    assert getattr(mods["breccia"].cast, "__breccia_b200__", False)
    plugin.uninstall()
    assert not getattr(mods["breccia"].cast, "__breccia_b200__", False)
    assert mods["breccia"].cast(x, None) == "breccia.cast"


def test_install_rebinds_cast_ste(fake_breccia):
    mods, calls = fake_breccia
    breccia_b200.install()
    for modname in ("breccia", "breccia.autograd"):
        for fn in ("cast_ste", "cast_ste_clipped"):
            f = getattr(mods[modname], fn)
            assert getattr(f, "__breccia_b200__", False)
            # non-CUDA inputs keep breccia's own function
            assert f(np.zeros((2, 32), np.float32), None) == f"{modname}.{fn}"
    plugin.uninstall()
    assert mods["breccia"].cast_ste(np.zeros(1), None) == "breccia.cast_ste"


def test_cuda_check_without_gpu():
    assert not plugin._on_cuda(np.zeros(3))
    assert not plugin._on_cuda(torch.zeros(3))


def test_backend_rejects_cpu_tensors():
    with pytest.raises(TypeError, match="CUDA torch tensors"):
        breccia_b200.cast(torch.zeros(2, 32), breccia_b200.MXFP8BlockScaling())
    with pytest.raises(TypeError, match="CUDA torch tensors"):
        breccia_b200.cast(np.zeros((2, 32), np.float32), breccia_b200.Float8CurrentScaling())
