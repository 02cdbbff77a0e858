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
    for modname in ("breccia.bridges", "breccia.bridges._huggingface"):
        m = types.ModuleType(modname)
        for fn in ("save_safetensors", "load_safetensors"):
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


def test_install_routes_bridges(fake_breccia, tmp_path):
    """Plain saves / loads keep breccia's bridge; CUDA tensors, pack_4bit and
    device= come here."""
    mods, calls = fake_breccia
    breccia_b200.install()
    for modname in ("breccia.bridges", "breccia.bridges._huggingface"):
        save, load = mods[modname].save_safetensors, mods[modname].load_safetensors
        assert getattr(save, "__breccia_b200__", False)
        cpu_st = breccia_b200.ScaledTensor(data=torch.zeros(2, 32, dtype=torch.uint8),
                                           scale=torch.ones(2, 2), recipe=breccia_b200.NVFP4BlockScaling(),
                                           layout=breccia_b200.PerBlockMN(1, 16))
        path = str(tmp_path / "x.safetensors")
        assert save({"w": cpu_st}, path) == f"{modname}.save_safetensors"
        assert load(path) == f"{modname}.load_safetensors"
        with pytest.raises(TypeError, match="CUDA"):  # ours: packing needs CUDA tensors
            save({"w": cpu_st}, path, pack_4bit=True)
        with pytest.raises(TypeError, match="CUDA device"):  # ours
            load(path, device="cpu")
    plugin.uninstall()
    assert not getattr(mods["breccia.bridges"].save_safetensors, "__breccia_b200__", False)


def test_cuda_check_without_gpu():
    assert not plugin._on_cuda(np.zeros(3))
    assert not plugin._on_cuda(torch.zeros(3))


def test_backend_rejects_cpu_tensors():
    with pytest.raises(TypeError, match="CUDA torch tensors"):
        breccia_b200.cast(torch.zeros(2, 32), breccia_b200.MXFP8BlockScaling())
    with pytest.raises(TypeError, match="CUDA torch tensors"):
        breccia_b200.cast(np.zeros((2, 32), np.float32), breccia_b200.Float8CurrentScaling())
