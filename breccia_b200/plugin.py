"""Install this backend behind the real ``breccia`` package.

breccia has no registry: its public functions are plain module attributes
(``src/breccia/__init__.py:23`` re-exports ``cast, dequantize, requantize,
matmul`` from ``breccia.kernels.reference`` and ``__init__.py:24``
``cast_ste, cast_ste_clipped`` from ``breccia.autograd``;
``breccia/autograd.py:47`` imports ``cast`` and ``dequantize`` by name; the
safetensors bridge is ``breccia.bridges.save_safetensors`` /
``load_safetensors``). ``install()`` rebinds each of those names to a wrapper
that sends CUDA torch inputs (and the bridge's ``pack_4bit`` / ``device``
extensions) to breccia_b200 and calls breccia's original function for
everything else (NumPy, CPU torch, JAX, MLX). ``uninstall()`` restores the
originals.
"""

from __future__ import annotations

import functools
import importlib

_SITES = [
    ("breccia", ("cast", "dequantize", "requantize", "matmul", "cast_ste", "cast_ste_clipped")),
    ("breccia.kernels.reference", ("cast", "dequantize", "requantize", "matmul")),
    ("breccia.kernels.reference.cast", ("cast", "dequantize", "requantize")),
    ("breccia.kernels.reference.matmul", ("dequantize",)),
    ("breccia.autograd", ("cast", "dequantize", "cast_ste", "cast_ste_clipped")),
    ("breccia.bridges", ("save_safetensors", "load_safetensors")),
    ("breccia.bridges._huggingface", ("save_safetensors", "load_safetensors")),
]
_saved: dict = {}


def _on_cuda(obj) -> bool:
    import torch
    if isinstance(obj, torch.Tensor):
        return obj.is_cuda
    data = getattr(obj, "data", None)
    return isinstance(data, torch.Tensor) and data.is_cuda and hasattr(obj, "recipe")


def _wrap(name, original):
    from . import api, autograd, bridges

    if name.endswith("_safetensors"):
        ours = getattr(bridges, name)
    else:
        ours = getattr(autograd if name.startswith("cast_ste") else api, name)

    @functools.wraps(original)
    def dispatch(*args, **kwargs):
        if name == "save_safetensors":
            # CUDA tensors and the packed format here; NumPy / CPU data on breccia's bridge
            tensors = args[0] if args else kwargs.get("scaled_tensors", {})
            if kwargs.get("pack_4bit") or any(_on_cuda(st) for st in dict(tensors).values()):
                return ours(*args, **kwargs)
            return original(*args, **kwargs)
        if name == "load_safetensors":
            # device= (loading onto the GPU) is this backend's; plain loads stay breccia's
            if kwargs.get("device") is not None:
                return ours(*args, **kwargs)
            return original(*args, **kwargs)
        if name == "matmul":
            a, b = args[0], args[1]
            if _on_cuda(a) or _on_cuda(b):
                return ours(*args, **kwargs)
        elif args and _on_cuda(args[0]):
            return ours(*args, **kwargs)
        return original(*args, **kwargs)

    dispatch.__breccia_b200__ = True
    return dispatch


def install() -> None:
    """Route breccia's cast/dequantize/requantize/matmul for CUDA tensors to
    this backend. Idempotent."""
    for modname, names in _SITES:
        try:
            mod = importlib.import_module(modname)
        except ImportError:
            if modname.startswith("breccia.bridges"):
                continue  # the bridges are optional in a stripped breccia install
            raise
        for name in names:
            fn = getattr(mod, name, None)
            if fn is None or getattr(fn, "__breccia_b200__", False):
                continue
            _saved[(modname, name)] = fn
            setattr(mod, name, _wrap(name, fn))


def uninstall() -> None:
    """Restore breccia's original functions."""
    for (modname, name), fn in list(_saved.items()):
        setattr(importlib.import_module(modname), name, fn)
        del _saved[(modname, name)]
