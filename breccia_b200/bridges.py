"""safetensors save / load of ``ScaledTensor`` objects, with an optional
packed 4-bit format and a GPU load path that leaves NVFP4, MXFP8 and INT4
tensors ready for the tensor-core GEMMs.

Reference: ``src/breccia/bridges/_huggingface.py:118-188`` (``save_safetensors``
/ ``load_safetensors``). The file layout is the reference's: for each name,
tensors ``{name}.data``, ``{name}.scale`` and (asymmetric INT4)
``{name}.zero_point``, and a JSON ``{name}.config`` metadata entry holding the
recipe and layout names and dataclass fields (``_huggingface.py:75-96``). Files
written with the default arguments are read by the reference's loader and
vice versa.

Extensions:

* ``save_safetensors(..., pack_4bit=True)`` stores NVFP4 and INT4 codes two
  per byte, in breccia's own nibble order (``_formats.py:227-243``:
  element 2i in the high nibble), as ``{name}.data_packed`` with a
  ``{name}.packing`` metadata entry (format, shape, dtype) instead of
  ``{name}.data``. A loader that does not know the entry skips it (the
  reference's requires ``.data``) rather than misreading it. Packing runs on
  the GPU (``brc_pack_nibbles_hi``), so it needs CUDA tensors.
* ``load_safetensors(path, device="cuda")`` reads the tensors onto the GPU,
  unpacks packed entries there (``brc_unpack_nibbles_hi``, which also
  writes the tensor-core nibble order), and rebuilds the GEMM side operands
  (``attach_gemm_operands``): the loaded tensors take the same tensor-core
  GEMM path as freshly cast ones. With ``device=None`` the tensors stay on
  the CPU exactly as stored, as in the reference.
"""

from __future__ import annotations

import dataclasses
import json
from typing import Any, Dict, Mapping, Optional

import torch

from . import _lib
from . import types as T
from .api import _aligned, _remember, _stream, attach_gemm_operands

__all__ = ["save_safetensors", "load_safetensors", "to_transformer_engine",
           "from_transformer_engine"]

_PACKED_FORMAT = "breccia_nibbles_high_first"
_FOUR_BIT = ("nvfp4", "int4")


def _require_safetensors():
    try:
        import safetensors  # noqa: F401
        return safetensors
    except ImportError as e:  # _huggingface.py:63-72
        raise ImportError(
            "safetensors is required for the HF bridge. "
            "Install with: pip install safetensors") from e


def _registries():
    """Recipe and layout classes by name: breccia's own when it is importable
    (so loaded tensors are breccia objects), else this package's mirrors."""
    try:
        import breccia
        mod = breccia
    except ImportError:
        mod = T
    recipes = {c.name: c for c in (mod.DelayedScaling, mod.Float8CurrentScaling,
                                   mod.Float8BlockScaling, mod.MXFP8BlockScaling,
                                   mod.NVFP4BlockScaling, mod.INT4Scaling)}
    layouts = {c.name: c for c in (mod.PerTensor, mod.PerBlockK, mod.PerChannel,
                                   mod.PerBlockMN)}
    return mod.ScaledTensor, recipes, layouts


def _fields(obj: Any):
    return dataclasses.fields(obj) if dataclasses.is_dataclass(obj) else []


def _config_to_json(recipe: Any, layout: Any) -> str:
    """``_huggingface.py:75-87``."""
    return json.dumps({
        "recipe": {"name": recipe.name,
                   "fields": {f.name: getattr(recipe, f.name) for f in _fields(recipe)}},
        "layout": {"name": layout.name,
                   "fields": {f.name: getattr(layout, f.name) for f in _fields(layout)}},
    })


def _json_to_config(s: str, recipes: dict, layouts: dict):
    """``_huggingface.py:90-96``."""
    obj = json.loads(s)
    recipe = recipes[obj["recipe"]["name"]](**obj["recipe"]["fields"])
    layout = layouts[obj["layout"]["name"]](**obj["layout"]["fields"])
    return recipe, layout


def _as_torch(arr: Any) -> torch.Tensor:
    """``_huggingface.py:107-115``: a contiguous torch tensor for safetensors."""
    if isinstance(arr, torch.Tensor):
        return arr.contiguous()
    import numpy as np
    return torch.as_tensor(np.asarray(arr)).contiguous()


def _pack(data: torch.Tensor, name: str) -> torch.Tensor:
    if not data.is_cuda:
        raise TypeError(f"pack_4bit packs on the GPU: {name}.data must be a CUDA tensor, "
                        f"got one on {data.device}")
    codes = _aligned(data.contiguous().view(torch.uint8))
    n = codes.numel()
    if n % 2:
        raise ValueError(f"pack_4bit requires an even number of codes, {name} has {n}")
    out = torch.empty(n // 2, dtype=torch.uint8, device=codes.device)
    with torch.cuda.device(codes.device):
        _lib.call("brc_pack_nibbles_hi", codes.data_ptr(), n, out.data_ptr(),
                  _stream(codes.device))
    return out


def save_safetensors(scaled_tensors: Mapping[str, Any], path: str,
                     extra_metadata: Optional[Dict[str, str]] = None, *,
                     pack_4bit: bool = False) -> None:
    """Save ``ScaledTensor`` objects to a safetensors file
    (``_huggingface.py:118-151``). ``pack_4bit``: store NVFP4 / INT4 codes two
    per byte (see the module docstring); CUDA tensors only."""
    _require_safetensors()
    from safetensors.torch import save_file

    tensors: Dict[str, torch.Tensor] = {}
    metadata: Dict[str, str] = dict(extra_metadata or {})
    for name, st in scaled_tensors.items():
        data = _as_torch(st.data)
        if pack_4bit and getattr(st.recipe, "name", None) in _FOUR_BIT:
            tensors[f"{name}.data_packed"] = _pack(data, name)
            metadata[f"{name}.packing"] = json.dumps(
                {"format": _PACKED_FORMAT, "shape": list(data.shape),
                 "dtype": str(data.dtype).replace("torch.", "")})
        else:
            tensors[f"{name}.data"] = data
        tensors[f"{name}.scale"] = _as_torch(st.scale)
        if st.zero_point is not None:
            tensors[f"{name}.zero_point"] = _as_torch(st.zero_point)
        metadata[f"{name}.config"] = _config_to_json(st.recipe, st.layout)
    # safetensors writes host memory: copy device tensors back first
    tensors = {k: v.cpu() for k, v in tensors.items()}
    save_file(tensors, path, metadata=metadata)


def _unpack(packed: torch.Tensor, info: dict, name: str):
    if info.get("format") != _PACKED_FORMAT:
        raise ValueError(f"{name}.packing: unknown format {info.get('format')!r}")
    shape = tuple(int(d) for d in info["shape"])
    n = 1
    for d in shape:
        n *= d
    if packed.numel() * 2 != n or n % 2:
        raise ValueError(f"{name}.data_packed holds {packed.numel()} bytes, "
                         f"not half of {n} codes")
    dev = packed.device
    src = _aligned(packed.contiguous().view(torch.uint8).reshape(-1))
    codes = torch.empty(shape, dtype=torch.uint8, device=dev)
    K = shape[-1] if shape else n
    lo = torch.empty(shape[:-1] + (K // 2,), dtype=torch.uint8, device=dev) \
        if K % 2 == 0 else None
    with torch.cuda.device(dev):
        _lib.call("brc_unpack_nibbles_hi", src.data_ptr(), n, codes.data_ptr(),
                  None if lo is None else lo.data_ptr(), _stream(dev))
    dtype = getattr(torch, info.get("dtype", "uint8"))
    return (codes if dtype == torch.uint8 else codes.view(dtype)), lo


def load_safetensors(path: str, *, device: Any = None) -> Dict[str, Any]:
    """Load ``ScaledTensor`` objects (``_huggingface.py:154-188``): every name
    with a ``.config`` entry and its tensors; other tensors are skipped.
    ``device`` (extension): a CUDA device to load onto, unpacking packed
    entries and attaching the tensor-core GEMM operands there."""
    _require_safetensors()
    from safetensors import safe_open

    dev = None if device is None else torch.device(device)
    if dev is not None and dev.type != "cuda":
        raise TypeError(f"device must be a CUDA device or None, got {dev}")
    if dev is not None and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    ST, recipes, layouts = _registries()
    with safe_open(path, framework="pt", device="cpu" if dev is None else str(dev)) as f:
        metadata = f.metadata() or {}
        keys = set(f.keys())
        out: Dict[str, Any] = {}
        for cfg_key in [k for k in metadata if k.endswith(".config")]:
            name = cfg_key[: -len(".config")]
            scale_key = f"{name}.scale"
            packed_key = f"{name}.data_packed"
            if scale_key not in keys:
                continue
            lo = None
            if f"{name}.data" in keys:
                data = f.get_tensor(f"{name}.data")
            elif packed_key in keys and f"{name}.packing" in metadata:
                if dev is None:
                    raise ValueError(
                        f"{name} is stored packed (two codes per byte); load it with "
                        f"device='cuda', which unpacks on the GPU")
                data, lo = _unpack(f.get_tensor(packed_key), json.loads(metadata[f"{name}.packing"]),
                                   name)
            else:
                continue
            recipe, layout = _json_to_config(metadata[cfg_key], recipes, layouts)
            zp_key = f"{name}.zero_point"
            st = ST(data=data, scale=f.get_tensor(scale_key), recipe=recipe, layout=layout,
                    zero_point=f.get_tensor(zp_key) if zp_key in keys else None)
            if dev is not None:
                if lo is not None and recipe.name == "nvfp4":
                    _remember(st.data, (st.scale, st.zero_point), packed=lo)
                attach_gemm_operands(st)
            out[name] = st
    return out


# ------------------------------------------------------------ TransformerEngine
# Reference: src/breccia/bridges/_transformer_engine.py:63-196. A TE
# Float8Tensor carries `_data` (uint8 FP8 bytes), `_scale_inv` (float32 of
# shape (1,), the dequantization scale -- breccia's ScaledTensor.scale) and
# `_fp8_dtype`. The per-tensor GPU outputs of this backend already have that
# form, so both directions share the buffers: no copy, no kernel. TE rounds
# ties to even in its own casts; codes made here round ties toward zero, as
# breccia's NumPy path does (the values they decode to are the same ones).

_TE_MODULES = ("transformer_engine.pytorch.tensor.float8_tensor",
               "transformer_engine.pytorch.tensor", "transformer_engine.pytorch.float8_tensor",
               "transformer_engine.pytorch")
_TE_DTYPE_MODULES = ("transformer_engine_torch", "transformer_engine.pytorch.cpp_extensions",
                     "transformer_engine.pytorch.tensor.float8_tensor", "transformer_engine.pytorch",
                     "transformer_engine.common.recipe")


def _te_attr(modules, attr):
    import importlib
    for name in modules:
        try:
            mod = importlib.import_module(name)
        except ImportError:
            continue
        if hasattr(mod, attr):
            return getattr(mod, attr)
    return None


def _require_te():
    try:
        import transformer_engine.pytorch  # noqa: F401
    except ImportError as e:  # the reference's message (_transformer_engine.py:41-52)
        raise ImportError("TransformerEngine is required for the TE bridge. Install with: "
                          "pip install transformer-engine (Linux + CUDA only)") from e


def to_transformer_engine(scaled):
    """Per-tensor FP8 ScaledTensor on the GPU -> TE ``Float8Tensor`` sharing
    its buffers (``_transformer_engine.py:91-196``): ``data`` viewed as
    uint8, the 0-d float32 scale viewed as shape (1,)."""
    _require_te()
    if getattr(scaled.recipe, "name", None) not in ("delayed", "current"):
        raise NotImplementedError(
            "to_transformer_engine supports DelayedScaling / Float8CurrentScaling only, got "
            f"{type(scaled.recipe).__name__}")
    data = scaled.data
    if not isinstance(data, torch.Tensor) or not data.is_cuda:
        raise TypeError("to_transformer_engine here takes CUDA tensors")
    if data.element_size() != 1:
        raise ValueError("to_transformer_engine requires 1-byte data dtype (uint8 or "
                         f"torch.float8_*), got {data.dtype}")
    Float8Tensor = _te_attr(_TE_MODULES, "Float8Tensor")
    DType = _te_attr(_TE_DTYPE_MODULES, "DType")
    if Float8Tensor is None or DType is None:
        raise RuntimeError("Could not locate TransformerEngine's Float8Tensor / DType")
    scale_inv = scaled.scale
    if scale_inv.dtype != torch.float32:
        scale_inv = scale_inv.to(torch.float32)
    fp8 = DType.kFloat8E4M3 if scaled.recipe.fp8_format == "E4M3" else DType.kFloat8E5M2
    return Float8Tensor(data=data.view(torch.uint8), fp8_scale_inv=scale_inv.reshape(1),
                        fp8_dtype=fp8)


def from_transformer_engine(te_tensor, recipe=None):
    """TE ``Float8Tensor`` -> ScaledTensor sharing ``_data`` and
    ``_scale_inv`` (``_transformer_engine.py:63-88``): the (1,)-shaped scale
    viewed as 0-d, recipe ``DelayedScaling`` with the TE dtype's format
    unless given."""
    _require_te()
    data = te_tensor._data
    scale = te_tensor._scale_inv
    if hasattr(scale, "squeeze") and scale.ndim == 1 and scale.shape[0] == 1:
        scale = scale.squeeze(0)
    if recipe is None:
        name = repr(getattr(te_tensor, "_fp8_dtype", "E4M3")).lower()
        if "e4m3" in name:
            fmt = "E4M3"
        elif "e5m2" in name:
            fmt = "E5M2"
        else:
            raise ValueError(f"unknown TE FP8 dtype: {te_tensor._fp8_dtype!r}")
        recipe = T.DelayedScaling(fp8_format=fmt)
    from .api import _classes
    ST, L = _classes(recipe)
    return ST(data=data, scale=scale, recipe=recipe, layout=L.PerTensor())
