"""safetensors bridge, host side (no GPU): the file format is the reference's.

``tests/golden/bridge_ref.safetensors`` was written by the reference's own
``save_safetensors`` (``src/breccia/bridges/_huggingface.py:118-151``; see
``tests/golden/make_bridge_golden.py``). Loading it must give the stored
tensors and the recipes / layouts it describes, and saving those objects again
must reproduce the reference's keys, dtypes, values and ``.config`` strings.
Mirrors the reference's tests/test_bridges.py HF cases.
"""

import json
import os

import numpy as np
import pytest
import torch

from safetensors import safe_open
from safetensors.torch import save_file

from breccia_b200 import bridges
import breccia_b200 as bb

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "bridge_ref.safetensors")
NAMES = ["current", "delayed_e5m2", "block", "mxfp8", "nvfp4", "int4_sym", "int4_asym",
         "int4_u_g64"]


def _raw(path):
    with safe_open(path, framework="pt") as f:
        return f.metadata(), {k: f.get_tensor(k) for k in f.keys()}


def test_load_reference_file():
    meta, raw = _raw(GOLDEN)
    out = bridges.load_safetensors(GOLDEN)
    assert sorted(out) == sorted(NAMES)
    for name, st in out.items():
        assert torch.equal(st.data, raw[f"{name}.data"])
        assert st.data.dtype == raw[f"{name}.data"].dtype
        assert torch.equal(st.scale, raw[f"{name}.scale"])
        if f"{name}.zero_point" in raw:
            assert torch.equal(st.zero_point, raw[f"{name}.zero_point"])
        else:
            assert st.zero_point is None
        cfg = json.loads(meta[f"{name}.config"])
        assert st.recipe.name == cfg["recipe"]["name"]
        assert st.layout.name == cfg["layout"]["name"]
        for k, v in cfg["recipe"]["fields"].items():
            assert getattr(st.recipe, k) == v
        for k, v in cfg["layout"]["fields"].items():
            assert getattr(st.layout, k) == v
    assert type(out["int4_asym"].recipe).__name__ == "INT4Scaling"
    assert out["int4_asym"].recipe.scale_dtype == "fp32"


def test_resave_matches_reference_file(tmp_path):
    meta, raw = _raw(GOLDEN)
    loaded = bridges.load_safetensors(GOLDEN)
    path = str(tmp_path / "again.safetensors")
    bridges.save_safetensors(loaded, path,
                             extra_metadata={"generator": meta["generator"]})
    meta2, raw2 = _raw(path)
    want = {k: v for k, v in raw.items() if not k.endswith(".packed_ref")}
    assert sorted(raw2) == sorted(want)
    for k, v in want.items():
        assert raw2[k].dtype == v.dtype and torch.equal(raw2[k], v), k
    assert meta2 == meta  # the .config strings are the reference's, byte for byte


def test_extra_metadata_and_skips(tmp_path):
    path = str(tmp_path / "mixed.safetensors")
    save_file({"foo.data": torch.zeros(4, dtype=torch.uint8)}, path, metadata=None)
    assert bridges.load_safetensors(path) == {}
    st = bridges.load_safetensors(GOLDEN)["current"]
    path2 = str(tmp_path / "md.safetensors")
    bridges.save_safetensors({"w": st}, path2, extra_metadata={"model_version": "v0.0.1"})
    meta, _ = _raw(path2)
    assert meta["model_version"] == "v0.0.1" and "w.config" in meta


def test_packed_needs_gpu(tmp_path):
    """Packing and unpacking run on the GPU: CPU tensors are refused, and a
    packed entry cannot be loaded with device=None."""
    st = bridges.load_safetensors(GOLDEN)["nvfp4"]
    with pytest.raises(TypeError, match="CUDA"):
        bridges.save_safetensors({"w": st}, str(tmp_path / "p.safetensors"), pack_4bit=True)
    meta, raw = _raw(GOLDEN)
    path = str(tmp_path / "packed.safetensors")
    save_file({"w.data_packed": raw["nvfp4.packed_ref"], "w.scale": raw["nvfp4.scale"]}, path,
              metadata={"w.config": meta["nvfp4.config"],
                        "w.packing": json.dumps({"format": "breccia_nibbles_high_first",
                                                 "shape": list(raw["nvfp4.data"].shape),
                                                 "dtype": "uint8"})})
    with pytest.raises(ValueError, match="device='cuda'"):
        bridges.load_safetensors(path)
    with pytest.raises(TypeError, match="CUDA device"):
        bridges.load_safetensors(path, device="cpu")


def test_golden_packing_is_breccias_order():
    """The golden packed bytes (the reference's pack_nibbles) against the
    oracle restatement, which the GPU kernels are tested against."""
    from oracle import codec
    _, raw = _raw(GOLDEN)
    for name in ("nvfp4", "int4_sym", "int4_asym", "int4_u_g64"):
        codes = raw[f"{name}.data"].numpy()
        np.testing.assert_array_equal(codec.pack_nibbles(codes), raw[f"{name}.packed_ref"].numpy())
        np.testing.assert_array_equal(codec.unpack_nibbles(raw[f"{name}.packed_ref"].numpy(),
                                                           codes.size), codes.ravel())


def test_module_exports():
    assert bb.bridges.save_safetensors is bridges.save_safetensors
    assert callable(bb.attach_gemm_operands)
