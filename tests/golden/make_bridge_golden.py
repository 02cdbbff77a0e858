"""Generate the safetensors golden file with the reference's own bridge.

Usage::

    python tests/golden/make_bridge_golden.py <path-to-breccia-src>

``<path-to-breccia-src>`` is the ``src/`` directory of jvoltci/breccia v0.1.3.
The script casts seeded inputs with the reference's NumPy path for every
recipe, saves them with the reference's ``breccia.bridges.save_safetensors``
(``src/breccia/bridges/_huggingface.py:118-151``) into
``tests/golden/bridge_ref.safetensors``, and also stores the reference's
``pack_nibbles`` of each 4-bit tensor (``_formats.py:227-243``) under
``{name}.packed_ref``. Nothing here runs at test time: the tests read the
file only.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(src: str) -> None:
    sys.path.insert(0, src)
    import breccia
    from breccia import _formats
    from breccia.bridges import save_safetensors
    from safetensors import safe_open
    from safetensors.torch import save_file
    import torch

    rng = np.random.default_rng(11)
    cases = {
        "current": (breccia.Float8CurrentScaling(), (16, 128)),
        "delayed_e5m2": (breccia.DelayedScaling(fp8_format="E5M2"), (8, 64)),
        "block": (breccia.Float8BlockScaling(block_k=128), (32, 256)),
        "mxfp8": (breccia.MXFP8BlockScaling(), (130, 96)),
        "nvfp4": (breccia.NVFP4BlockScaling(), (48, 512)),
        "int4_sym": (breccia.INT4Scaling(group_size=128), (32, 256)),
        "int4_asym": (breccia.INT4Scaling(group_size=128, signed=False, symmetric=False,
                                          scale_dtype="fp32"), (48, 384)),
        "int4_u_g64": (breccia.INT4Scaling(group_size=64, signed=False), (16, 128)),
    }
    sts = {}
    for name, (recipe, shape) in cases.items():
        x = (rng.standard_normal(shape) * np.exp2(rng.integers(-6, 6, (shape[0], 1)))).astype(
            np.float32)
        sts[name] = breccia.cast(x, recipe)
    path = os.path.join(HERE, "bridge_ref.safetensors")
    save_safetensors(sts, path, extra_metadata={"generator": "breccia v0.1.3 save_safetensors"})
    # add the reference's nibble packing of the 4-bit tensors, keeping the file's metadata
    with safe_open(path, framework="pt") as f:
        meta = f.metadata()
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    for name in ("nvfp4", "int4_sym", "int4_asym", "int4_u_g64"):
        tensors[f"{name}.packed_ref"] = torch.from_numpy(
            _formats.pack_nibbles(np.asarray(sts[name].data)))
    save_file(tensors, path, metadata=meta)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/path/to/breccia/src")
