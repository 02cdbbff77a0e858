import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def golden_recipes():
    """The recipes the golden casts were generated with, keyed by case name."""
    from breccia_b200.types import (DelayedScaling, Float8CurrentScaling, Float8BlockScaling,
                                    MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling)
    return {
        "delayed_e4m3": DelayedScaling(fp8_format="E4M3"),
        "current_e4m3": Float8CurrentScaling(fp8_format="E4M3"),
        "current_e5m2": Float8CurrentScaling(fp8_format="E5M2"),
        "block128_e4m3": Float8BlockScaling(fp8_format="E4M3", block_k=128),
        "block64_e5m2": Float8BlockScaling(fp8_format="E5M2", block_k=64),
        "block32_e4m3": Float8BlockScaling(fp8_format="E4M3", block_k=32),
        "mxfp8_e4m3": MXFP8BlockScaling(fp8_format="E4M3"),
        "mxfp8_e5m2": MXFP8BlockScaling(fp8_format="E5M2"),
        "nvfp4": NVFP4BlockScaling(),
        "int4_sym_s_fp16_g128": INT4Scaling(group_size=128),
        "int4_sym_u_fp32_g64": INT4Scaling(group_size=64, signed=False, scale_dtype="fp32"),
        "int4_sym_s_bf16_g32": INT4Scaling(group_size=32, scale_dtype="bf16"),
        "int4_asym_fp16_g128": INT4Scaling(group_size=128, signed=False, symmetric=False),
        "int4_asym_fp32_g64": INT4Scaling(group_size=64, signed=False, symmetric=False,
                                          scale_dtype="fp32"),
    }


def golden_requant_pairs():
    from breccia_b200.types import (Float8CurrentScaling, Float8BlockScaling,
                                    MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling)
    return {
        "nvfp4_to_mxfp8": (NVFP4BlockScaling(), MXFP8BlockScaling()),
        "mxfp8_to_nvfp4": (MXFP8BlockScaling(), NVFP4BlockScaling()),
        "block128_to_current": (Float8BlockScaling(block_k=128), Float8CurrentScaling()),
        "current_to_int4": (Float8CurrentScaling(), INT4Scaling(group_size=128)),
        "int4asym_to_block": (INT4Scaling(group_size=64, signed=False, symmetric=False),
                              Float8BlockScaling(block_k=64)),
    }


def golden_cases(z):
    """(recipe_name, input_name) pairs present in a golden cast file."""
    keys = sorted({k.rsplit("__", 1)[0] for k in z})
    return [tuple(k.split("__")) for k in keys]


def same_bits(a, b):
    """Bitwise equality that treats NaN payloads as equal only if identical bits."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert a.dtype.itemsize == b.dtype.itemsize, (a.dtype, b.dtype)
    u = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[a.dtype.itemsize]
    return np.array_equal(a.view(u), b.view(u))
