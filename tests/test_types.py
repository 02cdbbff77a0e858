"""The mirror types keep the reference's fields, checks and messages
(src/breccia/_core.py, recipes.py, layouts.py of jvoltci/breccia v0.1.3)."""

import numpy as np
import pytest

from breccia_b200.types import (ScaledTensor, from_buffer, DelayedScaling, Float8CurrentScaling,
                                Float8BlockScaling, MXFP8BlockScaling, NVFP4BlockScaling,
                                INT4Scaling, PerTensor, PerBlockK, PerChannel, PerBlockMN)


def test_recipe_names_and_defaults():
    assert DelayedScaling().name == "delayed" and DelayedScaling().amax_history_len == 16
    assert Float8CurrentScaling().name == "current"
    assert Float8BlockScaling().block_k == 128
    assert MXFP8BlockScaling().block_size == 32
    assert NVFP4BlockScaling().block_size == 16
    r = INT4Scaling()
    assert (r.group_size, r.signed, r.scale_dtype, r.symmetric) == (128, True, "fp16", True)


@pytest.mark.parametrize("ctor,msg", [
    (lambda: Float8CurrentScaling(fp8_format="E3M4"), "fp8_format must be"),
    (lambda: DelayedScaling(amax_history_len=0), "amax_history_len must be >= 1"),
    (lambda: Float8BlockScaling(block_k=0), "block_k must be > 0"),
    (lambda: MXFP8BlockScaling(block_size=16), "fixed at 32"),
    (lambda: NVFP4BlockScaling(block_size=32), "fixed at 16"),
    (lambda: INT4Scaling(scale_dtype="fp8"), "scale_dtype must be one of"),
    (lambda: INT4Scaling(symmetric=False), "requires signed=False"),
    (lambda: INT4Scaling(group_size=0), "group_size must be > 0"),
])
def test_recipe_validation(ctor, msg):
    with pytest.raises(ValueError, match=msg):
        ctor()


def test_layout_validation():
    d = np.zeros((4, 64), np.uint8)
    PerTensor().validate(d, np.float32(1.0) * np.ones(()))
    PerBlockK(32).validate(d, np.zeros((4, 2)))
    PerBlockMN(1, 32).validate(d, np.zeros((4, 2)))
    PerChannel().validate(d, np.zeros((4,)))
    with pytest.raises(ValueError, match="PerTensor requires a scalar"):
        PerTensor().validate(d, np.zeros((1,)))
    with pytest.raises(ValueError, match="must be divisible by"):
        PerBlockK(48).validate(d, np.zeros((4, 1)))
    with pytest.raises(ValueError, match="scale.shape must be"):
        PerBlockMN(1, 32).validate(d, np.zeros((4, 3)))


def test_scaled_tensor_checks():
    d = np.zeros((4, 64), np.uint8)
    st = from_buffer(d, np.zeros((4, 2), np.float32), Float8BlockScaling(block_k=32),
                     PerBlockK(32))
    assert st.shape == (4, 64) and st.ndim == 2
    assert "ScaledTensor" in repr(st)
    with pytest.raises(ValueError, match="recipe is required"):
        ScaledTensor(d, np.zeros(()), None, PerTensor())
    with pytest.raises(ValueError, match="zero_point.shape"):
        ScaledTensor(d, np.zeros((4, 2)), INT4Scaling(group_size=32), PerBlockK(32),
                     zero_point=np.zeros((4, 3)))
    with pytest.raises(TypeError, match="data must be array-like"):
        ScaledTensor([1, 2], np.zeros(()), Float8CurrentScaling(), PerTensor())
