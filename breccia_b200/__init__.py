"""breccia_b200 -- a B200 (sm_100a) backend for breccia's hot path.

``cast`` / ``dequantize`` / ``requantize`` / ``matmul`` with the reference's
interface (jvoltci/breccia v0.1.3, ``src/breccia/__init__.py:23``), running
hand-written CUDA kernels on CUDA torch tensors, plus the types
(``ScaledTensor``, recipes, layouts) with the reference's names and checks.

``install()`` puts this backend behind an imported ``breccia`` package:
breccia's own functions then send CUDA tensors here and keep their NumPy
path for everything else.
"""

from .types import (  # noqa: F401
    ScaledTensor, from_buffer,
    ScalingRecipe, DelayedScaling, Float8CurrentScaling, Float8BlockScaling,
    MXFP8BlockScaling, NVFP4BlockScaling, INT4Scaling,
    Layout, PerTensor, PerBlockK, PerChannel, PerBlockMN,
)
from .api import (cast, dequantize, requantize, matmul, linear, gemm_operands,  # noqa: F401
                  attach_gemm_operands, AmaxHistory, cast_matmul)
from . import bridges  # noqa: F401
from .autograd import cast_ste, cast_ste_clipped  # noqa: F401
from .plugin import install, uninstall  # noqa: F401

__version__ = "0.1.0"
