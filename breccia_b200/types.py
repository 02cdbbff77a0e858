"""breccia's value type, recipes and layouts, with the reference's interface.

These classes mirror, field for field and message for message, the public
types of jvoltci/breccia v0.1.3 so that code written against breccia runs
unchanged on this backend:

* :class:`ScaledTensor` / :func:`from_buffer` -- ``src/breccia/_core.py:37-196``
* recipes -- ``src/breccia/recipes.py:28-199``
* layouts -- ``src/breccia/layouts.py:31-164``

When the real ``breccia`` package is importable the backend accepts its
recipe objects too (dispatch reads the ``name`` class attribute) and returns
results built from the caller's own classes; see :mod:`breccia_b200.api`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, ClassVar, Tuple

__all__ = [
    "ScaledTensor", "from_buffer",
    "ScalingRecipe", "DelayedScaling", "Float8CurrentScaling", "Float8BlockScaling",
    "MXFP8BlockScaling", "NVFP4BlockScaling", "INT4Scaling",
    "Layout", "PerTensor", "PerBlockK", "PerChannel", "PerBlockMN",
]


# ------------------------------------------------------------------ recipes


class ScalingRecipe:
    """Base class of all recipes (``recipes.py:28-35``)."""

    name: ClassVar[str] = ""


def _check_fp8_format(fmt: str) -> None:  # recipes.py:38-40
    if fmt not in {"E4M3", "E5M2"}:
        raise ValueError(f"fp8_format must be 'E4M3' or 'E5M2', got {fmt!r}")


@dataclass(frozen=True)
class DelayedScaling(ScalingRecipe):
    """Per-tensor FP8 with a TE-style amax history (``recipes.py:43-77``).
    The cast itself uses the current tensor's amax, as the reference does,
    unless an ``AmaxHistory`` is passed to ``cast`` (extension)."""

    name: ClassVar[str] = "delayed"
    fp8_format: str = "E4M3"
    amax_history_len: int = 16
    margin: int = 0

    def __post_init__(self) -> None:
        _check_fp8_format(self.fp8_format)
        if self.amax_history_len < 1:
            raise ValueError(f"amax_history_len must be >= 1, got {self.amax_history_len}")


@dataclass(frozen=True)
class Float8CurrentScaling(ScalingRecipe):
    """Per-tensor FP8 from the current amax (``recipes.py:80-93``)."""

    name: ClassVar[str] = "current"
    fp8_format: str = "E4M3"

    def __post_init__(self) -> None:
        _check_fp8_format(self.fp8_format)


@dataclass(frozen=True)
class Float8BlockScaling(ScalingRecipe):
    """FP8 with one float32 scale per ``block_k`` run of the last axis
    (``recipes.py:96-112``)."""

    name: ClassVar[str] = "block"
    fp8_format: str = "E4M3"
    block_k: int = 128

    def __post_init__(self) -> None:
        _check_fp8_format(self.fp8_format)
        if self.block_k <= 0:
            raise ValueError(f"block_k must be > 0, got {self.block_k}")


@dataclass(frozen=True)
class MXFP8BlockScaling(ScalingRecipe):
    """OCP MX FP8: 32-element blocks, E8M0 scale (``recipes.py:115-134``)."""

    name: ClassVar[str] = "mxfp8"
    fp8_format: str = "E4M3"
    block_size: int = 32

    def __post_init__(self) -> None:
        _check_fp8_format(self.fp8_format)
        if self.block_size != 32:
            raise ValueError(
                "MXFP8 block_size is fixed at 32 by the OCP MX spec, "
                f"got {self.block_size}")


@dataclass(frozen=True)
class NVFP4BlockScaling(ScalingRecipe):
    """NVFP4: E2M1 data, 16-element blocks, E4M3 scale (``recipes.py:137-160``)."""

    name: ClassVar[str] = "nvfp4"
    fp4_format: str = "E2M1"
    block_size: int = 16
    scale_format: str = "E4M3"

    def __post_init__(self) -> None:
        if self.fp4_format != "E2M1":
            raise ValueError(f"NVFP4 fp4_format is fixed at 'E2M1', got {self.fp4_format!r}")
        if self.block_size != 16:
            raise ValueError(f"NVFP4 block_size is fixed at 16, got {self.block_size}")
        if self.scale_format != "E4M3":
            raise ValueError(
                f"NVFP4 scale_format is fixed at 'E4M3', got {self.scale_format!r}")


@dataclass(frozen=True)
class INT4Scaling(ScalingRecipe):
    """Group-wise INT4 weight quantization (``recipes.py:163-199``)."""

    name: ClassVar[str] = "int4"
    group_size: int = 128
    signed: bool = True
    scale_dtype: str = "fp16"
    symmetric: bool = True

    def __post_init__(self) -> None:
        if self.group_size <= 0:
            raise ValueError(f"group_size must be > 0, got {self.group_size}")
        if self.scale_dtype not in {"fp16", "bf16", "fp32"}:
            raise ValueError(
                "scale_dtype must be one of 'fp16', 'bf16', 'fp32', "
                f"got {self.scale_dtype!r}")
        if not self.symmetric and self.signed:
            raise ValueError(
                "asymmetric INT4 (symmetric=False) requires signed=False; "
                "the zero-point shifts an unsigned [0, 15] range into the "
                "values' actual distribution")


# ------------------------------------------------------------------ layouts


class Layout:
    """Base class of layouts (``layouts.py:31-42``)."""

    name: ClassVar[str] = ""

    def validate(self, data: Any, scale: Any) -> None:  # pragma: no cover
        raise NotImplementedError("Layout subclasses must implement validate()")


@dataclass(frozen=True)
class PerTensor(Layout):
    """One scalar scale (``layouts.py:45-59``)."""

    name: ClassVar[str] = "per_tensor"

    def validate(self, data: Any, scale: Any) -> None:
        if scale.ndim != 0:
            raise ValueError(
                f"PerTensor requires a scalar scale (ndim=0), "
                f"got ndim={scale.ndim} with shape={tuple(scale.shape)}")


@dataclass(frozen=True)
class PerBlockK(Layout):
    """One scale per ``block_size`` run of the last axis (``layouts.py:62-94``)."""

    name: ClassVar[str] = "per_block_k"
    block_size: int = 128

    def __post_init__(self) -> None:
        if self.block_size <= 0:
            raise ValueError(f"block_size must be > 0, got {self.block_size}")

    def validate(self, data: Any, scale: Any) -> None:
        if data.ndim < 2:
            raise ValueError(
                f"PerBlockK requires data.ndim >= 2 (matmul shape), got ndim={data.ndim}")
        K = data.shape[-1]
        if K % self.block_size != 0:
            raise ValueError(
                f"PerBlockK: data.shape[-1]={K} must be divisible by "
                f"block_size={self.block_size}")
        expected = tuple(data.shape[:-1]) + (K // self.block_size,)
        if tuple(scale.shape) != expected:
            raise ValueError(
                f"PerBlockK: scale.shape must be {expected}, got {tuple(scale.shape)}")


@dataclass(frozen=True)
class PerChannel(Layout):
    """One scale per row (``layouts.py:97-119``)."""

    name: ClassVar[str] = "per_channel"

    def validate(self, data: Any, scale: Any) -> None:
        if data.ndim < 2:
            raise ValueError(f"PerChannel requires data.ndim >= 2, got ndim={data.ndim}")
        M = data.shape[-2]
        valid = {(M,), tuple(data.shape[:-1]) + (1,)}
        if tuple(scale.shape) not in valid:
            raise ValueError(
                f"PerChannel: scale.shape must be one of {sorted(valid)}, "
                f"got {tuple(scale.shape)}")


@dataclass(frozen=True)
class PerBlockMN(Layout):
    """One scale per ``block_m x block_n`` tile of the last two axes
    (``layouts.py:122-164``)."""

    name: ClassVar[str] = "per_block_mn"
    block_m: int = 1
    block_n: int = 32

    def __post_init__(self) -> None:
        if self.block_m <= 0 or self.block_n <= 0:
            raise ValueError(
                f"block_m and block_n must be > 0, got ({self.block_m}, {self.block_n})")

    def validate(self, data: Any, scale: Any) -> None:
        if data.ndim < 2:
            raise ValueError(f"PerBlockMN requires data.ndim >= 2, got ndim={data.ndim}")
        M, N = data.shape[-2], data.shape[-1]
        if M % self.block_m != 0:
            raise ValueError(
                f"PerBlockMN: data.shape[-2]={M} not divisible by block_m={self.block_m}")
        if N % self.block_n != 0:
            raise ValueError(
                f"PerBlockMN: data.shape[-1]={N} not divisible by block_n={self.block_n}")
        expected = tuple(data.shape[:-2]) + (M // self.block_m, N // self.block_n)
        if tuple(scale.shape) != expected:
            raise ValueError(
                f"PerBlockMN: scale.shape must be {expected}, got {tuple(scale.shape)}")


# ------------------------------------------------------------- ScaledTensor


@dataclass(frozen=True)
class ScaledTensor:
    """Low-precision data with its scale, recipe and layout (``_core.py:37-155``).

    ``scale`` is the dequantization scale: ``x ~= decode(data) * scale``
    (asymmetric INT4: ``(data - zero_point) * scale``).
    """

    data: Any
    scale: Any
    recipe: Any
    layout: Any
    zero_point: Any = None

    def __post_init__(self) -> None:
        if not hasattr(self.data, "shape") or not hasattr(self.data, "dtype"):
            raise TypeError(
                f"data must be array-like with .shape and .dtype, "
                f"got {type(self.data).__name__}")
        if not hasattr(self.scale, "shape") or not hasattr(self.scale, "dtype"):
            raise TypeError(
                f"scale must be array-like with .shape and .dtype, "
                f"got {type(self.scale).__name__}")
        if self.data.ndim < 1:
            raise ValueError(f"data must be at least 1-D, got {self.data.ndim}-D")
        if self.recipe is None:
            raise ValueError("recipe is required (see breccia.recipes)")
        if self.layout is None:
            raise ValueError("layout is required (see breccia.layouts)")
        if self.zero_point is not None:
            if not hasattr(self.zero_point, "shape"):
                raise TypeError(
                    f"zero_point must be array-like, got {type(self.zero_point).__name__}")
            if tuple(self.zero_point.shape) != tuple(self.scale.shape):
                raise ValueError(
                    f"zero_point.shape ({tuple(self.zero_point.shape)}) must "
                    f"match scale.shape ({tuple(self.scale.shape)})")
        validate = getattr(self.layout, "validate", None)
        if callable(validate):
            validate(self.data, self.scale)

    @property
    def shape(self) -> Tuple[int, ...]:
        return tuple(self.data.shape)

    @property
    def data_dtype(self) -> Any:
        return self.data.dtype

    @property
    def scale_dtype(self) -> Any:
        return self.scale.dtype

    @property
    def ndim(self) -> int:
        return self.data.ndim

    def __repr__(self) -> str:
        return (f"breccia.ScaledTensor(shape={self.shape}, data_dtype={self.data_dtype}, "
                f"scale_shape={tuple(self.scale.shape)}, recipe={type(self.recipe).__name__}, "
                f"layout={type(self.layout).__name__})")


def from_buffer(data: Any, scale: Any, recipe: Any, layout: Any,
                zero_point: Any = None) -> ScaledTensor:
    """Wrap existing buffers without copying (``_core.py:158-196``)."""
    return ScaledTensor(data=data, scale=scale, recipe=recipe, layout=layout,
                        zero_point=zero_point)
