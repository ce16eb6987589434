"""batchaug_b200 — B200-native backend for batchaug's hot path.

A drop-in for the reference's transform API on that path
(``import batchaug_b200 as batchaug``): the same class names, constructors,
``sample_params`` / ``apply`` / ``to_affine`` and dict wrappers, and
``Compose(transforms, lazy, mode, padding_mode)``.  Work runs in hand-written
sm_100a CUDA kernels behind the C ABI in ``include/batchaug_b200.h``; there
is no Triton, no multi-backend dispatch and no CPU fallback.

Replaces the reference's backend dispatch (batchaug/__init__.py:64-74,
batchaug/_backend.py) with a single backend.  ``set_backend`` /
``get_backend`` / ``resolve_backend`` remain for API compatibility and only
accept this backend.
"""
from __future__ import annotations

from . import _lib  # noqa: F401  (loads libbatchaug_b200.so or raises ImportError)
from ._rng import get_shard, set_shard, shard
from .base import BatchDictTransform, BatchTransform
from .compose import Compose
from .ops import resample_exact, set_resample_exact
from .geometric import (
    Rand3DElastic,
    Rand3DElasticd,
    RandAffine,
    RandAffined,
    RandAxisFlip,
    RandAxisFlipd,
    RandFlip,
    RandFlipd,
    RandRotate,
    RandRotate90,
    RandRotate90d,
    RandRotated,
    RandZoom,
    RandZoomd,
)
from .intensity import (
    RandAdjustContrast,
    RandAdjustContrastd,
    RandBiasField,
    RandBiasFieldd,
    RandGaussianNoise,
    RandGaussianNoised,
    RandGaussianSharpen,
    RandGaussianSharpend,
    RandGaussianSmooth,
    RandGaussianSmoothd,
    RandRicianNoise,
    RandRicianNoised,
    RandScaleIntensity,
    RandScaleIntensityd,
    RandScaleIntensityFixedMean,
    RandScaleIntensityFixedMeand,
    RandShiftIntensity,
    RandShiftIntensityd,
    RandSimulateLowResolution,
    RandSimulateLowResolutiond,
    RandStdShiftIntensity,
    RandStdShiftIntensityd,
    ScaleIntensity,
    ScaleIntensityd,
)

_BACKEND = "b200"


def set_backend(name: str) -> None:
    """Accepts only this backend ("b200"; "auto" is an alias)."""
    if name not in ("auto", "b200"):
        raise ValueError(f"Unknown backend {name!r}: batchaug_b200 has the single backend 'b200'")


def get_backend() -> str:
    return _BACKEND


def resolve_backend() -> str:
    return _BACKEND


__all__ = [
    "BatchTransform", "BatchDictTransform", "Compose", "set_backend", "get_backend",
    "resolve_backend", "set_shard", "get_shard", "shard", "resample_exact", "set_resample_exact",
    "Rand3DElastic", "Rand3DElasticd", "RandAffine", "RandAffined", "RandAxisFlip",
    "RandAxisFlipd", "RandFlip", "RandFlipd", "RandRotate", "RandRotated", "RandRotate90",
    "RandRotate90d", "RandZoom", "RandZoomd",
    "RandAdjustContrast", "RandAdjustContrastd", "RandBiasField", "RandBiasFieldd",
    "RandGaussianNoise", "RandGaussianNoised", "RandGaussianSharpen", "RandGaussianSharpend",
    "RandGaussianSmooth", "RandGaussianSmoothd",
    "RandRicianNoise", "RandRicianNoised", "RandScaleIntensity", "RandScaleIntensityd",
    "RandScaleIntensityFixedMean", "RandScaleIntensityFixedMeand", "RandShiftIntensity",
    "RandShiftIntensityd", "RandSimulateLowResolution", "RandSimulateLowResolutiond",
    "RandStdShiftIntensity", "RandStdShiftIntensityd",
    "ScaleIntensity", "ScaleIntensityd",
]
