"""Whole-step CPU pipelines of the reference's headline configurations —
TEST INFRASTRUCTURE ONLY (the CPU baseline and the reference arm of
``bench.py``).

Each step restates what the reference's PyTorch backend does for one call of
the configuration's transform or ``Compose`` (halleewong/batchaug):
parameters are drawn per element in numpy with the reference's distributions
and draw order, and the tensor work runs in this package's C restatement of
torch's CPU kernels (``oracle.c``, ``oracle_intensity.c``).  Nothing here
imports ``batchaug_b200``: the reference arm must not run the product.

Random draws use numpy's PCG64 streams, not torch's generator, so the
*values* of the parameters differ from a torch run with the same seed; the
distributions, shapes and the work done per step are the reference's.
"""
from __future__ import annotations

import concurrent.futures as cf
import os

import numpy as np

from . import adjust_contrast, noise_add, rand_scale, rand_shift, resample3d, scale_intensity

_EYE = np.eye(4, dtype=np.float32)


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# Parameter sampling (numpy restatement of the reference's sample_params)
# ---------------------------------------------------------------------------

def _uniform(rng: np.random.Generator, n: int) -> np.ndarray:
    """torch.rand(n): float32 in [0, 1)."""
    return rng.random(n, dtype=np.float32)


def sample_mask(rng, B: int, prob: float) -> np.ndarray:
    """BatchTransform.sample_params: rand(B) < prob (batchaug/base.py:21-38)."""
    return _uniform(rng, B) < np.float32(prob)


def _sample_range(rng, spec, ndim: int, B: int, add_scalar: float = 0.0) -> np.ndarray:
    """_sample_range (pytorch/geometric/affine.py:119-151): None -> add_scalar;
    scalar s -> U(-s, s) + add_scalar; (lo, hi) -> U(lo, hi) + add_scalar;
    one rand(B) draw per axis, in axis order."""
    if isinstance(spec, (int, float)):
        spec = [spec] * ndim
    out = np.zeros((B, ndim), np.float32)
    for i, s in enumerate(spec):
        if s is None:
            out[:, i] = add_scalar
        elif isinstance(s, (int, float)):
            out[:, i] = _uniform(rng, B) * np.float32(2 * s) - np.float32(s) + np.float32(add_scalar)
        else:
            lo, hi = s
            out[:, i] = _uniform(rng, B) * np.float32(hi - lo) + np.float32(lo) + np.float32(add_scalar)
    return out


def _eye(B: int) -> np.ndarray:
    return np.broadcast_to(_EYE, (B, 4, 4)).copy()


def _rotation(angles: np.ndarray) -> np.ndarray:
    """Rx(a0) @ Ry(a1) @ Rz(a2) (pytorch/geometric/affine.py:9-58)."""
    B = angles.shape[0]
    c = np.cos(angles).astype(np.float32)
    s = np.sin(angles).astype(np.float32)
    rx, ry, rz = _eye(B), _eye(B), _eye(B)
    rx[:, 1, 1], rx[:, 1, 2], rx[:, 2, 1], rx[:, 2, 2] = c[:, 0], -s[:, 0], s[:, 0], c[:, 0]
    ry[:, 0, 0], ry[:, 0, 2], ry[:, 2, 0], ry[:, 2, 2] = c[:, 1], s[:, 1], -s[:, 1], c[:, 1]
    rz[:, 0, 0], rz[:, 0, 1], rz[:, 1, 0], rz[:, 1, 1] = c[:, 2], -s[:, 2], s[:, 2], c[:, 2]
    return (rx @ ry @ rz).astype(np.float32)


def sample_rand_affine(rng, B: int, prob: float, rotate_range=None, shear_range=None,
                       translate_range=None, scale_range=None):
    """RandAffine.sample_params (pytorch/geometric/affine.py:229-269): mask,
    then I @ R @ Sh @ T @ Sc per element; returns (mask, affine) with the
    affine already the identity where masked out (to_affine, :271-282)."""
    mask = sample_mask(rng, B, prob)
    a = _eye(B)
    if rotate_range is not None:
        a = a @ _rotation(_sample_range(rng, rotate_range, 3, B))
    if shear_range is not None:
        spec = [shear_range] * 6 if isinstance(shear_range, (int, float)) else shear_range
        sh = _sample_range(rng, spec, 6, B)
        m = _eye(B)
        m[:, 0, 1], m[:, 0, 2], m[:, 1, 0] = sh[:, 0], sh[:, 1], sh[:, 2]
        m[:, 1, 2], m[:, 2, 0], m[:, 2, 1] = sh[:, 3], sh[:, 4], sh[:, 5]
        a = a @ m
    if translate_range is not None:
        t = _sample_range(rng, translate_range, 3, B)
        m = _eye(B)
        m[:, :3, 3] = t
        a = a @ m
    if scale_range is not None:
        sc = _sample_range(rng, scale_range, 3, B, add_scalar=1.0)
        m = _eye(B)
        m[:, 0, 0], m[:, 1, 1], m[:, 2, 2] = sc[:, 0], sc[:, 1], sc[:, 2]
        a = a @ m
    a = a.astype(np.float32)
    return mask, np.where(mask[:, None, None], a, _EYE[None]).astype(np.float32)


def sample_rot90(rng, B: int, prob: float, max_k: int = 3, spatial_axes=(0, 1)):
    """RandRotate90.sample_params + to_affine (pytorch/geometric/rotate90.py:
    36-80): k in 1..max_k, exact cos/sin in the resampling convention."""
    mask = sample_mask(rng, B, prob)
    k = rng.integers(1, max_k + 1, B)
    a = _eye(B)
    ax0, ax1 = spatial_axes
    cos_t, sin_t = (0.0, -1.0, 0.0), (-1.0, 0.0, 1.0)
    for kk in range(1, max_k + 1):
        sel = mask & (k == kk)
        c, s = cos_t[(kk - 1) % 3], sin_t[(kk - 1) % 3]
        a[sel, ax0, ax0] = c
        a[sel, ax0, ax1] = -s
        a[sel, ax1, ax0] = s
        a[sel, ax1, ax1] = c
    return mask, a


def sample_axis_flip(rng, B: int, prob: float):
    """RandAxisFlip.sample_params + to_affine (pytorch/geometric/flip.py:
    28-52): one random spatial axis per element, diag -1 on it."""
    mask = sample_mask(rng, B, prob)
    axes = rng.integers(0, 3, B)
    a = _eye(B)
    for ax in range(3):
        a[mask & (axes == ax), ax, ax] = -1.0
    return mask, a


def normal_f32(rng, shape, nthreads: int) -> np.ndarray:
    """torch.randn(shape) stand-in: standard normal float32, generated in
    parallel chunks by independent PCG64 streams spawned from ``rng``."""
    out = np.empty(int(np.prod(shape)), np.float32)
    n = max(1, nthreads)
    bounds = np.linspace(0, out.size, n + 1).astype(np.int64)
    gens = [np.random.default_rng(int(s)) for s in rng.integers(0, 2**63, n)]

    def fill(i):
        gens[i].standard_normal(out=out[bounds[i]:bounds[i + 1]], dtype=np.float32)

    with cf.ThreadPoolExecutor(n) as ex:
        list(ex.map(fill, range(n)))
    return out.reshape(shape)


# ---------------------------------------------------------------------------
# Whole steps
# ---------------------------------------------------------------------------

AFFINE_CONFIG2 = dict(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=5,
                      scale_range=0.1)


def config2_step(x: np.ndarray, rng, nthreads: int) -> np.ndarray:
    """RandAffine(prob=1, rotate 0.785, shear 0.3, translate 5, scale 0.1)
    on (B,1,128^3) fp32 with bilinear/border padding
    (pytorch/geometric/affine.py:229-317)."""
    B = x.shape[0]
    mask, affine = sample_rand_affine(rng, B, **AFFINE_CONFIG2)
    return resample3d(x, affine=affine, mode="bilinear", padding="border", mask=mask,
                      nthreads=nthreads)


def _materialize(d: dict, pending: dict, modes: dict, nthreads: int) -> dict:
    """Compose._materialize (batchaug/compose.py:71-110): per key, skip when
    no element is selected, else one grid_sample through the accumulated
    affine with the key's mode (zeros padding) and the masked copy."""
    d = dict(d)
    for key, (affine, mask) in pending.items():
        if key not in d or not mask.any():
            continue
        d[key] = resample3d(d[key], affine=affine, mode=modes[key], padding="zeros", mask=mask,
                            nthreads=nthreads)
    return d


def config4_step(vol: np.ndarray, seg: np.ndarray, rng, nthreads: int):
    """Compose(lazy=True) of RandRotate90d(0.5, max_k 3, axes (0,1)),
    RandAxisFlipd(0.5), RandGaussianNoised(vol, std 0.5), RandAffined(0.5,
    rotate 0.785, shear 0.3, translate 5), ScaleIntensityd(vol); vol
    bilinear, seg nearest (batchaug/compose.py:116-164): {rot90, flip}
    materialised before the noise, {affine} before ScaleIntensity."""
    B = vol.shape[0]
    modes = {"vol": "bilinear", "seg": "nearest"}
    d = {"vol": vol, "seg": seg}
    m_r, a_r = sample_rot90(rng, B, 0.5, 3, (0, 1))
    m_f, a_f = sample_axis_flip(rng, B, 0.5)
    a1 = (a_r @ a_f).astype(np.float32)
    m1 = m_r | m_f
    d = _materialize(d, {"vol": (a1, m1), "seg": (a1, m1)}, modes, nthreads)
    # RandGaussianNoise(prob 0.1, std 0.5): randn of the whole tensor * std
    # + mean, added where the mask is set (pytorch/intensity/noise.py:34-66)
    m_n = sample_mask(rng, B, 0.1)
    noise = normal_f32(rng, d["vol"].shape, nthreads)
    noise *= np.float32(0.5)
    d["vol"] = noise_add(d["vol"], noise, m_n, nthreads=nthreads)
    m_a, a_a = sample_rand_affine(rng, B, 0.5, rotate_range=0.785, shear_range=0.3,
                                  translate_range=5)
    d = _materialize(d, {"vol": (a_a, m_a), "seg": (a_a, m_a)}, modes, nthreads)
    d["vol"] = scale_intensity(d["vol"], 0.0, 1.0, channel_wise=True, nthreads=nthreads)
    return d


def config3_step(x: np.ndarray, rng, nthreads: int) -> np.ndarray:
    """Noise (std U(0.1,0.5)) -> contrast (gamma U(0.5,2)) -> scale (0.2) ->
    shift (0.1) -> ScaleIntensity(0, 1), prob 1, on a bf16 tensor stored as
    uint16 bits (pytorch/intensity/{noise,contrast,scale_shift}.py)."""
    B = x.shape[0]
    mask = np.ones(B, bool)
    std = _uniform(rng, B) * np.float32(0.4) + np.float32(0.1)
    noise = normal_f32(rng, x.shape, nthreads)
    noise *= std.reshape((B,) + (1,) * (x.ndim - 1))
    y = noise_add(x, noise, mask, nthreads=nthreads)
    y = adjust_contrast(y, _uniform(rng, B) * np.float32(1.5) + np.float32(0.5), mask,
                        nthreads=nthreads)
    y = rand_scale(y, _uniform(rng, B) * np.float32(0.4) - np.float32(0.2), mask,
                   nthreads=nthreads)
    y = rand_shift(y, _uniform(rng, B) * np.float32(0.2) - np.float32(0.1), mask,
                   nthreads=nthreads)
    return scale_intensity(y, 0.0, 1.0, channel_wise=True, nthreads=nthreads)
