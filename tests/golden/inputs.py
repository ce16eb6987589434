"""Seeded synthetic inputs that regenerate bit for bit on any x86-64 host.

The Compose fixtures are recorded at the reference configurations' own sizes
(up to 2 x 4 x 128^3 and 2 x 2 x 160^3), too large to commit.  Their inputs,
the injected noise and the injected elastic grid are therefore regenerated
by the tests from a seed.  To make that exact on a host with other CPU
features, every value is built from numpy's PCG64 integer draws and
elementwise IEEE arithmetic only: no transcendental functions (whose SIMD
variants may differ in the last bit) and no reductions (whose summation
order may differ).

Each fixture stores a digest of the regenerated arrays so that a mismatch
shows up as such rather than as a parity failure.
"""
from __future__ import annotations

import hashlib

import numpy as np


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _unit(rng: np.random.Generator, shape) -> np.ndarray:
    """Uniform float64 in [0, 1) from 53-bit integers (exact conversion)."""
    return (rng.integers(0, 1 << 53, size=shape, dtype=np.int64).astype(np.float64)
            * (1.0 / (1 << 53)))


def normal(seed: int, shape) -> np.ndarray:
    """Approximately N(0, 1) float32: the sum of 12 uniforms minus 6
    (Irwin-Hall), summed in a fixed order."""
    rng = _rng(seed)
    acc = np.full(shape, -6.0)
    for _ in range(12):
        acc += _unit(rng, shape)
    return acc.astype(np.float32)


def uniform(seed: int, shape) -> np.ndarray:
    """Uniform [0, 1) float32."""
    return _unit(_rng(seed), shape).astype(np.float32)


def _upsample_blocks(coarse: np.ndarray, shape, block: int) -> np.ndarray:
    """Nearest upsampling of the last three axes by ``block``, cropped."""
    x = coarse
    for ax in (-3, -2, -1):
        x = np.repeat(x, block, axis=ax)
    H, W, D = shape[-3:]
    return x[..., :H, :W, :D]


def labels(seed: int, shape, n_labels: int, block: int = 12) -> np.ndarray:
    """Piecewise-constant label map 0..n_labels-1 (float32): random labels on
    a coarse lattice with one offset per (element, channel), repeated in
    ``block``-voxel blocks."""
    rng = _rng(seed)
    B, C, H, W, D = shape
    coarse_shape = (B, C, -(-H // block), -(-W // block), -(-D // block))
    coarse = rng.integers(0, n_labels, size=coarse_shape, dtype=np.int64)
    return _upsample_blocks(coarse, shape, block).astype(np.float32)


def _lerp_axis(coarse: np.ndarray, n: int, axis: int) -> np.ndarray:
    """Linear interpolation of ``coarse`` along ``axis`` to ``n`` samples
    spanning it end to end (elementwise float64 arithmetic)."""
    m = coarse.shape[axis]
    pos = np.arange(n, dtype=np.float64) * ((m - 1) / max(n - 1, 1))
    i0 = np.minimum(pos.astype(np.int64), m - 2)
    t = pos - i0
    a = np.take(coarse, i0, axis=axis)
    b = np.take(coarse, i0 + 1, axis=axis)
    shp = [1] * coarse.ndim
    shp[axis] = n
    t = t.reshape(shp)
    return a + (b - a) * t


def elastic_grid(seed: int, batch: int, spatial, max_disp: float, lattice: int = 6) -> np.ndarray:
    """A smooth grid_sample grid (B, H, W, D, 3) fp32 in the layout
    Rand3DElastic builds (last axis x = D, y = W, z = H, align_corners=True
    normalisation): the identity plus a displacement of at most
    ``max_disp`` voxels, interpolated from a random ``lattice``^3 field."""
    rng = _rng(seed)
    H, W, D = spatial
    disp = (_unit(rng, (batch, 3, lattice, lattice, lattice)) * 2.0 - 1.0) * max_disp
    f = disp
    for ax, n in ((2, H), (3, W), (4, D)):
        f = _lerp_axis(f, n, ax)
    out = np.empty((batch, H, W, D, 3), np.float64)
    for comp, (n, ax) in enumerate(((D, 4), (W, 3), (H, 2))):
        half = (n - 1) / 2.0 if n > 1 else 1.0
        shp = [1, 1, 1]
        shp[ax - 2] = n
        base = (np.arange(n, dtype=np.float64) - (n - 1) / 2.0).reshape(shp)
        # component order of grid_sample: x (D), y (W), z (H); the field's
        # channels are (H, W, D)
        out[..., comp] = (base[None] + f[:, 2 - comp]) / half
    return out.astype(np.float32)


def digest(*arrays) -> str:
    """sha256 of the arrays' bytes (shape and dtype included)."""
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str((a.shape, a.dtype.str)).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16), integer
    arithmetic only (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
