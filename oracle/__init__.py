"""CPU oracle for the batchaug hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in plain C (``oracle.c``, ``oracle_intensity.c``),
the reference PyTorch backend of batchaug for the geometric resample and the
intensity chain.  It is the parity checker for ``batchaug_b200``'s CUDA
kernels and the timed CPU baseline in ``bench.py``.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import it; the
``batchaug_b200`` package never does.

Parity is pinned: ``tests/golden/*.npz`` hold outputs of the reference
itself (``batchaug.pytorch`` on torch 2.11 CPU), produced by
``tests/golden/gen_golden.py``, and ``tests/test_oracle_golden.py`` checks
this oracle against every fixture.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_ba.so")
_lib = None

F32, BF16 = 0, 1
BILINEAR, NEAREST = 0, 1
PAD_ZEROS, PAD_BORDER, PAD_REFLECTION = 0, 1, 2
XFORM_AFFINE, XFORM_THETA, XFORM_GRID = 0, 1, 2

_MODES = {"bilinear": BILINEAR, "nearest": NEAREST}
_PADS = {"zeros": PAD_ZEROS, "border": PAD_BORDER, "reflection": PAD_REFLECTION}


def build(force: bool = False) -> str:
    """Compile liboracle_ba.so with the Makefile beside this file."""
    if force or not os.path.exists(_LIB_PATH) or _stale():
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "liboracle_ba.so"],
                       check=True)
    return _LIB_PATH


def _stale() -> bool:
    lib_t = os.path.getmtime(_LIB_PATH)
    for f in ("oracle.c", "oracle_intensity.c", "oracle_lowres.c", "oracle_compose.c", "Makefile"):
        p = os.path.join(_HERE, f)
        if os.path.exists(p) and os.path.getmtime(p) > lib_t:
            return True
    return False


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    P, I64, I, F, D = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_double
    L.ora_resample3d.argtypes = [P, P, I, I64, I64, I64, I64, I64, I, P, I64, I, I, I, P, I]
    L.ora_resample3d.restype = I
    L.ora_affine_grid.argtypes = [P, I64, I64, I64, I64, I64, I, P]
    L.ora_affine_to_theta.argtypes = [P, I64, I64, I64, I64, P]
    L.ora_linspace_m1p1.argtypes = [I64, I64]
    L.ora_linspace_m1p1.restype = F
    L.ora_base_coord.argtypes = [I64, I64, I]
    L.ora_base_coord.restype = F
    L.ora_bf16_round.argtypes = [F]
    L.ora_bf16_round.restype = F
    L.ora_bf16_from_f32.argtypes = [P, P, I64]
    L.ora_bf16_to_f32.argtypes = [P, P, I64]
    L.ora_minmax.argtypes = [P, I, I64, I64, P, P, I]
    L.ora_noise_add.argtypes = [P, P, I, P, P, I64, I64, I]
    L.ora_adjust_contrast.argtypes = [P, P, I, P, P, I64, I64, I]
    L.ora_rand_scale.argtypes = [P, P, I, P, P, I64, I64, I]
    L.ora_rand_shift.argtypes = [P, P, I, P, P, I, I64, I64, I]
    L.ora_scale_intensity.argtypes = [P, P, I, I64, I64, I64, D, D, D, I, I]
    L.ora_bias_field.argtypes = [P, P, I, P, P, I64, I64, I64, I64, I64, I, I]
    L.ora_bias_field.restype = I
    L.ora_gaussian_1d_batch.argtypes = [P, I64, D, P]
    L.ora_gaussian_1d_batch.restype = I64
    L.ora_separable_gauss.argtypes = [P, P, I, P, I64, P, I64, P, I64, I64, I64, I64, I64, I64, I,
                                      I]
    L.ora_elastic_grid.argtypes = [P, P, I64, P, I64, I64, I64, I64, P, I]
    L.ora_std_shift.argtypes = [P, P, I, P, P, I64, I64, I64, I, I, I]
    L.ora_fixed_mean.argtypes = [P, P, I, P, P, I64, I64, I64, I, I]
    L.ora_rician.argtypes = [P, P, I, P, P, P, D, I, P, I64, I64, I]
    L.ora_sharpen_combine.argtypes = [P, P, P, P, I, P, P, I64, I64, I]
    L.ora_lowres.argtypes = [P, P, I, I64, I64, I64, I64, I64, P, P, I, I, I, I]
    L.ora_lowres.restype = I
    L.ora_compose_field.argtypes = [P, P, P, P, I64, I64, I64, I64, P]


# ---------------------------------------------------------------------------
# bf16 storage in numpy: arrays of uint16 holding the upper half of fp32.
# ---------------------------------------------------------------------------

def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().ora_bf16_from_f32(a.ctypes.data, out.ctypes.data, a.size)
    return out


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, np.float32)
    lib().ora_bf16_to_f32(a.ctypes.data, out.ctypes.data, a.size)
    return out


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(f"oracle arrays are float32 or uint16 (bf16 bits), got {a.dtype}")


def _c(a, dtype=None):
    if a is None:
        return None
    return np.ascontiguousarray(a if dtype is None else a.astype(dtype, copy=False))


def _p(a):
    return None if a is None else a.ctypes.data


def _mask(mask, B):
    if mask is None:
        return None
    m = np.ascontiguousarray(np.asarray(mask).astype(np.uint8).reshape(B))
    return m


# ---------------------------------------------------------------------------
# Geometric
# ---------------------------------------------------------------------------

def resample3d(x: np.ndarray, *, affine=None, theta=None, grid=None, mode="bilinear",
               padding="zeros", align_corners=False, mask=None, nthreads=0) -> np.ndarray:
    """grid_sample of (B,C,H,W,D) x through a MONAI affine (B,4,4), a theta
    (B,3|4,4) or an explicit grid (B,H,W,D,3); masked-out elements copy x."""
    x = _c(x)
    B, C, H, W, D = x.shape
    out = np.empty_like(x)
    if affine is not None:
        kind, xf, stride = XFORM_AFFINE, _c(affine, np.float32), 16
    elif theta is not None:
        xf = _c(theta, np.float32)
        kind, stride = XFORM_THETA, int(np.prod(xf.shape[1:]))
    elif grid is not None:
        kind, xf, stride = XFORM_GRID, _c(grid, np.float32), 0
    else:
        raise ValueError("one of affine, theta or grid is required")
    m = _mask(mask, B)
    rc = lib().ora_resample3d(x.ctypes.data, out.ctypes.data, _dt(x), B, C, H, W, D, kind,
                              xf.ctypes.data, stride, _MODES[mode], _PADS[padding],
                              int(bool(align_corners)), _p(m), int(nthreads))
    if rc != 0:
        raise ValueError("ora_resample3d: bad arguments")
    return out


def affine_to_theta(affine: np.ndarray, spatial_shape) -> np.ndarray:
    a = _c(affine, np.float32)
    B = a.shape[0]
    out = np.empty((B, 3, 4), np.float32)
    H, W, D = spatial_shape
    lib().ora_affine_to_theta(a.ctypes.data, B, H, W, D, out.ctypes.data)
    return out


def affine_grid(theta: np.ndarray, shape, align_corners=False) -> np.ndarray:
    th = _c(theta, np.float32)
    B, _, H, W, D = shape
    out = np.empty((B, H, W, D, 3), np.float32)
    stride = int(np.prod(th.shape[1:]))
    lib().ora_affine_grid(th.ctypes.data, stride, B, H, W, D, int(bool(align_corners)),
                          out.ctypes.data)
    return out


# ---------------------------------------------------------------------------
# Intensity
# ---------------------------------------------------------------------------

def minmax(x: np.ndarray, n_groups: int, nthreads=0):
    x = _c(x)
    mins = np.empty(n_groups, np.float32)
    maxs = np.empty(n_groups, np.float32)
    lib().ora_minmax(x.ctypes.data, _dt(x), n_groups, x.size // n_groups, mins.ctypes.data,
                     maxs.ctypes.data, int(nthreads))
    return mins, maxs


def noise_add(x, noise, mask=None, nthreads=0):
    x = _c(x)
    nz = _c(noise, np.float32)
    B = x.shape[0]
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_noise_add(x.ctypes.data, out.ctypes.data, _dt(x), nz.ctypes.data, _p(m), B,
                        x.size // B, int(nthreads))
    return out


def adjust_contrast(x, gamma, mask=None, nthreads=0):
    x = _c(x)
    B = x.shape[0]
    g = _c(np.asarray(gamma, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_adjust_contrast(x.ctypes.data, out.ctypes.data, _dt(x), g.ctypes.data, _p(m), B,
                              x.size // B, int(nthreads))
    return out


def rand_scale(x, factor, mask=None, nthreads=0):
    x = _c(x)
    B = x.shape[0]
    f = _c(np.asarray(factor, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_rand_scale(x.ctypes.data, out.ctypes.data, _dt(x), f.ctypes.data, _p(m), B,
                         x.size // B, int(nthreads))
    return out


def rand_shift(x, offset, mask=None, safe=False, nthreads=0):
    x = _c(x)
    B = x.shape[0]
    o = _c(np.asarray(offset, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_rand_shift(x.ctypes.data, out.ctypes.data, _dt(x), o.ctypes.data, _p(m),
                         int(bool(safe)), B, x.size // B, int(nthreads))
    return out


def scale_intensity(x, minv=0.0, maxv=1.0, factor=None, channel_wise=True, nthreads=0):
    x = _c(x)
    B, C = x.shape[:2]
    out = np.empty_like(x)
    flags = (minv is not None) | ((maxv is not None) << 1) | (bool(channel_wise) << 2)
    flags |= (factor is not None) << 3
    lib().ora_scale_intensity(x.ctypes.data, out.ctypes.data, _dt(x), B, C, x.size // (B * C),
                              float(minv or 0.0), float(maxv or 0.0), float(factor or 0.0),
                              int(flags), int(nthreads))
    return out


def bias_field(x, coeffs, mask=None, degree=3, nthreads=0):
    x = _c(x)
    B, C, H, W, D = x.shape
    co = _c(coeffs, np.float32)
    out = np.empty_like(x)
    m = _mask(mask, B)
    rc = lib().ora_bias_field(x.ctypes.data, out.ctypes.data, _dt(x), co.ctypes.data, _p(m), B,
                              C, H, W, D, int(degree), int(nthreads))
    if rc:
        raise ValueError("bias_field: unsupported degree")
    return out


def gaussian_1d_batch(sigmas, truncated=4.0):
    s = _c(np.asarray(sigmas, np.float32).ravel())
    B = s.size
    K = lib().ora_gaussian_1d_batch(s.ctypes.data, B, float(truncated), None)
    out = np.empty((B, K), np.float32)
    lib().ora_gaussian_1d_batch(s.ctypes.data, B, float(truncated), out.ctypes.data)
    return out


_SMOOTH_PADS = {None: 0, "constant": 0, "reflect": 1, "replicate": 2}


def separable_gauss(x, kh, kw, kd, padding_mode=None, nthreads=0):
    x = _c(x)
    B, C, H, W, D = x.shape
    kh, kw, kd = _c(kh, np.float32), _c(kw, np.float32), _c(kd, np.float32)
    out = np.empty_like(x)
    lib().ora_separable_gauss(x.ctypes.data, out.ctypes.data, _dt(x), kh.ctypes.data,
                              kh.shape[1], kw.ctypes.data, kw.shape[1], kd.ctypes.data,
                              kd.shape[1], B, C, H, W, D, _SMOOTH_PADS[padding_mode],
                              int(nthreads))
    return out


def elastic_grid(u, taps, magnitude, nthreads=0):
    """Grid (B,H,W,D,3) from a uniform draw u (B,3,H,W,D), taps (B,K) and
    per-element magnitude, as Rand3DElastic.sample_params builds it."""
    u = _c(u, np.float32)
    B, _, H, W, D = u.shape
    taps = _c(taps, np.float32)
    mag = _c(np.asarray(magnitude, np.float32).reshape(B))
    out = np.empty((B, H, W, D, 3), np.float32)
    lib().ora_elastic_grid(u.ctypes.data, taps.ctypes.data, taps.shape[1], mag.ctypes.data, B,
                           H, W, D, out.ctypes.data, int(nthreads))
    return out


def std_shift(x, factor, mask=None, nonzero=False, channel_wise=False, nthreads=0):
    """RandStdShiftIntensity.apply (scale_shift.py:130-198)."""
    x = _c(x)
    B, C = x.shape[:2]
    f = _c(np.asarray(factor, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_std_shift(x.ctypes.data, out.ctypes.data, _dt(x), f.ctypes.data, _p(m), B, C,
                        x.size // (B * C) if B * C else 0, int(bool(nonzero)),
                        int(bool(channel_wise)), int(nthreads))
    return out


def fixed_mean(x, factor, mask=None, channel_wise=False, nthreads=0):
    """RandScaleIntensityFixedMean.apply (scale_shift.py:201-274)."""
    x = _c(x)
    B, C = x.shape[:2]
    f = _c(np.asarray(factor, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_fixed_mean(x.ctypes.data, out.ctypes.data, _dt(x), f.ctypes.data, _p(m), B, C,
                         x.size // (B * C) if B * C else 0, int(bool(channel_wise)),
                         int(nthreads))
    return out


def rician(x, u1, u2, noise_std, mean=0.0, relative=False, mask=None, nthreads=0):
    """RandRicianNoise.apply (noise.py:146-164) with injected unit normals."""
    x = _c(x)
    B = x.shape[0]
    a1, a2 = _c(u1, np.float32), _c(u2, np.float32)
    sd = _c(np.asarray(noise_std, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_rician(x.ctypes.data, out.ctypes.data, _dt(x), a1.ctypes.data, a2.ctypes.data,
                     sd.ctypes.data, float(mean), int(bool(relative)), _p(m), B,
                     x.size // B if B else 0, int(nthreads))
    return out


def sharpen_combine(blurred, double_blurred, x, alpha, mask=None, nthreads=0):
    """blurred + alpha * (blurred - double_blurred) in the dtype, masked-out
    elements keep x (sharpen.py:117-136)."""
    bl, db, x = _c(blurred), _c(double_blurred), _c(x)
    B = x.shape[0]
    al = _c(np.asarray(alpha, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    lib().ora_sharpen_combine(bl.ctypes.data, db.ctypes.data, x.ctypes.data, out.ctypes.data,
                              _dt(x), al.ctypes.data, _p(m), B, x.size // max(B, 1),
                              int(nthreads))
    return out


def sharpen(x, kernels1, kernels2, alpha, mask=None, padding_mode=None, nthreads=0):
    """RandGaussianSharpen.apply (sharpen.py:117-136): two separable blurs,
    each cast to the dtype, then the unsharp-mask combination."""
    bl = separable_gauss(x, *kernels1, padding_mode=padding_mode, nthreads=nthreads)
    db = separable_gauss(bl, *kernels2, padding_mode=padding_mode, nthreads=nthreads)
    return sharpen_combine(bl, db, x, alpha, mask, nthreads=nthreads)


LOWRES_MODES = {"nearest": 0, "nearest-exact": 1, "trilinear": 2, "area": 3}


def lowres(x, zoom, mask=None, downsample_mode="nearest", upsample_mode="trilinear",
           align_corners=False, nthreads=0):
    """RandSimulateLowResolution.apply (resolution.py:74-118)."""
    x = _c(x)
    B, C, H, W, D = x.shape
    z = _c(np.asarray(zoom, np.float32).reshape(B))
    out = np.empty_like(x)
    m = _mask(mask, B)
    rc = lib().ora_lowres(x.ctypes.data, out.ctypes.data, _dt(x), B, C, H, W, D, z.ctypes.data,
                          _p(m), LOWRES_MODES[downsample_mode], LOWRES_MODES[upsample_mode],
                          int(bool(align_corners)), int(nthreads))
    if rc:
        raise ValueError("lowres: unsupported mode")
    return out


def compose_field(field, theta, mask_field=None, mask_affine=None):
    """The elastic grid (B,H,W,D,3) composed with the affine theta (B,3,4)
    that follows it (an extension; see oracle_compose.c)."""
    field = _c(field, np.float32)
    B, H, W, D, _ = field.shape
    th = _c(np.asarray(theta, np.float32).reshape(B, -1)[:, :12])
    out = np.empty_like(field)
    mf, ma = _mask(mask_field, B), _mask(mask_affine, B)  # held until the call returns
    lib().ora_compose_field(field.ctypes.data, th.ctypes.data, _p(mf), _p(ma), B, H, W, D,
                            out.ctypes.data)
    return out
