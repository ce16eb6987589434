"""Geometric transforms: RandAffine, RandAxisFlip, RandFlip, RandRotate90,
RandRotate, RandZoom, Rand3DElastic (+ dict wrappers).

Same constructors, params keys and ``to_affine`` convention as the reference
(batchaug/pytorch/geometric/*.py).  Every resample, eager or lazily fused,
is one ``ba_resample3d`` launch; eager flips and square-plane rot90s are the
nearest-mode resample of their exact affine, which lands on voxel centres and
therefore copies voxels bit for bit, as torch.flip / torch.rot90 do.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib as L
from . import _rng, ops
from .base import BatchDictTransform, BatchTransform, upload

_EYE = np.eye(4, dtype=np.float32)


def _eye_batch(B: int) -> np.ndarray:
    return np.broadcast_to(_EYE, (B, 4, 4)).copy()


def monai_affine_to_theta(affine: np.ndarray, spatial_shape) -> np.ndarray:
    """theta = P @ S_norm @ A @ S_inv @ P (affine.py:154-195).  Every product
    of the chain has one nonzero term, so theta[i][j] is
    fl(fl(sn[p(i)] * A[p(i)][p(j)]) * si[p(j)]) in fp32 — bit-identical to the
    reference's torch computation and to the kernel's in-register version."""
    H, W, D = spatial_shape
    a = np.asarray(affine, dtype=np.float32)
    sn = np.array([2.0 / H, 2.0 / W, 2.0 / D, 1.0], dtype=np.float32)
    si = np.array([H / 2.0, W / 2.0, D / 2.0, 1.0], dtype=np.float32)
    perm = [2, 1, 0, 3]
    pa = a[:, perm][:, :, perm]                       # A[p(i)][p(j)]
    th = (sn[perm][None, :, None] * pa).astype(np.float32)
    th = (th * si[perm][None, None, :]).astype(np.float32)
    return th


def _range_cols(spec, u: np.ndarray, ndim: int, add_scalar: float = 0.0) -> np.ndarray:
    """_sample_range (affine.py:119-151): None -> add_scalar; scalar s ->
    U(-s, s) + add_scalar; (lo, hi) -> U(lo, hi) + add_scalar, per axis."""
    if isinstance(spec, (int, float)):
        spec = [spec] * ndim
    B = u.shape[0]
    out = np.zeros((B, ndim), np.float32)
    for i, s in enumerate(spec):
        if s is None:
            out[:, i] = add_scalar
        elif isinstance(s, (int, float)):
            out[:, i] = u[:, i] * np.float32(2 * s) - np.float32(s) + np.float32(add_scalar)
        else:
            lo, hi = s
            out[:, i] = u[:, i] * np.float32(hi - lo) + np.float32(lo) + np.float32(add_scalar)
    return out


def _rotation(angles: np.ndarray) -> np.ndarray:
    """Rx(a0) @ Ry(a1) @ Rz(a2), MONAI order (affine.py:9-58)."""
    B = angles.shape[0]
    c, s = np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)
    rx, ry, rz = _eye_batch(B), _eye_batch(B), _eye_batch(B)
    rx[:, 1, 1], rx[:, 1, 2], rx[:, 2, 1], rx[:, 2, 2] = c[:, 0], -s[:, 0], s[:, 0], c[:, 0]
    ry[:, 0, 0], ry[:, 0, 2], ry[:, 2, 0], ry[:, 2, 2] = c[:, 1], s[:, 1], -s[:, 1], c[:, 1]
    rz[:, 0, 0], rz[:, 0, 1], rz[:, 1, 0], rz[:, 1, 1] = c[:, 2], -s[:, 2], s[:, 2], c[:, 2]
    return (rx @ ry @ rz).astype(np.float32)


def _masked_affine(mask: np.ndarray, affine: np.ndarray) -> np.ndarray:
    """to_affine: identity where masked out (affine.py:272-282)."""
    return np.where(mask[:, None, None], affine, _EYE[None]).astype(np.float32)


class _AffineFamily(BatchTransform):
    """Shared apply/to_affine of transforms whose params carry a MONAI
    affine and its theta (RandAffine, RandZoom)."""

    mode = "bilinear"
    padding_mode = "zeros"
    _host_keys = ("affine",)

    def _device_params(self, host, shape, device):
        theta = host.get("theta")
        if theta is None:
            theta = monai_affine_to_theta(host["affine"], shape[2:])
        p = upload({"mask": host["mask"], "affine": host["affine"], "theta": theta}, device)
        p["spatial_shape"] = tuple(shape[2:])
        return p

    def to_affine(self, params: dict) -> torch.Tensor:
        """(B,4,4) MONAI affine, identity for masked-out elements."""
        affine, mask = params["affine"], params["mask"]
        eye = torch.eye(4, device=affine.device, dtype=affine.dtype).expand(mask.shape[0], 4, 4)
        return torch.where(mask[:, None, None], affine, eye)

    def host_affine(self, params: dict) -> np.ndarray:
        h = params["_host"]
        return _masked_affine(h["mask"], h["affine"])

    def apply(self, tensor, params, mode=None, padding_mode=None):
        """grid_sample through params["theta"] (affine.py:284-317)."""
        return ops.resample3d(tensor, theta=params["theta"], mask=params["mask"],
                              modes=mode or self.mode,
                              paddings=padding_mode or self.padding_mode)

    def apply_keys(self, tensors, params, modes, paddings):
        """``apply`` of several tensors (same batch and spatial shape) with
        one launch: the coordinates are computed once for all of them."""
        return ops.resample3d(list(tensors), theta=params["theta"], mask=params["mask"],
                              modes=list(modes), paddings=list(paddings))


class RandAffine(_AffineFamily):
    """Random affine I @ R @ Sh @ T @ Sc per element (affine.py:198-317)."""

    _stream = _rng.S_AFFINE

    def __init__(self, prob: float = 0.1, rotate_range=None, shear_range=None,
                 translate_range=None, scale_range=None, mode: str = "bilinear",
                 padding_mode: str = "zeros"):
        super().__init__(prob=prob)
        self.rotate_range = rotate_range
        self.shear_range = shear_range
        self.translate_range = translate_range
        self.scale_range = scale_range
        self.mode = mode
        self.padding_mode = padding_mode

    def _n_uniforms(self, shape):
        return 16  # mask, 3 angles, 6 shears, 3 shifts, 3 scales

    def _range_table(self):
        """(a, b, c, present, groups) of ba_host_rand_affine for this
        transform's ranges, following _sample_range (affine.py:119-151):
        None -> the fixed value c; scalar s -> U(-s, s) + c; (lo, hi) ->
        U(lo, hi) + c."""
        key = (self.rotate_range, self.shear_range, self.translate_range, self.scale_range)
        if getattr(self, "_table_key", None) == key:
            return self._table
        a = np.zeros(15, np.float32)
        b = np.zeros(15, np.float32)
        c = np.zeros(15, np.float32)
        present = groups = 0
        for g, (spec, first, n, add) in enumerate([(self.rotate_range, 0, 3, 0.0),
                                                    (self.shear_range, 3, 6, 0.0),
                                                    (self.translate_range, 9, 3, 0.0),
                                                    (self.scale_range, 12, 3, 1.0)]):
            if spec is None:
                continue
            groups |= 1 << g
            entries = [spec] * n if isinstance(spec, (int, float)) else list(spec)
            for i, e in enumerate(entries):
                k = first + i
                c[k] = add
                if e is None:
                    continue
                present |= 1 << k
                if isinstance(e, (int, float)):
                    a[k], b[k] = np.float32(2 * e), -np.float32(e)
                else:
                    lo, hi = e
                    a[k], b[k] = np.float32(hi - lo), np.float32(lo)
        self._table_key, self._table = key, (a, b, c, present, groups)
        return self._table

    def _host_params(self, B, shape, u, seed):
        a, b, c, present, groups = self._range_table()
        H, W, D = shape[2:]
        u = np.ascontiguousarray(u, dtype=np.float32)
        mask = np.empty(B, np.uint8)
        affine = np.empty((B, 4, 4), np.float32)
        theta = np.empty((B, 4, 4), np.float32)
        ops.host_rand_affine(u, self.prob, a, b, c, present, groups, (H, W, D), mask, affine,
                             theta)
        return {"mask": mask.view(np.bool_), "affine": affine, "theta": theta}


class RandZoom(_AffineFamily):
    """Isotropic zoom z ~ U(min_zoom, max_zoom), affine diag 1/z (zoom.py:10-121)."""

    _stream = _rng.S_ZOOM

    def __init__(self, prob: float = 0.1, min_zoom: float = 0.9, max_zoom: float = 1.1,
                 mode: str = "bilinear", padding_mode: str = "border"):
        super().__init__(prob=prob)
        self.min_zoom, self.max_zoom = min_zoom, max_zoom
        self.mode, self.padding_mode = mode, padding_mode

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        zoom = (u[:, 1] * np.float32(self.max_zoom - self.min_zoom)
                + np.float32(self.min_zoom)).astype(np.float32)
        scale = (np.float32(1.0) / zoom).astype(np.float32)
        affine = _eye_batch(B)
        affine[:, 0, 0] = affine[:, 1, 1] = affine[:, 2, 2] = scale
        return {"mask": u[:, 0] < self.prob, "affine": affine, "zoom": zoom}

    def _device_params(self, host, shape, device):
        p = super()._device_params(host, shape, device)
        p["zoom"] = upload({"zoom": host["zoom"]}, device)["zoom"]
        return p


class RandRotate(RandAffine):
    """RandAffine with rotation only (rotate.py:6-40)."""

    def __init__(self, prob: float = 0.1, range_x=0.0, range_y=0.0, range_z=0.0,
                 mode: str = "bilinear", padding_mode: str = "border"):
        super().__init__(prob=prob, rotate_range=[range_x, range_y, range_z], mode=mode,
                         padding_mode=padding_mode)


class RandAxisFlip(BatchTransform):
    """Flip one random spatial axis per element (flip.py:8-66)."""

    _stream = _rng.S_FLIP
    _host_keys = ("axes",)

    def __init__(self, prob: float = 0.1):
        super().__init__(prob=prob)

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        n = len(shape) - 2
        axes = np.minimum((u[:, 1] * n).astype(np.int64), n - 1)
        return {"mask": u[:, 0] < self.prob, "axes": axes}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "axes": host["axes"]}, device)

    @staticmethod
    def _flip_affine(mask: np.ndarray, axes: np.ndarray) -> np.ndarray:
        a = _eye_batch(mask.shape[0])
        for ax in range(3):
            sel = mask & (axes == ax)
            a[sel, ax, ax] = -1.0
        return a

    def host_affine(self, params):
        h = params["_host"] if "_host" in params else _to_host(params, ("mask", "axes"))
        return self._flip_affine(h["mask"], h["axes"])

    def to_affine(self, params):
        return torch.from_numpy(self.host_affine(params)).to(params["mask"].device)

    def apply(self, tensor, params):
        # An exact voxel permutation: the nearest resample of the flip affine.
        return ops.resample3d(tensor, affine=self.host_affine(params), modes="nearest",
                              mask=_host_mask(params))


class RandFlip(BatchTransform):
    """Flip the listed spatial axes (all when None) together (flip.py:80-148)."""

    _stream = _rng.S_FLIP

    def __init__(self, prob: float = 0.1, spatial_axis=None):
        super().__init__(prob=prob)
        if spatial_axis is None:
            self._spatial_axes = None
        elif isinstance(spatial_axis, int):
            self._spatial_axes = [spatial_axis]
        else:
            self._spatial_axes = list(spatial_axis)

    def host_affine(self, params):
        h = params["_host"] if "_host" in params else _to_host(params, ("mask",))
        mask = h["mask"]
        a = _eye_batch(mask.shape[0])
        for ax in (self._spatial_axes if self._spatial_axes is not None else [0, 1, 2]):
            a[mask, ax, ax] = -1.0
        return a

    def to_affine(self, params):
        return torch.from_numpy(self.host_affine(params)).to(params["mask"].device)

    def apply(self, tensor, params):
        return ops.resample3d(tensor, affine=self.host_affine(params), modes="nearest",
                              mask=_host_mask(params))


class RandRotate90(BatchTransform):
    """k*90 degree rotation, k in 1..max_k, in spatial_axes (rotate90.py:10-112)."""

    _stream = _rng.S_ROT90
    _host_keys = ("k",)

    def __init__(self, prob: float = 0.1, max_k: int = 3, spatial_axes=(0, 1)):
        super().__init__(prob=prob)
        self.max_k = max_k
        self.spatial_axes = spatial_axes

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        k = 1 + np.minimum((u[:, 1] * self.max_k).astype(np.int64), self.max_k - 1)
        return {"mask": u[:, 0] < self.prob, "k": k}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "k": host["k"]}, device)

    def host_affine(self, params):
        h = params["_host"] if "_host" in params else _to_host(params, ("mask", "k"))
        mask, kv = h["mask"], h["k"]
        a = _eye_batch(mask.shape[0])
        ax0, ax1 = self.spatial_axes
        # resampling (inverse) convention, rotate90.py:61-62
        cos_t, sin_t = [0.0, -1.0, 0.0], [-1.0, 0.0, 1.0]
        for k in range(1, self.max_k + 1):
            sel = mask & (kv == k)
            c, s = cos_t[(k - 1) % 3], sin_t[(k - 1) % 3]
            a[sel, ax0, ax0] = c
            a[sel, ax0, ax1] = -s
            a[sel, ax1, ax0] = s
            a[sel, ax1, ax1] = c
        return a

    def to_affine(self, params):
        return torch.from_numpy(self.host_affine(params)).to(params["mask"].device)

    def apply(self, tensor, params):
        ax = [a + 2 for a in self.spatial_axes]
        if tensor.shape[ax[0]] == tensor.shape[ax[1]]:
            # square plane: torch.rot90 is an exact voxel permutation
            return ops.resample3d(tensor, affine=self.host_affine(params), modes="nearest",
                                  mask=_host_mask(params))
        # non-square plane: the reference's bilinear/zeros grid_sample fallback
        return ops.resample3d(tensor, affine=self.host_affine(params), modes="bilinear",
                              paddings="zeros", mask=_host_mask(params))


class Rand3DElastic(BatchTransform):
    """Smoothed random displacement field + grid_sample(align_corners=True)
    (elastic.py:10-125).  No ``to_affine``: as in the reference, a lazy
    Compose materialises pending affines before it and resamples eagerly."""

    _stream = _rng.S_ELASTIC

    def __init__(self, prob: float = 0.1, sigma_range=(3.0, 3.0), magnitude_range=(0.0, 0.1),
                 mode: str = "bilinear", padding_mode: str = "zeros"):
        super().__init__(prob=prob)
        self.sigma_range = sigma_range
        self.magnitude_range = magnitude_range
        self.mode = mode
        self.padding_mode = padding_mode

    def sample_host(self, batch_size, shape):
        seed = _rng.draw_seed()
        u_all, row = _rng.global_uniforms(seed, self._stream, batch_size, 3)
        s_lo, s_hi = self.sigma_range
        m_lo, m_hi = self.magnitude_range
        sig_all = (u_all[:, 1] * np.float32(s_hi - s_lo) + np.float32(s_lo)).astype(np.float32)
        u = u_all[row:row + batch_size]
        return {"mask": u[:, 0] < self.prob,
                "sigma": sig_all[row:row + batch_size],
                "magnitude": (u[:, 2] * np.float32(m_hi - m_lo) + np.float32(m_lo)).astype(np.float32),
                # gaussian_1d_batch pads to the (global) batch-max tail (smooth.py:24-25)
                "max_sigma": float(np.maximum(sig_all, np.float32(1e-6)).max()) if len(sig_all) else 1e-6,
                "seed": seed}

    def sample_params(self, batch_size, shape, device):
        host = self.sample_host(batch_size, shape)
        p = upload({"mask": host["mask"], "sigma": host["sigma"],
                    "magnitude": host["magnitude"]}, device)
        H, W, D = shape[2:]
        K = ops.gauss_taps_len(host["max_sigma"], 3.0)
        taps = ops.gauss_taps(p["sigma"], K)
        p["grid"] = ops.elastic_grid((batch_size, H, W, D), taps, p["magnitude"],
                                     seed=host["seed"], elem_offset=_rng.element_offset(),
                                     device=torch.device(device))
        p["_host"] = host
        return p

    def apply(self, tensor, params, mode=None, padding_mode=None):
        return ops.resample3d(tensor, grid=params["grid"], mask=params["mask"],
                              modes=mode or self.mode,
                              paddings=padding_mode or self.padding_mode, align_corners=True)

    def apply_keys(self, tensors, params, modes, paddings):
        """``apply`` of several tensors (same batch and spatial shape) with
        one launch reading the grid once."""
        return ops.resample3d(list(tensors), grid=params["grid"], mask=params["mask"],
                              modes=list(modes), paddings=list(paddings), align_corners=True)


def _host_mask(params: dict) -> np.ndarray:
    """The params' mask on the host: the copy sample_params keeps, else a
    device read of an injected mask.  A host mask (with a host transform)
    travels in the resample's kernel parameters."""
    if "_host" in params and "mask" in params["_host"]:
        return np.asarray(params["_host"]["mask"])
    m = params["mask"]
    return m.detach().cpu().numpy() if isinstance(m, torch.Tensor) else np.asarray(m)


def _to_host(params: dict, keys) -> dict:
    """Host copies of injected device params (a device read; only used when
    params did not come from this package's sample_params)."""
    return {k: params[k].detach().cpu().numpy() for k in keys}


# ---------------------------------------------------------------------------
# Dict wrappers
# ---------------------------------------------------------------------------

class _PerKeyModes:
    """Dict wrapper with per-key mode/padding (affine.py:320-378)."""

    _default_padding = "zeros"

    def __init__(self, keys, transform, mode="bilinear", padding_mode=None):
        self.keys = keys
        self.transform = transform
        padding_mode = self._default_padding if padding_mode is None else padding_mode
        self._mode = {k: mode for k in keys} if isinstance(mode, str) else mode
        self._padding_mode = ({k: padding_mode for k in keys} if isinstance(padding_mode, str)
                              else padding_mode)

    def __call__(self, data, params: dict | None = None):
        """``params``: optional injected params (as ``sample_params`` returns
        them, e.g. the reference's own) instead of sampling."""
        d = dict(data)
        if params is None:
            first = d[self.keys[0]]
            params = self.transform.sample_params(first.shape[0], first.shape, first.device)
        else:
            params = self.transform.adopt_params(params)
        mode = lambda k: self._mode.get(k, "bilinear")  # noqa: E731
        pad = lambda k: self._padding_mode.get(k, self._default_padding)  # noqa: E731
        keys = [k for k in self.keys if k in d]
        if hasattr(self.transform, "apply_keys"):
            # keys with one batch and spatial shape share one launch (the
            # same per-key arithmetic as applying them one at a time)
            groups: dict[tuple, list] = {}
            for k in keys:
                t = d[k]
                groups.setdefault((t.shape[0], tuple(t.shape[2:]), t.device), []).append(k)
            for ks in groups.values():
                for i in range(0, len(ks), L.BA_MAX_KEYS):
                    chunk = ks[i:i + L.BA_MAX_KEYS]
                    outs = self.transform.apply_keys([d[k] for k in chunk], params,
                                                     [mode(k) for k in chunk],
                                                     [pad(k) for k in chunk])
                    for k, o in zip(chunk, outs):
                        d[k] = o
            return d
        for key in keys:
            d[key] = self.transform.apply(d[key], params, mode=mode(key), padding_mode=pad(key))
        return d


class RandAffined(_PerKeyModes):
    def __init__(self, keys, prob: float = 0.1, rotate_range=None, shear_range=None,
                 translate_range=None, scale_range=None, mode="bilinear", padding_mode="zeros"):
        super().__init__(keys, RandAffine(prob=prob, rotate_range=rotate_range,
                                          shear_range=shear_range,
                                          translate_range=translate_range,
                                          scale_range=scale_range), mode, padding_mode)


class RandZoomd(_PerKeyModes):
    _default_padding = "border"

    def __init__(self, keys, prob: float = 0.1, min_zoom: float = 0.9, max_zoom: float = 1.1,
                 mode="bilinear", padding_mode="border"):
        super().__init__(keys, RandZoom(prob=prob, min_zoom=min_zoom, max_zoom=max_zoom), mode,
                         padding_mode)


class Rand3DElasticd(_PerKeyModes):
    def __init__(self, keys, prob: float = 0.1, sigma_range=(3.0, 3.0),
                 magnitude_range=(0.0, 0.1), mode="bilinear", padding_mode="zeros"):
        super().__init__(keys, Rand3DElastic(prob=prob, sigma_range=sigma_range,
                                             magnitude_range=magnitude_range), mode,
                         padding_mode)


class RandRotated:
    """Dict RandRotate (rotate.py:43-77).  Like the reference it wraps a
    RandAffined privately and exposes no ``transform``, so a lazy Compose
    applies it eagerly rather than fusing it."""

    def __init__(self, keys, prob: float = 0.1, range_x=0.0, range_y=0.0, range_z=0.0,
                 mode="bilinear", padding_mode="border"):
        self._inner = RandAffined(keys=keys, prob=prob, rotate_range=[range_x, range_y, range_z],
                                  mode=mode, padding_mode=padding_mode)

    def __call__(self, data, params: dict | None = None):
        return self._inner(data, params=params)


class RandAxisFlipd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1):
        super().__init__(keys=keys, transform=RandAxisFlip(prob=prob))


class RandFlipd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, spatial_axis=None):
        super().__init__(keys=keys, transform=RandFlip(prob=prob, spatial_axis=spatial_axis))


class RandRotate90d(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, max_k: int = 3, spatial_axes=(0, 1)):
        super().__init__(keys=keys, transform=RandRotate90(prob=prob, max_k=max_k,
                                                           spatial_axes=spatial_axes))
