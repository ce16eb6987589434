"""Intensity transforms: RandGaussianNoise, RandRicianNoise,
RandAdjustContrast, RandScaleIntensity, RandShiftIntensity,
RandStdShiftIntensity, RandScaleIntensityFixedMean, RandBiasField,
ScaleIntensity, RandGaussianSmooth, RandGaussianSharpen,
RandSimulateLowResolution (+ dict wrappers).

Constructors, params keys and results follow the reference PyTorch backend
(batchaug/pytorch/intensity/*.py), op by op in the tensor dtype.  Each
``apply`` is one fused ``ba_intensity_chain`` (or ``ba_smooth3d``) call; a
``Compose`` fuses consecutive transforms of this module into a single chain
per key (see :meth:`_FusibleIntensity.chain_op`).

Gaussian (and Rician) noise is generated in-kernel from the params'
``noise_seed`` (Philox4x32-10 keyed on the global element index and voxel
position) and is never materialised; params holding explicit ``"noise"`` (or
``"u1"``/``"u2"``) tensors (the reference's params, or a test's injected
noise) are applied as given.  The statistics that RandStdShiftIntensity,
RandScaleIntensityFixedMean and relative RandRicianNoise read (mean, std of
their input) are reduced in the pass that produces that input.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib as L
from . import _rng, ops
from .base import BatchDictTransform, BatchTransform, upload


def _parse_range(param) -> tuple[float, float]:
    """Scalar v -> (-v, v); (lo, hi) unchanged (scale_shift.py:8-16)."""
    if isinstance(param, (int, float)):
        v = float(param)
        return (-v, v)
    return (float(param[0]), float(param[1]))


def _dev(params: dict, key: str, device) -> torch.Tensor:
    t = params[key]
    return t if t.device == device else t.to(device)


def _mask_u8(params: dict, device) -> torch.Tensor:
    m = params["mask"]
    if m.device != device:
        m = m.to(device)
    return m.view(torch.uint8) if m.dtype == torch.bool else (m != 0).to(torch.uint8)


class _FusibleIntensity(BatchTransform):
    """An intensity transform that is one op of ba_intensity_chain."""

    def chain_op(self, params: dict, tensor: torch.Tensor) -> ops.ChainOp:
        raise NotImplementedError

    def chain_params(self, batch_size: int, shape, device) -> dict:
        """``sample_params`` for a Compose chain, which reads the host copies:
        the same draws, but device tensors only when the op selects some
        element (a chain leaves an op that selects none out)."""
        host = self.sample_host(batch_size, shape)
        if not np.asarray(host["mask"]).any():
            return {"_host": host}
        params = self._device_params(host, tuple(shape), device)
        params["_host"] = host
        return params

    def apply(self, tensor: torch.Tensor, params: dict) -> torch.Tensor:
        return ops.intensity_chain(tensor, [self.chain_op(params, tensor)])


class RandGaussianNoise(_FusibleIntensity):
    """x + noise * mask with noise ~ N(mean, std) per element (noise.py:8-66)."""

    _stream = _rng.S_NOISE

    def __init__(self, prob: float = 0.1, mean=0.0, std=0.1):
        super().__init__(prob=prob)
        self.mean = mean
        self.std = std

    def _n_uniforms(self, shape):
        return 3

    @staticmethod
    def _scalar(param, col: np.ndarray) -> np.ndarray:
        if isinstance(param, (list, tuple)):
            lo, hi = param
            return (col * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)
        return np.full(col.shape, param, np.float32)

    def _host_params(self, B, shape, u, seed):
        return {"mask": u[:, 0] < self.prob, "std": self._scalar(self.std, u[:, 1]),
                "mean": self._scalar(self.mean, u[:, 2]), "noise_seed": seed}

    def _device_params(self, host, shape, device):
        p = upload({"mask": host["mask"], "std": host["std"], "mean": host["mean"]}, device)
        p["noise_seed"] = host["noise_seed"]
        p["elem_offset"] = _rng.element_offset()
        return p

    def chain_op(self, params, tensor):
        dev = tensor.device
        if "noise" in params:  # injected noise tensor (already * std + mean)
            noise = params["noise"].to(device=dev, dtype=torch.float32).contiguous()
            if noise.shape != tensor.shape:
                raise ValueError(f"noise shape {tuple(noise.shape)} != tensor shape "
                                 f"{tuple(tensor.shape)}")
            return ops.ChainOp(L.BA_OP_NOISE, mask=_mask_u8(params, dev), noise=noise)
        return ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, mask=_mask_u8(params, dev),
                           param=_dev(params, "std", dev), param2=_dev(params, "mean", dev),
                           seed=params["noise_seed"], elem_offset=params.get("elem_offset", 0))


class RandAdjustContrast(_FusibleIntensity):
    """Gamma on per-element min/max, fp32 (contrast.py:88-131)."""

    _stream = _rng.S_CONTRAST

    def __init__(self, prob: float = 0.1, gamma=(0.5, 4.5)):
        super().__init__(prob=prob)
        self.gamma = gamma

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        lo, hi = self.gamma
        return {"mask": u[:, 0] < self.prob,
                "gamma": (u[:, 1] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "gamma": host["gamma"]}, device)

    def chain_op(self, params, tensor):
        dev = tensor.device
        return ops.ChainOp(L.BA_OP_CONTRAST, mask=_mask_u8(params, dev),
                           param=_dev(params, "gamma", dev))


class RandScaleIntensity(_FusibleIntensity):
    """x * (1 + factor) in the tensor dtype (scale_shift.py:19-56)."""

    _stream = _rng.S_SCALE

    def __init__(self, prob: float = 0.1, factors=(0.0, 0.5)):
        super().__init__(prob=prob)
        self.factors = _parse_range(factors)

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        lo, hi = self.factors
        return {"mask": u[:, 0] < self.prob,
                "factor": (u[:, 1] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "factor": host["factor"]}, device)

    def chain_op(self, params, tensor):
        dev = tensor.device
        return ops.ChainOp(L.BA_OP_SCALE, mask=_mask_u8(params, dev),
                           param=_dev(params, "factor", dev))


class RandShiftIntensity(_FusibleIntensity):
    """x + offset in the tensor dtype, optional clamp (scale_shift.py:72-113)."""

    _stream = _rng.S_SHIFT

    def __init__(self, prob: float = 0.1, offsets=(-0.1, 0.1), safe: bool = False):
        super().__init__(prob=prob)
        self.offsets = _parse_range(offsets)
        self.safe = safe

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        lo, hi = self.offsets
        return {"mask": u[:, 0] < self.prob,
                "offset": (u[:, 1] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "offset": host["offset"]}, device)

    def chain_op(self, params, tensor):
        dev = tensor.device
        return ops.ChainOp(L.BA_OP_SHIFT, flags=L.BA_SHIFT_SAFE if self.safe else 0,
                           mask=_mask_u8(params, dev), param=_dev(params, "offset", dev))


class RandBiasField(_FusibleIntensity):
    """x * exp(sum c * L_i L_j L_k), Legendre basis evaluated in-kernel
    (bias_field.py:56-112)."""

    _stream = _rng.S_BIAS
    _subsettable = True

    def __init__(self, prob: float = 0.1, degree: int = 3, coeff_range=(0.0, 0.1)):
        super().__init__(prob=prob)
        if degree < 1:
            raise ValueError(f"degree should be no less than 1, got {degree}.")
        self.degree = degree
        self.coeff_range = coeff_range

    @property
    def n_coeff(self) -> int:
        d = self.degree
        return (d + 1) * (d + 2) * (d + 3) // 6

    def _n_uniforms(self, shape):
        return 1 + self.n_coeff

    def _host_params(self, B, shape, u, seed):
        lo, hi = self.coeff_range
        return {"mask": u[:, 0] < self.prob,
                "coeffs": (u[:, 1:] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "coeffs": host["coeffs"]}, device)

    def chain_op(self, params, tensor):
        dev = tensor.device
        coeffs = params["coeffs"].to(device=dev, dtype=torch.float32).contiguous()
        if tuple(coeffs.shape) != (tensor.shape[0], self.n_coeff):
            raise ValueError(f"coeffs must be {(tensor.shape[0], self.n_coeff)} for degree "
                             f"{self.degree}, got {tuple(coeffs.shape)}")
        return ops.ChainOp(L.BA_OP_BIAS_FIELD, mask=_mask_u8(params, dev), param=coeffs,
                           degree=self.degree)


class RandRicianNoise(_FusibleIntensity):
    """sqrt((x + n1)^2 + n2^2) with n = mean + std * u, u ~ N(0, 1) per
    voxel, in fp32 (noise.py:86-164).  ``relative`` multiplies the element's
    std by the (unbiased) std of its input over all channels.

    The unit draws u1, u2 come from Philox in-kernel (keyed on the params'
    ``noise_seed``, the global element index and the voxel); params holding
    explicit ``"u1"`` and ``"u2"`` tensors (the reference's params) are
    applied as given."""

    _stream = _rng.S_RICIAN

    def __init__(self, prob: float = 0.1, mean: float = 0.0, std: float = 0.1,
                 relative: bool = False, sample_std: bool = True):
        super().__init__(prob=prob)
        self.mean = mean
        self.std = std
        self.relative = relative
        self.sample_std = sample_std

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        if self.sample_std:
            noise_std = (u[:, 1] * np.float32(self.std)).astype(np.float32)
        else:
            noise_std = np.full((B,), self.std, np.float32)
        return {"mask": u[:, 0] < self.prob, "noise_std": noise_std, "noise_seed": seed}

    def _device_params(self, host, shape, device):
        p = upload({"mask": host["mask"], "noise_std": host["noise_std"]}, device)
        p["noise_seed"] = host["noise_seed"]
        p["elem_offset"] = _rng.element_offset()
        return p

    def chain_op(self, params, tensor):
        dev = tensor.device
        flags = L.BA_RICIAN_RELATIVE if self.relative else 0
        std = _dev(params, "noise_std", dev).to(torch.float32).contiguous()
        if "u1" in params or "u2" in params:
            u = []
            for name in ("u1", "u2"):
                t = params[name].to(device=dev, dtype=torch.float32).contiguous()
                if t.shape != tensor.shape:
                    raise ValueError(f"{name} shape {tuple(t.shape)} != tensor shape "
                                     f"{tuple(tensor.shape)}")
                u.append(t)
            return ops.ChainOp(L.BA_OP_RICIAN, flags=flags, mask=_mask_u8(params, dev), param=std,
                               noise=u[0], param2=u[1], c0=float(self.mean))
        return ops.ChainOp(L.BA_OP_RICIAN, flags=flags | L.BA_RICIAN_PHILOX,
                           mask=_mask_u8(params, dev), param=std, c0=float(self.mean),
                           seed=params["noise_seed"], elem_offset=params.get("elem_offset", 0))


class _FactorIntensity(_FusibleIntensity):
    """A transform with one factor ~ U(lo, hi) per element."""

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        lo, hi = self.factors
        return {"mask": u[:, 0] < self.prob,
                "factor": (u[:, 1] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)}

    def _device_params(self, host, shape, device):
        return upload({"mask": host["mask"], "factor": host["factor"]}, device)


class RandStdShiftIntensity(_FactorIntensity):
    """x + factor * std, fp32 then one cast (scale_shift.py:120-198).  The
    std is unbiased, over the element (or each channel with
    ``channel_wise``); ``nonzero`` takes it over the nonzero voxels when
    there are at least two of them."""

    _stream = _rng.S_STD_SHIFT

    def __init__(self, prob: float = 0.1, factors=(-3.0, 3.0), nonzero: bool = False,
                 channel_wise: bool = False):
        super().__init__(prob=prob)
        self.factors = _parse_range(factors)
        self.nonzero = nonzero
        self.channel_wise = channel_wise

    def chain_op(self, params, tensor):
        dev = tensor.device
        flags = (L.BA_STD_NONZERO if self.nonzero else 0) | \
            (L.BA_STAT_CHANNEL if self.channel_wise else 0)
        return ops.ChainOp(L.BA_OP_STD_SHIFT, flags=flags, mask=_mask_u8(params, dev),
                           param=_dev(params, "factor", dev).to(torch.float32).contiguous())


class RandScaleIntensityFixedMean(_FactorIntensity):
    """mean + (x - mean) * (1 + factor), fp32 then one cast, the mean over
    the element (or each channel with ``channel_wise``)
    (scale_shift.py:219-274)."""

    _stream = _rng.S_FIXED_MEAN

    def __init__(self, prob: float = 0.1, factors=(-0.5, 0.5), channel_wise: bool = False):
        super().__init__(prob=prob)
        self.factors = _parse_range(factors)
        self.channel_wise = channel_wise

    def chain_op(self, params, tensor):
        dev = tensor.device
        return ops.ChainOp(L.BA_OP_FIXED_MEAN,
                           flags=L.BA_STAT_CHANNEL if self.channel_wise else 0,
                           mask=_mask_u8(params, dev),
                           param=_dev(params, "factor", dev).to(torch.float32).contiguous())


class ScaleIntensity(_FusibleIntensity):
    """Rescale to [minv, maxv] with per-(element, channel) or per-element
    min/max, in the tensor dtype (contrast.py:8-68)."""

    def __init__(self, minv=0.0, maxv=1.0, factor=None, channel_wise: bool = True):
        super().__init__(prob=1.0)
        self.minv = minv
        self.maxv = maxv
        self.factor = factor
        self.channel_wise = channel_wise

    def takes_stats(self) -> bool:
        """True when the rescale can use per-(element, channel) min/max made
        elsewhere (``ops.resample3d(..., minmax=...)``) instead of reducing
        its input itself."""
        return self.factor is None and self.channel_wise and (
            self.minv is not None or self.maxv is not None)

    def chain_op(self, params, tensor, stats=None):
        if self.factor is not None:
            return ops.ChainOp(L.BA_OP_RESCALE, flags=L.BA_RESCALE_FACTOR, c0=self.factor)
        flags = 0
        if self.minv is not None:
            flags |= L.BA_RESCALE_MINV
        if self.maxv is not None:
            flags |= L.BA_RESCALE_MAXV
        if self.channel_wise:
            flags |= L.BA_RESCALE_CHANNEL
        if stats is not None and self.takes_stats():
            flags |= L.BA_RESCALE_GIVEN
        else:
            stats = None
        return ops.ChainOp(L.BA_OP_RESCALE, flags=flags, c0=self.minv or 0.0,
                           c1=self.maxv or 0.0, stats=stats)

    def chain_params(self, batch_size, shape, device):
        # chain_op reads no params: nothing to upload
        return {"_host": self.sample_host(batch_size, shape)}

    def apply(self, tensor, params):
        if self.factor is None and self.minv is None and self.maxv is None:
            return tensor
        return super().apply(tensor, params)


class RandGaussianSmooth(BatchTransform):
    """Separable Gaussian blur with per-element, per-axis sigma
    (smooth.py:91-143)."""

    _stream = _rng.S_SMOOTH
    _subsettable = True

    def __init__(self, prob: float = 0.1, sigma_x=(0.25, 1.5), sigma_y=(0.25, 1.5),
                 sigma_z=(0.25, 1.5), padding_mode=None):
        super().__init__(prob=prob)
        self.sigma_x, self.sigma_y, self.sigma_z = sigma_x, sigma_y, sigma_z
        self.padding_mode = padding_mode

    def sample_host(self, batch_size, shape):
        seed = _rng.draw_seed()
        u_all, row = _rng.global_uniforms(seed, self._stream, batch_size, 4)
        host = {"mask": u_all[row:row + batch_size, 0] < self.prob}
        for i, (name, rng) in enumerate((("sigma_x", self.sigma_x), ("sigma_y", self.sigma_y),
                                         ("sigma_z", self.sigma_z))):
            lo, hi = rng
            s_all = (u_all[:, 1 + i] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)
            host[name] = s_all[row:row + batch_size]
            # gaussian_1d_batch pads every kernel to the batch-max tail
            host["K_" + name] = ops.gauss_taps_len(
                float(np.maximum(s_all, np.float32(1e-6)).max()) if len(s_all) else 1e-6, 4.0)
        return host

    def sample_params(self, batch_size, shape, device):
        host = self.sample_host(batch_size, shape)
        p = upload({k: host[k] for k in ("mask", "sigma_x", "sigma_y", "sigma_z")}, device)
        p["kernel_h"] = ops.gauss_taps(p["sigma_x"], host["K_sigma_x"])
        p["kernel_w"] = ops.gauss_taps(p["sigma_y"], host["K_sigma_y"])
        p["kernel_d"] = ops.gauss_taps(p["sigma_z"], host["K_sigma_z"])
        p["_host"] = host
        return p

    def apply(self, tensor, params):
        return ops.smooth3d(tensor, params["kernel_h"], params["kernel_w"], params["kernel_d"],
                            mask=params["mask"], padding_mode=self.padding_mode)


class RandGaussianSharpen(BatchTransform):
    """Unsharp masking blurred + alpha * (blurred - double_blurred) with two
    separable Gaussian blurs (sharpen.py:9-136).  A scalar sigma2 samples
    from [sigma2, sigma1] per element, a tuple from its range.  One
    ``ba_sharpen3d`` call: the second blur's last pass writes the
    combination."""

    _stream = _rng.S_SHARPEN
    _subsettable = True

    def __init__(self, prob: float = 0.1, sigma1_x=(0.5, 1.0), sigma1_y=(0.5, 1.0),
                 sigma1_z=(0.5, 1.0), sigma2_x=0.5, sigma2_y=0.5, sigma2_z=0.5,
                 alpha=(10.0, 30.0), padding_mode=None):
        super().__init__(prob=prob)
        self.sigma1_x, self.sigma1_y, self.sigma1_z = sigma1_x, sigma1_y, sigma1_z
        self.sigma2_x, self.sigma2_y, self.sigma2_z = sigma2_x, sigma2_y, sigma2_z
        self.alpha = alpha
        self.padding_mode = padding_mode

    @staticmethod
    def _range(col: np.ndarray, rng) -> np.ndarray:
        lo, hi = rng
        return (col * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)

    @staticmethod
    def _sigma2(col: np.ndarray, param, sigma1: np.ndarray) -> np.ndarray:
        """sharpen.py:61-75: scalar -> U(param, sigma1), tuple -> U(lo, hi)."""
        if isinstance(param, (int, float)):
            lo = np.float32(param)
            return (col * (sigma1 - lo) + lo).astype(np.float32)
        return RandGaussianSharpen._range(col, param)

    def sample_host(self, batch_size, shape):
        # draw order of sharpen.py:77-113: mask, sigma1 x/y/z, sigma2 x/y/z, alpha
        seed = _rng.draw_seed()
        u_all, row = _rng.global_uniforms(seed, self._stream, batch_size, 8)
        full = {"mask": u_all[:, 0] < self.prob}
        for i, a in enumerate("xyz"):
            full[f"sigma1_{a}"] = self._range(u_all[:, 1 + i], getattr(self, f"sigma1_{a}"))
        for i, a in enumerate("xyz"):
            full[f"sigma2_{a}"] = self._sigma2(u_all[:, 4 + i], getattr(self, f"sigma2_{a}"),
                                               full[f"sigma1_{a}"])
        full["alpha"] = self._range(u_all[:, 7], self.alpha)
        host = {k: v[row:row + batch_size] for k, v in full.items()}
        # gaussian_1d_batch sizes each kernel set by its batch-max sigma
        for k in ("sigma1_x", "sigma1_y", "sigma1_z", "sigma2_x", "sigma2_y", "sigma2_z"):
            s_all = full[k]
            host["K_" + k] = ops.gauss_taps_len(
                float(np.maximum(s_all, np.float32(1e-6)).max()) if len(s_all) else 1e-6, 4.0)
        return host

    def sample_params(self, batch_size, shape, device):
        host = self.sample_host(batch_size, shape)
        keys = ("mask", "alpha", "sigma1_x", "sigma1_y", "sigma1_z", "sigma2_x", "sigma2_y",
                "sigma2_z")
        p = upload({k: host[k] for k in keys}, device)
        for n in "12":
            for a, ax in zip("xyz", "hwd"):
                p[f"kernel{n}_{ax}"] = ops.gauss_taps(p[f"sigma{n}_{a}"], host[f"K_sigma{n}_{a}"])
        p["_host"] = host
        return p

    def apply(self, tensor, params):
        return ops.sharpen3d(tensor, [params[f"kernel1_{a}"] for a in "hwd"],
                             [params[f"kernel2_{a}"] for a in "hwd"], params["alpha"],
                             mask=params["mask"], padding_mode=self.padding_mode)


class RandSimulateLowResolution(BatchTransform):
    """Downsample each element by a zoom factor ~ U(zoom_range) and upsample
    back (resolution.py:9-118); any of the 5-D F.interpolate modes
    ("nearest", "nearest-exact", "trilinear", "area") for either step,
    align_corners on a trilinear step.  One ``ba_lowres3d`` call; the
    per-target-size groups of the reference need no grouping here."""

    _stream = _rng.S_LOWRES

    def __init__(self, prob: float = 0.1, zoom_range=(0.5, 1.0), downsample_mode="nearest",
                 upsample_mode="trilinear", align_corners: bool = False):
        super().__init__(prob=prob)
        self.zoom_range = zoom_range
        self.downsample_mode = downsample_mode
        self.upsample_mode = upsample_mode
        self.align_corners = align_corners

    def _n_uniforms(self, shape):
        return 2

    def _host_params(self, B, shape, u, seed):
        lo, hi = self.zoom_range
        return {"mask": u[:, 0] < self.prob,
                "zoom_factor": (u[:, 1] * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)}

    def _device_params(self, host, shape, device):
        p = upload({"mask": host["mask"], "zoom_factor": host["zoom_factor"]}, device)
        p["_max_zoom"] = float(host["zoom_factor"].max()) if len(host["zoom_factor"]) else 1.0
        return p

    def apply(self, tensor, params):
        return ops.lowres3d(tensor, params["zoom_factor"], mask=params["mask"],
                            downsample_mode=self.downsample_mode,
                            upsample_mode=self.upsample_mode, align_corners=self.align_corners,
                            max_zoom=params.get("_max_zoom"))


# ---------------------------------------------------------------------------
# Dict wrappers (same keys/params sharing as the reference)
# ---------------------------------------------------------------------------

class RandGaussianNoised(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, mean=0.0, std=0.1):
        super().__init__(keys=keys, transform=RandGaussianNoise(prob=prob, mean=mean, std=std))


class RandAdjustContrastd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, gamma=(0.5, 4.5)):
        super().__init__(keys=keys, transform=RandAdjustContrast(prob=prob, gamma=gamma))


class RandScaleIntensityd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, factors=(0.0, 0.5)):
        super().__init__(keys=keys, transform=RandScaleIntensity(prob=prob, factors=factors))


class RandShiftIntensityd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, offsets=(-0.1, 0.1), safe: bool = False):
        super().__init__(keys=keys,
                         transform=RandShiftIntensity(prob=prob, offsets=offsets, safe=safe))


class RandBiasFieldd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, degree: int = 3, coeff_range=(0.0, 0.1)):
        super().__init__(keys=keys, transform=RandBiasField(prob=prob, degree=degree,
                                                            coeff_range=coeff_range))


class RandRicianNoised(BatchDictTransform):
    """Every key gets the same unit draws and mask (noise.py:167-185)."""

    def __init__(self, keys, prob: float = 0.1, mean: float = 0.0, std: float = 0.1,
                 relative: bool = False, sample_std: bool = True):
        super().__init__(keys=keys, transform=RandRicianNoise(
            prob=prob, mean=mean, std=std, relative=relative, sample_std=sample_std))


class RandStdShiftIntensityd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, factors=(-3.0, 3.0), nonzero: bool = False,
                 channel_wise: bool = False):
        super().__init__(keys=keys, transform=RandStdShiftIntensity(
            prob=prob, factors=factors, nonzero=nonzero, channel_wise=channel_wise))


class RandScaleIntensityFixedMeand(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, factors=(-0.5, 0.5), channel_wise: bool = False):
        super().__init__(keys=keys, transform=RandScaleIntensityFixedMean(
            prob=prob, factors=factors, channel_wise=channel_wise))


class ScaleIntensityd(BatchDictTransform):
    def __init__(self, keys, minv=0.0, maxv=1.0, factor=None, channel_wise: bool = True):
        super().__init__(keys=keys, transform=ScaleIntensity(minv=minv, maxv=maxv, factor=factor,
                                                             channel_wise=channel_wise))


class RandGaussianSmoothd(BatchDictTransform):
    def __init__(self, keys, prob: float = 0.1, sigma_x=(0.25, 1.5), sigma_y=(0.25, 1.5),
                 sigma_z=(0.25, 1.5), padding_mode=None):
        super().__init__(keys=keys, transform=RandGaussianSmooth(
            prob=prob, sigma_x=sigma_x, sigma_y=sigma_y, sigma_z=sigma_z,
            padding_mode=padding_mode))


class RandGaussianSharpend(BatchDictTransform):
    """Every key gets the same sharpening params (sharpen.py:139-169)."""

    def __init__(self, keys, prob: float = 0.1, sigma1_x=(0.5, 1.0), sigma1_y=(0.5, 1.0),
                 sigma1_z=(0.5, 1.0), sigma2_x=0.5, sigma2_y=0.5, sigma2_z=0.5,
                 alpha=(10.0, 30.0), padding_mode=None):
        super().__init__(keys=keys, transform=RandGaussianSharpen(
            prob=prob, sigma1_x=sigma1_x, sigma1_y=sigma1_y, sigma1_z=sigma1_z,
            sigma2_x=sigma2_x, sigma2_y=sigma2_y, sigma2_z=sigma2_z, alpha=alpha,
            padding_mode=padding_mode))


class RandSimulateLowResolutiond(BatchDictTransform):
    """Every key gets the same zoom factor and mask (resolution.py:121-147)."""

    def __init__(self, keys, prob: float = 0.1, zoom_range=(0.5, 1.0), downsample_mode="nearest",
                 upsample_mode="trilinear", align_corners: bool = False):
        super().__init__(keys=keys, transform=RandSimulateLowResolution(
            prob=prob, zoom_range=zoom_range, downsample_mode=downsample_mode,
            upsample_mode=upsample_mode, align_corners=align_corners))
