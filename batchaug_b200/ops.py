"""Functional entry points: torch tensors in, C-ABI calls out.

Each function validates tensors (CUDA, contiguous, fp32/bf16), allocates the
outputs and scratch with torch's caching allocator, and enqueues the kernels
on torch's current stream.  These are what the transform classes call; they
can also be used directly.
"""
from __future__ import annotations

import contextlib
import ctypes
import os

import numpy as np
import torch

from . import _lib as L
from . import _timing


def _contig(t: torch.Tensor, name: str) -> torch.Tensor:
    L.require_cuda(t, name)
    return t if t.is_contiguous() else t.contiguous()


def _to_device(arr: np.ndarray, device) -> torch.Tensor:
    """Asynchronous small host-to-device copy through pinned memory."""
    t = torch.from_numpy(np.ascontiguousarray(arr))
    return t.pin_memory().to(device, non_blocking=True)


def _dev_f32(x, device, name):
    """Small parameter arrays (numpy or tensor) as contiguous fp32 on device."""
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=torch.float32).contiguous()
    return _to_device(np.asarray(x, dtype=np.float32), device)


def _dev_mask(mask, B, device):
    if mask is None:
        return None
    if isinstance(mask, torch.Tensor):
        m = mask.to(device=device).reshape(B)
        if m.dtype in (torch.bool, torch.uint8):
            return m.contiguous().view(torch.uint8)  # a view: no kernel
        return (m != 0).to(torch.uint8).contiguous()
    return _to_device(np.asarray(mask).reshape(B).astype(np.uint8), device)


# ---------------------------------------------------------------------------
# Geometric
# ---------------------------------------------------------------------------

# Trilinear arithmetic of the resample: False (default) interpolates with
# fused multiply-add lerps, within 1e-5 (fp32) / 2 bf16 ulp of torch's CPU
# grid_sample; True rounds every weight product and sum as torch's CPU code
# does (bit for bit).  Coordinates, and so nearest keys, are exact either way.
# BATCHAUG_B200_EXACT=1 in the environment starts in exact mode.
_EXACT = [os.environ.get("BATCHAUG_B200_EXACT", "0") == "1"]


def set_resample_exact(flag: bool) -> bool:
    """Set the default trilinear arithmetic (see above); returns the old one."""
    old, _EXACT[0] = _EXACT[0], bool(flag)
    return old


@contextlib.contextmanager
def resample_exact(flag: bool = True):
    """``with resample_exact():`` runs its body's resamples in exact mode."""
    old = set_resample_exact(flag)
    try:
        yield
    finally:
        set_resample_exact(old)


def resample3d(tensors, *, affine=None, theta=None, grid=None, modes="bilinear",
               paddings="zeros", align_corners=False, mask=None, out=None, exact=None,
               minmax=None):
    """Resample one or more (B,C,H,W,D) tensors through one shared map.

    Exactly one of ``affine`` (MONAI (B,4,4)), ``theta`` (affine_grid
    (B,3|4,4)) or ``grid`` (grid_sample (B,H,W,D,3)) gives the map.  ``modes``
    and ``paddings`` are a string or one entry per tensor.  Masked-out
    elements are copied.  ``exact`` overrides the default trilinear
    arithmetic (``set_resample_exact``).  ``minmax`` (one entry per tensor,
    None or an int32 (B, C, 2) device tensor) receives each output's
    per-(element, channel) min/max as statistics for a following
    ScaleIntensity (``ChainOp(stats=...)``).  Returns a list of new tensors
    (or fills ``out``).
    """
    single = isinstance(tensors, torch.Tensor)
    ts = [tensors] if single else list(tensors)
    if not 1 <= len(ts) <= L.BA_MAX_KEYS:
        raise ValueError(f"resample3d takes 1..{L.BA_MAX_KEYS} tensors")
    ts = [_contig(t, "tensor") for t in ts]
    for t in ts:
        if t.dim() != 5:
            raise ValueError(f"expected (B,C,H,W,D) tensors, got shape {tuple(t.shape)}")
    B, _, H, W, D = ts[0].shape
    device = ts[0].device
    for t in ts[1:]:
        if t.shape[0] != B or tuple(t.shape[2:]) != (H, W, D) or t.device != device:
            raise ValueError("resample3d: tensors must share batch, spatial shape and device")
    modes = [modes] * len(ts) if isinstance(modes, str) else list(modes)
    paddings = [paddings] * len(ts) if isinstance(paddings, str) else list(paddings)
    for m in modes:
        if m not in L.MODES:
            raise ValueError(f"unsupported interpolation mode {m!r} (bilinear or nearest)")
    for p in paddings:
        if p not in L.PADDINGS:
            raise ValueError(f"unsupported padding_mode {p!r} (zeros, border or reflection)")
    if sum(x is not None for x in (affine, theta, grid)) != 1:
        raise ValueError("resample3d needs exactly one of affine, theta or grid")
    # host (numpy) transforms and masks ride in the kernels' parameters
    # (BA_RESAMPLE_HOST_PARAMS): no upload, no device allocation
    host = not isinstance(affine if affine is not None else theta, torch.Tensor) and \
        (grid is None or isinstance(grid, torch.Tensor)) and not isinstance(mask, torch.Tensor)
    if affine is not None:
        xf = (np.ascontiguousarray(affine, np.float32).reshape(B, -1) if host
              else _dev_f32(affine, device, "affine").reshape(B, -1))
        kind, stride = L.BA_XFORM_AFFINE, xf.shape[1]
        if stride != 16:
            raise ValueError("affine must be (B,4,4)")
    elif theta is not None:
        xf = (np.ascontiguousarray(theta, np.float32).reshape(B, -1) if host
              else _dev_f32(theta, device, "theta").reshape(B, -1))
        kind, stride = L.BA_XFORM_THETA, xf.shape[1]
        if stride not in (12, 16):
            raise ValueError("theta must be (B,3,4) or (B,4,4)")
    else:
        xf = _dev_f32(grid, device, "grid")
        if tuple(xf.shape) != (B, H, W, D, 3):
            raise ValueError(f"grid must be {(B, H, W, D, 3)}, got {tuple(xf.shape)}")
        kind, stride = L.BA_XFORM_GRID, 0
    if host:
        m = None if mask is None else np.ascontiguousarray(np.asarray(mask).reshape(B) != 0,
                                                           np.uint8)
    else:
        m = _dev_mask(mask, B, device)
    outs = list(out) if out is not None else [torch.empty_like(t) for t in ts]
    d = L.ResampleDesc()
    d.batch, d.H, d.W, d.D = B, H, W, D
    d.xform_kind = kind
    d.align_corners = int(bool(align_corners))
    d.flags = L.BA_RESAMPLE_EXACT if (_EXACT[0] if exact is None else exact) else 0
    d.n_keys = len(ts)
    if host:
        d.flags |= L.BA_RESAMPLE_HOST_PARAMS
        d.xform = xf.ctypes.data if kind != L.BA_XFORM_GRID else xf.data_ptr()
        d.mask = None if m is None else m.ctypes.data
    else:
        d.xform = xf.data_ptr()
        d.mask = L.ptr(m)
    d.xform_stride = stride
    mms = list(minmax) if minmax is not None else [None] * len(ts)
    if len(mms) != len(ts):
        raise ValueError("resample3d: minmax needs one entry per tensor")
    for i, (t, o) in enumerate(zip(ts, outs)):
        k = d.keys[i]
        k.src, k.dst = t.data_ptr(), o.data_ptr()
        mm = mms[i]
        if mm is not None:
            if (mm.dtype != torch.int32 or tuple(mm.shape) != (B, t.shape[1], 2)
                    or not mm.is_contiguous() or mm.device != device):
                raise ValueError(f"resample3d: minmax[{i}] must be a contiguous int32 "
                                 f"{(B, t.shape[1], 2)} tensor on {device}")
            k.minmax = mm.data_ptr()
        k.channels = t.shape[1]
        k.dtype = L.dtype_code(t)
        k.mode = L.MODES[modes[i]]
        k.padding = L.PADDINGS[paddings[i]]
    tok = _timing.begin("ba_resample3d", sum(2 * t.numel() * t.element_size() for t in ts),
                        device)
    L.check(L.lib.ba_resample3d(ctypes.byref(d), L.stream_ptr(device)), "ba_resample3d")
    _timing.end(tok)
    return outs[0] if single else outs


# ---------------------------------------------------------------------------
# Intensity chain
# ---------------------------------------------------------------------------

class ChainOp:
    """One op of a fused intensity chain (device tensors for its params)."""

    __slots__ = ("kind", "flags", "mask", "param", "param2", "noise", "seed", "elem_offset",
                 "degree", "c0", "c1", "stats")

    def __init__(self, kind, flags=0, mask=None, param=None, param2=None, noise=None, seed=0,
                 elem_offset=0, degree=0, c0=0.0, c1=0.0, stats=None):
        self.kind, self.flags, self.mask = kind, flags, mask
        self.param, self.param2, self.noise = param, param2, noise
        self.seed, self.elem_offset, self.degree = seed, elem_offset, degree
        self.c0, self.c1 = c0, c1
        self.stats = stats  # RESCALE with BA_RESCALE_GIVEN: resample3d's minmax


def intensity_chain(x: torch.Tensor, ops, out: torch.Tensor | None = None,
                    inplace: bool = False) -> torch.Tensor:
    """Apply a list of ChainOp to x in as few HBM passes as possible."""
    x = _contig(x, "tensor")
    if x.dim() != 5:
        raise ValueError(f"expected a (B,C,H,W,D) tensor, got shape {tuple(x.shape)}")
    if not 1 <= len(ops) <= L.BA_MAX_OPS:
        raise ValueError(f"intensity_chain takes 1..{L.BA_MAX_OPS} ops")
    B, C, H, W, D = x.shape
    if out is None:
        out = x if inplace else torch.empty_like(x)
    d = L.ChainDesc()
    d.src, d.dst = x.data_ptr(), out.data_ptr()
    d.batch, d.channels, d.H, d.W, d.D = B, C, H, W, D
    d.dtype = L.dtype_code(x)
    d.n_ops = len(ops)
    keep = []
    for i, op in enumerate(ops):
        o = d.ops[i]
        o.kind, o.flags = op.kind, op.flags
        for name in ("mask", "param", "param2", "noise", "stats"):
            t = getattr(op, name)
            if t is not None:
                if t.device != x.device:
                    raise ValueError(f"op {i} {name} is on {t.device}, tensor on {x.device}")
                keep.append(t)
            setattr(o, name, L.ptr(t))
        o.seed = int(op.seed) & 0xFFFFFFFFFFFFFFFF
        o.elem_offset = int(op.elem_offset)
        o.degree = int(op.degree)
        o.c0, o.c1 = float(op.c0), float(op.c1)
    nbytes = L.lib.ba_intensity_workspace_bytes(ctypes.byref(d))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device) if nbytes else None
    tok = _timing.begin("ba_intensity_chain", 2 * x.numel() * x.element_size(), x.device)
    L.check(L.lib.ba_intensity_chain(ctypes.byref(d), L.ptr(ws), nbytes, L.stream_ptr(x.device)),
            "ba_intensity_chain")
    _timing.end(tok)
    return out


def minmax(x: torch.Tensor, n_groups: int):
    """Per-group (min, max) of x viewed as (n_groups, -1), fp32 tensors."""
    x = _contig(x, "tensor")
    if x.numel() % max(n_groups, 1):
        raise ValueError("minmax: numel is not a multiple of n_groups")
    stats = torch.empty(n_groups, 2, dtype=torch.float32, device=x.device)
    tok = _timing.begin("ba_minmax", x.numel() * x.element_size(), x.device)
    L.check(L.lib.ba_minmax(x.data_ptr(), L.dtype_code(x), n_groups,
                            x.numel() // max(n_groups, 1), stats.data_ptr(),
                            L.stream_ptr(x.device)), "ba_minmax")
    _timing.end(tok)
    return stats[:, 0], stats[:, 1]


# ---------------------------------------------------------------------------
# Smoothing / elastic
# ---------------------------------------------------------------------------

def gauss_taps_len(max_sigma: float, truncated: float) -> int:
    return int(L.lib.ba_gauss_taps_len(float(max_sigma), float(truncated)))


def gauss_taps(sigmas: torch.Tensor, K: int) -> torch.Tensor:
    """(B,K) taps of gaussian_1d_batch for sigmas already on device."""
    s = sigmas.to(torch.float32).contiguous()
    L.require_cuda(s, "sigmas")
    taps = torch.empty(s.numel(), K, dtype=torch.float32, device=s.device)
    L.check(L.lib.ba_gauss_taps(s.data_ptr(), s.numel(), K, taps.data_ptr(),
                                L.stream_ptr(s.device)), "ba_gauss_taps")
    return taps


def smooth3d(x: torch.Tensor, taps_h, taps_w, taps_d, mask=None,
             padding_mode=None) -> torch.Tensor:
    """Separable Gaussian smoothing with per-element taps; padding_mode is
    None/"constant" (zeros), "reflect" or "replicate" as in F.pad."""
    if padding_mode not in L.SMOOTH_PADS:
        raise ValueError(f"unsupported padding_mode {padding_mode!r}")
    x = _contig(x, "tensor")
    B, C, H, W, D = x.shape
    th, tw, td = (_dev_f32(t, x.device, "taps") for t in (taps_h, taps_w, taps_d))
    m = _dev_mask(mask, B, x.device)
    out = torch.empty_like(x)
    nbytes = L.lib.ba_smooth_workspace_bytes(B, C, H, W, D)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    tok = _timing.begin("ba_smooth3d", 2 * x.numel() * x.element_size(), x.device)
    L.check(L.lib.ba_smooth3d(x.data_ptr(), out.data_ptr(), L.dtype_code(x), B, C, H, W, D,
                              th.data_ptr(), th.shape[1], tw.data_ptr(), tw.shape[1],
                              td.data_ptr(), td.shape[1], L.SMOOTH_PADS[padding_mode], L.ptr(m),
                              ws.data_ptr(), nbytes,
                              L.stream_ptr(x.device)), "ba_smooth3d")
    _timing.end(tok)
    return out


def sharpen3d(x: torch.Tensor, taps1, taps2, alpha, mask=None,
              padding_mode=None) -> torch.Tensor:
    """Unsharp masking blurred + alpha * (blurred - double_blurred) with
    per-element taps: taps1 / taps2 are (H, W, D) triples of (B, K) for the
    first and second blur."""
    if padding_mode not in L.SMOOTH_PADS:
        raise ValueError(f"unsupported padding_mode {padding_mode!r}")
    x = _contig(x, "tensor")
    B, C, H, W, D = x.shape
    t1 = [_dev_f32(t, x.device, "taps1") for t in taps1]
    t2 = [_dev_f32(t, x.device, "taps2") for t in taps2]
    for t in t1 + t2:
        if t.dim() != 2 or t.shape[0] != B:
            raise ValueError(f"taps must be (B={B}, K), got {tuple(t.shape)}")
    al = _dev_f32(alpha, x.device, "alpha").reshape(-1)
    if al.numel() != B:
        raise ValueError(f"alpha has {al.numel()} values for a batch of {B}")
    m = _dev_mask(mask, B, x.device)
    out = torch.empty_like(x)
    d = L.SharpenDesc()
    d.src, d.dst = x.data_ptr(), out.data_ptr()
    d.dtype, d.padding = L.dtype_code(x), L.SMOOTH_PADS[padding_mode]
    d.batch, d.channels, d.H, d.W, d.D = B, C, H, W, D
    for i in range(3):
        d.taps1[i], d.K1[i] = t1[i].data_ptr(), t1[i].shape[1]
        d.taps2[i], d.K2[i] = t2[i].data_ptr(), t2[i].shape[1]
    d.alpha, d.mask = al.data_ptr(), L.ptr(m)
    nbytes = L.lib.ba_sharpen_workspace_bytes(ctypes.byref(d))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    tok = _timing.begin("ba_sharpen3d", 2 * x.numel() * x.element_size(), x.device)
    L.check(L.lib.ba_sharpen3d(ctypes.byref(d), ws.data_ptr(), nbytes, L.stream_ptr(x.device)),
            "ba_sharpen3d")
    _timing.end(tok)
    return out


def lowres3d(x: torch.Tensor, zoom, mask=None, downsample_mode="nearest",
             upsample_mode="trilinear", align_corners=False, max_zoom=None) -> torch.Tensor:
    """Down to max(1, rint(s * zoom[b])) per axis and back up, per element
    (RandSimulateLowResolution.apply).  max_zoom bounds zoom (read from it
    when None, which costs a device-to-host copy for a device tensor)."""
    for m in (downsample_mode, upsample_mode):
        if m not in L.INTERP_MODES:
            raise ValueError(f"unsupported interpolation mode {m!r} for a 5-D tensor "
                             f"(expected one of {sorted(L.INTERP_MODES)})")
    x = _contig(x, "tensor")
    B, C, H, W, D = x.shape
    z = _dev_f32(zoom, x.device, "zoom").reshape(-1)
    if z.numel() != B:
        raise ValueError(f"zoom has {z.numel()} values for a batch of {B}")
    if max_zoom is None:
        max_zoom = float(z.max()) if B else 1.0
    m = _dev_mask(mask, B, x.device)
    out = torch.empty_like(x)
    d = L.LowresDesc()
    d.src, d.dst, d.dtype = x.data_ptr(), out.data_ptr(), L.dtype_code(x)
    d.down_mode, d.up_mode = L.INTERP_MODES[downsample_mode], L.INTERP_MODES[upsample_mode]
    d.align_corners = int(bool(align_corners))
    d.batch, d.channels, d.H, d.W, d.D = B, C, H, W, D
    d.zoom, d.mask, d.max_zoom = z.data_ptr(), L.ptr(m), float(max(max_zoom, 1e-30))
    nbytes = L.lib.ba_lowres_workspace_bytes(ctypes.byref(d))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    tok = _timing.begin("ba_lowres3d", 2 * x.numel() * x.element_size(), x.device)
    L.check(L.lib.ba_lowres3d(ctypes.byref(d), ws.data_ptr(), nbytes, L.stream_ptr(x.device)),
            "ba_lowres3d")
    _timing.end(tok)
    return out


def compose_field(field: torch.Tensor, theta, mask_field=None, mask_affine=None) -> torch.Tensor:
    """Grid (B,H,W,D,3) of the elastic field ``field`` followed by the affine
    ``theta`` (B,3,4) (see ba_compose_field): one grid_sample with it
    (align_corners=True) gives I(field(A(p)))."""
    field = _contig(field.to(torch.float32), "field")
    if field.dim() != 5 or field.shape[-1] != 3:
        raise ValueError(f"field must be (B,H,W,D,3), got {tuple(field.shape)}")
    B, H, W, D, _ = field.shape
    th = _dev_f32(theta, field.device, "theta").reshape(B, -1)
    if th.shape[1] == 16:
        th = th.reshape(B, 4, 4)[:, :3, :].contiguous()
    th = th.reshape(B, 3, 4).contiguous()
    mf = _dev_mask(mask_field, B, field.device)
    ma = _dev_mask(mask_affine, B, field.device)
    out = torch.empty_like(field)
    tok = _timing.begin("ba_compose_field", 2 * field.numel() * 4, field.device)
    L.check(L.lib.ba_compose_field(field.data_ptr(), th.data_ptr(), L.ptr(mf), L.ptr(ma), B, H, W,
                                   D, out.data_ptr(), L.stream_ptr(field.device)),
            "ba_compose_field")
    _timing.end(tok)
    return out


def elastic_grid(shape, taps, magnitude, *, u=None, seed=0, elem_offset=0,
                 device=None) -> torch.Tensor:
    """grid_sample grid (B,H,W,D,3) of Rand3DElastic from taps (B,K) and
    magnitude (B,); the uniform draw u (B,3,H,W,D) is generated in-kernel
    from (seed, elem_offset) unless given."""
    B, H, W, D = shape
    device = device or (u.device if u is not None else taps.device)
    tp = _dev_f32(taps, device, "taps")
    mg = _dev_f32(magnitude, device, "magnitude").reshape(B)
    uu = None if u is None else _contig(u.to(torch.float32), "u")
    grid = torch.empty(B, H, W, D, 3, dtype=torch.float32, device=device)
    nbytes = L.lib.ba_elastic_workspace_bytes(B, H, W, D)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    tok = _timing.begin("ba_elastic_grid", grid.numel() * 4, device)
    L.check(L.lib.ba_elastic_grid(L.ptr(uu), int(seed) & 0xFFFFFFFFFFFFFFFF, int(elem_offset),
                                  B, H, W, D, tp.data_ptr(), tp.shape[1], mg.data_ptr(),
                                  grid.data_ptr(), ws.data_ptr(), nbytes,
                                  L.stream_ptr(device)), "ba_elastic_grid")
    _timing.end(tok)
    return grid


def host_rand_affine(u, prob, a, b, c, present, groups, spatial_shape, mask, affine, theta):
    """ba_host_rand_affine into the given numpy outputs (mask u8 (B,),
    affine and theta (B,4,4) float32)."""
    H, W, D = spatial_shape
    B = u.shape[0]
    L.lib.ba_host_rand_affine(u.ctypes.data, B, u.shape[1], float(prob), a.ctypes.data,
                              b.ctypes.data, c.ctypes.data, int(present), int(groups), H, W, D,
                              mask.ctypes.data, affine.ctypes.data, theta.ctypes.data)


def host_uniform(seed: int, stream: int, elem_offset: int, n_elems: int,
                 per_elem: int) -> np.ndarray:
    """(n_elems, per_elem) uniforms in [0,1) keyed on global element index."""
    out = np.empty((n_elems, per_elem), np.float32)
    if n_elems and per_elem:
        L.lib.ba_host_uniform(int(seed) & 0xFFFFFFFFFFFFFFFF, int(stream) & 0xFFFF,
                              int(elem_offset), n_elems, per_elem, out.ctypes.data)
    return out

