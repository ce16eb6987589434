"""The oracle replays the reference's recorded Compose runs (CPU).

The fixtures of tests/golden/gen_golden.py (``compose_*``) hold the params
the reference's ``Compose(lazy=True)`` sampled and its outputs.  Replaying
the lazy schedule with the oracle's restated kernels — one resample per
accumulated affine (batchaug/compose.py:71-110), then the eager transform —
must reproduce them: bit for bit where the reference is deterministic on
CPU, within the parity tolerance where it goes through conv3d / einsum.
Also checks that the seeded inputs regenerate to the generator's digest on
this host, and that the host-side affine composition rounds as torch's
batched matmul.
"""
from __future__ import annotations

import importlib.util
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from helpers import assert_close_dtype

_spec = importlib.util.spec_from_file_location("golden_inputs", os.path.join(GOLDEN, "inputs.py"))
inputs = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(inputs)

_EYE = np.eye(4, dtype=np.float32)


def _compose(a, b):
    """Sequential fp32 products and sums: torch's CPU (B,4,4) @ (B,4,4)."""
    acc = a[:, :, 0, None] * b[:, None, 0, :]
    for k in range(1, 4):
        acc = acc + a[:, :, k, None] * b[:, None, k, :]
    return acc.astype(np.float32)


def _masked(mask, a):
    return np.where(mask[:, None, None], a, _EYE[None]).astype(np.float32)


def _flip_affine(mask, axes):
    a = np.broadcast_to(_EYE, (len(mask), 4, 4)).copy()
    for ax in range(3):
        a[mask & (axes == ax), ax, ax] = -1.0
    return a


def _rot90_affine(mask, k, axes=(0, 1)):
    a = np.broadcast_to(_EYE, (len(mask), 4, 4)).copy()
    cos_t, sin_t = (0.0, -1.0, 0.0), (-1.0, 0.0, 1.0)
    ax0, ax1 = axes
    for kk in (1, 2, 3):
        sel = mask & (k == kk)
        a[sel, ax0, ax0], a[sel, ax0, ax1] = cos_t[kk - 1], -sin_t[kk - 1]
        a[sel, ax1, ax0], a[sel, ax1, ax1] = sin_t[kk - 1], cos_t[kk - 1]
    return a


def _m(z, i):
    return z[f"p{i}_mask"].astype(bool)


def _noise(z, i, shape):
    std = z[f"p{i}_std"].astype(np.float32).reshape(-1, 1, 1, 1, 1)
    mean = z[f"p{i}_mean"].astype(np.float32).reshape(-1, 1, 1, 1, 1)
    return (inputs.normal(int(z["seed_noise"]), shape) * std + mean).astype(np.float32)


def _summary(a):
    vals = (a.astype(np.uint32) << 16).view(np.float32) if a.dtype == np.uint16 else a
    flat = vals.astype(np.float64).reshape(a.shape[0] * a.shape[1], -1)
    H = a.shape[2]
    return a[:, :, (H * 3) // 5], a[:, :, ::9, ::9, ::9], flat.sum(1), (flat * flat).sum(1)


def test_affine_composition_rounds_as_torch():
    from batchaug_b200.compose import compose_affines
    g = torch.Generator().manual_seed(5)
    a, b = torch.randn(512, 4, 4, generator=g), torch.randn(512, 4, 4, generator=g)
    ref = (a @ b).numpy()
    assert np.array_equal(compose_affines(a.numpy(), b.numpy()), ref)
    assert np.array_equal(_compose(a.numpy(), b.numpy()), ref)


def test_seeded_inputs_regenerate():
    z = load_golden("compose_cfg1")
    shp = (2, 1, 64, 64, 64)
    d = {"vol": inputs.normal(int(z["seed_vol"]), shp),
         "seg": inputs.labels(int(z["seed_seg"]), shp, 5, block=10)}
    assert inputs.digest(d["seg"], d["vol"]) == str(z["input_digest"])


def test_oracle_replays_reference_compose_cfg1(oracle_lib):
    """Config 1 at full size: {flip, affine} -> noise -> ScaleIntensity."""
    o = oracle_lib
    z = load_golden("compose_cfg1")
    shp = (2, 1, 64, 64, 64)
    vol = inputs.normal(int(z["seed_vol"]), shp)
    seg = inputs.labels(int(z["seed_seg"]), shp, 5, block=10)
    a = _compose(_flip_affine(_m(z, 0), z["p0_axes"]), _masked(_m(z, 1), z["p1_affine"]))
    mask = _m(z, 0) | _m(z, 1)
    vo = o.resample3d(vol, affine=a, mode="bilinear", mask=mask)
    so = o.resample3d(seg, affine=a, mode="nearest", mask=mask)
    vo = o.noise_add(vo, _noise(z, 2, shp), _m(z, 2))
    vo = o.scale_intensity(vo, 0.0, 1.0)
    assert np.array_equal(so, z["out_seg"])
    assert np.array_equal(vo, z["out_vol"])


def test_oracle_replays_reference_compose_cfg4(oracle_lib):
    """Config 4 slice: {rot90, flip} -> noise -> {affine} -> ScaleIntensity
    (two materialisations)."""
    o = oracle_lib
    z = load_golden("compose_cfg4")
    shp = (2, 4, 128, 128, 128)
    vol = inputs.normal(int(z["seed_vol"]), shp)
    seg = (inputs.labels(int(z["seed_seg"]), shp, 2, block=16) > 0).astype(np.float32)
    a1 = _compose(_rot90_affine(_m(z, 0), z["p0_k"]), _flip_affine(_m(z, 1), z["p1_axes"]))
    m1 = _m(z, 0) | _m(z, 1)
    vol = o.resample3d(vol, affine=a1, mode="bilinear", mask=m1)
    seg = o.resample3d(seg, affine=a1, mode="nearest", mask=m1)
    vol = o.noise_add(vol, _noise(z, 2, shp), _m(z, 2))
    a2 = _masked(_m(z, 3), z["p3_affine"])
    vol = o.resample3d(vol, affine=a2, mode="bilinear", mask=_m(z, 3))
    seg = o.resample3d(seg, affine=a2, mode="nearest", mask=_m(z, 3))
    vol = o.scale_intensity(vol, 0.0, 1.0)
    for key, out in (("vol", vol), ("seg", seg)):
        plane, stride, s, ss = _summary(out)
        assert np.array_equal(plane, z[f"out_{key}_plane"]), key
        assert np.array_equal(stride, z[f"out_{key}_stride"]), key
        np.testing.assert_array_equal(s, z[f"out_{key}_sum"])


def test_oracle_replays_reference_compose_cfg5(oracle_lib):
    """Config 5 slice: elastic (injected grid) -> {affine} -> bias ->
    smooth -> ScaleIntensity, vol bf16; the smoothing and bias field go
    through torch's conv3d / einsum, so vol is held to 2 bf16 ulp."""
    o = oracle_lib
    z = load_golden("compose_cfg5")
    shp = (2, 2, 160, 160, 160)
    vol = inputs.bf16_bits(inputs.uniform(int(z["seed_vol"]), shp))
    seg = inputs.labels(int(z["seed_seg"]), shp, 8, block=20)
    grid = inputs.elastic_grid(int(z["seed_grid"]), 2, shp[2:], 4.0)
    m0 = _m(z, 0)
    vol = o.resample3d(vol, grid=grid, mode="bilinear", align_corners=True, mask=m0)
    seg = o.resample3d(seg, grid=grid, mode="nearest", align_corners=True, mask=m0)
    a1 = _masked(_m(z, 1), z["p1_affine"])
    vol = o.resample3d(vol, affine=a1, mode="bilinear", mask=_m(z, 1))
    seg = o.resample3d(seg, affine=a1, mode="nearest", mask=_m(z, 1))
    vol = o.bias_field(vol, z["p2_coeffs"], _m(z, 2))
    sm = o.separable_gauss(vol, z["p3_kernel_h"], z["p3_kernel_w"], z["p3_kernel_d"])
    vol = np.where(_m(z, 3)[:, None, None, None, None], sm, vol)
    vol = o.scale_intensity(vol, 0.0, 1.0)
    plane, stride, s, _ = _summary(seg)
    assert np.array_equal(plane, z["out_seg_plane"])
    assert np.array_equal(stride, z["out_seg_stride"])
    np.testing.assert_array_equal(s, z["out_seg_sum"])
    plane, stride, s, _ = _summary(vol)
    assert_close_dtype(plane, z["out_vol_plane"])
    assert_close_dtype(stride, z["out_vol_stride"])


@pytest.mark.parametrize("name", ["compose_keysets", "compose_partial_mask"])
def test_oracle_replays_reference_nearest_cases(oracle_lib, name):
    """The reference's key-set and partial-mask Compose cases
    (tests/test_compose.py:217-253, :287-308), all nearest."""
    o = oracle_lib
    z = load_golden(name)
    shp = (4, 3, 16, 16, 16)
    vol = inputs.uniform(int(z["seed_vol"]), shp)
    if name == "compose_keysets":
        seg = inputs.labels(int(z["seed_seg"]), shp, 5, block=3)
        af = _flip_affine(_m(z, 0), z["p0_axes"])
        av = _compose(af, _rot90_affine(_m(z, 1), z["p1_k"]))
        vo = o.resample3d(vol, affine=av, mode="nearest", mask=_m(z, 0) | _m(z, 1))
        so = o.resample3d(seg, affine=af, mode="nearest", mask=_m(z, 0))
        assert np.array_equal(so, z["out_seg"])
    else:
        vo = o.resample3d(vol, affine=_flip_affine(_m(z, 0), z["p0_axes"]), mode="nearest",
                          mask=_m(z, 0))
        keep = ~_m(z, 0)
        assert np.array_equal(vo[keep], vol[keep])  # masked-out elements untouched
    assert np.array_equal(vo, z["out_vol"])


def test_oracle_zoom_flip_rotate_eager(oracle_lib):
    """RandZoom.apply (zoom.py:90-121), RandFlip.apply (flip.py:128-137) and
    RandRotate.apply (rotate.py:6-40 through affine.py:284-317) of the
    reference, replayed with their recorded params."""
    o = oracle_lib
    z = load_golden("zoom_flip_rotate_eager")
    x = z["x"]
    m = z["zoom_mask"].astype(bool)
    assert np.array_equal(o.resample3d(x, theta=z["zoom_theta"], padding="border", mask=m),
                          z["zoom_out"])
    assert np.array_equal(o.resample3d(x, theta=z["zoom_theta"], mode="nearest", mask=m),
                          z["zoom_nearest_zeros_out"])
    for tag, axes in (("all", (0, 1, 2)), ("h", (0,)), ("wd", (1, 2))):
        mk = z[f"flip_{tag}_mask"].astype(bool)
        a = np.broadcast_to(_EYE, (len(mk), 4, 4)).copy()
        for ax in axes:
            a[mk, ax, ax] = -1.0
        assert np.array_equal(o.resample3d(x, affine=a, mode="nearest", mask=mk),
                              z[f"flip_{tag}_out"]), tag
    mr = z["rotate_mask"].astype(bool)
    assert np.array_equal(o.resample3d(x, theta=z["rotate_theta"], padding="border", mask=mr),
                          z["rotate_out"])
