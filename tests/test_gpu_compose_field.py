"""The elastic∘affine single-resample extension (Compose(fuse_elastic=True),
ba_compose_field) against its CPU restatement in the oracle, plus the
properties that tie it to the reference's two-resample order: without an
affine it is exactly the elastic resample, and with a zero field it is the
affine resample (to fp32 rounding of the coordinates).  The reference has no
such mode, so there are no golden fixtures for it."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu


def _field_and_theta(rng, B, H, W, D, scale=0.15):
    """An elastic-like grid (identity plus a smooth displacement) and random
    affines converted to theta."""
    from batchaug_b200.geometric import monai_affine_to_theta
    import oracle as O
    ident = O.compose_field(np.zeros((1, H, W, D, 3), np.float32),
                            np.eye(4, dtype=np.float32)[None, :3], mask_field=np.zeros(1, np.uint8),
                            mask_affine=np.zeros(1, np.uint8))
    hh, ww, dd = np.meshgrid(np.linspace(0, np.pi, H), np.linspace(0, np.pi, W),
                             np.linspace(0, np.pi, D), indexing="ij")
    field = np.repeat(ident, B, axis=0)
    for b in range(B):
        ph = rng.uniform(0, np.pi, 3)
        field[b, ..., 0] += scale * np.sin(hh + ph[0]) * np.cos(ww)
        field[b, ..., 1] += scale * np.sin(dd + ph[1])
        field[b, ..., 2] += scale * np.cos(ww + ph[2]) * np.sin(dd)
    A = np.tile(np.eye(4, dtype=np.float32), (B, 1, 1))
    for b in range(B):
        a = rng.uniform(-0.4, 0.4)
        c, s = np.cos(a), np.sin(a)
        A[b, :2, :2] = [[c, -s], [s, c]]
        A[b, :3, 3] = rng.uniform(-3, 3, 3)
    return field.astype(np.float32), A, monai_affine_to_theta(A, (H, W, D))


@pytest.mark.parametrize("shape", [(3, 11, 14, 17), (2, 16, 16, 16)])
def test_compose_field_vs_oracle(ba, oracle_lib, shape):
    from batchaug_b200 import ops
    rng = np.random.default_rng(sum(shape))
    B, H, W, D = shape
    field, _, theta = _field_and_theta(rng, B, H, W, D)
    mf = np.array([1, 0, 1][:B], np.uint8)
    ma = np.array([1, 1, 0][:B], np.uint8)
    g = ops.compose_field(to_dev(field), to_dev(theta), mask_field=to_dev(mf.astype(bool)),
                          mask_affine=to_dev(ma.astype(bool)))
    ref = oracle_lib.compose_field(field, theta, mask_field=mf, mask_affine=ma)
    assert np.array_equal(to_np(g), ref)
    # no affine: the grid is the field itself
    g0 = ops.compose_field(to_dev(field), to_dev(theta),
                           mask_affine=torch.zeros(B, dtype=torch.bool, device="cuda"))
    assert np.array_equal(to_np(g0), field)


def _pipeline(ba, fuse, magnitude=(50.0, 150.0), affine_prob=1.0):
    return ba.Compose([ba.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5.0, 7.0),
                                         magnitude_range=magnitude,
                                         mode={"vol": "bilinear", "seg": "nearest"}),
                       ba.RandAffined(["vol", "seg"], prob=affine_prob, rotate_range=0.5,
                                      translate_range=3)],
                      lazy=True, mode={"vol": "bilinear", "seg": "nearest"}, fuse_elastic=fuse)


def test_fused_compose_vs_oracle(ba, oracle_lib):
    """Compose(fuse_elastic=True): the grid the library composes and the one
    resample it runs, against the oracle on the same sampled params."""
    from batchaug_b200.geometric import monai_affine_to_theta
    B, H, W, D = 3, 20, 24, 28
    g = torch.Generator(device="cuda").manual_seed(5)
    vol = torch.rand(B, 2, H, W, D, device="cuda", generator=g).bfloat16()
    seg = torch.randint(0, 5, (B, 1, H, W, D), device="cuda", generator=g).float()
    c = _pipeline(ba, True, affine_prob=0.6)
    torch.manual_seed(11)
    out = c({"vol": vol, "seg": seg})
    # the same draws, in Compose's order: elastic params, then the affine
    torch.manual_seed(11)
    el, af = c.transforms[0].transform, c.transforms[1].transform
    pe = el.sample_params(B, vol.shape, vol.device)
    ha = af.sample_host(B, vol.shape)
    A = af.host_affine({"_host": ha})
    mf, ma = pe["_host"]["mask"].astype(np.uint8), ha["mask"].astype(np.uint8)
    grid = oracle_lib.compose_field(to_np(pe["grid"]), monai_affine_to_theta(A, (H, W, D)),
                                    mask_field=mf, mask_affine=ma)
    m = (mf | ma).astype(np.uint8)
    rv = oracle_lib.resample3d(to_np(vol), grid=grid, mode="bilinear", padding="zeros",
                               align_corners=True, mask=m)
    rs = oracle_lib.resample3d(to_np(seg), grid=grid, mode="nearest", padding="zeros",
                               align_corners=True, mask=m)
    assert_close_dtype(to_np(out["vol"]), rv)
    assert np.array_equal(to_np(out["seg"]), rs)
    assert set(np.unique(to_np(out["seg"]))) <= set(range(5))


def test_fused_without_affine_is_the_elastic_resample(ba):
    B = 2
    g = torch.Generator(device="cuda").manual_seed(6)
    vol = torch.rand(B, 1, 24, 24, 24, device="cuda", generator=g)
    seg = torch.randint(0, 4, (B, 1, 24, 24, 24), device="cuda", generator=g).float()
    outs = []
    for fuse in (False, True):
        torch.manual_seed(3)
        outs.append(_pipeline(ba, fuse, affine_prob=0.0)({"vol": vol, "seg": seg}))
    assert torch.equal(outs[0]["vol"], outs[1]["vol"])
    assert torch.equal(outs[0]["seg"], outs[1]["seg"])


def test_fused_with_zero_field_is_the_affine_resample(ba):
    """Magnitude 0: the composed coordinates are the affine's (rounding of
    the fp32 coordinate steps only), so trilinear results agree to 1e-5."""
    B = 2
    g = torch.Generator(device="cuda").manual_seed(7)
    # smooth content so a coordinate difference of ~1e-6 voxel stays tiny
    base = torch.linspace(0, 1, 24, device="cuda")
    vol = (base[None, None, :, None, None] * base[None, None, None, :, None]
           + 0.5 * base[None, None, None, None, :]).expand(B, 1, 24, 24, 24).contiguous()
    vol = vol + 0.01 * torch.rand(B, 1, 24, 24, 24, device="cuda", generator=g)
    outs = []
    for fuse in (False, True):
        torch.manual_seed(4)
        c = ba.Compose([ba.Rand3DElasticd(["vol"], prob=1.0, magnitude_range=(0.0, 0.0)),
                        ba.RandAffined(["vol"], prob=1.0, rotate_range=0.5, translate_range=3)],
                       lazy=True, fuse_elastic=fuse)
        outs.append(c({"vol": vol})["vol"])
    # unfused: elastic with a zero field is an exact copy, then the affine
    assert (outs[0] - outs[1]).abs().max().item() <= 1e-5
