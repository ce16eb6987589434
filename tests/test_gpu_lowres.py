"""CUDA RandSimulateLowResolution (ba_lowres3d) against the reference's
golden outputs and the oracle.  Bar: bit-exact in fp32 and bf16 for every
downsample/upsample mode pair (the kernel follows torch's CPU interpolate
arithmetic step by step)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import to_dev, to_np

pytestmark = pytest.mark.gpu

MODES = (("nearest", "trilinear", False), ("nearest-exact", "trilinear", False),
         ("nearest", "trilinear", True), ("trilinear", "trilinear", False),
         ("trilinear", "nearest", True), ("area", "trilinear", False),
         ("nearest-exact", "area", False), ("area", "nearest-exact", False))


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_lowres(ba, tag):
    from batchaug_b200 import ops
    g = load_golden(f"lowres_{tag}")
    x = to_dev(g["x"])
    for i, (dm, um, ac) in enumerate(MODES):
        out = ops.lowres3d(x, to_dev(g[f"m{i}_zoom"]), mask=to_dev(g[f"m{i}_mask"]),
                           downsample_mode=dm, upsample_mode=um, align_corners=ac)
        assert np.array_equal(to_np(out), g[f"m{i}_out"]), (dm, um, ac)
        t = ba.RandSimulateLowResolution(prob=0.8, zoom_range=(0.3, 1.0), downsample_mode=dm,
                                         upsample_mode=um, align_corners=ac)
        out2 = t.apply(x, {"mask": to_dev(g[f"m{i}_mask"]), "zoom_factor": to_dev(g[f"m{i}_zoom"])})
        assert torch.equal(out, out2)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("modes", MODES)
def test_lowres_vs_oracle(ba, oracle_lib, dt, modes):
    """Odd sizes, zoom factors from 0.05 (targets of one voxel) to 1.6
    (upsampling first), a masked-out element."""
    from batchaug_b200 import ops
    dm, um, ac = modes
    rng = np.random.default_rng(len(dm) * 7 + len(um) + ac)
    x = rng.random((5, 2, 13, 20, 27)).astype(np.float32)
    if dt == "bf16":
        x = oracle_lib.to_bf16_bits(x)
    zoom = np.array([0.05, 0.37, 0.5, 1.0, 1.6], np.float32)
    mask = np.array([1, 1, 1, 1, 0], np.uint8) if um != "area" else np.ones(5, np.uint8)
    ref = oracle_lib.lowres(x, zoom, mask, dm, um, ac)
    out = ops.lowres3d(to_dev(x), to_dev(zoom), mask=to_dev(mask.astype(bool)),
                       downsample_mode=dm, upsample_mode=um, align_corners=ac)
    assert np.array_equal(to_np(out), ref)


def test_lowres_transform_sampling_and_keys(ba):
    torch.manual_seed(2)
    x = torch.rand(4, 1, 24, 20, 16, device="cuda")
    t = ba.RandSimulateLowResolution(prob=1.0, zoom_range=(0.4, 0.8))
    p = t.sample_params(4, x.shape, x.device)
    z = p["zoom_factor"].cpu()
    assert bool(((z >= 0.4) & (z < 0.8)).all())
    y = t.apply(x, p)
    assert y.shape == x.shape and not torch.equal(y, x)
    td = ba.RandSimulateLowResolutiond(["a", "b"], prob=1.0)
    torch.manual_seed(3)
    out = td({"a": x, "b": x.clone()})
    assert torch.equal(out["a"], out["b"])
    assert torch.equal(ba.RandSimulateLowResolution(prob=0.0)(x), x)
    # zoom 1: every target equals the input, nearest then trilinear is a copy
    same = ba.ops.lowres3d(x, torch.ones(4, device="cuda"))
    assert torch.equal(same, x)
    with pytest.raises(ValueError):
        ba.ops.lowres3d(x, torch.ones(4, device="cuda"), downsample_mode="bicubic")
