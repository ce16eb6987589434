"""CUDA Gaussian taps, separable smoothing and elastic field vs the oracle and
the reference's golden outputs (fp32 within 1e-5, bf16 within 2 ulp)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu


def test_gauss_taps(ba):
    from batchaug_b200 import ops
    g = load_golden("intensity_f32")
    s = g["sigma_x"]
    K = ops.gauss_taps_len(float(np.maximum(s, 1e-6).max()), 4.0)
    assert K == g["kernel_h"].shape[1]
    taps = to_np(ops.gauss_taps(to_dev(s), K))
    np.testing.assert_allclose(taps, g["kernel_h"], rtol=0, atol=1e-7)
    ge = load_golden("elastic")
    Ke = ops.gauss_taps_len(float(ge["sigma"].max()), 3.0)
    assert Ke == ge["taps"].shape[1]


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_smooth_golden(ba, tag):
    g = load_golden(f"intensity_{tag}")
    x = to_dev(g["x"])
    t = ba.RandGaussianSmooth(prob=0.5)
    params = {"mask": to_dev(g["smooth_mask"]), "kernel_h": to_dev(g["kernel_h"]),
              "kernel_w": to_dev(g["kernel_w"]), "kernel_d": to_dev(g["kernel_d"])}
    assert_close_dtype(to_np(t.apply(x, params)), g["smooth_out"])
    ones = {**params, "mask": torch.ones(x.shape[0], dtype=torch.bool, device="cuda")}
    for pm in ("reflect", "replicate"):
        tp = ba.RandGaussianSmooth(prob=1.0, padding_mode=pm)
        assert_close_dtype(to_np(tp.apply(x, ones)), g[f"smooth_{pm}_out"])


@pytest.mark.parametrize("shape", [(2, 3, 9, 17, 12), (1, 1, 40, 8, 33)])
def test_smooth_vs_oracle(ba, oracle_lib, shape):
    from batchaug_b200 import ops
    rng = np.random.default_rng(5)
    x = rng.standard_normal(shape).astype(np.float32)
    B = shape[0]
    sig = rng.uniform(0.5, 3.0, (3, B)).astype(np.float32)
    taps = [oracle_lib.gaussian_1d_batch(s, 4.0) for s in sig]
    ref = oracle_lib.separable_gauss(x, *taps)
    out = ops.smooth3d(to_dev(x), *[to_dev(t) for t in taps])
    np.testing.assert_allclose(to_np(out), ref, rtol=0, atol=1e-5)


def test_elastic_grid_injected_u(ba):
    from batchaug_b200 import ops
    g = load_golden("elastic")
    B, _, H, W, D = g["u"].shape
    grid = ops.elastic_grid((B, H, W, D), to_dev(g["taps"]), to_dev(g["magnitude"]),
                            u=to_dev(g["u"]))
    np.testing.assert_allclose(to_np(grid), g["grid"], rtol=0, atol=1e-5)


def test_elastic_transform_end_to_end(ba):
    """Philox field: deterministic per seed, displacement statistics sane,
    magnitude 0 gives the identity grid's resample (an exact copy)."""
    torch.manual_seed(0)
    t = ba.Rand3DElastic(prob=1.0, sigma_range=(5.0, 7.0), magnitude_range=(50.0, 150.0))
    x = torch.rand(2, 2, 32, 32, 32, device="cuda")
    torch.manual_seed(1)
    p = t.sample_params(2, x.shape, x.device)
    torch.manual_seed(1)
    p2 = t.sample_params(2, x.shape, x.device)
    assert torch.equal(p["grid"], p2["grid"])
    out = t.apply(x, p)
    assert out.shape == x.shape and torch.isfinite(out).all()
    t0 = ba.Rand3DElastic(prob=1.0, sigma_range=(5.0, 7.0), magnitude_range=(0.0, 0.0))
    p0 = t0.sample_params(2, x.shape, x.device)
    out0 = t0.apply(x, p0, mode="nearest")
    assert torch.equal(out0, x)
