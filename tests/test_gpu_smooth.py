"""CUDA Gaussian taps, separable smoothing and elastic field vs the oracle and
the reference's golden outputs (fp32 within 1e-5, bf16 within 2 ulp)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import as_f32, assert_close_dtype, to_dev, to_np

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


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("pm", [None, "reflect", "replicate"])
@pytest.mark.parametrize("shape,sig", [
    ((2, 2, 130, 20, 40), (0.3, 1.2)),   # K <= 11, H split into chunks
    ((2, 1, 50, 18, 20), (0.6, 1.0)),    # K 7..9: KMAX 9
    ((2, 2, 40, 24, 36), (1.2, 1.5)),    # K 11..13: KMAX 13
    ((1, 3, 136, 35, 33), (1.0, 2.8)),   # K 9..23, ragged W/D, H in chunks for K <= 15
    ((3, 1, 24, 16, 32), (2.0, 2.7)),    # K = 23, one chunk, exact tiles
])
def test_smooth_stream_vs_oracle(ba, oracle_lib, dt, pm, shape, sig):
    """The streaming smoother (taps up to 23) across padding modes, ragged
    W/D blocks and H chunks, with a masked-out element.  Intensities in
    [0, 1): with positive taps nothing cancels, so the bf16 bar (2 ulp)
    applies to every voxel; zero-mean data is covered in fp32 above."""
    from batchaug_b200 import ops
    O = oracle_lib
    rng = np.random.default_rng(sum(shape) + len(str(pm)))
    x = rng.random(shape).astype(np.float32)
    if dt == "bf16":
        x = O.to_bf16_bits(x)
    B = shape[0]
    s = rng.uniform(*sig, (3, B)).astype(np.float32)
    taps = [O.gaussian_1d_batch(si, 4.0) for si in s]
    mask = np.ones(B, bool)
    mask[0] = False
    ref = O.separable_gauss(x, *taps, padding_mode=pm)
    ref[0] = x[0]
    out = ops.smooth3d(to_dev(x), *[to_dev(t) for t in taps], mask=to_dev(mask),
                       padding_mode=pm)
    o = to_np(out)
    diff = np.abs(as_f32(o).astype(np.float64) - as_f32(ref))
    try:
        assert_close_dtype(o, ref)
    except AssertionError:
        at = np.unravel_index(diff.argmax(), diff.shape)
        raise AssertionError(f"max |diff| {diff.max()} at {at}: {as_f32(o)[at]} vs "
                             f"{as_f32(ref)[at]}") from None


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("pm", [None, "reflect", "replicate"])
@pytest.mark.parametrize("shape,sig", [
    ((2, 2, 40, 36, 44), (3.0, 3.8)),    # K 25..31: KMAX 31
    ((2, 2, 34, 40, 36), (4.0, 5.2)),    # K 33..43: KMAX 43 (39 and 41 pad it)
    ((1, 3, 30, 50, 33), (4.5, 5.5)),    # K 37..45: KMAX 43 or 47, ragged D
    ((2, 1, 70, 64, 66), (7.0, 7.8)),    # K 57..63: KMAX 63
    ((1, 2, 760, 20, 20), (3.0, 3.8)),   # H line too long to stage: the ring walk
])
def test_smooth_wide_vs_oracle(ba, oracle_lib, dt, pm, shape, sig):
    """The wide-tap path (D rows, then W and H as staged column tiles, or
    the register-ring walk for lines too long to stage) across padding
    modes, sizes and a masked-out element."""
    from batchaug_b200 import ops
    O = oracle_lib
    rng = np.random.default_rng(sum(shape) * 3 + len(str(pm)))
    x = rng.random(shape).astype(np.float32)
    if dt == "bf16":
        x = O.to_bf16_bits(x)
    B = shape[0]
    s = rng.uniform(*sig, (3, B)).astype(np.float32)
    taps = [O.gaussian_1d_batch(si, 4.0) for si in s]
    if pm == "reflect" and max(t.shape[1] for t in taps) // 2 >= min(shape[2:]):
        pytest.skip("reflect needs K/2 < size")
    mask = np.ones(B, bool)
    mask[-1] = B == 1
    ref = O.separable_gauss(x, *taps, padding_mode=pm)
    if not mask[-1]:
        ref[-1] = x[-1]
    out = ops.smooth3d(to_dev(x), *[to_dev(t) for t in taps], mask=to_dev(mask),
                       padding_mode=pm)
    assert_close_dtype(to_np(out), ref)


def test_elastic_grid_wide_path_properties(ba, oracle_lib):
    """Philox field generated inside the D pass: deterministic, keyed on the
    global element (a shard with an offset reproduces the same grid), and
    the D-unaligned fallback (draw through scratch) agrees with the oracle
    on an injected field."""
    from batchaug_b200 import ops
    B, H, W, D = 3, 20, 22, 24
    taps = ops.gauss_taps(torch.tensor([5.0, 6.0, 7.0], device="cuda"),
                          ops.gauss_taps_len(7.0, 3.0))
    mag = torch.tensor([50.0, 100.0, 150.0], device="cuda")
    g1 = ops.elastic_grid((B, H, W, D), taps, mag, seed=99)
    g2 = ops.elastic_grid((B, H, W, D), taps, mag, seed=99)
    assert torch.equal(g1, g2)
    g3 = ops.elastic_grid((2, H, W, D), taps[1:], mag[1:], seed=99, elem_offset=1)
    assert torch.equal(g3, g1[1:])
    rng = np.random.default_rng(0)
    u = rng.random((2, 3, 9, 10, 13)).astype(np.float32)  # D = 13: not a multiple of 4
    t2 = oracle_lib.gaussian_1d_batch(np.array([5.5, 6.5], np.float32), 3.0)
    ref = oracle_lib.elastic_grid(u, t2, np.array([60.0, 120.0], np.float32))
    got = ops.elastic_grid((2, 9, 10, 13), to_dev(t2), to_dev(np.array([60.0, 120.0], np.float32)),
                           u=to_dev(u))
    np.testing.assert_allclose(to_np(got), ref, rtol=0, atol=1e-5)
