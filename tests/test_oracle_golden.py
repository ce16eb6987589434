"""Pin the CPU oracle against the reference's own outputs (tests/golden).

Resample, noise, scale, shift and ScaleIntensity are bit-exact restatements of
the reference; contrast (pow), bias field (exp) and the Gaussian smoothing
(conv3d accumulation order) differ from torch's CPU kernels only by libm /
summation-order rounding, bounded here by a few fp32 ulp."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden

MODES = ("bilinear", "nearest")
PADS = ("zeros", "border", "reflection")


def f32(a: np.ndarray) -> np.ndarray:
    import oracle
    return oracle.bf16_bits_to_f32(a) if a.dtype == np.uint16 else a


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("pad", PADS)
@pytest.mark.parametrize("align", [0, 1])
def test_resample_modes_exact(oracle_lib, dt, mode, pad, align):
    g = load_golden("resample_modes")
    x = g["x"] if dt == "f32" else g["x_bf16"]
    ref = g[f"{dt}_{mode}_{pad}_{align}"]
    out = oracle_lib.resample3d(x, theta=g["theta"], mode=mode, padding=pad,
                                align_corners=bool(align))
    assert np.array_equal(out, ref)
    if not align:
        # monai_affine_to_theta restated exactly: same output from the affine
        out2 = oracle_lib.resample3d(x, affine=g["affine"], mode=mode, padding=pad)
        assert np.array_equal(out2, ref)


def test_affine_to_theta_exact(oracle_lib):
    g = load_golden("resample_modes")
    th = oracle_lib.affine_to_theta(g["affine"], g["x"].shape[2:])
    assert np.array_equal(th, g["theta"][:, :3, :])


def test_affine_apply_partial_mask(oracle_lib):
    g = load_golden("affine_apply_border")
    out = oracle_lib.resample3d(g["x"], theta=g["theta"], padding="border", mask=g["mask"])
    assert np.array_equal(out, g["out"])
    # masked-out element is a bit copy of the input
    assert np.array_equal(out[1], g["x"][1])


def test_compose_materialize(oracle_lib):
    g = load_golden("compose_materialize")
    vo = oracle_lib.resample3d(g["vol"], affine=g["affine"], mode="bilinear", mask=g["mask"])
    so = oracle_lib.resample3d(g["seg"], affine=g["affine"], mode="nearest", mask=g["mask"])
    assert np.array_equal(vo, g["vol_out"])
    assert np.array_equal(so, g["seg_out"])


def test_flip_rot90_are_exact_nearest_resamples(oracle_lib):
    g = load_golden("flip_rot90")
    fo = oracle_lib.resample3d(g["x"], affine=g["flip_affine"], mode="nearest")
    assert np.array_equal(fo, g["flip_out"])
    ro = oracle_lib.resample3d(g["x"], affine=g["rot_affine"], mode="nearest")
    assert np.array_equal(ro, g["rot_out"])


def test_elastic_grid_and_resample(oracle_lib):
    g = load_golden("elastic")
    taps = oracle_lib.gaussian_1d_batch(g["sigma"], truncated=3.0)
    assert taps.shape == g["taps"].shape
    np.testing.assert_allclose(taps, g["taps"], rtol=0, atol=1e-7)
    grid = oracle_lib.elastic_grid(g["u"], g["taps"], g["magnitude"])
    np.testing.assert_allclose(grid, g["grid"], rtol=0, atol=1e-6)
    vo = oracle_lib.resample3d(g["vol"], grid=g["grid"], mode="bilinear", align_corners=True)
    so = oracle_lib.resample3d(g["seg"], grid=g["grid"], mode="nearest", align_corners=True)
    assert np.array_equal(vo, g["vol_out"])
    assert np.array_equal(so, g["seg_out"])


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_intensity_ops(oracle_lib, tag):
    O = oracle_lib
    g = load_golden(f"intensity_{tag}")
    x = g["x"]
    assert np.array_equal(O.noise_add(x, g["noise"], g["noise_mask"]), g["noise_out"])
    assert np.array_equal(O.rand_scale(x, g["factor"], g["scale_mask"]), g["scale_out"])
    assert np.array_equal(O.rand_shift(x, g["offset"], g["shift_mask"], safe=True), g["shift_out"])
    xc = g["xconst"]
    assert np.array_equal(O.scale_intensity(xc, 0.0, 1.0), g["scaleint_cw_out"])
    assert np.array_equal(O.scale_intensity(xc, 0.0, 1.0, channel_wise=False),
                          g["scaleint_el_out"])
    assert np.array_equal(O.scale_intensity(x, -1.0, 3.0), g["scaleint_m13_out"])
    assert np.array_equal(O.scale_intensity(x, factor=0.5), g["scaleint_factor_out"])
    # libm pow / exp and conv summation order: a few fp32 ulp (bf16: exact or 1 ulp)
    tol = 2e-7 if tag == "f32" else 1e-2
    np.testing.assert_allclose(f32(O.adjust_contrast(x, g["gamma"], g["contrast_mask"])),
                               f32(g["contrast_out"]), rtol=0, atol=tol)
    np.testing.assert_allclose(f32(O.bias_field(x, g["coeffs"], g["bias_mask"])),
                               f32(g["bias_out"]), rtol=0, atol=4 * tol)
    sm = O.separable_gauss(x, g["kernel_h"], g["kernel_w"], g["kernel_d"])
    sm = np.where(g["smooth_mask"].astype(bool)[:, None, None, None, None], sm, x)
    np.testing.assert_allclose(f32(sm), f32(g["smooth_out"]), rtol=0, atol=tol)
    for pm in ("reflect", "replicate"):
        smp = O.separable_gauss(x, g["kernel_h"], g["kernel_w"], g["kernel_d"], padding_mode=pm)
        np.testing.assert_allclose(f32(smp), f32(g[f"smooth_{pm}_out"]), rtol=0, atol=tol)


def test_gaussian_taps(oracle_lib):
    g = load_golden("intensity_f32")
    taps = oracle_lib.gaussian_1d_batch(g["sigma_x"], truncated=4.0)
    assert taps.shape == g["kernel_h"].shape
    np.testing.assert_allclose(taps, g["kernel_h"], rtol=0, atol=1e-7)


def test_chain_cfg3(oracle_lib):
    O = oracle_lib
    g = load_golden("chain_cfg3")
    y = O.noise_add(g["x"], g["noise"])
    y = O.adjust_contrast(y, g["gamma"])
    y = O.rand_scale(y, g["factor"])
    y = O.rand_shift(y, g["offset"])
    y = O.scale_intensity(y, 0.0, 1.0)
    ref = g["out"]
    # the only non-restated op is pow (libm vs torch): at most 1 bf16 ulp, rarely
    diff = np.abs(f32(y) - f32(ref))
    assert diff.max() <= 2 ** -7
    assert (y != ref).mean() < 1e-3


def test_pipeline_cfg1(oracle_lib):
    O = oracle_lib
    g = load_golden("pipeline_cfg1")
    vo = O.resample3d(g["vol"], affine=g["affine"], mode="bilinear", mask=g["mask"])
    so = O.resample3d(g["seg"], affine=g["affine"], mode="nearest", mask=g["mask"])
    vo = O.noise_add(vo, g["noise"], g["noise_mask"])
    vo = O.scale_intensity(vo, 0.0, 1.0)
    assert np.array_equal(so, g["seg_out"])
    assert np.array_equal(vo, g["vol_out"])


def _close(out, ref, f32_atol=2e-6, bf16_ulp=1):
    """fp32 within a few ulp of values ~1; bf16 within one ulp (the reductions
    and libm differ from torch's only in the last bits)."""
    if ref.dtype == np.uint16:
        from helpers import bf16_ulp_diff
        assert bf16_ulp_diff(out, ref) <= bf16_ulp
    else:
        np.testing.assert_allclose(out, ref, rtol=0, atol=f32_atol)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_stats_ops(oracle_lib, tag):
    """Rician noise (absolute and relative std), std shift (per element / per
    channel, all values / nonzero values) and fixed-mean scaling against the
    reference's outputs."""
    g = load_golden(f"intensity_stats_{tag}")
    x = g["x"]
    for k, rel in (("rician", False), ("rician_rel", True)):
        out = oracle_lib.rician(x, g[f"{k}_u1"], g[f"{k}_u2"], g[f"{k}_std"], relative=rel,
                                mask=g[f"{k}_mask"])
        _close(out, g[f"{k}_out"])
    for cw in (0, 1):
        for nz in (0, 1):
            k = f"stdshift_cw{cw}_nz{nz}"
            out = oracle_lib.std_shift(x, g[f"{k}_factor"], mask=g[f"{k}_mask"], nonzero=nz,
                                       channel_wise=cw)
            _close(out, g[f"{k}_out"])
        k = f"fixedmean_cw{cw}"
        out = oracle_lib.fixed_mean(x, g[f"{k}_factor"], mask=g[f"{k}_mask"], channel_wise=cw)
        _close(out, g[f"{k}_out"])


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_sharpen(oracle_lib, tag):
    """RandGaussianSharpen: the combination step is bit-exact on the
    reference's own blurs; each blur is within the smoothing bar, and the
    whole op within that bar amplified by the unsharp mask, (1 + 2 alpha)."""
    O = oracle_lib
    g = load_golden(f"sharpen_{tag}")
    x = g["x"]
    for name, pm in (("none", None), ("reflect", "reflect"), ("replicate", "replicate")):
        k1 = [g[f"{name}_kernel1_{a}"] for a in "hwd"]
        k2 = [g[f"{name}_kernel2_{a}"] for a in "hwd"]
        alpha, mask = g[f"{name}_alpha"], g[f"{name}_mask"]
        comb = O.sharpen_combine(g[f"{name}_blurred"], g[f"{name}_double_blurred"], x, alpha,
                                 mask)
        assert np.array_equal(comb, g[f"{name}_out"])
        blur_tol = 2e-7 if tag == "f32" else 2.0 ** -8
        bl = O.separable_gauss(x, *k1, padding_mode=pm)
        np.testing.assert_allclose(f32(bl), f32(g[f"{name}_blurred"]), rtol=0, atol=blur_tol)
        db = O.separable_gauss(g[f"{name}_blurred"], *k2, padding_mode=pm)
        np.testing.assert_allclose(f32(db), f32(g[f"{name}_double_blurred"]), rtol=0,
                                   atol=blur_tol)
        full = O.sharpen(x, k1, k2, alpha, mask, padding_mode=pm)
        amp = 1.0 + 2.0 * float(np.max(alpha))
        np.testing.assert_allclose(f32(full), f32(g[f"{name}_out"]), rtol=0, atol=amp * blur_tol)
        # the sampled params: sigma2 in [sigma2, sigma1] (scalar) or its range
        for a in "xyz":
            s1, s2 = g[f"{name}_sigma1_{a}"], g[f"{name}_sigma2_{a}"]
            assert np.all((s1 >= 0.5) & (s1 < 1.0))
            if name == "reflect":
                assert np.all((s2 >= 0.3) & (s2 < 0.6))
            else:
                assert np.all((s2 >= 0.5) & (s2 <= s1))
        for a, s in zip("hwd", "xyz"):
            np.testing.assert_allclose(O.gaussian_1d_batch(g[f"{name}_sigma1_{s}"]),
                                       g[f"{name}_kernel1_{a}"], rtol=0, atol=1e-7)


LOWRES_MODES = (("nearest", "trilinear", False), ("nearest-exact", "trilinear", False),
                ("nearest", "trilinear", True), ("trilinear", "trilinear", False),
                ("trilinear", "nearest", True), ("area", "trilinear", False),
                ("nearest-exact", "area", False), ("area", "nearest-exact", False))


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_lowres(oracle_lib, tag):
    """RandSimulateLowResolution for every downsample/upsample pair: bit-exact
    against the reference's outputs in fp32 and bf16."""
    g = load_golden(f"lowres_{tag}")
    for i, (dm, um, ac) in enumerate(LOWRES_MODES):
        out = oracle_lib.lowres(g["x"], g[f"m{i}_zoom"], g[f"m{i}_mask"], dm, um, ac)
        assert np.array_equal(out, g[f"m{i}_out"]), (dm, um, ac)
