"""CUDA intensity chain (ba_intensity_chain, ba_minmax) against the oracle and
the reference's golden outputs.

Bar: noise (injected), scale, shift and ScaleIntensity are bit-exact; contrast
(powf), bias field (expf) are within 1e-5 abs in fp32 and 2 bf16 ulp in bf16;
in-kernel Philox noise is checked statistically and for determinism."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import as_f32, assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu


def _ops():
    from batchaug_b200 import _lib as L
    from batchaug_b200 import ops
    return L, ops


def _m(a):
    return to_dev(a).to(torch.uint8)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_single_ops(ba, tag):
    L, ops = _ops()
    g = load_golden(f"intensity_{tag}")
    x = to_dev(g["x"])
    one = lambda op: to_np(ops.intensity_chain(x, [op]))  # noqa: E731
    nz = to_dev(g["noise"])
    assert np.array_equal(one(ops.ChainOp(L.BA_OP_NOISE, mask=_m(g["noise_mask"]), noise=nz)),
                          g["noise_out"])
    assert np.array_equal(one(ops.ChainOp(L.BA_OP_SCALE, mask=_m(g["scale_mask"]),
                                          param=to_dev(g["factor"]))), g["scale_out"])
    assert np.array_equal(one(ops.ChainOp(L.BA_OP_SHIFT, flags=L.BA_SHIFT_SAFE,
                                          mask=_m(g["shift_mask"]),
                                          param=to_dev(g["offset"]))), g["shift_out"])
    assert_close_dtype(one(ops.ChainOp(L.BA_OP_CONTRAST, mask=_m(g["contrast_mask"]),
                                       param=to_dev(g["gamma"]))), g["contrast_out"])
    assert_close_dtype(one(ops.ChainOp(L.BA_OP_BIAS_FIELD, mask=_m(g["bias_mask"]),
                                       param=to_dev(g["coeffs"]), degree=3)), g["bias_out"])
    xc = to_dev(g["xconst"])
    resc = lambda flags, c0=0.0, c1=1.0, src=xc: to_np(ops.intensity_chain(  # noqa: E731
        src, [ops.ChainOp(L.BA_OP_RESCALE, flags=flags, c0=c0, c1=c1)]))
    both = L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV
    assert np.array_equal(resc(both | L.BA_RESCALE_CHANNEL), g["scaleint_cw_out"])
    assert np.array_equal(resc(both), g["scaleint_el_out"])
    assert np.array_equal(resc(both | L.BA_RESCALE_CHANNEL, -1.0, 3.0, x), g["scaleint_m13_out"])
    assert np.array_equal(resc(L.BA_RESCALE_FACTOR, 0.5, 0.0, x), g["scaleint_factor_out"])


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_via_transform_api(ba, tag):
    """The reference-facing classes with the reference's own params."""
    g = load_golden(f"intensity_{tag}")
    x = to_dev(g["x"])
    n = ba.RandGaussianNoise(prob=0.5, std=(0.1, 0.5))
    out = n.apply(x, {"mask": to_dev(g["noise_mask"]), "noise": to_dev(g["noise"])})
    assert np.array_equal(to_np(out), g["noise_out"])
    s = ba.RandScaleIntensity(prob=0.5, factors=0.2)
    out = s.apply(x, {"mask": to_dev(g["scale_mask"]), "factor": to_dev(g["factor"])})
    assert np.array_equal(to_np(out), g["scale_out"])
    c = ba.RandAdjustContrast(prob=0.5, gamma=(0.5, 2.0))
    out = c.apply(x, {"mask": to_dev(g["contrast_mask"]), "gamma": to_dev(g["gamma"])})
    assert_close_dtype(to_np(out), g["contrast_out"])
    b = ba.RandBiasField(prob=0.5)
    out = b.apply(x, {"mask": to_dev(g["bias_mask"]), "coeffs": to_dev(g["coeffs"])})
    assert_close_dtype(to_np(out), g["bias_out"])
    assert np.array_equal(to_np(ba.ScaleIntensity().apply(to_dev(g["xconst"]), {})),
                          g["scaleint_cw_out"])


def test_golden_chain_cfg3_fused(ba):
    """noise -> contrast -> scale -> shift -> ScaleIntensity as ONE chain call
    (three segments cut at the two min/max barriers)."""
    L, ops = _ops()
    g = load_golden("chain_cfg3")
    x = to_dev(g["x"])
    chain = [ops.ChainOp(L.BA_OP_NOISE, noise=to_dev(g["noise"])),
             ops.ChainOp(L.BA_OP_CONTRAST, param=to_dev(g["gamma"])),
             ops.ChainOp(L.BA_OP_SCALE, param=to_dev(g["factor"])),
             ops.ChainOp(L.BA_OP_SHIFT, param=to_dev(g["offset"])),
             ops.ChainOp(L.BA_OP_RESCALE, flags=L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV
                         | L.BA_RESCALE_CHANNEL, c0=0.0, c1=1.0)]
    out = to_np(ops.intensity_chain(x, chain))
    assert_close_dtype(out, g["out"])


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(4, 2, 10, 12, 8), (3, 3, 7, 9, 5), (2, 1, 32, 33, 31)])
def test_chain_vs_oracle(ba, oracle_lib, dt, shape):
    """Every op in one chain, odd shapes (scalar path), masks; vs the oracle
    applying the ops one at a time."""
    L, ops = _ops()
    O = oracle_lib
    rng = np.random.default_rng(sum(shape))
    B = shape[0]
    x = np.clip(0.5 + 0.2 * rng.standard_normal(shape), 0, 1).astype(np.float32)
    if dt == "bf16":
        x = O.to_bf16_bits(x)
    noise = (rng.standard_normal(shape) * 0.2).astype(np.float32)
    masks = [rng.random(B) < 0.6 for _ in range(6)]
    gamma = rng.uniform(0.5, 2.0, B).astype(np.float32)
    factor = rng.uniform(-0.2, 0.2, B).astype(np.float32)
    offset = rng.uniform(-0.1, 0.1, B).astype(np.float32)
    coeffs = rng.uniform(0, 0.1, (B, 20)).astype(np.float32)
    ref = O.noise_add(x, noise, masks[0])
    ref = O.adjust_contrast(ref, gamma, masks[1])
    ref = O.rand_scale(ref, factor, masks[2])
    ref = O.rand_shift(ref, offset, masks[3], safe=True)
    ref = O.bias_field(ref, coeffs, masks[4])
    ref = O.scale_intensity(ref, 0.0, 1.0, channel_wise=False)
    chain = [ops.ChainOp(L.BA_OP_NOISE, mask=_m(masks[0].astype(np.uint8)), noise=to_dev(noise)),
             ops.ChainOp(L.BA_OP_CONTRAST, mask=_m(masks[1].astype(np.uint8)), param=to_dev(gamma)),
             ops.ChainOp(L.BA_OP_SCALE, mask=_m(masks[2].astype(np.uint8)), param=to_dev(factor)),
             ops.ChainOp(L.BA_OP_SHIFT, flags=L.BA_SHIFT_SAFE, mask=_m(masks[3].astype(np.uint8)),
                         param=to_dev(offset)),
             ops.ChainOp(L.BA_OP_BIAS_FIELD, mask=_m(masks[4].astype(np.uint8)),
                         param=to_dev(coeffs), degree=3),
             ops.ChainOp(L.BA_OP_RESCALE, flags=L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV,
                         c0=0.0, c1=1.0)]
    out = to_np(ops.intensity_chain(to_dev(x), chain))
    # pow/exp differences propagate through the rescale: fp32 1e-5, bf16 2 ulp
    assert_close_dtype(out, ref)


def test_inplace_chain(ba, oracle_lib):
    L, ops = _ops()
    rng = np.random.default_rng(3)
    x = rng.random((2, 2, 8, 8, 8)).astype(np.float32)
    off = np.array([0.1, -0.2], np.float32)
    xd = to_dev(x)
    out = ops.intensity_chain(xd, [ops.ChainOp(L.BA_OP_SHIFT, param=to_dev(off)),
                                   ops.ChainOp(L.BA_OP_RESCALE, flags=3, c0=0.0, c1=1.0)],
                              inplace=True)
    assert out.data_ptr() == xd.data_ptr()
    ref = oracle_lib.scale_intensity(oracle_lib.rand_shift(x, off), 0.0, 1.0, channel_wise=False)
    assert np.array_equal(to_np(out), ref)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_minmax(ba, dt):
    _, ops = _ops()
    torch.manual_seed(0)
    x = torch.randn(6, 3, 17, 19, 23, device="cuda").to(dt)
    mn, mx = ops.minmax(x, 18)
    flat = x.float().reshape(18, -1)
    assert torch.equal(mn, flat.min(1).values) and torch.equal(mx, flat.max(1).values)
    x[2, 1, 3, 4, 5] = float("nan")
    mn, mx = ops.minmax(x, 18)
    assert torch.isnan(mn[7]) and torch.isnan(mx[7])
    assert not torch.isnan(mn[6])


def test_philox_noise_statistics_and_determinism(ba):
    """In-kernel noise: N(mean, std) per element, independent across voxels
    and channels, identical across keys / calls / shard layouts."""
    L, ops = _ops()
    B, C, H, W, D = 4, 2, 64, 64, 64
    x = torch.zeros(B, C, H, W, D, device="cuda")
    std = torch.tensor([0.1, 0.5, 1.0, 2.0], device="cuda")
    mean = torch.tensor([0.0, 1.0, -1.0, 0.5], device="cuda")
    op = ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, param=std, param2=mean, seed=1234)
    y = ops.intensity_chain(x, [op]).double()
    for b in range(B):
        v = y[b].flatten()
        assert abs(v.mean().item() - mean[b].item()) < 5 * std[b].item() / v.numel() ** 0.5
        assert abs(v.std().item() / std[b].item() - 1) < 0.01
    # standardized moments: skew ~0, kurtosis ~3
    z = ((y[0] - mean[0]) / std[0]).flatten()
    assert abs((z ** 3).mean().item()) < 0.02 and abs((z ** 4).mean().item() - 3) < 0.05
    # channels and neighbours uncorrelated
    assert abs(torch.corrcoef(torch.stack([y[1, 0].flatten(), y[1, 1].flatten()]))[0, 1]) < 0.01
    zz = y[2, 0].flatten()
    assert abs(torch.corrcoef(torch.stack([zz[:-1], zz[1:]]))[0, 1]) < 0.01
    # deterministic, and element b of a shard with offset o equals element o+b
    y2 = ops.intensity_chain(x, [op]).double()
    assert torch.equal(y, y2)
    op_shard = ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, param=std[2:],
                           param2=mean[2:], seed=1234, elem_offset=2)
    y3 = ops.intensity_chain(x[2:], [op_shard]).double()
    assert torch.equal(y3, y[2:])
    # mask 0 leaves the element untouched
    op_m = ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, param=std, param2=mean,
                       seed=1234, mask=torch.tensor([1, 0, 1, 0], dtype=torch.uint8,
                                                     device="cuda"))
    ym = ops.intensity_chain(x, [op_m])
    assert torch.equal(ym[1], x[1]) and torch.equal(ym[0].double(), y[0])


def test_noise_same_for_every_key(ba):
    """One sample_params, two keys of different dtype: same noise values."""
    torch.manual_seed(0)
    t = ba.RandGaussianNoised(keys=["a", "b"], prob=1.0, std=0.3)
    a = torch.zeros(2, 1, 16, 16, 16, device="cuda")
    out = t({"a": a, "b": a.bfloat16()})
    assert torch.equal(out["a"].bfloat16(), out["b"])


def test_errors(ba):
    L, ops = _ops()
    x = torch.zeros(2, 1, 4, 4, 4, device="cuda")
    with pytest.raises(ValueError):
        ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_BIAS_FIELD, param=torch.zeros(
            2, 20, device="cuda"), degree=9)])
    with pytest.raises(ValueError):
        ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_SCALE)])  # missing factor
    with pytest.raises(ValueError):
        ops.intensity_chain(x.half(), [ops.ChainOp(L.BA_OP_RESCALE, flags=3, c1=1.0)])
    with pytest.raises(ValueError):
        ba.RandBiasField(degree=0)


def test_full_size_config3_chain_properties(ba, oracle_lib):
    """Config 3 at full size (B=16, C=4, 128^3 bf16, prob 1): the L2-sliced
    three-segment chain equals the oracle on two elements, and the result of
    ScaleIntensity spans exactly [0, 1] per (element, channel)."""
    L, ops = _ops()
    torch.manual_seed(0)
    B, C = 16, 4
    x = (0.5 + 0.2 * torch.randn(B, C, 128, 128, 128, device="cuda")).clamp(0, 1).bfloat16()
    gen = np.random.default_rng(0)
    std = torch.tensor(gen.uniform(0.1, 0.5, B), dtype=torch.float32, device="cuda")
    gam = torch.tensor(gen.uniform(0.5, 2.0, B), dtype=torch.float32, device="cuda")
    fac = torch.tensor(gen.uniform(-0.2, 0.2, B), dtype=torch.float32, device="cuda")
    off = torch.tensor(gen.uniform(-0.1, 0.1, B), dtype=torch.float32, device="cuda")
    zero = torch.zeros(B, device="cuda")
    noise_op = ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, param=std, param2=zero, seed=9)
    rest = [ops.ChainOp(L.BA_OP_CONTRAST, param=gam), ops.ChainOp(L.BA_OP_SCALE, param=fac),
            ops.ChainOp(L.BA_OP_SHIFT, param=off),
            ops.ChainOp(L.BA_OP_RESCALE, flags=7, c0=0.0, c1=1.0)]
    out = ops.intensity_chain(x, [noise_op] + rest)
    # the same noise materialised by a noise-only chain on zeros (exact in fp32)
    nz = ops.intensity_chain(torch.zeros(2, C, 128, 128, 128, device="cuda"),
                             [ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, param=std[:2],
                                          param2=zero[:2], seed=9)])
    O = oracle_lib
    xs = to_np(x[:2])
    r = O.noise_add(xs, to_np(nz))
    r = O.adjust_contrast(r, to_np(gam[:2]))
    r = O.rand_scale(r, to_np(fac[:2]))
    r = O.rand_shift(r, to_np(off[:2]))
    r = O.scale_intensity(r, 0.0, 1.0)
    assert_close_dtype(to_np(out[:2]), r)
    f = out.float().reshape(B * C, -1)
    assert torch.equal(f.min(1).values, torch.zeros(B * C, device="cuda"))
    assert torch.equal(f.max(1).values, torch.ones(B * C, device="cuda"))
    assert as_f32(to_np(out[0, 0, 0, 0, :4])).dtype == np.float32
