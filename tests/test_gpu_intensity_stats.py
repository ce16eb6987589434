"""CUDA intensity ops that read a statistic of their own input
(RandRicianNoise, RandStdShiftIntensity, RandScaleIntensityFixedMean) against
the reference's golden outputs and the oracle.

Bar: fp32 within 1e-5 abs, bf16 within 2 ulp.  Rician noise with injected
unit normals and an absolute std is bit-exact against the oracle (one
correctly rounded fp32 op at a time); the reference's own fp32 outputs differ
from that by 1 ulp on a few elements because torch's CPU sqrt is not
correctly rounded.  In-kernel Philox draws are checked statistically and for
determinism."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu


def _ops():
    from batchaug_b200 import _lib as L
    from batchaug_b200 import ops
    return L, ops


def _m(a):
    return to_dev(np.asarray(a).astype(np.uint8)).to(torch.uint8)


def _rician_op(L, ops, g, k, rel):
    return ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_RELATIVE if rel else 0,
                       mask=_m(g[f"{k}_mask"]), param=to_dev(g[f"{k}_std"]),
                       noise=to_dev(g[f"{k}_u1"]), param2=to_dev(g[f"{k}_u2"]), c0=0.0)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_stats_ops(ba, oracle_lib, tag):
    L, ops = _ops()
    g = load_golden(f"intensity_stats_{tag}")
    x = to_dev(g["x"])
    one = lambda op: to_np(ops.intensity_chain(x, [op]))  # noqa: E731
    for k, rel in (("rician", False), ("rician_rel", True)):
        out = one(_rician_op(L, ops, g, k, rel))
        assert_close_dtype(out, g[f"{k}_out"])
        if not rel:
            ref = oracle_lib.rician(g["x"], g[f"{k}_u1"], g[f"{k}_u2"], g[f"{k}_std"],
                                    mask=g[f"{k}_mask"])
            assert np.array_equal(out, ref)
    for cw in (0, 1):
        for nz in (0, 1):
            k = f"stdshift_cw{cw}_nz{nz}"
            flags = (L.BA_STD_NONZERO if nz else 0) | (L.BA_STAT_CHANNEL if cw else 0)
            out = one(ops.ChainOp(L.BA_OP_STD_SHIFT, flags=flags, mask=_m(g[f"{k}_mask"]),
                                  param=to_dev(g[f"{k}_factor"])))
            assert_close_dtype(out, g[f"{k}_out"])
        k = f"fixedmean_cw{cw}"
        out = one(ops.ChainOp(L.BA_OP_FIXED_MEAN, flags=L.BA_STAT_CHANNEL if cw else 0,
                              mask=_m(g[f"{k}_mask"]), param=to_dev(g[f"{k}_factor"])))
        assert_close_dtype(out, g[f"{k}_out"])


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_stats_via_transform_api(ba, tag):
    """The reference-facing classes given the reference's own params."""
    g = load_golden(f"intensity_stats_{tag}")
    x = to_dev(g["x"])
    for k, rel in (("rician", False), ("rician_rel", True)):
        t = ba.RandRicianNoise(prob=0.7, std=0.2, relative=rel)
        p = {"mask": to_dev(g[f"{k}_mask"]), "noise_std": to_dev(g[f"{k}_std"]),
             "u1": to_dev(g[f"{k}_u1"]), "u2": to_dev(g[f"{k}_u2"])}
        assert_close_dtype(to_np(t.apply(x, p)), g[f"{k}_out"])
    for cw in (False, True):
        for nz in (False, True):
            k = f"stdshift_cw{int(cw)}_nz{int(nz)}"
            t = ba.RandStdShiftIntensity(prob=0.7, factors=(-2.0, 2.0), nonzero=nz,
                                         channel_wise=cw)
            p = {"mask": to_dev(g[f"{k}_mask"]), "factor": to_dev(g[f"{k}_factor"])}
            assert_close_dtype(to_np(t.apply(x, p)), g[f"{k}_out"])
        k = f"fixedmean_cw{int(cw)}"
        t = ba.RandScaleIntensityFixedMean(prob=0.7, factors=0.5, channel_wise=cw)
        p = {"mask": to_dev(g[f"{k}_mask"]), "factor": to_dev(g[f"{k}_factor"])}
        assert_close_dtype(to_np(t.apply(x, p)), g[f"{k}_out"])


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(4, 2, 10, 12, 8), (3, 3, 7, 9, 5), (2, 2, 32, 33, 31)])
def test_stats_chain_vs_oracle(ba, oracle_lib, dt, shape):
    """scale -> std shift -> fixed mean -> relative Rician -> std shift as
    one chain: every statistic is reduced in the segment that produces its
    input (odd shapes take the scalar path, even ones the vector path)."""
    L, ops = _ops()
    O = oracle_lib
    rng = np.random.default_rng(sum(shape) + 7)
    B = shape[0]
    x = np.clip(0.5 + 0.2 * rng.standard_normal(shape), 0, 1).astype(np.float32)
    x[0, 0, : shape[2] // 2] = 0.0
    if dt == "bf16":
        x = O.to_bf16_bits(x)
    masks = [rng.random(B) < 0.7 for _ in range(5)]
    for m in masks:
        m[0] = True
    f_scale = rng.uniform(-0.2, 0.2, B).astype(np.float32)
    f_std = rng.uniform(-2, 2, B).astype(np.float32)
    f_mean = rng.uniform(-0.5, 0.5, B).astype(np.float32)
    sd = rng.uniform(0, 0.2, B).astype(np.float32)
    u1 = rng.standard_normal(shape).astype(np.float32)
    u2 = rng.standard_normal(shape).astype(np.float32)
    f_std2 = rng.uniform(-1, 1, B).astype(np.float32)
    ref = O.rand_scale(x, f_scale, masks[0])
    ref = O.std_shift(ref, f_std, masks[1], nonzero=True, channel_wise=True)
    ref = O.fixed_mean(ref, f_mean, masks[2], channel_wise=False)
    ref = O.rician(ref, u1, u2, sd, mean=0.05, relative=True, mask=masks[3])
    ref = O.std_shift(ref, f_std2, masks[4], nonzero=False, channel_wise=False)
    chain = [ops.ChainOp(L.BA_OP_SCALE, mask=_m(masks[0]), param=to_dev(f_scale)),
             ops.ChainOp(L.BA_OP_STD_SHIFT, flags=L.BA_STD_NONZERO | L.BA_STAT_CHANNEL,
                         mask=_m(masks[1]), param=to_dev(f_std)),
             ops.ChainOp(L.BA_OP_FIXED_MEAN, mask=_m(masks[2]), param=to_dev(f_mean)),
             ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_RELATIVE, mask=_m(masks[3]),
                         param=to_dev(sd), noise=to_dev(u1), param2=to_dev(u2), c0=0.05),
             ops.ChainOp(L.BA_OP_STD_SHIFT, mask=_m(masks[4]), param=to_dev(f_std2))]
    out = to_np(ops.intensity_chain(to_dev(x), chain))
    assert_close_dtype(out, ref)


def test_stats_after_minmax_ops(ba, oracle_lib):
    """Moments and min/max consumers interleaved: contrast (min/max) ->
    fixed mean (mean) -> ScaleIntensity (min/max) -> std shift (std)."""
    L, ops = _ops()
    O = oracle_lib
    rng = np.random.default_rng(11)
    shape = (3, 2, 16, 16, 16)
    x = rng.random(shape).astype(np.float32)
    gam = rng.uniform(0.5, 2.0, 3).astype(np.float32)
    fm = rng.uniform(-0.5, 0.5, 3).astype(np.float32)
    fs = rng.uniform(-2, 2, 3).astype(np.float32)
    ref = O.adjust_contrast(x, gam)
    ref = O.fixed_mean(ref, fm, channel_wise=True)
    ref = O.scale_intensity(ref, 0.0, 1.0, channel_wise=True)
    ref = O.std_shift(ref, fs)
    chain = [ops.ChainOp(L.BA_OP_CONTRAST, param=to_dev(gam)),
             ops.ChainOp(L.BA_OP_FIXED_MEAN, flags=L.BA_STAT_CHANNEL, param=to_dev(fm)),
             ops.ChainOp(L.BA_OP_RESCALE, flags=L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV
                         | L.BA_RESCALE_CHANNEL, c0=0.0, c1=1.0),
             ops.ChainOp(L.BA_OP_STD_SHIFT, param=to_dev(fs))]
    assert_close_dtype(to_np(ops.intensity_chain(to_dev(x), chain)), ref)


def test_philox_rician_statistics_and_determinism(ba):
    """In-kernel draws on a zero volume: sqrt(n1^2 + n2^2) with
    n ~ N(mu, s) has E[y^2] = 2 (mu^2 + s^2), and for mu = 0 is Rayleigh
    (mean s sqrt(pi/2)); identical across calls and shard layouts; masked
    elements untouched."""
    L, ops = _ops()
    B, C, H, W, D = 4, 2, 64, 64, 64
    x = torch.zeros(B, C, H, W, D, device="cuda")
    sd = torch.tensor([0.1, 0.5, 1.0, 2.0], device="cuda")
    op = ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_PHILOX, param=sd, seed=77)
    y = ops.intensity_chain(x, [op]).double()
    n = y[0].numel()
    for b in range(B):
        s = sd[b].item()
        v = y[b].flatten()
        assert abs(v.mean().item() / (s * (np.pi / 2) ** 0.5) - 1) < 0.005
        assert abs((v ** 2).mean().item() / (2 * s * s) - 1) < 0.01
    assert bool((y >= 0).all())
    # with a mean: E[y^2] = 2 (mu^2 + s^2)
    opm = ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_PHILOX, param=sd, seed=77, c0=0.5)
    ym = ops.intensity_chain(x, [opm]).double()
    for b in range(B):
        s = sd[b].item()
        assert abs((ym[b] ** 2).mean().item() / (2 * (0.25 + s * s)) - 1) < 0.01
    # neighbours and channels uncorrelated
    z = y[1, 0].flatten()
    assert abs(torch.corrcoef(torch.stack([z[:-1], z[1:]]))[0, 1]) < 0.01
    assert abs(torch.corrcoef(torch.stack([y[1, 0].flatten(), y[1, 1].flatten()]))[0, 1]) < 0.01
    assert n > 0
    # the Rician draws are a different stream from the Gaussian noise
    gn = ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_NOISE, flags=L.BA_NOISE_PHILOX, param=sd,
                                             param2=torch.zeros(B, device="cuda"), seed=77)])
    assert not torch.equal(gn.abs().double(), y)
    # deterministic, shard-invariant, masks respected
    assert torch.equal(ops.intensity_chain(x, [op]).double(), y)
    op_s = ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_PHILOX, param=sd[1:], seed=77,
                       elem_offset=1)
    assert torch.equal(ops.intensity_chain(x[1:], [op_s]).double(), y[1:])
    xr = torch.rand(B, C, H, W, D, device="cuda")
    op_m = ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_PHILOX, param=sd, seed=77,
                       mask=torch.tensor([0, 1, 0, 1], dtype=torch.uint8, device="cuda"))
    ym = ops.intensity_chain(xr, [op_m])
    assert torch.equal(ym[0], xr[0]) and torch.equal(ym[2], xr[2])
    assert not torch.equal(ym[1], xr[1])


def test_philox_rician_scalar_and_vector_paths_agree(ba):
    """The same draws whether the chain runs its 4/8-wide path or the
    scalar path (an odd voxel count forces the scalar path)."""
    L, ops = _ops()
    B, C = 2, 3
    sd = torch.tensor([0.3, 0.7], device="cuda")
    x = torch.rand(B, C, 8, 8, 9, device="cuda")
    op = ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_PHILOX, param=sd, seed=5)
    vec = ops.intensity_chain(x, [op])
    # a strided view of a larger buffer is made contiguous at an odd offset
    big = torch.zeros(B * C * 8 * 8 * 9 + 1, device="cuda")
    big[1:] = x.flatten()
    xs = big[1:].view(B, C, 8, 8, 9)
    sca = ops.intensity_chain(xs, [op])
    assert torch.equal(vec, sca)


def test_transforms_sample_and_apply(ba):
    """sample_params -> apply through the classes, dict wrappers share the
    draws across keys, and a relative Rician with a zero-variance input
    leaves it unchanged."""
    torch.manual_seed(3)
    a = torch.rand(2, 1, 16, 16, 16, device="cuda")
    t = ba.RandRicianNoised(keys=["a", "b"], prob=1.0, std=0.3)
    out = t({"a": a, "b": a.bfloat16()})
    ref = out["a"].bfloat16()
    diff = (ref.float() - out["b"].float()).abs()
    assert float(diff.max()) <= 2 ** -7 * float(ref.float().abs().max())
    const = torch.full((2, 1, 8, 8, 8), 0.25, device="cuda")
    rel = ba.RandRicianNoise(prob=1.0, std=0.5, relative=True)
    assert torch.equal(rel(const), const)
    s = ba.RandStdShiftIntensity(prob=1.0, factors=(1.0, 1.0))
    y = s(a)
    std = a.flatten(1).std(1)
    assert torch.allclose(y - a, std[:, None, None, None, None].expand_as(a), atol=1e-5)
    fm = ba.RandScaleIntensityFixedMean(prob=1.0, factors=(0.5, 0.5), channel_wise=True)
    y = fm(a)
    assert torch.allclose(y.mean((2, 3, 4)), a.mean((2, 3, 4)), atol=1e-5)
    assert torch.allclose(y.std((2, 3, 4)), 1.5 * a.std((2, 3, 4)), rtol=1e-4)


def test_compose_fuses_stats_ops(ba):
    """Compose runs a run of fusible dict transforms as one chain per key;
    the result equals applying them one by one with the same draws (to the
    last bits of the fp32 statistics, which the two plans sum in different
    orders)."""
    keys = ["img"]
    mk = lambda: [ba.RandScaleIntensityd(keys, prob=1.0, factors=0.2),  # noqa: E731
                  ba.RandStdShiftIntensityd(keys, prob=1.0, factors=(-1, 1), nonzero=True),
                  ba.RandRicianNoised(keys, prob=1.0, std=0.1, relative=True),
                  ba.RandScaleIntensityFixedMeand(keys, prob=1.0, channel_wise=True)]
    x = torch.rand(2, 2, 20, 24, 16, device="cuda")
    torch.manual_seed(21)
    fused = ba.Compose(mk())({"img": x})["img"]
    torch.manual_seed(21)
    d = {"img": x}
    for t in mk():
        d = t(d)
    assert (fused - d["img"]).abs().max().item() <= 1e-5


def test_stats_errors(ba):
    L, ops = _ops()
    x = torch.zeros(2, 1, 4, 4, 4, device="cuda")
    sd = torch.ones(2, device="cuda")
    with pytest.raises(ValueError):  # injected u1 without u2
        ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_RICIAN, param=sd, noise=torch.zeros_like(x))])
    with pytest.raises(ValueError):  # no noise_std
        ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_RICIAN, flags=L.BA_RICIAN_PHILOX)])
    with pytest.raises(ValueError):
        ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_STD_SHIFT)])
    with pytest.raises(ValueError):
        ops.intensity_chain(x, [ops.ChainOp(L.BA_OP_FIXED_MEAN)])
    t = ba.RandRicianNoise(prob=1.0)
    with pytest.raises(ValueError):
        t.apply(x, {"mask": torch.ones(2, dtype=torch.bool, device="cuda"), "noise_std": sd,
                    "u1": torch.zeros(2, 1, 4, 4, 5), "u2": torch.zeros(2, 1, 4, 4, 5)})
