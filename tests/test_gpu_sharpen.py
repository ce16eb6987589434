"""CUDA unsharp masking (ba_sharpen3d, RandGaussianSharpen) against the
reference's golden outputs and the oracle.

The op is blurred + alpha * (blurred - double_blurred) with alpha in
[10, 30], so any difference in a blur is amplified up to (1 + 2 alpha)
times.  The bar is therefore stated per stage: each blur within the
smoothing bar (fp32 1e-5, bf16 2 ulp); the combination bit-exact given the
two blurs (the kernel's epilogue against the oracle's per-op arithmetic on
the same blurs); the whole op within the smoothing bar times (1 + 2 alpha)
in fp32."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import as_f32, assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu

CASES = (("none", None), ("reflect", "reflect"), ("replicate", "replicate"))


def _ops():
    from batchaug_b200 import ops
    return ops


def _check_composition(ops, O, x, k1, k2, alpha, mask, pm, out):
    """out equals the oracle's combination of the GPU's own two blurs."""
    bl = ops.smooth3d(x, *k1, padding_mode=pm)
    db = ops.smooth3d(bl, *k2, padding_mode=pm)
    ref = O.sharpen_combine(to_np(bl), to_np(db), to_np(x), to_np(alpha),
                            None if mask is None else to_np(mask).astype(np.uint8))
    assert np.array_equal(to_np(out), ref)
    return bl, db


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_sharpen(ba, oracle_lib, tag):
    ops = _ops()
    g = load_golden(f"sharpen_{tag}")
    x = to_dev(g["x"])
    for name, pm in CASES:
        k1 = [to_dev(g[f"{name}_kernel1_{a}"]) for a in "hwd"]
        k2 = [to_dev(g[f"{name}_kernel2_{a}"]) for a in "hwd"]
        alpha, mask = to_dev(g[f"{name}_alpha"]), to_dev(g[f"{name}_mask"])
        out = ops.sharpen3d(x, k1, k2, alpha, mask=mask, padding_mode=pm)
        bl, _ = _check_composition(ops, oracle_lib, x, k1, k2, alpha, mask, pm, out)
        # each blur within the smoothing bar of the reference's
        assert_close_dtype(to_np(bl), g[f"{name}_blurred"])
        db_ref_input = ops.smooth3d(to_dev(g[f"{name}_blurred"]), *k2, padding_mode=pm)
        assert_close_dtype(to_np(db_ref_input), g[f"{name}_double_blurred"])
        # masked-out elements are the input, bit for bit
        m = g[f"{name}_mask"].astype(bool)
        assert np.array_equal(to_np(out)[~m], g["x"][~m])
        if tag == "f32":
            amp = 1.0 + 2.0 * float(g[f"{name}_alpha"].max())
            np.testing.assert_allclose(to_np(out), g[f"{name}_out"], rtol=0, atol=amp * 1e-5)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_golden_via_transform_api(ba, tag):
    """RandGaussianSharpen.apply given the reference's own params."""
    g = load_golden(f"sharpen_{tag}")
    x = to_dev(g["x"])
    ops = _ops()
    for name, pm in CASES:
        t = ba.RandGaussianSharpen(prob=0.7, padding_mode=pm)
        p = {"mask": to_dev(g[f"{name}_mask"]), "alpha": to_dev(g[f"{name}_alpha"])}
        for n in "12":
            for a in "hwd":
                p[f"kernel{n}_{a}"] = to_dev(g[f"{name}_kernel{n}_{a}"])
        out = t.apply(x, p)
        direct = ops.sharpen3d(x, [p[f"kernel1_{a}"] for a in "hwd"],
                               [p[f"kernel2_{a}"] for a in "hwd"], p["alpha"], mask=p["mask"],
                               padding_mode=pm)
        assert torch.equal(out, direct)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,sig1,pm", [
    ((3, 2, 20, 24, 28), (0.5, 1.0), "reflect"),     # tiled smoother, small taps
    ((2, 3, 17, 9, 40), (2.0, 5.0), "replicate"),    # tiled, K up to 41
    ((2, 2, 30, 28, 36), (5.0, 6.0), "replicate"),   # K up to 49: wide-tap passes
    ((2, 1, 12, 10, 70), (15.0, 16.0), None),        # K = 129: axis-pass smoother
])
def test_sharpen_vs_oracle(ba, oracle_lib, dt, shape, sig1, pm):
    ops = _ops()
    O = oracle_lib
    gen = np.random.default_rng(sum(shape))
    B = shape[0]
    x = torch.from_numpy(np.clip(0.5 + 0.2 * gen.standard_normal(shape), 0, 1)
                         .astype(np.float32)).to(dt).cuda()
    s1 = gen.uniform(*sig1, (3, B)).astype(np.float32)
    s2 = (gen.random((3, B)) * (s1 - 0.5) + 0.5).astype(np.float32)
    k1 = [O.gaussian_1d_batch(s) for s in s1]
    k2 = [O.gaussian_1d_batch(s) for s in s2]
    alpha = gen.uniform(10, 30, B).astype(np.float32)
    mask = np.ones(B, bool)
    mask[-1] = False
    out = ops.sharpen3d(x, [to_dev(k) for k in k1], [to_dev(k) for k in k2], to_dev(alpha),
                        mask=to_dev(mask), padding_mode=pm)
    bl, db = _check_composition(ops, O, x, [to_dev(k) for k in k1], [to_dev(k) for k in k2],
                                to_dev(alpha), to_dev(mask), pm, out)
    xn = to_np(x)
    bl_o = O.separable_gauss(xn, *k1, padding_mode=pm)
    assert_close_dtype(to_np(bl), bl_o)
    assert_close_dtype(to_np(db), O.separable_gauss(to_np(bl), *k2, padding_mode=pm))
    assert np.array_equal(to_np(out)[-1], xn[-1])
    if dt == torch.float32:
        ref = O.sharpen(xn, k1, k2, alpha, mask, padding_mode=pm)
        amp = 1.0 + 2.0 * float(alpha.max())
        np.testing.assert_allclose(to_np(out), ref, rtol=0, atol=amp * 1e-5)
    else:
        # bf16: a blur that lands one ulp away moves the result by at most
        # (1 + 2 alpha) ulps of the blur's magnitude (<= 1 here, ulp 2^-8)
        ref = O.sharpen(xn, k1, k2, alpha, mask, padding_mode=pm)
        amp = 1.0 + 2.0 * float(alpha.max())
        d = np.abs(as_f32(to_np(out)) - as_f32(ref))
        assert d.max() <= amp * 2.0 * 2.0 ** -8


def test_sample_apply_and_dict_keys(ba):
    """sample_params -> apply; every key of the dict wrapper gets the same
    params; all-masked batches come back unchanged."""
    torch.manual_seed(4)
    x = torch.rand(3, 1, 16, 18, 20, device="cuda")
    t = ba.RandGaussianSharpen(prob=1.0)
    p = t.sample_params(3, x.shape, x.device)
    for n in "12":
        for a in "hwd":
            assert p[f"kernel{n}_{a}"].shape[0] == 3
            assert torch.allclose(p[f"kernel{n}_{a}"].sum(1), torch.ones(3, device="cuda"))
    y = t.apply(x, p)
    assert y.shape == x.shape and torch.isfinite(y).all() and not torch.equal(y, x)
    td = ba.RandGaussianSharpend(keys=["a", "b"], prob=1.0)
    torch.manual_seed(5)
    out = td({"a": x, "b": x.clone()})
    assert torch.equal(out["a"], out["b"])
    t0 = ba.RandGaussianSharpen(prob=0.0)
    assert torch.equal(t0(x), x)
    empty = torch.zeros(0, 1, 4, 4, 4, device="cuda")
    assert t.apply(empty, t.sample_params(0, empty.shape, empty.device)).shape == empty.shape


def test_sharpen_errors(ba):
    ops = _ops()
    x = torch.zeros(2, 1, 4, 4, 4, device="cuda")
    k = torch.ones(2, 3, device="cuda") / 3
    with pytest.raises(ValueError):  # reflect with K/2 >= size
        big = torch.ones(2, 9, device="cuda") / 9
        ops.sharpen3d(x, [big] * 3, [k] * 3, torch.ones(2, device="cuda"),
                      padding_mode="reflect")
    with pytest.raises(ValueError):  # alpha of the wrong length
        ops.sharpen3d(x, [k] * 3, [k] * 3, torch.ones(3, device="cuda"))
    with pytest.raises(ValueError):  # taps of the wrong batch
        ops.sharpen3d(x, [k[:1]] * 3, [k] * 3, torch.ones(2, device="cuda"))
