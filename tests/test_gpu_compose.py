"""Compose (lazy fusion + intensity chain fusion) through the reference-facing
API, modelled on the reference's tests/test_compose.py and with the config-1
pipeline checked against the reference's golden output."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture
def vol():
    torch.manual_seed(42)
    return torch.rand(4, 3, 16, 16, 16, device="cuda")


@pytest.fixture
def seg():
    torch.manual_seed(42)
    return torch.randint(0, 5, (4, 3, 16, 16, 16), device="cuda").float()


def test_eager_matches_sequential(ba, vol, seg):
    ts = [ba.RandAxisFlipd(keys=["vol", "seg"], prob=1.0),
          ba.RandGaussianNoised(keys=["vol"], prob=1.0, mean=0.0, std=0.1),
          ba.RandRotate90d(keys=["vol", "seg"], prob=1.0)]
    torch.manual_seed(0)
    r = ba.Compose(ts, lazy=False)({"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(0)
    d = {"vol": vol.clone(), "seg": seg.clone()}
    for t in ts:
        d = t(d)
    assert torch.equal(r["vol"], d["vol"]) and torch.equal(r["seg"], d["seg"])


@pytest.mark.parametrize("make", [
    lambda ba: ba.RandAxisFlipd(keys=["vol", "seg"], prob=1.0),
    lambda ba: ba.RandRotate90d(keys=["vol", "seg"], prob=1.0, max_k=3),
])
def test_lazy_exact_maps_equal_eager(ba, vol, seg, make):
    t = make(ba)
    c = ba.Compose([t], lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    torch.manual_seed(7)
    lazy = c({"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(7)
    eager = t({"vol": vol.clone(), "seg": seg.clone()})
    assert torch.allclose(lazy["vol"], eager["vol"], atol=1e-5)
    assert torch.equal(lazy["seg"], eager["seg"])


def test_lazy_affine_equals_eager(ba, vol, seg):
    t = ba.RandAffined(keys=["vol", "seg"], prob=1.0, rotate_range=0.3, scale_range=0.1,
                       mode={"vol": "bilinear", "seg": "nearest"})
    c = ba.Compose([t], lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    torch.manual_seed(22)
    lazy = c({"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(22)
    eager = t({"vol": vol.clone(), "seg": seg.clone()})
    # same theta (derived in-kernel from the affine vs given): bit-identical
    assert torch.equal(lazy["vol"], eager["vol"])
    assert torch.equal(lazy["seg"], eager["seg"])


def test_fusion_flip_rot90_affine(ba, vol, seg):
    t1 = ba.RandAxisFlipd(keys=["vol", "seg"], prob=1.0)
    t2 = ba.RandRotate90d(keys=["vol", "seg"], prob=1.0)
    t3 = ba.RandAffined(keys=["vol", "seg"], prob=1.0, rotate_range=0.2, scale_range=0.1)
    c = ba.Compose([t1, t2], lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    torch.manual_seed(33)
    lazy = c({"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(33)
    p1 = t1.transform.sample_params(4, vol.shape, vol.device)
    p2 = t2.transform.sample_params(4, vol.shape, vol.device)
    ev = t2.transform.apply(t1.transform.apply(vol.clone(), p1), p2)
    es = t2.transform.apply(t1.transform.apply(seg.clone(), p1), p2)
    assert torch.allclose(lazy["vol"], ev, atol=1e-5)
    assert torch.equal(lazy["seg"], es)
    c3 = ba.Compose([t1, t2, t3], lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    torch.manual_seed(44)
    lazy3 = c3({"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(44)
    p1 = t1.transform.sample_params(4, vol.shape, vol.device)
    p2 = t2.transform.sample_params(4, vol.shape, vol.device)
    p3 = t3.transform.sample_params(4, vol.shape, vol.device)
    ev = t3.transform.apply(t2.transform.apply(t1.transform.apply(vol.clone(), p1), p2), p3)
    assert torch.allclose(lazy3["vol"], ev, atol=1e-4)


def test_geo_intensity_geo(ba, vol, seg):
    ts = [ba.RandAxisFlipd(keys=["vol", "seg"], prob=1.0),
          ba.RandGaussianNoised(keys=["vol"], prob=1.0, mean=0.0, std=0.01),
          ba.RandRotate90d(keys=["vol", "seg"], prob=1.0)]
    torch.manual_seed(55)
    lazy = ba.Compose(ts, lazy=True, mode={"vol": "bilinear", "seg": "nearest"})(
        {"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(55)
    eager = ba.Compose(ts, lazy=False)({"vol": vol.clone(), "seg": seg.clone()})
    assert torch.allclose(lazy["vol"], eager["vol"], atol=1e-5)
    assert torch.equal(lazy["seg"], eager["seg"])


def test_mask_preserved(ba, vol, seg):
    t = ba.RandAffined(keys=["vol", "seg"], prob=0.0, rotate_range=0.5)
    r = ba.Compose([t], lazy=True, mode={"vol": "bilinear", "seg": "nearest"})(
        {"vol": vol.clone(), "seg": seg.clone()})
    assert torch.equal(r["vol"], vol) and torch.equal(r["seg"], seg)
    x = torch.rand(4, 1, 8, 8, 8, device="cuda")
    t = ba.RandAxisFlipd(keys=["vol"], prob=0.5)
    torch.manual_seed(123)
    res = ba.Compose([t], lazy=True, mode="nearest")({"vol": x.clone()})
    torch.manual_seed(123)
    m = t.transform.sample_params(4, x.shape, x.device)["mask"]
    for i in range(4):
        if not m[i]:
            assert torch.equal(res["vol"][i], x[i])


def test_per_key_modes_label_set(ba, vol, seg):
    t = ba.RandAffined(keys=["vol", "seg"], prob=1.0, rotate_range=0.3)
    r = ba.Compose([t], lazy=True, mode={"vol": "bilinear", "seg": "nearest"})(
        {"vol": vol.clone(), "seg": seg.clone()})
    assert set(r["seg"].unique().tolist()) <= {0.0, 1.0, 2.0, 3.0, 4.0}


def test_different_key_sets(ba, vol, seg):
    t1 = ba.RandAxisFlipd(keys=["vol", "seg"], prob=1.0)
    t2 = ba.RandRotate90d(keys=["vol"], prob=1.0)
    torch.manual_seed(66)
    r = ba.Compose([t1, t2], lazy=True, mode="nearest")({"vol": vol.clone(), "seg": seg.clone()})
    torch.manual_seed(66)
    p1 = t1.transform.sample_params(4, vol.shape, vol.device)
    p2 = t2.transform.sample_params(4, vol.shape, vol.device)
    ev = t2.transform.apply(t1.transform.apply(vol.clone(), p1), p2)
    es = t1.transform.apply(seg.clone(), p1)
    assert torch.equal(r["vol"], ev) and torch.equal(r["seg"], es)


def test_edge_cases(ba, vol, seg):
    r = ba.Compose([], lazy=True)({"vol": vol.clone(), "seg": seg.clone()})
    assert torch.equal(r["vol"], vol)
    t = ba.RandGaussianNoised(keys=["vol"], prob=1.0, std=0.1)
    torch.manual_seed(5)
    lazy = ba.Compose([t], lazy=True)({"vol": vol.clone()})
    torch.manual_seed(5)
    eager = t({"vol": vol.clone()})
    assert torch.equal(lazy["vol"], eager["vol"])


def test_non_cubic_and_bf16(ba):
    torch.manual_seed(42)
    v = torch.rand(2, 1, 12, 16, 20, device="cuda")
    s = torch.randint(0, 5, (2, 1, 12, 16, 20), device="cuda").float()
    ts = [ba.RandAxisFlipd(keys=["vol", "seg"], prob=1.0),
          ba.RandRotate90d(keys=["vol", "seg"], prob=1.0),
          ba.RandAffined(keys=["vol", "seg"], prob=1.0, rotate_range=0.3, scale_range=0.1)]
    r = ba.Compose(ts, lazy=True, mode={"vol": "bilinear", "seg": "nearest"})(
        {"vol": v, "seg": s})
    assert r["vol"].shape == v.shape and not torch.isnan(r["vol"]).any()
    assert set(r["seg"].unique().tolist()) <= {0.0, 1.0, 2.0, 3.0, 4.0}
    vb = torch.rand(4, 3, 16, 16, 16, device="cuda", dtype=torch.bfloat16)
    rb = ba.Compose([ba.RandAffined(keys=["vol"], prob=1.0, rotate_range=0.2)], lazy=True)(
        {"vol": vb})
    assert rb["vol"].dtype == torch.bfloat16 and not torch.isnan(rb["vol"]).any()


def test_intensity_run_fusion_equals_sequential(ba):
    """A fused run (one chain per key) equals applying each transform alone."""
    torch.manual_seed(0)
    x = (0.5 + 0.2 * torch.randn(3, 2, 16, 16, 16, device="cuda")).clamp(0, 1).bfloat16()
    ts = [ba.RandGaussianNoised(keys=["v"], prob=0.7, std=(0.1, 0.5)),
          ba.RandAdjustContrastd(keys=["v"], prob=0.7, gamma=(0.5, 2.0)),
          ba.RandScaleIntensityd(keys=["v"], prob=0.7, factors=0.2),
          ba.RandShiftIntensityd(keys=["v"], prob=0.7, offsets=0.1),
          ba.RandBiasFieldd(keys=["v"], prob=0.7),
          ba.ScaleIntensityd(keys=["v"])]
    torch.manual_seed(9)
    fused = ba.Compose(ts, lazy=True)({"v": x})["v"]
    torch.manual_seed(9)
    d = {"v": x}
    for t in ts:
        d = t(d)
    assert torch.equal(fused, d["v"])


def test_golden_pipeline_cfg1(ba):
    """Config 1 with the reference's params: materialise (flip∘affine, two
    keys, one launch) -> noise (injected) -> ScaleIntensity == reference."""
    from batchaug_b200 import _lib as L
    from batchaug_b200 import ops
    g = load_golden("pipeline_cfg1")
    vo, so = ops.resample3d([to_dev(g["vol"]), to_dev(g["seg"])], affine=g["affine"],
                            mask=g["mask"], modes=["bilinear", "nearest"], exact=True)
    vo = ops.intensity_chain(vo, [
        ops.ChainOp(L.BA_OP_NOISE, mask=to_dev(g["noise_mask"]).to(torch.uint8),
                    noise=to_dev(g["noise"])),
        ops.ChainOp(L.BA_OP_RESCALE, flags=7, c0=0.0, c1=1.0)])
    assert np.array_equal(to_np(so), g["seg_out"])
    assert np.array_equal(to_np(vo), g["vol_out"])


def test_config_pipelines_run(ba):
    """Configs 1, 4 and a scaled-down 5 end to end through Compose."""
    torch.manual_seed(0)
    v = torch.randn(2, 1, 64, 64, 64, device="cuda")
    s = torch.randint(0, 5, (2, 1, 64, 64, 64), device="cuda").float()
    c1 = ba.Compose([ba.RandAxisFlipd(["vol", "seg"], prob=0.5),
                     ba.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.785,
                                    shear_range=0.3, translate_range=5),
                     ba.RandGaussianNoised(["vol"], std=0.1), ba.ScaleIntensityd(["vol"])],
                    lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    r = c1({"vol": v, "seg": s})
    assert float(r["vol"].min()) == 0.0 and float(r["vol"].max()) == 1.0
    assert set(r["seg"].unique().tolist()) <= {0.0, 1.0, 2.0, 3.0, 4.0}
    v5 = torch.rand(2, 2, 48, 48, 48, device="cuda").bfloat16()
    s5 = torch.randint(0, 8, (2, 2, 48, 48, 48), device="cuda").float()
    c5 = ba.Compose([ba.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5, 7),
                                       magnitude_range=(50, 150),
                                       mode={"vol": "bilinear", "seg": "nearest"}),
                     ba.RandAffined(["vol", "seg"], prob=0.1, rotate_range=0.5),
                     ba.RandBiasFieldd(["vol"], prob=0.1, degree=3, coeff_range=(0, 0.1)),
                     ba.RandGaussianSmoothd(["vol"], prob=0.1, sigma_x=(0.5, 1.5),
                                            sigma_y=(0.5, 1.5), sigma_z=(0.5, 1.5)),
                     ba.ScaleIntensityd(["vol"])],
                    lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    r5 = c5({"vol": v5, "seg": s5})
    assert r5["vol"].dtype == torch.bfloat16 and torch.isfinite(r5["vol"].float()).all()
    assert set(r5["seg"].unique().tolist()) <= set(float(i) for i in range(8))


def _owned_pipeline(ba):
    return [ba.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.3, translate_range=2),
            ba.RandGaussianSmoothd(["vol"], prob=0.2, sigma_x=(0.5, 1.5), sigma_y=(0.5, 1.5),
                                   sigma_z=(0.5, 1.5)),
            ba.RandBiasFieldd(["vol"], prob=0.2),
            ba.RandGaussianSharpend(["vol"], prob=0.2),
            ba.RandAffined(["vol", "seg"], prob=0.2, rotate_range=0.5),
            ba.RandGaussianSmoothd(["vol"], prob=0.7),
            ba.RandGaussianSmoothd(["vol"], prob=0.0),
            ba.ScaleIntensityd(["vol"])]


@pytest.mark.parametrize("lazy", [False, True])
def test_owned_keys_in_place_equal_copying(ba, monkeypatch, lazy):
    """Keys the pipeline created are updated on the selected elements only
    (gather, transform, scatter back); the result equals the copying path
    (every transform writing a new tensor), and the inputs are untouched."""
    B = 6
    g = torch.Generator(device="cuda").manual_seed(3)
    vol = torch.rand(B, 2, 18, 20, 16, device="cuda", generator=g).bfloat16()
    seg = torch.randint(0, 4, (B, 1, 18, 20, 16), device="cuda", generator=g).float()
    v0, s0 = vol.clone(), seg.clone()
    subsets = []
    orig = ba.Compose._subset_index
    monkeypatch.setattr(ba.Compose, "_subset_index",
                        staticmethod(lambda m, dev: subsets.append(1) or orig(m, dev)))
    outs = []
    for in_place in (True, False):
        if not in_place:
            monkeypatch.setattr(ba.Compose, "_owned", lambda self, d, keys, inputs: False)
        for seed in range(4):
            torch.manual_seed(seed)
            r = ba.Compose(_owned_pipeline(ba), lazy=lazy,
                           mode={"vol": "bilinear", "seg": "nearest"})({"vol": vol, "seg": seg})
            outs.append((r["vol"], r["seg"]))
    for (a, b), (c, e) in zip(outs[:4], outs[4:]):
        assert torch.equal(a, c) and torch.equal(b, e)
    assert torch.equal(vol, v0) and torch.equal(seg, s0)
    assert subsets, "the in-place subset path never ran"


def test_owned_keys_never_the_inputs(ba):
    """A transform selecting no element, or keys sharing one tensor, never
    write in place into the caller's tensors."""
    x = torch.rand(3, 1, 8, 8, 8, device="cuda")
    x0 = x.clone()
    c = ba.Compose([ba.RandGaussianSmoothd(["a", "b"], prob=0.5),
                    ba.RandBiasFieldd(["a", "b"], prob=0.5)], lazy=True)
    for seed in range(4):
        torch.manual_seed(seed)
        r = c({"a": x, "b": x})
        assert torch.equal(x, x0)
        assert torch.equal(r["a"], r["b"])


def test_owned_key_noise_runs_equal_full_chain(ba):
    """A pipeline-owned key gets its intensity run in place on the runs of
    selected elements only; with the same params, the selected elements get
    exactly the noise a full-batch chain gives them (Philox keyed on the
    global element index), the others are untouched."""
    torch.manual_seed(4)
    vol = torch.randn(7, 2, 12, 10, 16, device="cuda")
    flip = ba.RandAxisFlipd(["vol"], prob=1.0)
    noise = ba.RandGaussianNoised(["vol"], prob=0.5, std=0.3)
    pf = flip.transform.sample_params(7, vol.shape, vol.device)
    pn = noise.transform.sample_params(7, vol.shape, vol.device)
    sel = np.array([True, True, False, True, False, False, True])
    pn["mask"] = torch.from_numpy(sel).cuda()
    pn["_host"]["mask"] = sel
    out = ba.Compose([flip, noise], lazy=True)({"vol": vol}, params=[pf, pn])["vol"]
    # the Compose's own materialisation of the flip (bilinear, its mode)
    flipped = ba.Compose([flip], lazy=True)({"vol": vol}, params=[pf])["vol"]
    full = noise.transform.apply(flipped, pn)
    assert torch.equal(out[torch.from_numpy(sel)], full[torch.from_numpy(sel)])
    assert torch.equal(out[torch.from_numpy(~sel)], flipped[torch.from_numpy(~sel)])
