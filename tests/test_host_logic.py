"""Host logic of the drop-in API on CPU: parameter distributions and affine
conventions, and Compose's lazy accumulation, key grouping, mask skipping
and intensity-run fusion — with the two kernel entry points replaced by
oracle-backed fakes that record their calls (the CUDA kernels themselves are
covered by the -m gpu tests)."""
from __future__ import annotations

import numpy as np
import pytest
import torch


def test_affine_params_distribution(ba):
    torch.manual_seed(0)
    t = ba.RandAffine(prob=0.3, rotate_range=0.785, shear_range=0.3, translate_range=5,
                      scale_range=0.1)
    h = t.sample_host(4000, (4000, 1, 8, 8, 8))
    assert abs(h["mask"].mean() - 0.3) < 0.03
    a = h["affine"]
    assert np.allclose(a[:, 3], [0, 0, 0, 1])
    assert np.abs(a[:, :3, 3]).max() <= 5 * 2.5  # rotated/sheared translations stay bounded
    # masked elements map to the identity in to_affine
    m = t.host_affine({"_host": h})
    assert np.array_equal(m[~h["mask"]], np.broadcast_to(np.eye(4), m[~h["mask"]].shape))


def test_theta_formula_matches_reference_chain(ba):
    """monai_affine_to_theta restated: equals P @ S_norm @ A @ S_inv @ P."""
    from batchaug_b200.geometric import monai_affine_to_theta
    rng = np.random.default_rng(0)
    A = rng.standard_normal((5, 4, 4)).astype(np.float32)
    H, W, D = 12, 16, 20
    P = np.eye(4, dtype=np.float32)[[2, 1, 0, 3]]
    Sn = np.diag(np.array([2 / H, 2 / W, 2 / D, 1], np.float32))
    Si = np.diag(np.array([H / 2, W / 2, D / 2, 1], np.float32))
    ref = P @ Sn @ A @ Si @ P
    assert np.allclose(monai_affine_to_theta(A, (H, W, D)), ref, rtol=1e-6, atol=1e-6)


def test_flip_rot90_affines(ba):
    h = {"mask": np.array([True, True, False]), "axes": np.array([0, 2, 1])}
    a = ba.RandAxisFlip(prob=1.0).host_affine({"_host": h})
    assert np.array_equal(np.diagonal(a, axis1=1, axis2=2),
                          [[-1, 1, 1, 1], [1, 1, -1, 1], [1, 1, 1, 1]])
    r = ba.RandRotate90(prob=1.0, max_k=3)
    hk = {"mask": np.array([True, True, True]), "k": np.array([1, 2, 3])}
    ar = r.host_affine({"_host": hk})
    assert np.array_equal(ar[0, :2, :2], [[0, 1], [-1, 0]])
    assert np.array_equal(ar[1, :2, :2], [[-1, 0], [0, -1]])
    assert np.array_equal(ar[2, :2, :2], [[0, -1], [1, 0]])


def test_ranges_and_k(ba):
    torch.manual_seed(1)
    h = ba.RandRotate90(prob=1.0, max_k=3).sample_host(3000, (3000, 1, 4, 4, 4))
    assert set(np.unique(h["k"])) == {1, 2, 3}
    f = ba.RandAxisFlip(prob=1.0).sample_host(3000, (3000, 1, 4, 4, 4))
    assert set(np.unique(f["axes"])) == {0, 1, 2}
    s = ba.RandScaleIntensity(prob=1.0, factors=0.2).sample_host(3000, (3000, 1, 4, 4, 4))
    assert s["factor"].min() >= -0.2 and s["factor"].max() < 0.2
    b = ba.RandBiasField(degree=3).sample_host(10, (10, 1, 4, 4, 4))
    assert b["coeffs"].shape == (10, 20)


class _Recorder:
    """Oracle-backed stand-ins for ops.resample3d / ops.intensity_chain on CPU
    tensors, recording each call."""

    def __init__(self, oracle):
        self.O = oracle
        self.calls = []
        self.minmax = []     # each resample call's minmax argument
        self.chain_ops = []  # each chain call's ops

    def resample3d(self, tensors, *, affine=None, modes="bilinear", paddings="zeros",
                   mask=None, **kw):
        single = isinstance(tensors, torch.Tensor)
        ts = [tensors] if single else list(tensors)
        modes = [modes] * len(ts) if isinstance(modes, str) else modes
        paddings = [paddings] * len(ts) if isinstance(paddings, str) else paddings
        self.calls.append(("resample", len(ts), np.array(mask)))
        self.minmax.append(kw.get("minmax"))
        outs = [torch.from_numpy(self.O.resample3d(t.numpy(), affine=affine, mode=m, padding=p,
                                                   mask=mask)) for t, m, p in zip(ts, modes,
                                                                                  paddings)]
        return outs[0] if single else outs

    def intensity_chain(self, x, ops_, **kw):
        self.calls.append(("chain", len(ops_), [o.kind for o in ops_]))
        self.chain_ops.append(list(ops_))
        return x + 0  # values are not checked here, only the plan


@pytest.fixture
def rec(ba, oracle_lib, monkeypatch):
    from batchaug_b200 import compose, intensity
    r = _Recorder(oracle_lib)
    monkeypatch.setattr(compose.ops, "resample3d", r.resample3d)
    monkeypatch.setattr(compose.ops, "intensity_chain", r.intensity_chain)

    def fake_chain_op(self, params, tensor):
        from batchaug_b200 import ops
        return ops.ChainOp(type(self).__name__ and _KIND[type(self).__name__])
    _KIND.update({"RandGaussianNoise": 1, "RandAdjustContrast": 2, "RandScaleIntensity": 3,
                  "RandShiftIntensity": 4, "RandBiasField": 5, "ScaleIntensity": 6})
    monkeypatch.setattr(intensity._FusibleIntensity, "chain_op", fake_chain_op)
    monkeypatch.setattr(intensity.BatchTransform, "_device_params",
                        lambda self, host, shape, device: {"mask": torch.from_numpy(host["mask"])})
    return r


_KIND: dict = {}


def test_compose_plan_config4(ba, rec, oracle_lib):
    """rot90, flip -> noise -> affine -> ScaleIntensity: two resamples of the
    (vol, seg) pair, each ONE launch for both keys; intensity runs fused."""
    torch.manual_seed(0)
    vol = torch.randn(3, 2, 8, 8, 8)
    seg = (torch.rand(3, 1, 8, 8, 8) > 0.5).float()
    c = ba.Compose([ba.RandRotate90d(["vol", "seg"], prob=1.0, max_k=3),
                    ba.RandAxisFlipd(["vol", "seg"], prob=1.0),
                    ba.RandGaussianNoised(["vol"], prob=1.0, std=0.5),
                    ba.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.785),
                    ba.ScaleIntensityd(["vol"]),
                    ba.RandShiftIntensityd(["vol"], prob=1.0)],
                   lazy=True, mode={"vol": "bilinear", "seg": "nearest"})
    out = c({"vol": vol, "seg": seg})
    kinds = [k[0] for k in rec.calls]
    assert kinds == ["resample", "chain", "resample", "chain"]
    assert rec.calls[0][1] == 2 and rec.calls[2][1] == 2
    assert rec.calls[3][2] == [6, 4]  # ScaleIntensity then shift, one chain
    # nearest keeps binary labels
    assert set(np.unique(out["seg"].numpy())) <= {0.0, 1.0}


def test_compose_hands_resample_stats_to_scale_intensity(ba, rec, oracle_lib):
    """A materialisation followed by a channel-wise ScaleIntensity(d) asks
    the resample for the rescaled keys' per-(element, channel) min/max, and
    the rescale takes them as given statistics; a factor rescale, a
    per-element one and keys the rescale does not list get none."""
    from batchaug_b200 import _lib as L
    torch.manual_seed(0)
    vol = torch.randn(3, 2, 8, 8, 8)
    seg = (torch.rand(3, 1, 8, 8, 8) > 0.5).float()
    mode = {"vol": "bilinear", "seg": "nearest"}
    c = ba.Compose([ba.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.5),
                    ba.ScaleIntensityd(["vol"])], lazy=True, mode=mode)
    c({"vol": vol, "seg": seg})
    mm = rec.minmax[-1]
    assert mm is not None
    given = [m for m in mm if m is not None]
    assert len(given) == 1 and tuple(given[0].shape) == (3, 2, 2)  # vol's (B, C, 2) only
    assert given[0].dtype == torch.int32
    (op,) = rec.chain_ops[-1]
    assert op.kind == L.BA_OP_RESCALE and op.stats is given[0]
    assert op.flags & L.BA_RESCALE_GIVEN
    for last in (ba.ScaleIntensityd(["vol"], factor=0.1),
                 ba.ScaleIntensityd(["vol"], channel_wise=False),
                 ba.ScaleIntensityd(["seg"], minv=None, maxv=None)):
        rec.minmax.clear()
        rec.chain_ops.clear()
        ba.Compose([ba.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.5), last],
                   lazy=True, mode=mode)({"vol": vol, "seg": seg})
        assert all(m is None for m in (rec.minmax[-1] or []))
        assert all(getattr(o, "stats", None) is None for ops_ in rec.chain_ops for o in ops_)


def test_owned_key_chain_runs_on_selected_elements_only(ba, rec, oracle_lib):
    """On a key the pipeline created (the first resample's output), an
    intensity run touches only the runs of elements its ops select, in place:
    no launch when none is selected, one per run of consecutive elements."""
    torch.manual_seed(0)
    vol = torch.randn(6, 1, 8, 8, 8)
    for prob, launches in ((0.0, 0), (1.0, 1)):
        rec.calls.clear()
        c = ba.Compose([ba.RandAxisFlipd(["vol"], prob=1.0),
                        ba.RandGaussianNoised(["vol"], prob=prob, std=0.5)], lazy=True)
        c({"vol": vol})
        assert [k[0] for k in rec.calls].count("chain") == launches
    rec.calls.clear()
    from batchaug_b200 import compose
    sel = np.array([True, True, False, True, False, False])
    assert compose.Compose._runs(np.flatnonzero(sel)) == [(0, 2), (3, 1)]
    p = {"mask": torch.tensor(sel), "std": torch.arange(6.0), "elem_offset": 10,
         "_host": {"mask": sel}}
    q = compose._slice_params(p, 3, 1)
    assert q["elem_offset"] == 13 and q["std"].tolist() == [3.0] and q["_host"]["mask"].tolist() == [True]


def test_compose_accumulates_like_reference(ba, rec, oracle_lib):
    """flip then rot90 on the pair: one resample through flip_A @ rot_A."""
    torch.manual_seed(3)
    vol = torch.randn(2, 1, 6, 6, 6)
    t1 = ba.RandAxisFlipd(["vol", "seg"], prob=1.0)
    t2 = ba.RandRotate90d(["vol", "seg"], prob=1.0)
    torch.manual_seed(3)
    out = ba.Compose([t1, t2], lazy=True, mode="nearest")({"vol": vol, "seg": vol.clone()})
    torch.manual_seed(3)
    h1 = t1.transform.sample_host(2, vol.shape)
    h2 = t2.transform.sample_host(2, vol.shape)
    A = t1.transform.host_affine({"_host": h1}) @ t2.transform.host_affine({"_host": h2})
    ref = oracle_lib.resample3d(vol.numpy(), affine=A, mode="nearest")
    assert np.array_equal(out["vol"].numpy(), ref)
    assert len([c for c in rec.calls if c[0] == "resample"]) == 1


def test_compose_skips_all_masked_and_splits_key_sets(ba, rec):
    torch.manual_seed(0)
    v = torch.randn(2, 1, 4, 4, 4)
    c = ba.Compose([ba.RandAffined(["vol"], prob=0.0, rotate_range=0.5)], lazy=True)
    out = c({"vol": v})
    assert out["vol"] is v and rec.calls == []  # mask all false: no launch, same tensor
    c2 = ba.Compose([ba.RandAxisFlipd(["vol", "seg"], prob=1.0),
                     ba.RandRotate90d(["vol"], prob=1.0)], lazy=True, mode="nearest")
    c2({"vol": v, "seg": v.clone()})
    res = [k for k in rec.calls if k[0] == "resample"]
    assert len(res) == 2 and sorted(r[1] for r in res) == [1, 1]  # different histories


def _numpy_rand_affine(u, rot, shear, trans, scale):
    """RandAffine's affine chain I @ R @ Sh @ T @ Sc restated in numpy
    (affine.py:9-151), used to check the native host builder."""
    B = u.shape[0]
    eye = lambda: np.broadcast_to(np.eye(4, dtype=np.float32), (B, 4, 4)).copy()

    def cols(spec, uu, n, add=0.0):
        spec = [spec] * n if isinstance(spec, (int, float)) else list(spec)
        out = np.zeros((B, n), np.float32)
        for i, s in enumerate(spec):
            if s is None:
                out[:, i] = add
            elif isinstance(s, (int, float)):
                out[:, i] = uu[:, i] * np.float32(2 * s) - np.float32(s) + np.float32(add)
            else:
                out[:, i] = uu[:, i] * np.float32(s[1] - s[0]) + np.float32(s[0]) + np.float32(add)
        return out

    A = eye()
    if rot is not None:
        a = cols(rot, u[:, 1:4], 3)
        c, s = np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)
        rx, ry, rz = eye(), eye(), eye()
        rx[:, 1, 1], rx[:, 1, 2], rx[:, 2, 1], rx[:, 2, 2] = c[:, 0], -s[:, 0], s[:, 0], c[:, 0]
        ry[:, 0, 0], ry[:, 0, 2], ry[:, 2, 0], ry[:, 2, 2] = c[:, 1], s[:, 1], -s[:, 1], c[:, 1]
        rz[:, 0, 0], rz[:, 0, 1], rz[:, 1, 0], rz[:, 1, 1] = c[:, 2], -s[:, 2], s[:, 2], c[:, 2]
        A = A @ (rx @ ry @ rz)
    if shear is not None:
        sh = cols(shear, u[:, 4:10], 6)
        m = eye()
        m[:, 0, 1], m[:, 0, 2], m[:, 1, 0] = sh[:, 0], sh[:, 1], sh[:, 2]
        m[:, 1, 2], m[:, 2, 0], m[:, 2, 1] = sh[:, 3], sh[:, 4], sh[:, 5]
        A = A @ m
    if trans is not None:
        t = cols(trans, u[:, 10:13], 3)
        m = eye()
        m[:, 0, 3], m[:, 1, 3], m[:, 2, 3] = t[:, 0], t[:, 1], t[:, 2]
        A = A @ m
    if scale is not None:
        sc = cols(scale, u[:, 13:16], 3, 1.0)
        m = eye()
        m[:, 0, 0], m[:, 1, 1], m[:, 2, 2] = sc[:, 0], sc[:, 1], sc[:, 2]
        A = A @ m
    return A.astype(np.float32)


@pytest.mark.parametrize("ranges", [
    (0.785, 0.3, 5, 0.1),
    ((0.1, 0.5), None, (None, 2, (1, 3)), None),
    (None, (0.1, None, 0.2, None, 0.3, None), None, (0.9, 1.1)),
])
def test_native_affine_builder_matches_numpy_chain(ba, ranges):
    from batchaug_b200.geometric import monai_affine_to_theta
    rot, shear, trans, scale = ranges
    t = ba.RandAffine(prob=0.6, rotate_range=rot, shear_range=shear, translate_range=trans,
                      scale_range=scale)
    u = np.random.default_rng(3).random((64, 16), dtype=np.float32)
    h = t._host_params(64, (64, 1, 12, 16, 20), u, 0)
    ref = _numpy_rand_affine(u, rot, shear, trans, scale)
    np.testing.assert_allclose(h["affine"], ref, rtol=0, atol=2e-6)
    assert np.array_equal(h["mask"], u[:, 0] < 0.6)
    np.testing.assert_array_equal(h["theta"], monai_affine_to_theta(h["affine"], (12, 16, 20)))


def test_stats_transforms_host_params_and_ops(ba):
    """RandRicianNoise / RandStdShiftIntensity / RandScaleIntensityFixedMean:
    parameter ranges (noise.py:125-141, scale_shift.py:158-166, 245-250) and
    the chain op each one asks for (built on CPU tensors, not launched)."""
    from batchaug_b200 import _lib as L
    torch.manual_seed(5)
    shape = (4000, 1, 4, 4, 4)
    r = ba.RandRicianNoise(prob=0.25, std=0.3).sample_host(4000, shape)
    assert abs(r["mask"].mean() - 0.25) < 0.03
    assert r["noise_std"].dtype == np.float32
    assert r["noise_std"].min() >= 0 and r["noise_std"].max() < 0.3
    assert abs(r["noise_std"].mean() - 0.15) < 0.01
    fixed = ba.RandRicianNoise(std=0.3, sample_std=False).sample_host(8, (8, 1, 4, 4, 4))
    assert np.array_equal(fixed["noise_std"], np.full(8, 0.3, np.float32))
    s = ba.RandStdShiftIntensity(prob=1.0, factors=2.5).sample_host(4000, shape)
    assert s["factor"].min() >= -2.5 and s["factor"].max() < 2.5
    assert ba.RandStdShiftIntensity().factors == (-3.0, 3.0)
    f = ba.RandScaleIntensityFixedMean(prob=1.0).sample_host(4000, shape)
    assert f["factor"].min() >= -0.5 and f["factor"].max() < 0.5
    # draws differ from transform to transform for one seed (own streams)
    torch.manual_seed(9)
    a = ba.RandStdShiftIntensity(prob=1.0, factors=(0, 1)).sample_host(16, (16, 1, 2, 2, 2))
    torch.manual_seed(9)
    b = ba.RandScaleIntensityFixedMean(prob=1.0, factors=(0, 1)).sample_host(16, (16, 1, 2, 2, 2))
    assert not np.array_equal(a["factor"], b["factor"])

    x = torch.zeros(2, 1, 4, 4, 4)
    mask = torch.tensor([True, False])
    p = {"mask": mask, "noise_std": torch.tensor([0.1, 0.2]), "noise_seed": 7, "elem_offset": 3}
    op = ba.RandRicianNoise(mean=0.25, relative=True).chain_op(p, x)
    assert op.kind == L.BA_OP_RICIAN and op.seed == 7 and op.elem_offset == 3
    assert op.flags == L.BA_RICIAN_PHILOX | L.BA_RICIAN_RELATIVE and op.c0 == 0.25
    u = torch.ones_like(x)
    op = ba.RandRicianNoise().chain_op({"mask": mask, "noise_std": p["noise_std"], "u1": u,
                                        "u2": 2 * u}, x)
    assert op.flags == 0 and op.noise is not None and float(op.param2.max()) == 2.0
    with pytest.raises(ValueError):
        ba.RandRicianNoise().chain_op({"mask": mask, "noise_std": p["noise_std"],
                                       "u1": u[:, :, :2], "u2": u}, x)
    pf = {"mask": mask, "factor": torch.tensor([0.5, -0.5])}
    op = ba.RandStdShiftIntensity(nonzero=True, channel_wise=True).chain_op(pf, x)
    assert op.kind == L.BA_OP_STD_SHIFT and op.flags == L.BA_STD_NONZERO | L.BA_STAT_CHANNEL
    op = ba.RandScaleIntensityFixedMean(channel_wise=True).chain_op(pf, x)
    assert op.kind == L.BA_OP_FIXED_MEAN and op.flags == L.BA_STAT_CHANNEL
    assert ba.RandRicianNoised(["a"]).transform.std == 0.1


def test_sharpen_host_params(ba):
    """RandGaussianSharpen params (sharpen.py:61-113): sigma1 in its range,
    a scalar sigma2 in [sigma2, sigma1], a tuple sigma2 in its range, alpha
    in its range, and each kernel set sized by its batch-max sigma."""
    torch.manual_seed(2)
    t = ba.RandGaussianSharpen(prob=0.4, sigma1_x=(1.0, 2.0), sigma2_y=(0.2, 0.3))
    h = t.sample_host(3000, (3000, 1, 4, 4, 4))
    assert abs(h["mask"].mean() - 0.4) < 0.03
    assert h["sigma1_x"].min() >= 1.0 and h["sigma1_x"].max() < 2.0
    assert np.all(h["sigma2_x"] >= 0.5) and np.all(h["sigma2_x"] <= h["sigma1_x"])
    assert h["sigma2_y"].min() >= 0.2 and h["sigma2_y"].max() < 0.3
    assert h["alpha"].min() >= 10.0 and h["alpha"].max() < 30.0
    assert h["K_sigma1_x"] == ba.ops.gauss_taps_len(float(h["sigma1_x"].max()), 4.0) == 17
    assert h["K_sigma2_y"] == 3
    # a shard of the global batch draws exactly that slice of the params
    torch.manual_seed(3)
    full = t.sample_host(8, (8, 1, 4, 4, 4))
    torch.manual_seed(3)
    with ba.shard(4, 8):
        part = t.sample_host(4, (4, 1, 4, 4, 4))
    for k in ("mask", "sigma1_x", "sigma2_z", "alpha"):
        assert np.array_equal(part[k], full[k][4:])
    assert part["K_sigma1_x"] == full["K_sigma1_x"]
