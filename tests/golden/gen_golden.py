"""Generate the golden fixtures of tests/golden/ from the reference itself.

Runs halleewong/batchaug's PyTorch backend (``batchaug.pytorch``,
``batchaug.compose``) on CPU with seeded inputs and stores inputs, the
sampled params and the reference outputs as small .npz files (bf16 tensors
as uint16 bit patterns).  The oracle is pinned against these
(tests/test_oracle_golden.py) and the CUDA path is checked against both.

    python tests/golden/gen_golden.py --reference /path/to/batchaug

Needs the reference checkout on disk; the fixtures it writes are committed so
nothing at test time reads the reference.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, OUT)
import inputs  # noqa: E402  (tests/golden/inputs.py: seeded regenerable inputs)


def npy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.bool:
        return t.numpy().astype(np.uint8)
    return t.numpy().copy()


def save(name: str, **arrays):
    np.savez_compressed(os.path.join(OUT, name + ".npz"),
                        **{k: (npy(v) if isinstance(v, torch.Tensor) else np.asarray(v))
                           for k, v in arrays.items()})
    print("wrote", name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BATCHAUG_REFERENCE", ""))
    ap.add_argument("--only", choices=["stats", "sharpen", "lowres", "compose"], default=None,
                    help="write only this group of fixtures")
    args = ap.parse_args()
    if args.reference:
        sys.path.insert(0, args.reference)
    import torch.nn.functional as F

    import batchaug.pytorch as P
    if args.only == "compose":
        gen_compose(P)
        return
    if args.only == "stats":
        gen_stats_ops(P)
        return
    if args.only == "sharpen":
        gen_sharpen(P)
        return
    if args.only == "lowres":
        gen_lowres(P)
        return
    from batchaug.pytorch.geometric.affine import monai_affine_to_theta
    from batchaug.pytorch.intensity.smooth import gaussian_1d_batch
    dev = torch.device("cpu")
    torch.set_num_threads(1)

    # --- resample: every mode/padding/align, fp32 and bf16, non-cubic -------
    torch.manual_seed(101)
    B, C, H, W, D = 2, 2, 9, 10, 12
    x = torch.randn(B, C, H, W, D)
    t = P.RandAffine(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=3,
                     scale_range=0.1)
    p = t.sample_params(B, x.shape, dev)
    out = {}
    for dt in ("f32", "bf16"):
        xt = x if dt == "f32" else x.bfloat16()
        for mode in ("bilinear", "nearest"):
            for pad in ("zeros", "border", "reflection"):
                for align in (0, 1):
                    grid = F.affine_grid(p["theta"][:, :3, :], list(x.shape), align_corners=bool(align))
                    r = F.grid_sample(xt.float(), grid, mode=mode, padding_mode=pad,
                                      align_corners=bool(align)).to(xt.dtype)
                    out[f"{dt}_{mode}_{pad}_{align}"] = r
    save("resample_modes", x=x, x_bf16=x.bfloat16(), affine=p["affine"], theta=p["theta"], **out)

    # --- RandAffine.apply with a partial mask, border padding (config 2 style)
    torch.manual_seed(102)
    x = torch.rand(3, 1, 12, 12, 12)
    t = P.RandAffine(prob=0.5, rotate_range=0.785, shear_range=0.3, translate_range=5,
                     scale_range=0.1, padding_mode="border")
    p = t.sample_params(3, x.shape, dev)
    p["mask"] = torch.tensor([True, False, True])
    save("affine_apply_border", x=x, mask=p["mask"], theta=p["theta"], affine=p["affine"],
         out=t.apply(x, p))

    # --- Compose._materialize of flip∘affine on vol (bilinear) + seg (nearest)
    torch.manual_seed(103)
    vol = torch.randn(2, 1, 16, 16, 16)
    seg = torch.randint(0, 5, (2, 1, 16, 16, 16)).float()
    flip = P.RandAxisFlip(prob=0.5)
    aff = P.RandAffine(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=5)
    pf = flip.sample_params(2, vol.shape, dev)
    pa = aff.sample_params(2, vol.shape, dev)
    A = flip.to_affine(pf) @ aff.to_affine(pa)
    m = pf["mask"] | pa["mask"]
    theta = monai_affine_to_theta(A, vol.shape[2:], dev)
    grid = F.affine_grid(theta[:, :3, :], list(vol.shape), align_corners=False)
    vo = F.grid_sample(vol, grid, mode="bilinear", padding_mode="zeros", align_corners=False)
    so = F.grid_sample(seg, grid, mode="nearest", padding_mode="zeros", align_corners=False)
    vo = torch.where(m[:, None, None, None, None], vo, vol)
    so = torch.where(m[:, None, None, None, None], so, seg)
    save("compose_materialize", vol=vol, seg=seg, affine=A, mask=m, vol_out=vo, seg_out=so)

    # --- exact voxel maps: eager flip and rot90 vs their affines -------------
    torch.manual_seed(104)
    v = torch.randn(4, 2, 8, 8, 6)
    fl = P.RandAxisFlip(prob=1.0)
    pfl = fl.sample_params(4, v.shape, dev)
    r9 = P.RandRotate90(prob=1.0, max_k=3, spatial_axes=(0, 1))
    pr = r9.sample_params(4, v.shape, dev)
    save("flip_rot90", x=v, flip_axes=pfl["axes"], flip_affine=fl.to_affine(pfl),
         flip_out=fl.apply(v, pfl), rot_k=pr["k"], rot_affine=r9.to_affine(pr),
         rot_out=r9.apply(v, pr))

    # --- elastic: grid from its uniform draw, and the resample with it -------
    torch.manual_seed(105)
    B, H, W, D = 2, 12, 14, 16
    el = P.Rand3DElastic(prob=1.0, sigma_range=(5.0, 7.0), magnitude_range=(50.0, 150.0))
    pe = el.sample_params(B, (B, 1, H, W, D), dev)
    torch.manual_seed(105)
    _mask = torch.rand(B)
    u = torch.rand(B, 3, H, W, D)
    sigma = torch.rand(B) * 2.0 + 5.0
    magnitude = torch.rand(B) * 100.0 + 50.0
    taps = gaussian_1d_batch(sigma, truncated=3.0)
    vol = torch.rand(B, 2, H, W, D)
    seg = torch.randint(0, 8, (B, 1, H, W, D)).float()
    save("elastic", u=u, sigma=sigma, magnitude=magnitude, taps=taps, grid=pe["grid"],
         vol=vol, seg=seg, vol_out=el.apply(vol, pe, mode="bilinear"),
         seg_out=el.apply(seg, pe, mode="nearest"))

    # --- intensity ops, fp32 and bf16 ----------------------------------------
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        torch.manual_seed(106)
        B, C, H, W, D = 3, 2, 9, 10, 11
        x = (0.5 + 0.2 * torch.randn(B, C, H, W, D)).clamp(0, 1).to(dt)
        rec = {"x": x}
        tn = P.RandGaussianNoise(prob=0.5, std=(0.1, 0.5))
        pn = tn.sample_params(B, x.shape, dev)
        rec.update(noise=pn["noise"], noise_mask=pn["mask"], noise_out=tn.apply(x, pn))
        tc = P.RandAdjustContrast(prob=0.5, gamma=(0.5, 2.0))
        pc = tc.sample_params(B, x.shape, dev)
        rec.update(gamma=pc["gamma"], contrast_mask=pc["mask"], contrast_out=tc.apply(x, pc))
        ts = P.RandScaleIntensity(prob=0.5, factors=0.2)
        ps = ts.sample_params(B, x.shape, dev)
        rec.update(factor=ps["factor"], scale_mask=ps["mask"], scale_out=ts.apply(x, ps))
        th = P.RandShiftIntensity(prob=0.5, offsets=0.1, safe=True)
        ph = th.sample_params(B, x.shape, dev)
        rec.update(offset=ph["offset"], shift_mask=ph["mask"], shift_out=th.apply(x, ph))
        tb = P.RandBiasField(prob=0.5, degree=3, coeff_range=(0.0, 0.1))
        pb = tb.sample_params(B, x.shape, dev)
        rec.update(coeffs=pb["coeffs"], bias_mask=pb["mask"], bias_out=tb.apply(x, pb))
        xc = x.clone()
        xc[1, 0] = 0.25  # a constant (element, channel) group
        rec.update(xconst=xc, scaleint_cw_out=P.ScaleIntensity().apply(xc, {}),
                   scaleint_el_out=P.ScaleIntensity(channel_wise=False).apply(xc, {}),
                   scaleint_m13_out=P.ScaleIntensity(minv=-1.0, maxv=3.0).apply(x, {}),
                   scaleint_factor_out=P.ScaleIntensity(factor=0.5).apply(x, {}))
        tg = P.RandGaussianSmooth(prob=0.5, sigma_x=(0.5, 1.5), sigma_y=(0.5, 1.5),
                                  sigma_z=(0.5, 1.5))
        pg = tg.sample_params(B, x.shape, dev)
        rec.update(kernel_h=pg["kernel_h"], kernel_w=pg["kernel_w"], kernel_d=pg["kernel_d"],
                   sigma_x=pg["sigma_x"], smooth_mask=pg["mask"], smooth_out=tg.apply(x, pg))
        for pm in ("reflect", "replicate"):
            tgp = P.RandGaussianSmooth(prob=1.0, sigma_x=(0.5, 1.5), sigma_y=(0.5, 1.5),
                                       sigma_z=(0.5, 1.5), padding_mode=pm)
            rec[f"smooth_{pm}_out"] = tgp.apply(x, {**pg, "mask": torch.ones(B, dtype=torch.bool)})
        save(f"intensity_{tag}", **rec)

    # --- config 3 chain (noise -> contrast -> scale -> shift -> ScaleIntensity)
    torch.manual_seed(107)
    B, C, H, W, D = 4, 2, 10, 12, 8
    x = (0.5 + 0.2 * torch.randn(B, C, H, W, D)).clamp(0, 1).bfloat16()
    chain = [P.RandGaussianNoise(prob=1.0, std=(0.1, 0.5)),
             P.RandAdjustContrast(prob=1.0, gamma=(0.5, 2.0)),
             P.RandScaleIntensity(prob=1.0, factors=0.2),
             P.RandShiftIntensity(prob=1.0, offsets=0.1),
             P.ScaleIntensity(minv=0.0, maxv=1.0)]
    ps = [c.sample_params(B, x.shape, dev) for c in chain]
    y = x
    for c, pp in zip(chain, ps):
        y = c.apply(y, pp)
    save("chain_cfg3", x=x, noise=ps[0]["noise"], gamma=ps[1]["gamma"], factor=ps[2]["factor"],
         offset=ps[3]["offset"], out=y)

    # --- config 1 pipeline with the reference's own params --------------------
    torch.manual_seed(108)
    vol = torch.randn(2, 1, 16, 16, 16)
    seg = torch.randint(0, 5, (2, 1, 16, 16, 16)).float()
    flip = P.RandAxisFlip(prob=0.5)
    aff = P.RandAffine(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=5)
    pf = flip.sample_params(2, vol.shape, dev)
    pa = aff.sample_params(2, vol.shape, dev)
    A = flip.to_affine(pf) @ aff.to_affine(pa)
    m = pf["mask"] | pa["mask"]
    theta = monai_affine_to_theta(A, vol.shape[2:], dev)
    grid = F.affine_grid(theta[:, :3, :], list(vol.shape), align_corners=False)
    vo = torch.where(m[:, None, None, None, None],
                     F.grid_sample(vol, grid, mode="bilinear", align_corners=False), vol)
    so = torch.where(m[:, None, None, None, None],
                     F.grid_sample(seg, grid, mode="nearest", align_corners=False), seg)
    tn = P.RandGaussianNoise(prob=0.1, std=0.1)
    pn = tn.sample_params(2, vol.shape, dev)
    pn["mask"] = torch.tensor([True, False])
    vo = tn.apply(vo, pn)
    vo = P.ScaleIntensity().apply(vo, {})
    save("pipeline_cfg1", vol=vol, seg=seg, affine=A, mask=m, noise=pn["noise"],
         noise_mask=pn["mask"], vol_out=vo, seg_out=so)
    gen_stats_ops(P)
    gen_sharpen(P)
    gen_lowres(P)
    gen_compose(P)


def gen_stats_ops(P):
    """RandRicianNoise, RandStdShiftIntensity and RandScaleIntensityFixedMean:
    the intensity ops that reduce their own input to a mean or std."""
    dev = torch.device("cpu")
    torch.set_num_threads(1)
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        torch.manual_seed(108)
        B, C, H, W, D = 3, 2, 9, 10, 12
        x = (0.5 + 0.2 * torch.randn(B, C, H, W, D)).clamp(0, 1)
        x[2, 1, :4] = 0.0  # zeros for the nonzero std
        x = x.to(dt)
        rec = {"x": x}
        for rel in (False, True):
            tr = P.RandRicianNoise(prob=0.7, std=0.2, relative=rel)
            pr = tr.sample_params(B, x.shape, dev)
            pr["mask"][0] = True
            k = "rician_rel" if rel else "rician"
            rec.update({f"{k}_mask": pr["mask"], f"{k}_std": pr["noise_std"],
                        f"{k}_u1": pr["u1"], f"{k}_u2": pr["u2"], f"{k}_out": tr.apply(x, pr)})
        for cw in (False, True):
            for nz in (False, True):
                ts = P.RandStdShiftIntensity(prob=0.7, factors=(-2.0, 2.0), nonzero=nz,
                                             channel_wise=cw)
                ps = ts.sample_params(B, x.shape, dev)
                ps["mask"][0] = True
                k = f"stdshift_cw{int(cw)}_nz{int(nz)}"
                rec.update({f"{k}_mask": ps["mask"], f"{k}_factor": ps["factor"],
                            f"{k}_out": ts.apply(x, ps)})
            tf = P.RandScaleIntensityFixedMean(prob=0.7, factors=0.5, channel_wise=cw)
            pf = tf.sample_params(B, x.shape, dev)
            pf["mask"][0] = True
            k = f"fixedmean_cw{int(cw)}"
            rec.update({f"{k}_mask": pf["mask"], f"{k}_factor": pf["factor"],
                        f"{k}_out": tf.apply(x, pf)})
        save(f"intensity_stats_{tag}", **rec)


def gen_sharpen(P):
    """RandGaussianSharpen: the two blurs, the unsharp-mask combination and
    the sampled params (scalar sigma2 -> [sigma2, sigma1] and tuple sigma2),
    for padding None / reflect / replicate."""
    from batchaug.pytorch.intensity.smooth import separable_gaussian_conv3d
    dev = torch.device("cpu")
    torch.set_num_threads(1)
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        torch.manual_seed(109)
        B, C, H, W, D = 3, 2, 11, 12, 13
        x = (0.5 + 0.2 * torch.randn(B, C, H, W, D)).clamp(0, 1).to(dt)
        rec = {"x": x}
        cases = (("none", None, 0.5), ("reflect", "reflect", (0.3, 0.6)),
                 ("replicate", "replicate", 0.5))
        for name, pm, s2 in cases:
            t = P.RandGaussianSharpen(prob=0.7, sigma2_x=s2, sigma2_y=s2, sigma2_z=s2,
                                      padding_mode=pm)
            p = t.sample_params(B, x.shape, dev)
            p["mask"][0] = True
            k1 = [p[f"kernel1_{a}"] for a in "hwd"]
            k2 = [p[f"kernel2_{a}"] for a in "hwd"]
            bl = separable_gaussian_conv3d(x, *k1, padding_mode=pm)
            db = separable_gaussian_conv3d(bl, *k2, padding_mode=pm)
            rec.update({f"{name}_mask": p["mask"], f"{name}_alpha": p["alpha"],
                        f"{name}_blurred": bl, f"{name}_double_blurred": db,
                        f"{name}_out": t.apply(x, p)})
            for a in "xyz":
                rec[f"{name}_sigma1_{a}"] = p[f"sigma1_{a}"]
                rec[f"{name}_sigma2_{a}"] = p[f"sigma2_{a}"]
            for a in "hwd":
                rec[f"{name}_kernel1_{a}"] = p[f"kernel1_{a}"]
                rec[f"{name}_kernel2_{a}"] = p[f"kernel2_{a}"]
        save(f"sharpen_{tag}", **rec)


LOWRES_MODES = (("nearest", "trilinear", False), ("nearest-exact", "trilinear", False),
                ("nearest", "trilinear", True), ("trilinear", "trilinear", False),
                ("trilinear", "nearest", True), ("area", "trilinear", False),
                ("nearest-exact", "area", False), ("area", "nearest-exact", False))


def gen_lowres(P):
    """RandSimulateLowResolution for every (downsample, upsample,
    align_corners) combination above, with the sampled zoom factors and
    masks; odd sizes so the targets round both ways."""
    dev = torch.device("cpu")
    torch.set_num_threads(1)
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        torch.manual_seed(110)
        B, C, H, W, D = 4, 1, 11, 14, 17
        x = torch.rand(B, C, H, W, D).to(dt)
        rec = {"x": x}
        for i, (dm, um, ac) in enumerate(LOWRES_MODES):
            t = P.RandSimulateLowResolution(prob=0.8, zoom_range=(0.3, 1.0), downsample_mode=dm,
                                            upsample_mode=um, align_corners=ac)
            p = t.sample_params(B, x.shape, dev)
            p["mask"][0] = True
            p["mask"][1] = False
            rec.update({f"m{i}_mask": p["mask"], f"m{i}_zoom": p["zoom_factor"],
                        f"m{i}_out": t.apply(x, p)})
        save(f"lowres_{tag}", **rec)


# ---------------------------------------------------------------------------
# Compose itself: the reference's batchaug.compose.Compose on recorded params
# ---------------------------------------------------------------------------

def _sampler_of(t):
    """The object whose sample_params a Compose step calls for ``t``."""
    inner = getattr(t, "transform", None)
    if inner is not None:
        return inner
    wrapped = getattr(t, "_inner", None)  # RandRotated wraps a RandAffined
    if wrapped is not None:
        return wrapped.transform
    return t


def _record(transforms, overrides):
    """Wrap every transform's sample_params: apply the override for its
    index (forced masks, regenerated large tensors) and log the params."""
    log = {}
    for i, t in enumerate(transforms):
        obj = _sampler_of(t)
        orig = obj.sample_params

        def wrapped(B, shape, device, _i=i, _orig=orig):
            p = _orig(B, shape, device)
            ov = overrides.get(_i)
            if ov is not None:
                p = ov(p, tuple(shape))
            log[_i] = p
            return p
        obj.sample_params = wrapped
    return log


# params regenerated by the tests from a recipe instead of being stored
_REGENERATED = {"noise", "grid", "basis"}


def _params_arrays(log, n):
    out = {}
    for i in range(n):
        for k, v in log.get(i, {}).items():
            if k in _REGENERATED or not isinstance(v, torch.Tensor):
                continue
            out[f"p{i}_{k}"] = v
    return out


def _summary(name, a):
    """A large output kept as: one H plane, a strided subsample and the
    per-(element, channel) sums and sums of squares (float64)."""
    a = np.asarray(a)
    vals = a.astype(np.float32) if a.dtype != np.uint16 else inputs.bf16_to_f32(a)
    H = a.shape[2]
    flat = vals.reshape(a.shape[0] * a.shape[1], -1).astype(np.float64)
    return {f"{name}_plane": a[:, :, (H * 3) // 5], f"{name}_stride": a[:, :, ::9, ::9, ::9],
            f"{name}_sum": flat.sum(1), f"{name}_sumsq": (flat * flat).sum(1)}


def _force(mask_values, extra=None):
    def ov(p, shape):
        p["mask"] = torch.tensor(mask_values)
        if extra is not None:
            p = extra(p, shape)
        return p
    return ov


def _noise_from(seed):
    """Replace the reference's randn noise by the seeded one (same formula:
    z * std + mean in fp32, per element)."""
    def ov(p, shape):
        z = inputs.normal(seed, shape)
        std = p["std"].numpy().astype(np.float32).reshape(-1, 1, 1, 1, 1)
        mean = p["mean"].numpy().astype(np.float32).reshape(-1, 1, 1, 1, 1)
        p["noise"] = torch.from_numpy((z * std + mean).astype(np.float32))
        return p
    return ov


def _grid_from(seed, max_disp):
    def ov(p, shape):
        B, _, H, W, D = shape
        p["grid"] = torch.from_numpy(inputs.elastic_grid(seed, B, (H, W, D), max_disp))
        return p
    return ov


def gen_compose(P):
    """Compose(lazy=True) of the reference at configs 1, 4 and 5 (full size
    for config 1, two-element slices of configs 4 and 5), the
    different-key-sets and mask cases of the reference's tests, and
    RandZoom / RandFlip / RandRotate eager and inside Compose."""
    from batchaug.compose import Compose
    torch.set_num_threads(8)
    dev = torch.device("cpu")

    def run(name, transforms, data, overrides, mode, padding="zeros", seeds=None,
            big=(), lazy=True):
        log = _record(transforms, overrides)
        c = Compose(transforms, lazy=lazy, mode=mode, padding_mode=padding)
        out = c({k: torch.from_numpy(v.copy()) if v.dtype != np.uint16 else
                 torch.from_numpy(v.view(np.int16).copy()).view(torch.bfloat16)
                 for k, v in data.items()})
        rec = _params_arrays(log, len(transforms))
        rec["n_transforms"] = np.int64(len(transforms))
        for k, v in out.items():
            a = npy(v)
            if k in big:
                rec.update(_summary(f"out_{k}", a))
            else:
                rec[f"out_{k}"] = a
        rec.update({f"seed_{k}": np.int64(v) for k, v in (seeds or {}).items()})
        rec["input_digest"] = np.array(inputs.digest(*[data[k] for k in sorted(data)]))
        save(name, **rec)
        return out

    # --- config 1, full size: 2 x 1 x 64^3, flip + affine fused, noise, scale
    shp = (2, 1, 64, 64, 64)
    vol, seg = inputs.normal(201, shp), inputs.labels(202, shp, 5, block=10)
    run("compose_cfg1", [P.RandAxisFlipd(["vol", "seg"], prob=0.5),
                         P.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.785,
                                       shear_range=0.3, translate_range=5),
                         P.RandGaussianNoised(["vol"], std=0.1),
                         P.ScaleIntensityd(["vol"])],
        {"vol": vol, "seg": seg},
        {0: _force([True, False]), 2: _force([True, False], _noise_from(203))},
        {"vol": "bilinear", "seg": "nearest"}, seeds={"vol": 201, "seg": 202, "noise": 203})

    # --- config 4 slice: 2 x 4 x 128^3, {rot90, flip} -> noise -> {affine} -> scale
    shp = (2, 4, 128, 128, 128)
    vol = inputs.normal(401, shp)
    seg = (inputs.labels(402, shp, 2, block=16) > 0).astype(np.float32)
    run("compose_cfg4", [P.RandRotate90d(["vol", "seg"], prob=0.5, max_k=3, spatial_axes=(0, 1)),
                         P.RandAxisFlipd(["vol", "seg"], prob=0.5),
                         P.RandGaussianNoised(["vol"], std=0.5),
                         P.RandAffined(["vol", "seg"], prob=0.5, rotate_range=0.785,
                                       shear_range=0.3, translate_range=5),
                         P.ScaleIntensityd(["vol"])],
        {"vol": vol, "seg": seg},
        {0: _force([True, False]), 1: _force([True, True]),
         2: _force([False, True], _noise_from(403)), 3: _force([True, False])},
        {"vol": "bilinear", "seg": "nearest"}, seeds={"vol": 401, "seg": 402, "noise": 403},
        big=("vol", "seg"))

    # --- config 5 slice: 2 x 2 x 160^3, vol bf16 + seg f32; elastic (grid
    # injected) -> {affine} -> bias -> smooth -> scale
    shp = (2, 2, 160, 160, 160)
    vol = inputs.bf16_bits(inputs.uniform(501, shp))
    seg = inputs.labels(502, shp, 8, block=20)
    run("compose_cfg5", [P.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5, 7),
                                          magnitude_range=(50, 150),
                                          mode={"vol": "bilinear", "seg": "nearest"}),
                         P.RandAffined(["vol", "seg"], prob=0.1, rotate_range=0.5),
                         P.RandBiasFieldd(["vol"], prob=0.1),
                         P.RandGaussianSmoothd(["vol"], prob=0.1, sigma_x=(0.5, 1.5),
                                               sigma_y=(0.5, 1.5), sigma_z=(0.5, 1.5)),
                         P.ScaleIntensityd(["vol"])],
        {"vol": vol, "seg": seg},
        {0: _grid_from(503, 4.0), 1: _force([True, False]), 2: _force([False, True]),
         3: _force([True, False])},
        {"vol": "bilinear", "seg": "nearest"}, seeds={"vol": 501, "seg": 502, "grid": 503},
        big=("vol", "seg"))

    # --- the reference's own Compose cases (tests/test_compose.py) --------
    shp = (4, 3, 16, 16, 16)
    vol, seg = inputs.uniform(601, shp), inputs.labels(602, shp, 5, block=3)
    run("compose_keysets", [P.RandAxisFlipd(["vol", "seg"], prob=1.0),
                            P.RandRotate90d(["vol"], prob=1.0)],
        {"vol": vol, "seg": seg}, {}, "nearest", seeds={"vol": 601, "seg": 602})
    run("compose_partial_mask", [P.RandAxisFlipd(["vol"], prob=0.5)], {"vol": vol},
        {0: _force([True, False, True, False])}, "nearest", seeds={"vol": 601})
    run("compose_mixed", [P.RandAxisFlipd(["vol", "seg"], prob=1.0),
                          P.RandGaussianNoised(["vol"], prob=1.0, std=0.1),
                          P.RandRotate90d(["vol", "seg"], prob=1.0)],
        {"vol": vol, "seg": seg}, {1: _noise_from(603)},
        {"vol": "bilinear", "seg": "nearest"}, seeds={"vol": 601, "seg": 602, "noise": 603})

    # --- RandZoom / RandFlip / RandRotate: eager, and inside Compose -----
    shp = (3, 2, 12, 14, 16)
    vol, seg = inputs.normal(701, shp), inputs.labels(702, shp, 6, block=4)
    mask3 = [True, False, True]
    run("compose_zoom_flip_rotate",
        [P.RandZoomd(["vol", "seg"], prob=0.7, min_zoom=0.7, max_zoom=1.3),
         P.RandFlipd(["vol", "seg"], prob=0.7),
         P.RandRotated(["vol", "seg"], prob=0.7, range_x=0.4, range_y=0.3, range_z=0.2,
                       mode={"vol": "bilinear", "seg": "nearest"}),
         P.RandFlipd(["vol", "seg"], prob=0.7, spatial_axis=[0, 2])],
        {"vol": vol, "seg": seg},
        {0: _force(mask3), 1: _force([False, True, True]), 2: _force(mask3),
         3: _force([True, True, False])},
        {"vol": "bilinear", "seg": "nearest"}, seeds={"vol": 701, "seg": 702})
    x = torch.from_numpy(vol)
    rec = {}
    z = P.RandZoom(prob=0.7, min_zoom=0.7, max_zoom=1.3)
    pz = z.sample_params(3, x.shape, dev)
    pz["mask"] = torch.tensor(mask3)
    rec.update(zoom_mask=pz["mask"], zoom_zoom=pz["zoom"], zoom_affine=pz["affine"],
               zoom_theta=pz["theta"], zoom_out=z.apply(x, pz),
               zoom_nearest_zeros_out=z.apply(x, pz, mode="nearest", padding_mode="zeros"))
    for tag, axis in (("all", None), ("h", 0), ("wd", [1, 2])):
        f = P.RandFlip(prob=0.7, spatial_axis=axis)
        pf = f.sample_params(3, x.shape, dev)
        pf["mask"] = torch.tensor(mask3)
        rec[f"flip_{tag}_mask"] = pf["mask"]
        rec[f"flip_{tag}_out"] = f.apply(x, pf)
    r = P.RandRotate(prob=0.7, range_x=0.4, range_y=(0.1, 0.3), range_z=0.2)
    pr = r.sample_params(3, x.shape, dev)
    pr["mask"] = torch.tensor(mask3)
    rec.update(rotate_mask=pr["mask"], rotate_affine=pr["affine"], rotate_theta=pr["theta"],
               rotate_out=r.apply(x, pr))
    rec["x"] = x
    save("zoom_flip_rotate_eager", **rec)


if __name__ == "__main__":
    main()
