"""Compose itself against the reference's Compose (batchaug/compose.py:116-164).

tests/golden/gen_golden.py ran the reference's ``Compose(lazy=True)`` on CPU
for config 1 (full size), two-element slices of configs 4 and 5, the
reference's own key-set and mask cases (tests/test_compose.py:217-253,
:287-308) and RandZoom / RandFlip / RandRotate inside a Compose, recording
every transform's params.  Here ``batchaug_b200.Compose`` replays the same
pipelines with those params injected (``Compose(...)(data, params=...)``)
and must give the reference's outputs: label maps (nearest) bit for bit,
volumes within 1e-5 (fp32) or 2 bf16 ulp.

Inputs, the injected noise and the injected elastic grid are regenerated
from their seeds (tests/golden/inputs.py) and checked against the digest the
generator stored.  Outputs too large to commit are compared through one H
plane, a strided subsample and the per-(element, channel) sums.
"""
from __future__ import annotations

import importlib.util
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from helpers import as_f32, assert_close_dtype, to_np

pytestmark = pytest.mark.gpu

_spec = importlib.util.spec_from_file_location("golden_inputs", os.path.join(GOLDEN, "inputs.py"))
inputs = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(inputs)

VB = {"vol": "bilinear", "seg": "nearest"}


def _cfg1(ba):
    return [ba.RandAxisFlipd(["vol", "seg"], prob=0.5),
            ba.RandAffined(["vol", "seg"], prob=1.0, rotate_range=0.785, shear_range=0.3,
                           translate_range=5),
            ba.RandGaussianNoised(["vol"], std=0.1),
            ba.ScaleIntensityd(["vol"])]


def _cfg4(ba):
    return [ba.RandRotate90d(["vol", "seg"], prob=0.5, max_k=3, spatial_axes=(0, 1)),
            ba.RandAxisFlipd(["vol", "seg"], prob=0.5),
            ba.RandGaussianNoised(["vol"], std=0.5),
            ba.RandAffined(["vol", "seg"], prob=0.5, rotate_range=0.785, shear_range=0.3,
                           translate_range=5),
            ba.ScaleIntensityd(["vol"])]


def _cfg5(ba):
    return [ba.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5, 7),
                              magnitude_range=(50, 150), mode=VB),
            ba.RandAffined(["vol", "seg"], prob=0.1, rotate_range=0.5),
            ba.RandBiasFieldd(["vol"], prob=0.1),
            ba.RandGaussianSmoothd(["vol"], prob=0.1, sigma_x=(0.5, 1.5), sigma_y=(0.5, 1.5),
                                   sigma_z=(0.5, 1.5)),
            ba.ScaleIntensityd(["vol"])]


def _zfr(ba):
    return [ba.RandZoomd(["vol", "seg"], prob=0.7, min_zoom=0.7, max_zoom=1.3),
            ba.RandFlipd(["vol", "seg"], prob=0.7),
            ba.RandRotated(["vol", "seg"], prob=0.7, range_x=0.4, range_y=0.3, range_z=0.2,
                           mode=VB),
            ba.RandFlipd(["vol", "seg"], prob=0.7, spatial_axis=[0, 2])]


def _in_cfg1(z):
    shp = (2, 1, 64, 64, 64)
    return {"vol": inputs.normal(int(z["seed_vol"]), shp),
            "seg": inputs.labels(int(z["seed_seg"]), shp, 5, block=10)}


def _in_cfg4(z):
    shp = (2, 4, 128, 128, 128)
    return {"vol": inputs.normal(int(z["seed_vol"]), shp),
            "seg": (inputs.labels(int(z["seed_seg"]), shp, 2, block=16) > 0).astype(np.float32)}


def _in_cfg5(z):
    shp = (2, 2, 160, 160, 160)
    return {"vol": inputs.bf16_bits(inputs.uniform(int(z["seed_vol"]), shp)),
            "seg": inputs.labels(int(z["seed_seg"]), shp, 8, block=20)}


def _in_small(z, shp=(4, 3, 16, 16, 16), n_labels=5, block=3, vol=inputs.uniform):
    d = {"vol": vol(int(z["seed_vol"]), shp)}
    if "seed_seg" in z:
        d["seg"] = inputs.labels(int(z["seed_seg"]), shp, n_labels, block=block)
    return d


def _in_zfr(z):
    return _in_small(z, (3, 2, 12, 14, 16), 6, 4, inputs.normal)


# name -> (transforms, Compose mode, inputs, {index: injected large tensor})
CASES = {
    "compose_cfg1": (_cfg1, VB, _in_cfg1, {2: "noise"}),
    "compose_cfg4": (_cfg4, VB, _in_cfg4, {2: "noise"}),
    "compose_cfg5": (_cfg5, VB, _in_cfg5, {0: "grid"}),
    "compose_keysets": (lambda ba: [ba.RandAxisFlipd(["vol", "seg"], prob=1.0),
                                    ba.RandRotate90d(["vol"], prob=1.0)], "nearest", _in_small, {}),
    "compose_partial_mask": (lambda ba: [ba.RandAxisFlipd(["vol"], prob=0.5)], "nearest",
                             _in_small, {}),
    "compose_mixed": (lambda ba: [ba.RandAxisFlipd(["vol", "seg"], prob=1.0),
                                  ba.RandGaussianNoised(["vol"], prob=1.0, std=0.1),
                                  ba.RandRotate90d(["vol", "seg"], prob=1.0)], VB, _in_small,
                      {1: "noise"}),
    "compose_zoom_flip_rotate": (_zfr, VB, _in_zfr, {}),
}


def _to_torch(a: np.ndarray, device) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _params(z, data, regen, device):
    """The recorded params, in transform order, with the regenerated noise /
    grid tensors put back."""
    n = int(z["n_transforms"])
    shape = data["vol"].shape
    out = []
    for i in range(n):
        p = {}
        pre = f"p{i}_"
        for k in z:
            if k.startswith(pre):
                a = z[k]
                t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
                p[k[len(pre):]] = t.bool() if k.endswith("_mask") else t
        kind = regen.get(i)
        if kind == "noise":
            std = z[f"{pre}std"].astype(np.float32).reshape(-1, 1, 1, 1, 1)
            mean = z[f"{pre}mean"].astype(np.float32).reshape(-1, 1, 1, 1, 1)
            nz = (inputs.normal(int(z["seed_noise"]), shape) * std + mean).astype(np.float32)
            p["noise"] = torch.from_numpy(nz).to(device)
        elif kind == "grid":
            B, _, H, W, D = shape
            p["grid"] = torch.from_numpy(
                inputs.elastic_grid(int(z["seed_grid"]), B, (H, W, D), 4.0)).to(device)
        out.append(p)
    return out


def _summary(a: np.ndarray):
    vals = as_f32(a).astype(np.float64)
    H = a.shape[2]
    flat = vals.reshape(a.shape[0] * a.shape[1], -1)
    return a[:, :, (H * 3) // 5], a[:, :, ::9, ::9, ::9], flat.sum(1), (flat * flat).sum(1)


def _check(name, key, out: np.ndarray, z, exact: bool):
    if f"out_{key}" in z:
        ref = z[f"out_{key}"]
        if exact:
            assert np.array_equal(out, ref), f"{name}/{key}: differs from the reference"
        else:
            assert_close_dtype(out, ref, bf16_abs=1e-6)
        return
    plane, stride, s, ss = _summary(out)
    for part, mine in (("plane", plane), ("stride", stride)):
        ref = z[f"out_{key}_{part}"]
        if exact:
            assert np.array_equal(mine, ref), f"{name}/{key} {part}: differs from the reference"
        else:
            assert_close_dtype(mine, ref, bf16_abs=1e-6)
    if exact:
        np.testing.assert_array_equal(s, z[f"out_{key}_sum"])
        np.testing.assert_array_equal(ss, z[f"out_{key}_sumsq"])
    else:
        n = out[0, 0].size
        tol = n * (1e-5 if out.dtype == np.float32 else 2 * 2.0 ** -8)
        np.testing.assert_allclose(s, z[f"out_{key}_sum"], rtol=0, atol=tol)


@pytest.mark.parametrize("name", sorted(CASES))
def test_compose_matches_reference(ba, name):
    make, mode, make_inputs, regen = CASES[name]
    z = load_golden(name)
    data_np = make_inputs(z)
    assert inputs.digest(*[data_np[k] for k in sorted(data_np)]) == str(z["input_digest"]), \
        "regenerated inputs differ from the generator's"
    dev = torch.device("cuda")
    data = {k: _to_torch(v, dev) for k, v in data_np.items()}
    params = _params(z, data_np, regen, dev)
    out = ba.Compose(make(ba), lazy=True, mode=mode)(dict(data), params=params)
    torch.cuda.synchronize()
    for key in data:
        exact = key == "seg" or mode == "nearest"
        _check(name, key, to_np(out[key]), z, exact)
    # the caller's tensors are never written
    for k, v in data_np.items():
        assert np.array_equal(to_np(data[k]), v)


@pytest.mark.parametrize("name", ["compose_mixed", "compose_keysets"])
def test_compose_eager_matches_lazy(ba, name):
    """The reference's lazy-vs-eager property (tests/test_compose.py:42-81,
    :173-214) with the same injected params: flips and rot90 land on voxel
    centres, so label maps are identical and volumes agree within 1e-5."""
    make, mode, make_inputs, regen = CASES[name]
    z = load_golden(name)
    data_np = make_inputs(z)
    dev = torch.device("cuda")
    data = {k: _to_torch(v, dev) for k, v in data_np.items()}
    params = _params(z, data_np, regen, dev)
    lazy = ba.Compose(make(ba), lazy=True, mode=mode)(dict(data), params=params)
    eager = ba.Compose(make(ba), lazy=False, mode=mode)(dict(data), params=params)
    torch.cuda.synchronize()
    for k in data:
        a, b = to_np(lazy[k]), to_np(eager[k])
        if k == "seg" or mode == "nearest":
            assert np.array_equal(a, b), k
        else:
            np.testing.assert_allclose(a, b, rtol=0, atol=1e-5)


def test_params_length_checked(ba):
    with pytest.raises(ValueError, match="entries"):
        ba.Compose(_cfg1(ba), lazy=True)({"vol": torch.zeros(2, 1, 4, 4, 4, device="cuda")},
                                         params=[None])
