"""RandZoom(d), RandFlip(d) and RandRotate(d) on the GPU against the
reference (batchaug/pytorch/geometric/zoom.py:10-121, flip.py:80-148,
rotate.py:6-77), eager, with the reference's recorded params injected.
Inside a lazy Compose they are covered by tests/test_gpu_compose_ref.py
(compose_zoom_flip_rotate).  Flips are exact voxel maps (bit-exact); the
trilinear zoom and rotation are held to 1e-5."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu


def _params(z, prefix, keys):
    p = {k: to_dev(z[f"{prefix}_{k}"]) for k in keys}
    p["mask"] = to_dev(z[f"{prefix}_mask"]).bool()
    return p


def test_rand_zoom_apply(ba):
    z = load_golden("zoom_flip_rotate_eager")
    x = to_dev(z["x"])
    t = ba.RandZoom(prob=0.7, min_zoom=0.7, max_zoom=1.3)
    p = t.adopt_params(_params(z, "zoom", ("zoom", "affine", "theta")))
    assert_close_dtype(to_np(t.apply(x, p)), z["zoom_out"])
    out = t.apply(x, p, mode="nearest", padding_mode="zeros")
    assert np.array_equal(to_np(out), z["zoom_nearest_zeros_out"])


@pytest.mark.parametrize("tag,axis", [("all", None), ("h", 0), ("wd", [1, 2])])
def test_rand_flip_apply(ba, tag, axis):
    z = load_golden("zoom_flip_rotate_eager")
    x = to_dev(z["x"])
    t = ba.RandFlip(prob=0.7, spatial_axis=axis)
    p = t.adopt_params({"mask": to_dev(z[f"flip_{tag}_mask"]).bool()})
    assert np.array_equal(to_np(t.apply(x, p)), z[f"flip_{tag}_out"])


def test_rand_rotate_apply(ba):
    z = load_golden("zoom_flip_rotate_eager")
    x = to_dev(z["x"])
    t = ba.RandRotate(prob=0.7, range_x=0.4, range_y=(0.1, 0.3), range_z=0.2)
    p = t.adopt_params(_params(z, "rotate", ("affine", "theta")))
    assert_close_dtype(to_np(t.apply(x, p)), z["rotate_out"])


def test_rand_rotated_dict_keys(ba):
    """RandRotated applies one rotation to every key, per-key modes."""
    z = load_golden("zoom_flip_rotate_eager")
    x = to_dev(z["x"])
    seg = torch.round(x.abs() * 3)
    t = ba.RandRotated(["vol", "seg"], prob=0.7, range_x=0.4, range_y=(0.1, 0.3), range_z=0.2,
                       mode={"vol": "bilinear", "seg": "nearest"})
    p = _params(z, "rotate", ("affine", "theta"))
    out = t({"vol": x, "seg": seg}, params=p)
    assert_close_dtype(to_np(out["vol"]), z["rotate_out"])
    ref = ba.RandRotate(prob=0.7).apply(seg, ba.RandRotate(prob=0.7).adopt_params(p),
                                        mode="nearest")
    assert torch.equal(out["seg"], ref)
    assert set(torch.unique(out["seg"]).tolist()) <= set(torch.unique(seg).tolist()) | {0.0}
