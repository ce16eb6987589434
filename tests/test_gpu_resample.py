"""CUDA resample (ba_resample3d) against the oracle and the reference's golden
outputs, in both trilinear modes.  Exact mode (BA_RESAMPLE_EXACT) restates
torch's CPU affine_grid/grid_sample operation by operation: bit-exact for
every mode, padding, align_corners and dtype.  The default fast mode
interpolates with fused lerps: trilinear within 1e-5 (fp32) / 2 bf16 ulp,
nearest still bit-exact (its coordinates are the exact ones)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import assert_close_dtype, to_dev, to_np

pytestmark = pytest.mark.gpu

_MODE = ["exact"]


@pytest.fixture(autouse=True, params=["exact", "fast"])
def resample_mode(request):
    from batchaug_b200 import ops
    old = ops.set_resample_exact(request.param == "exact")
    _MODE[0] = request.param
    yield request.param
    ops.set_resample_exact(old)


def _check(out: np.ndarray, ref: np.ndarray, nearest: bool, msg=None):
    """Bit-exact in exact mode and for nearest; the parity tolerance for the
    fast mode's trilinear output (bf16: 2 ulp, or 1e-6 absolute where the
    value cancels to near zero)."""
    if nearest or _MODE[0] == "exact":
        assert np.array_equal(out, ref), msg
    else:
        assert_close_dtype(out, ref, bf16_abs=1e-6)

MODES = ("bilinear", "nearest")
PADS = ("zeros", "border", "reflection")


def _rand_affine(rng, B, scale=True):
    """MONAI affines like RandAffine's (rotation, shear, translation, scale)."""
    a = np.zeros((B, 4, 4), np.float32)
    for b in range(B):
        ang = rng.uniform(-0.785, 0.785, 3)
        cx, cy, cz = np.cos(ang)
        sx, sy, sz = np.sin(ang)
        rx = np.array([[1, 0, 0], [0, cx, -sx], [0, sx, cx]])
        ry = np.array([[cy, 0, sy], [0, 1, 0], [-sy, 0, cy]])
        rz = np.array([[cz, -sz, 0], [sz, cz, 0], [0, 0, 1]])
        sh = np.eye(3) + rng.uniform(-0.3, 0.3, (3, 3)) * (1 - np.eye(3))
        sc = np.diag(1 + rng.uniform(-0.1, 0.1, 3)) if scale else np.eye(3)
        a[b, :3, :3] = rx @ ry @ rz @ sh @ sc
        a[b, :3, 3] = rng.uniform(-5, 5, 3)
        a[b, 3, 3] = 1
    return a


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("pad", PADS)
@pytest.mark.parametrize("align", [0, 1])
def test_golden_modes(ba, dt, mode, pad, align):
    from batchaug_b200 import ops
    g = load_golden("resample_modes")
    x = to_dev(g["x"] if dt == "f32" else g["x_bf16"])
    out = ops.resample3d(x, theta=to_dev(g["theta"]), modes=mode, paddings=pad,
                         align_corners=bool(align))
    _check(to_np(out), g[f"{dt}_{mode}_{pad}_{align}"], mode == "nearest")


@pytest.mark.parametrize("shape", [(2, 1, 16, 16, 16), (3, 2, 9, 10, 12), (1, 3, 7, 5, 33),
                                   (2, 1, 1, 8, 8), (2, 2, 12, 1, 1), (5, 1, 4, 4, 4)])
@pytest.mark.parametrize("dt", [np.float32, "bf16"])
def test_vs_oracle_random_shapes(ba, oracle_lib, shape, dt):
    """Odd, non-cubic and 1-voxel extents; all modes and paddings, with a mask."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(hash(shape) % 2**32)
    x = rng.standard_normal(shape).astype(np.float32)
    if dt == "bf16":
        x = oracle_lib.to_bf16_bits(x)
    A = _rand_affine(rng, shape[0])
    mask = rng.random(shape[0]) < 0.7
    mask[0] = True
    xd = to_dev(x)
    for mode in MODES:
        for pad in PADS:
            ref = oracle_lib.resample3d(x, affine=A, mode=mode, padding=pad, mask=mask)
            out = ops.resample3d(xd, affine=A, modes=mode, paddings=pad, mask=mask)
            _check(to_np(out), ref, mode == "nearest", (mode, pad))


def test_multi_key_one_launch(ba, oracle_lib):
    """vol bf16 bilinear + seg f32 nearest + a 3-channel key sharing one map."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(7)
    B, H, W, D = 3, 12, 10, 16
    vol = oracle_lib.to_bf16_bits(rng.random((B, 2, H, W, D)).astype(np.float32))
    seg = rng.integers(0, 8, (B, 1, H, W, D)).astype(np.float32)
    img = rng.standard_normal((B, 3, H, W, D)).astype(np.float32)
    A = _rand_affine(rng, B)
    mask = np.array([True, False, True])
    outs = ops.resample3d([to_dev(vol), to_dev(seg), to_dev(img)], affine=A, mask=mask,
                          modes=["bilinear", "nearest", "bilinear"],
                          paddings=["zeros", "zeros", "reflection"])
    _check(to_np(outs[0]), oracle_lib.resample3d(vol, affine=A, mask=mask), False)
    assert np.array_equal(to_np(outs[1]),
                          oracle_lib.resample3d(seg, affine=A, mode="nearest", mask=mask))
    assert np.array_equal(to_np(outs[2]),
                          oracle_lib.resample3d(img, affine=A, padding="reflection", mask=mask))
    # nearest keeps the label set; masked element copied bit for bit
    assert set(np.unique(to_np(outs[1]))) <= set(range(8))
    assert np.array_equal(to_np(outs[0])[1], vol[1])


def test_grid_mode_align_corners(ba, oracle_lib):
    from batchaug_b200 import ops
    g = load_golden("elastic")
    grid = to_dev(g["grid"])
    vo = ops.resample3d(to_dev(g["vol"]), grid=grid, modes="bilinear", align_corners=True)
    so = ops.resample3d(to_dev(g["seg"]), grid=grid, modes="nearest", align_corners=True)
    assert np.array_equal(to_np(vo), g["vol_out"])
    assert np.array_equal(to_np(so), g["seg_out"])


@pytest.mark.parametrize("pad", PADS)
@pytest.mark.parametrize("align", [True, False])
@pytest.mark.parametrize("shape", [(3, 12, 10, 16), (2, 9, 11, 14)])
def test_grid_map_keys_vs_oracle(ba, oracle_lib, pad, align, shape):
    """Grid maps (the lane-per-voxel grid kernel, whole and partial last
    CTAs): a bf16 bilinear key and an fp32 nearest key in one launch, an
    fp32 bilinear key alone, a masked-out element, displacements that leave
    the volume near its faces."""
    from batchaug_b200 import ops
    B, H, W, D = shape
    rng = np.random.default_rng(H * W + D + len(pad) + int(align))
    lin = [np.linspace(-1, 1, n, dtype=np.float32) for n in (H, W, D)]
    zz, yy, xx = np.meshgrid(*lin, indexing="ij")
    grid = np.empty((B, H, W, D, 3), np.float32)
    for b in range(B):
        ph = rng.uniform(0, np.pi, 3)
        grid[b, ..., 0] = xx + 0.2 * np.sin(3 * zz + ph[0])
        grid[b, ..., 1] = yy + 0.2 * np.cos(2 * xx + ph[1])
        grid[b, ..., 2] = zz + 0.2 * np.sin(2 * yy + ph[2])
    vol = rng.random((B, 2, H, W, D)).astype(np.float32)
    vol_bf = oracle_lib.to_bf16_bits(vol)
    seg = rng.integers(0, 6, (B, 1, H, W, D)).astype(np.float32)
    mask = np.ones(B, bool)
    mask[1] = False
    m = mask.astype(np.uint8)
    gd = to_dev(grid)
    vo, so = ops.resample3d([to_dev(vol_bf), to_dev(seg)], grid=gd, modes=["bilinear", "nearest"],
                            paddings=pad, align_corners=align, mask=to_dev(mask))
    assert np.array_equal(to_np(vo), oracle_lib.resample3d(vol_bf, grid=grid, mode="bilinear",
                                                           padding=pad, align_corners=align,
                                                           mask=m))
    assert np.array_equal(to_np(so), oracle_lib.resample3d(seg, grid=grid, mode="nearest",
                                                           padding=pad, align_corners=align,
                                                           mask=m))
    v32 = ops.resample3d(to_dev(vol), grid=gd, modes="bilinear", paddings=pad,
                         align_corners=align)
    assert np.array_equal(to_np(v32), oracle_lib.resample3d(vol, grid=grid, mode="bilinear",
                                                            padding=pad, align_corners=align))


def test_golden_compose_materialize(ba):
    from batchaug_b200 import ops
    g = load_golden("compose_materialize")
    vo, so = ops.resample3d([to_dev(g["vol"]), to_dev(g["seg"])], affine=g["affine"],
                            mask=g["mask"], modes=["bilinear", "nearest"])
    _check(to_np(vo), g["vol_out"], False)
    assert np.array_equal(to_np(so), g["seg_out"])


def test_golden_affine_apply_border(ba):
    g = load_golden("affine_apply_border")
    t = ba.RandAffine(prob=1.0, padding_mode="border")
    params = {"mask": to_dev(g["mask"]), "theta": to_dev(g["theta"]),
              "affine": to_dev(g["affine"]), "spatial_shape": g["x"].shape[2:]}
    out = t.apply(to_dev(g["x"]), params)
    _check(to_np(out), g["out"], False)


def test_golden_flip_rot90_exact(ba):
    g = load_golden("flip_rot90")
    x = to_dev(g["x"])
    fl = ba.RandAxisFlip(prob=1.0)
    pf = {"mask": torch.ones(4, dtype=torch.bool, device="cuda"),
          "axes": to_dev(g["flip_axes"])}
    assert np.array_equal(to_np(fl.apply(x, pf)), g["flip_out"])
    r9 = ba.RandRotate90(prob=1.0, max_k=3)
    pr = {"mask": torch.ones(4, dtype=torch.bool, device="cuda"), "k": to_dev(g["rot_k"])}
    assert np.array_equal(to_np(r9.apply(x, pr)), g["rot_out"])


def test_full_size_config2_properties(ba, oracle_lib):
    """Config 2 at full size (B=8, 128^3, border): compare two elements with
    the oracle exactly; the identity affine reproduces the input to fp32
    rounding (affine_grid's base grid is not exactly on voxel centres, so
    torch's own result is not a bit copy either) and matches the oracle
    exactly; masked-out elements are bit copies."""
    from batchaug_b200 import ops
    torch.manual_seed(0)
    x = torch.rand(8, 1, 128, 128, 128, device="cuda")
    rng = np.random.default_rng(2)
    A = _rand_affine(rng, 8)
    out = ops.resample3d(x, affine=A, paddings="border")
    xs = to_np(x[:2])
    ref = oracle_lib.resample3d(xs, affine=A[:2], padding="border")
    _check(to_np(out[:2]), ref, False)
    eye = np.broadcast_to(np.eye(4, dtype=np.float32), (8, 4, 4)).copy()
    ident = ops.resample3d(x, affine=eye, paddings="border")
    # unnormalised coordinates carry ~size * ulp(1) of rounding: 128 * 6e-8
    assert torch.allclose(ident, x, rtol=0, atol=2e-5)
    _check(to_np(ident[:1]), oracle_lib.resample3d(xs[:1], affine=eye[:1], padding="border"),
           False)
    m = np.zeros(8, bool)
    copy = ops.resample3d(x, affine=A, mask=m)
    assert torch.equal(copy, x)


def test_errors_are_value_errors(ba):
    from batchaug_b200 import ops
    x = torch.zeros(2, 1, 4, 4, 4, device="cuda")
    with pytest.raises(ValueError):
        ops.resample3d(x, modes="bicubic", affine=np.eye(4, dtype=np.float32)[None].repeat(2, 0))
    with pytest.raises(ValueError):
        ops.resample3d(x.double(), affine=np.eye(4, dtype=np.float32)[None].repeat(2, 0))
    with pytest.raises(ValueError):
        # out-of-place only: dst must not alias src
        ops.resample3d(x, affine=np.eye(4, dtype=np.float32)[None].repeat(2, 0), out=[x])


@pytest.mark.parametrize("dt", [np.float32, "bf16"])
@pytest.mark.parametrize("pad", ["zeros", "border"])
@pytest.mark.parametrize("align", [False, True])
def test_staged_tiles_vs_oracle(ba, oracle_lib, dt, pad, align):
    """Volumes spanning several partial 16x16x8 tiles with D % 4 == 0 (the
    shared-memory staged path), one element zoomed out so far that its tiles'
    source boxes do not fit and fall back to global gathers, and a masked-out
    element; a nearest label key rides along in the same launch."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(11)
    shape = (4, 2, 21, 35, 44)
    x = rng.standard_normal(shape).astype(np.float32)
    if dt == "bf16":
        x = oracle_lib.to_bf16_bits(x)
    seg = rng.integers(0, 5, (4, 1) + shape[2:]).astype(np.float32)
    A = _rand_affine(rng, 4)
    A[1, :3, :3] *= 3.5  # zoom out: large source footprints
    mask = np.array([True, True, False, True])
    outs = ops.resample3d([to_dev(x), to_dev(seg)], affine=A, modes=["bilinear", "nearest"],
                          paddings=pad, align_corners=align, mask=mask)
    ref = oracle_lib.resample3d(x, affine=A, mode="bilinear", padding=pad, mask=mask,
                                align_corners=align)
    ref_seg = oracle_lib.resample3d(seg, affine=A, mode="nearest", padding=pad, mask=mask,
                                    align_corners=align)
    _check(to_np(outs[0]), ref, False)
    assert np.array_equal(to_np(outs[1]), ref_seg)


@pytest.mark.parametrize("mode", ["bilinear", "nearest"])
def test_host_params_chunks_equal_device_params(ba, mode):
    """Host (numpy) affines and masks ride in the kernel parameters, 32
    elements per launch: a batch of 70 (three launches) gives exactly what
    the same transforms as device tensors give in one launch."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(70)
    x = to_dev(rng.standard_normal((70, 2, 6, 9, 16)).astype(np.float32))
    A = _rand_affine(rng, 70)
    mask = rng.random(70) < 0.6
    host = ops.resample3d(x, affine=A, mask=mask, modes=mode)
    dev = ops.resample3d(x, affine=torch.from_numpy(A).cuda(), mask=torch.from_numpy(mask).cuda(),
                         modes=mode)
    assert torch.equal(host, dev)
    keep = ~torch.from_numpy(mask).cuda()
    assert torch.equal(host[keep], x[keep])  # masked-out elements copied


def _signed_perm_affines(rng, B, square=True):
    """Products of axis flips and (H, W)-plane rot90s (the maps a Compose of
    RandAxisFlip / RandRotate90 accumulates), MONAI convention."""
    out = np.zeros((B, 4, 4), np.float32)
    for b in range(B):
        a = np.eye(4, dtype=np.float32)
        for ax in range(3):
            if rng.random() < 0.5:
                f = np.eye(4, dtype=np.float32)
                f[ax, ax] = -1
                a = a @ f
        if square and rng.random() < 0.7:
            k = int(rng.integers(1, 4))
            c, s = [0.0, -1.0, 0.0][k - 1], [-1.0, 0.0, 1.0][k - 1]
            r = np.eye(4, dtype=np.float32)
            r[0, 0], r[0, 1], r[1, 0], r[1, 1] = c, -s, s, c
            a = a @ r
        out[b] = a
    return out


@pytest.mark.parametrize("shape", [(3, 2, 16, 16, 32), (2, 3, 12, 12, 20), (4, 1, 9, 9, 8),
                                   (2, 2, 10, 14, 12), (2, 1, 8, 8, 13)])
@pytest.mark.parametrize("dt", [np.float32, "bf16"])
@pytest.mark.parametrize("pad", ["zeros", "border"])
def test_signed_permutations_vs_oracle(ba, oracle_lib, shape, dt, pad):
    """Flips and rot90s (the row-copy kernel in fast mode when D % 4 == 0
    and the rotated plane is square; the general kernels otherwise): a
    bilinear key with a nearest label key in one launch, masked elements,
    against the oracle."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(sum(shape))
    B = shape[0]
    x = rng.standard_normal(shape).astype(np.float32)
    if dt == "bf16":
        x = oracle_lib.to_bf16_bits(x)
    seg = rng.integers(0, 7, shape).astype(np.float32)
    A = _signed_perm_affines(rng, B, square=shape[2] == shape[3])
    mask = rng.random(B) < 0.8
    mask[0] = True
    vo, so = ops.resample3d([to_dev(x), to_dev(seg)], affine=A, modes=["bilinear", "nearest"],
                            paddings=pad, mask=mask)
    ref = oracle_lib.resample3d(x, affine=A, mode="bilinear", padding=pad, mask=mask)
    ref_seg = oracle_lib.resample3d(seg, affine=A, mode="nearest", padding=pad, mask=mask)
    _check(to_np(vo), ref, False)
    assert np.array_equal(to_np(so), ref_seg)
    # nearest alone (an eager flip / rot90) is an exact voxel permutation
    n1 = ops.resample3d(to_dev(seg), affine=A, modes="nearest", paddings=pad, mask=mask)
    assert np.array_equal(to_np(n1), ref_seg)


@pytest.mark.parametrize("shape", [(2, 2, 12, 12, 16), (3, 1, 8, 8, 256), (2, 1, 7, 7, 40),
                                   (5, 2, 20, 20, 24)])
@pytest.mark.parametrize("pad", ["zeros", "border"])
def test_signed_permutations_tma_keys(ba, oracle_lib, shape, pad):
    """The TMA-staged row copy (rows of 16-byte multiples, H, W, D <= 256):
    three keys of mixed mode and dtype in one launch (an fp32 and a bf16
    bilinear key, a bf16 label key), partial tiles, a D of 256 (two chunks
    per lane), masked elements; then no bounded device wait ran out."""
    from batchaug_b200 import _lib, ops
    rng = np.random.default_rng(sum(shape) + 7)
    B = shape[0]
    x = rng.standard_normal(shape).astype(np.float32)
    xb = oracle_lib.to_bf16_bits(rng.standard_normal(shape).astype(np.float32))
    seg = oracle_lib.to_bf16_bits(rng.integers(0, 9, shape).astype(np.float32))
    A = _signed_perm_affines(rng, B)
    mask = rng.random(B) < 0.7
    mask[0] = True
    outs = ops.resample3d([to_dev(x), to_dev(xb), to_dev(seg)], affine=A,
                          modes=["bilinear", "bilinear", "nearest"], paddings=pad, mask=mask)
    _lib.wait_status()
    for o, src, mode in zip(outs, (x, xb, seg), ("bilinear", "bilinear", "nearest")):
        ref = oracle_lib.resample3d(src, affine=A, mode=mode, padding=pad, mask=mask)
        _check(to_np(o), ref, mode == "nearest")


def test_signed_permutation_copies_keep_bits(ba):
    """Masked-out elements and nearest keys are bit copies: bf16 and fp32 NaN
    payloads and negative zeros come through unchanged."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(11)
    B, C, H, W, D = 3, 2, 8, 8, 32
    A = _signed_perm_affines(rng, B)
    mask = np.array([True, False, True])
    for dtype, nan_bits in ((torch.bfloat16, 0x7F85), (torch.float32, 0x7F800123)):
        itype = np.int16 if dtype == torch.bfloat16 else np.int32
        info = np.iinfo(itype)
        nb = rng.integers(info.min, info.max, (B, C, H, W, D), dtype=itype, endpoint=True)
        nb[..., 3] = nan_bits
        nb[..., 5] = info.min  # -0.0
        bits = torch.from_numpy(nb)
        t = bits.view(dtype).cuda()
        out = ops.resample3d(t, affine=A, modes="nearest", paddings="zeros", mask=mask)
        got = out.view(bits.dtype).cpu()
        assert torch.equal(got[1], bits[1])  # masked out: copied bit for bit
        ref = ops.resample3d(t.float(), affine=A, modes="nearest", paddings="zeros", mask=mask)
        fin = torch.isfinite(ref.cpu())
        assert torch.equal(out.float().cpu()[fin], ref.cpu()[fin])
        # every voxel of an active element is some source voxel's exact bits
        for b in (0, 2):
            assert torch.equal(torch.sort(got[b].flatten())[0], torch.sort(bits[b].flatten())[0])


@pytest.mark.parametrize("zoom", [1.5, 1.7, 2.2])
@pytest.mark.parametrize("pad", ["zeros", "border"])
def test_large_footprints_vs_oracle(ba, oracle_lib, zoom, pad):
    """Source footprints around and over the staging limit (a zoom-out of
    1.5-2.2 with a rotation and shear): some tiles stage their box, the others
    gather from global memory; partial tiles along every axis, two channels,
    a label key in the same launch."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(int(zoom * 10))
    shape = (2, 2, 37, 48, 60)
    x = rng.standard_normal(shape).astype(np.float32)
    seg = rng.integers(0, 5, (2, 1) + shape[2:]).astype(np.float32)
    A = _rand_affine(rng, 2, scale=False)
    A[:, :3, :3] *= zoom
    outs = ops.resample3d([to_dev(x), to_dev(seg)], affine=A, modes=["bilinear", "nearest"],
                          paddings=pad)
    ref = oracle_lib.resample3d(x, affine=A, mode="bilinear", padding=pad)
    ref_seg = oracle_lib.resample3d(seg, affine=A, mode="nearest", padding=pad)
    _check(to_np(outs[0]), ref, False)
    assert np.array_equal(to_np(outs[1]), ref_seg)


def test_tensor_map_cache_follows_shape(ba, oracle_lib):
    """The TMA kernel caches tensor maps by address, dtype and shape: two
    volumes of different shapes starting at the same address (views of one
    buffer) each resample correctly, in either order, twice."""
    from batchaug_b200 import _lib, ops
    rng = np.random.default_rng(5)
    buf = torch.empty(2 * 12 * 16 * 20 * 8, device="cuda")
    shapes = [(2, 2, 16, 16, 24), (3, 1, 12, 12, 32)]
    for _ in range(2):
        for shape in shapes + shapes[::-1]:
            n = int(np.prod(shape))
            x = rng.standard_normal(shape).astype(np.float32)
            src = buf[:n].view(shape)
            src.copy_(torch.from_numpy(x))
            A = _signed_perm_affines(rng, shape[0])
            out = ops.resample3d(src, affine=A, modes="nearest", paddings="zeros")
            ref = oracle_lib.resample3d(x, affine=A, mode="nearest", padding="zeros")
            assert np.array_equal(to_np(out), ref), shape
    _lib.wait_status()


def _decode_keys(keys: np.ndarray) -> np.ndarray:
    """The order-preserving int32 min/max keys as floats."""
    k = keys.astype(np.int64)
    bits = np.where(k >= 0, k, k ^ 0x7FFFFFFF) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("case", ["affine_pair", "affine_bf16", "perm", "exact", "grid_like"])
def test_resample_minmax_matches_output(ba, case):
    """minmax holds each output's per-(element, channel) min and max: folded
    by the staged affine kernel (masked-out copies included, 4 channels per
    pass), reduced from the output on every other path."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(17)
    B, C, H, W, D = 5, 4, 24, 20, 32
    vol = torch.from_numpy(rng.standard_normal((B, C, H, W, D)).astype(np.float32)).cuda()
    seg = torch.from_numpy(rng.integers(0, 3, (B, 2, H, W, D)).astype(np.float32)).cuda()
    if case == "affine_bf16":
        vol = vol.bfloat16()
    A = _signed_perm_affines(rng, B, square=False) if case == "perm" else _rand_affine(rng, B)
    mask = np.array([True, False, True, True, False])
    mm = [torch.empty(B, C, 2, dtype=torch.int32, device="cuda"),
          torch.empty(B, 2, 2, dtype=torch.int32, device="cuda")]
    kw = dict(affine=A, modes=["bilinear", "nearest"], paddings="zeros", mask=mask, minmax=mm)
    if case == "exact":
        kw["exact"] = True
    if case == "grid_like":
        kw["paddings"] = "reflection"  # the global-gather kernel
    outs = ops.resample3d([vol, seg], **kw)
    for o, m in zip(outs, mm):
        got = _decode_keys(m.cpu().numpy())
        of = o.float()
        assert np.array_equal(got[..., 0], of.amin(dim=(2, 3, 4)).cpu().numpy()), case
        assert np.array_equal(got[..., 1], of.amax(dim=(2, 3, 4)).cpu().numpy()), case


def test_scale_intensity_with_given_stats(ba):
    """A ScaleIntensity chain fed the resample's min/max gives the result of
    the chain that reduces its input itself, bit for bit."""
    from batchaug_b200 import ops
    rng = np.random.default_rng(23)
    B, C = 4, 3
    x = torch.from_numpy(rng.standard_normal((B, C, 16, 16, 32)).astype(np.float32)).cuda()
    mm = torch.empty(B, C, 2, dtype=torch.int32, device="cuda")
    y = ops.resample3d(x, affine=_rand_affine(rng, B), paddings="border", minmax=[mm])
    si = ba.ScaleIntensity(minv=0.0, maxv=1.0)
    ref = ops.intensity_chain(y, [si.chain_op(None, y)])
    got = ops.intensity_chain(y, [si.chain_op(None, y, stats=mm)])
    assert torch.equal(ref, got)
