"""Benchmark: augmented voxels/s of batchaug's hot path on B200, and the
fraction of the HBM roofline its dominant kernel reaches.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload config4|config2|config3|...]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

Headline workload (config 4 of the reference's headline set, the largest
configuration that fits one GPU as a whole Compose of both keys): per GPU a
dict batch vol + seg, each (5, 4, 128, 128, 128) fp32 (vol N(0,1); seg the
{0,1} threshold at 0 of Gaussian-smoothed (sigma 3) noise), through
Compose(lazy=True) of RandRotate90d(0.5, max_k 3, axes (0,1)),
RandAxisFlipd(0.5), RandGaussianNoised(vol, std 0.5), RandAffined(0.5,
rotate 0.785, shear 0.3, translate 5), ScaleIntensityd(vol), with bilinear
vol and nearest seg.  A step is one Compose call: host parameter sampling,
two fused resamples (one launch each for both keys) and the intensity
chains.  Ranks shard the batch (weak scaling: 5 elements per rank, global
element offset rank*5) with no collective on the data path; NCCL is used
only for the barrier and the max-over-ranks of the timings.

Timing: W untimed warm-up steps, then K steps between barrier +
cuda.synchronize, timed with CUDA events on the launching stream; inputs
alternate between 2 distinct batches of 671 MB each (larger than the 126 MB
L2).  ``value`` = voxels of all keys and ranks / max-over-ranks time.  Every
library call is also bracketed by CUDA events
(``batchaug_b200._timing``) in a second run of the same steps after the
timed one, each span behind a short device busy-wait so that it holds the
kernels alone and not the host's launch latency; ``roofline`` is the dominant entry point's
algorithmic bytes per launch over its mean event-timed duration, and
``roofline_step`` the whole step's algorithmic bytes over the step time.
``e2e`` is the same step through the public API from pinned host memory:
H2D of every input key, the Compose, D2H of every output key, every step,
with the copies on their own streams (double-buffered) so they overlap the
neighbouring steps' work; ``e2e.copy_bound`` times the same copies with no
transform between them (the host link's concurrent rate, which bounds it).

--impl reference runs the reference algorithm on the host CPU cores: the C
oracle (a restatement of the reference's PyTorch path; the Python reference
cannot be shipped to the GPU host) on the same workload, with parameters
drawn in numpy; it never imports batchaug_b200.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "augmented voxels/s at 1/2/4/8 B200; fraction of HBM roofline"
UNIT = "voxel/s"
HEADLINE = "config4"

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# dominant entry point's kernels, from ncu captures of those kernels.
#   config2: resample3d_fast_kernel<2,-1> on 8x1x128^3 fp32 (RandAffine,
#     border), one launch: 63,000,576 + 34,108,928 B.
#   config4: the step's two ba_resample3d launches, captured on a 2-element
#     slice of the workload (2x4x128^3 vol + seg) and scaled to the 5
#     elements of a launch (traffic grows with the elements): the permutation
#     kernel resample3d_permt_kernel<0,1> 136,066,816 + 89,412,352 B and the
#     affine kernel resample3d_fast_kernel<0,6,1> (min/max folded)
#     130,400,256 + 102,155,520 B, mean 229,017,472 B x 5 / 2.
DRAM_BYTES_PER_LAUNCH = {"config2": 97109504, "config4": 572543680}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples = []
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    hh = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(hh)
                    u = u.decode() if isinstance(u, bytes) else u
                    if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                        h = hh
            self.h = h or pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report no clocks rather than fail
            self.err = str(e)
        self.period = period_s
        self._stop = threading.Event()
        self._t = None

    def _sample(self):
        n = self.nvml
        sm = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
        try:
            r = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            r = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        self.samples.append((sm, r))

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._sample()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self.ok and self._t is not None:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "note": "NVML unavailable"}
        mhz = [s for s, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [name for bit, name in self.REASONS.items() if bits & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# Workloads.  Each describes one step and its shapes; ``config`` is shared
# verbatim by the b200 and reference arms.
# ---------------------------------------------------------------------------

class Workload:
    def __init__(self, name, text, dtype, keys, elements, volume, inputs_note,
                 build=None, reference=None, e2e=True):
        self.name, self.text, self.dtype = name, text, dtype
        self.keys = keys              # {key: (channels, bytes per voxel)}
        self.elements = elements      # batch elements per GPU
        self.volume = volume          # spatial shape
        self.inputs_note = inputs_note
        self.build = build            # (torch, ba, device, rank) -> (input sets, step)
        self.reference = reference    # (rng, nthreads) -> (inputs, step(inputs, rng)) or None
        self.e2e = e2e

    @property
    def voxels(self) -> int:
        n = int(np.prod(self.volume))
        return sum(self.elements * c * n for c, _ in self.keys.values())

    @property
    def alg_bytes(self) -> int:
        """Every key read once plus written once."""
        n = int(np.prod(self.volume))
        return sum(self.elements * c * n * 2 * b for c, b in self.keys.values())

    def config(self) -> dict:
        return {"workload": self.text, "elements_per_gpu": self.elements,
                "keys": {k: [c] + list(self.volume) for k, (c, _) in self.keys.items()},
                "l2": self.inputs_note}


def _smooth_noise(torch, ops, shape, sigma, device, g):
    u = torch.randn(*shape, device=device, generator=g)
    K = ops.gauss_taps_len(sigma, 4.0)
    taps = ops.gauss_taps(torch.full((shape[0],), float(sigma), device=device), K)
    return ops.smooth3d(u, taps, taps, taps)


def _config4_compose(ba):
    return ba.Compose([ba.RandRotate90d(["vol", "seg"], prob=0.5, max_k=3, spatial_axes=(0, 1)),
                       ba.RandAxisFlipd(["vol", "seg"], prob=0.5),
                       ba.RandGaussianNoised(["vol"], std=0.5),
                       ba.RandAffined(["vol", "seg"], prob=0.5, rotate_range=0.785,
                                      shear_range=0.3, translate_range=5),
                       ba.ScaleIntensityd(["vol"])], lazy=True,
                      mode={"vol": "bilinear", "seg": "nearest"})


def _build_config4(torch, ba, device, rank):
    from batchaug_b200 import ops
    g = torch.Generator(device=device)
    sets = []
    B = WORKLOADS["config4"].elements
    for i in range(2):
        g.manual_seed(100 * rank + i)
        vol = torch.randn(B, 4, 128, 128, 128, device=device, generator=g)
        seg = (_smooth_noise(torch, ops, (B, 4, 128, 128, 128), 3.0, device, g) > 0).float()
        sets.append({"vol": vol, "seg": seg})
    c = _config4_compose(ba)
    return sets, c


def _ref_config4(rng, nthreads):
    import oracle
    from oracle import pipelines as P
    vol = P.normal_f32(rng, (5, 4, 128, 128, 128), nthreads)
    noise = P.normal_f32(rng, (5, 4, 128, 128, 128), nthreads)
    taps = oracle.gaussian_1d_batch(np.full(5, 3.0, np.float32), 4.0)
    seg = (oracle.separable_gauss(noise, taps, taps, taps, nthreads=nthreads) > 0)
    inputs = {"vol": vol, "seg": seg.astype(np.float32)}
    return inputs, lambda d, r: P.config4_step(d["vol"], d["seg"], r, nthreads)


def _build_config2(torch, ba, device, rank):
    from batchaug_b200 import ops
    g = torch.Generator(device=device)
    sets = []
    for i in range(4):
        g.manual_seed(1000 * rank + i)
        u = torch.rand(8, 1, 128, 128, 128, device=device, generator=g)
        K = ops.gauss_taps_len(2.0, 4.0)
        taps = ops.gauss_taps(torch.full((8,), 2.0, device=device), K)
        sets.append({"vol": ops.smooth3d(u, taps, taps, taps)})
    t = ba.RandAffine(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=5,
                      scale_range=0.1, mode="bilinear", padding_mode="border")
    return sets, lambda d: {"vol": t(d["vol"])}


def _ref_config2(rng, nthreads):
    from oracle import pipelines as P
    x = rng.random((8, 1, 128, 128, 128), dtype=np.float32)
    return {"vol": x}, lambda d, r: {"vol": P.config2_step(d["vol"], r, nthreads)}


def _build_config3(torch, ba, device, rank):
    g = torch.Generator(device=device)
    g.manual_seed(7 + rank)
    sets = [{"v": (0.5 + 0.2 * torch.randn(16, 4, 128, 128, 128, device=device, generator=g))
             .clamp(0, 1).bfloat16()} for _ in range(2)]
    c = ba.Compose([ba.RandGaussianNoised(["v"], prob=1.0, std=(0.1, 0.5)),
                    ba.RandAdjustContrastd(["v"], prob=1.0, gamma=(0.5, 2.0)),
                    ba.RandScaleIntensityd(["v"], prob=1.0, factors=0.2),
                    ba.RandShiftIntensityd(["v"], prob=1.0, offsets=0.1),
                    ba.ScaleIntensityd(["v"], minv=0.0, maxv=1.0)], lazy=True)
    return sets, c


def _ref_config3(rng, nthreads):
    import oracle
    from oracle import pipelines as P
    x = np.clip(0.5 + 0.2 * P.normal_f32(rng, (16, 4, 128, 128, 128), nthreads), 0, 1)
    xb = oracle.to_bf16_bits(x)
    return {"v": xb}, lambda d, r: {"v": P.config3_step(d["v"], r, nthreads)}


def _config5_compose(ba, fuse=False):
    return ba.Compose([ba.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5, 7),
                                         magnitude_range=(50, 150),
                                         mode={"vol": "bilinear", "seg": "nearest"}),
                       ba.RandAffined(["vol", "seg"], prob=0.1, rotate_range=0.5),
                       ba.RandBiasFieldd(["vol"], prob=0.1),
                       ba.RandGaussianSmoothd(["vol"], prob=0.1, sigma_x=(0.5, 1.5),
                                              sigma_y=(0.5, 1.5), sigma_z=(0.5, 1.5)),
                       ba.ScaleIntensityd(["vol"])], lazy=True,
                      mode={"vol": "bilinear", "seg": "nearest"}, fuse_elastic=fuse)


def _build_config5(fuse):
    def build(torch, ba, device, rank):
        g = torch.Generator(device=device)
        g.manual_seed(7 + rank)
        vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
        seg = torch.randint(0, 8, (8, 2, 160, 160, 160), device=device, generator=g).float()
        return [{"vol": vol, "seg": seg}], _config5_compose(ba, fuse)
    return build


def _build_single(make):
    """A workload whose step is one transform or op on one tensor."""
    def build(torch, ba, device, rank):
        g = torch.Generator(device=device)
        g.manual_seed(7 + rank)
        sets, fn = make(torch, ba, device, g)
        return sets, fn
    return build


def _mk_smooth(torch, ba, device, g):
    vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
    sm = ba.RandGaussianSmooth(prob=1.0, sigma_x=(0.5, 1.5), sigma_y=(0.5, 1.5),
                               sigma_z=(0.5, 1.5))
    p = sm.sample_params(8, vol.shape, device)
    return [{"vol": vol}], lambda d: {"vol": sm.apply(d["vol"], p)}


def _mk_sharpen(torch, ba, device, g):
    vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
    sh = ba.RandGaussianSharpen(prob=1.0)
    p = sh.sample_params(8, vol.shape, device)
    return [{"vol": vol}], lambda d: {"vol": sh.apply(d["vol"], p)}


def _mk_stats(torch, ba, device, g):
    sets = [{"v": (0.5 + 0.2 * torch.randn(16, 4, 128, 128, 128, device=device, generator=g))
             .clamp(0, 1).bfloat16()} for _ in range(2)]
    c = ba.Compose([ba.RandStdShiftIntensityd(["v"], prob=1.0, nonzero=True),
                    ba.RandRicianNoised(["v"], prob=1.0, std=0.1, relative=True),
                    ba.RandScaleIntensityFixedMeand(["v"], prob=1.0, channel_wise=True)],
                   lazy=True)
    return sets, c


def _mk_lowres(down):
    def mk(torch, ba, device, g):
        sets = [{"vol": torch.rand(8, 1, 128, 128, 128, device=device, generator=g)}
                for _ in range(4)]
        lr = ba.RandSimulateLowResolution(prob=1.0, zoom_range=(0.5, 1.0), downsample_mode=down)
        return sets, lambda d: {"vol": lr(d["vol"])}
    return mk


def _mk_elastic(D):
    def mk(torch, ba, device, g):
        el = ba.Rand3DElastic(prob=1.0, sigma_range=(5, 7), magnitude_range=(50, 150))
        shape = (8, 2, 160, 160, D)
        return [{}], lambda d: {"grid": el.sample_params(8, shape, device)["grid"]}
    return mk


def _mk_eager(cls, shape=(8, 1, 128, 128, 128), **kw):
    def mk(torch, ba, device, g):
        sets = [{"vol": torch.rand(*shape, device=device, generator=g)} for _ in range(4)]
        t = getattr(ba, cls)(prob=1.0, **kw)
        return sets, lambda d: {"vol": t(d["vol"])}
    return mk


def _mk_minmax(torch, ba, device, g):
    from batchaug_b200 import ops
    sets = [{"v": torch.rand(16, 4, 128, 128, 128, device=device, generator=g).bfloat16()}
            for _ in range(2)]
    return sets, lambda d: dict(zip(("min", "max"), ops.minmax(d["v"], 64)))


def _mk_fallbacks(torch, ba, device, g):
    """One launch of each kernel that only fallback cases reach: the exact
    trilinear mode (resample3d_staged_kernel), an elastic field whose taps
    exceed the wide passes' 63 (elastic_draw4, axis passes, elastic grid),
    a smoothing with more than 63 taps (axis passes), and a smoothing whose
    H line is too long to stage (roll_axis)."""
    from batchaug_b200 import ops
    vol = torch.rand(8, 1, 128, 128, 128, device=device, generator=g)
    aff = ba.RandAffine(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=5,
                        scale_range=0.1, padding_mode="border")
    pa = aff.sample_params(8, vol.shape, device)
    el = ba.Rand3DElastic(prob=1.0, sigma_range=(11.0, 12.0), magnitude_range=(50, 150))
    v2 = torch.rand(2, 1, 96, 96, 96, device=device, generator=g)
    big = ba.RandGaussianSmooth(prob=1.0, sigma_x=(8.5, 9.0), sigma_y=(8.5, 9.0),
                                sigma_z=(8.5, 9.0))
    pb = big.sample_params(2, v2.shape, device)
    v3 = torch.rand(1, 1, 800, 64, 48, device=device, generator=g)
    long_h = ba.RandGaussianSmooth(prob=1.0, sigma_x=(5.0, 5.0), sigma_y=(5.0, 5.0),
                                   sigma_z=(5.0, 5.0))
    pl = long_h.sample_params(1, v3.shape, device)

    def step(d):
        with ops.resample_exact(True):
            a = aff.apply(d["vol"], pa)
        grid = el.sample_params(2, (2, 1, 96, 96, 96), device)["grid"]
        return {"a": a, "grid": grid, "b": big.apply(d["v2"], pb), "c": long_h.apply(d["v3"], pl)}
    return [{"vol": vol, "v2": v2, "v3": v3}], step


def _mk_compose_field(torch, ba, device, g):
    from batchaug_b200 import ops
    el = ba.Rand3DElastic(prob=1.0, sigma_range=(5, 7), magnitude_range=(50, 150))
    grid = el.sample_params(8, (8, 1, 160, 160, 160), device)["grid"]
    aff = ba.RandAffine(prob=1.0, rotate_range=0.5)
    theta = aff.sample_params(8, (8, 1, 160, 160, 160), device)["theta"]
    return [{"grid": grid}], lambda d: {"grid": ops.compose_field(d["grid"], theta)}


_C4_TEXT = ("config 4: Compose(lazy) rot90(0.5, max_k 3, axes (0,1)) -> axis flip(0.5) -> "
            "noise(vol, std 0.5) -> affine(0.5; rotate 0.785, shear 0.3, translate 5) -> "
            "ScaleIntensity(vol); vol bilinear + seg nearest, each 5x4x128^3 fp32 per GPU")
_ROT = "inputs rotate over distinct batches larger than the 126 MB L2, no flush"

WORKLOADS = {
    "config4": Workload("config4", _C4_TEXT, "f32", {"vol": (4, 4), "seg": (4, 4)}, 5,
                        (128, 128, 128), "inputs alternate over 2 distinct 671 MB batches "
                        "(> 126 MB L2), no flush", _build_config4, _ref_config4),
    "config2": Workload("config2", "config 2: RandAffine(prob=1, rotate_range=0.785, "
                        "shear_range=0.3, translate_range=5, scale_range=0.1), bilinear, border; "
                        "B=8 C=1 128^3 fp32 per GPU", "f32", {"vol": (1, 4)}, 8, (128, 128, 128),
                        "inputs rotate over 4 distinct 67 MB batches (268 MB > 126 MB L2), "
                        "no flush", _build_config2, _ref_config2),
    "config3": Workload("config3", "config 3 (prob=1 variant): noise -> contrast -> scale -> "
                        "shift -> ScaleIntensity, B=16 C=4 128^3 bf16", "bf16", {"v": (4, 2)},
                        16, (128, 128, 128), _ROT, _build_config3, _ref_config3),
    "config5": Workload("config5", "config 5 per-GPU shard: elastic + affine(0.1) -> bias(0.1) "
                        "-> smooth(0.1) -> ScaleIntensity, vol 8x2x160^3 bf16 + seg 8x2x160^3 "
                        "f32", "bf16+f32", {"vol": (2, 2), "seg": (2, 4)}, 8, (160, 160, 160),
                        "inputs larger than L2 (one 786 MB batch)", _build_config5(False)),
    "config5-fused": Workload("config5-fused", "config 5 per-GPU shard with the elastic∘affine "
                              "single resample (Compose(fuse_elastic=True), an extension)",
                              "bf16+f32", {"vol": (2, 2), "seg": (2, 4)}, 8, (160, 160, 160),
                              "inputs larger than L2", _build_config5(True)),
    "config5-smooth": Workload("config5-smooth", "RandGaussianSmooth(prob=1, sigma 0.5..1.5) on "
                               "config 5's vol shard (8x2x160^3 bf16)", "bf16", {"vol": (2, 2)},
                               8, (160, 160, 160), "input larger than L2",
                               _build_single(_mk_smooth)),
    "config5-elastic": Workload("config5-elastic", "Rand3DElastic.sample_params (sigma 5..7, "
                                "magnitude 50..150) for config 5's per-GPU shard: Philox field, "
                                "separable Gaussian (K=43), grid 8x160^3x3 fp32", "f32",
                                {"grid": (3, 2)}, 8, (160, 160, 160), "no input",
                                _build_single(_mk_elastic(160)), e2e=False),
    "elastic-draw": Workload("elastic-draw", "Rand3DElastic.sample_params on 8x160x160x158 (D not "
                             "a multiple of 4: the separate Philox draw kernel)", "f32",
                             {"grid": (3, 2)}, 8, (160, 160, 158), "no input",
                             _build_single(_mk_elastic(158)), e2e=False),
    "sharpen": Workload("sharpen", "RandGaussianSharpen(prob=1, sigma1 0.5..1, sigma2 0.5..sigma1,"
                        " alpha 10..30) on config 5's vol shard (8x2x160^3 bf16)", "bf16",
                        {"vol": (2, 2)}, 8, (160, 160, 160), "input larger than L2",
                        _build_single(_mk_sharpen)),
    "stats": Workload("stats", "std shift (nonzero std) -> relative Rician noise -> fixed-mean "
                      "scaling (channel-wise), prob 1, B=16 C=4 128^3 bf16", "bf16", {"v": (4, 2)},
                      16, (128, 128, 128), _ROT, _build_single(_mk_stats)),
    "lowres": Workload("lowres", "RandSimulateLowResolution(prob=1, zoom 0.5..1, nearest down, "
                       "trilinear up), B=8 C=1 128^3 fp32", "f32", {"vol": (1, 4)}, 8,
                       (128, 128, 128), _ROT, _build_single(_mk_lowres("nearest"))),
    "lowres-area": Workload("lowres-area", "RandSimulateLowResolution(prob=1, zoom 0.5..1, area "
                            "down, trilinear up), B=8 C=1 128^3 fp32", "f32", {"vol": (1, 4)}, 8,
                            (128, 128, 128), _ROT, _build_single(_mk_lowres("area"))),
    "flip": Workload("flip", "RandAxisFlip(prob=1) eager apply, B=8 C=1 128^3 fp32", "f32",
                     {"vol": (1, 4)}, 8, (128, 128, 128), _ROT,
                     _build_single(_mk_eager("RandAxisFlip"))),
    "flip-d260": Workload("flip-d260", "RandAxisFlip(prob=1) eager apply on rows longer than one "
                          "tensor-map box (D=260: the per-lane row-copy kernel), B=8 C=1 "
                          "128x128x260 fp32", "f32", {"vol": (1, 4)}, 8, (128, 128, 260), _ROT,
                          _build_single(_mk_eager("RandAxisFlip", shape=(8, 1, 128, 128, 260)))),
    "rot90": Workload("rot90", "RandRotate90(prob=1, max_k 3, axes (0,1)) eager apply, B=8 C=1 "
                      "128^3 fp32", "f32", {"vol": (1, 4)}, 8, (128, 128, 128), _ROT,
                      _build_single(_mk_eager("RandRotate90"))),
    "affine-reflection": Workload("affine-reflection", "config 2's RandAffine with reflection "
                                  "padding (the global-gather resample kernel), B=8 C=1 128^3 "
                                  "fp32", "f32", {"vol": (1, 4)}, 8, (128, 128, 128), _ROT,
                                  _build_single(_mk_eager(
                                      "RandAffine", rotate_range=0.785, shear_range=0.3,
                                      translate_range=5, scale_range=0.1,
                                      padding_mode="reflection"))),
    "fallbacks": Workload("fallbacks", "one launch of each fallback-only kernel: exact-mode "
                          "RandAffine (8x1x128^3), elastic field sigma 11..12 (2x96^3), smoothing "
                          "sigma 8.5..9 (2x1x96^3) and sigma 5 on an 800-long H line (1x1x800x64x48);"
                          " for ncu summaries, not a throughput line", "f32", {"vol": (1, 4)}, 8,
                          (128, 128, 128), "inputs larger than L2", _build_single(_mk_fallbacks),
                          e2e=False),
    "minmax": Workload("minmax", "per-(element, channel) min/max (ba_minmax) of 16x4x128^3 bf16",
                       "bf16", {"v": (4, 1)}, 16, (128, 128, 128), _ROT,
                       _build_single(_mk_minmax), e2e=False),
    "compose-field": Workload("compose-field", "elastic grid composed with the following affine "
                              "(ba_compose_field) on 8x160^3x3 fp32", "f32", {"grid": (3, 4)}, 8,
                              (160, 160, 160), "input larger than L2",
                              _build_single(_mk_compose_field), e2e=False),
}


# ---------------------------------------------------------------------------
# b200 arm
# ---------------------------------------------------------------------------

def _outputs(res) -> list:
    import torch
    if isinstance(res, dict):
        return [v for v in res.values() if isinstance(v, torch.Tensor)]
    return [res]


def run_b200(args, wl: Workload):
    import torch
    import torch.distributed as dist

    ws, rank, local = _dist()
    if ws != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    import batchaug_b200 as ba
    from batchaug_b200 import _lib as L
    from batchaug_b200 import _timing

    ba.set_shard(rank * wl.elements, ws * wl.elements)
    torch.manual_seed(1234)  # identical on every rank: same per-call seeds
    sets, step = wl.build(torch, ba, device, rank)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(sets[i % len(sets)])
    barrier()

    clocks = ClockSampler(local)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = L.kernel_launches()
    clocks.start()
    start.record(stream)
    for i in range(args.steps):
        step(sets[i % len(sets)])
    end.record(stream)
    barrier()
    clocks.stop()
    launches = L.kernel_launches() - launches0
    total_ms = start.elapsed_time(end)
    # attribution: the same steps again with every library call bracketed by
    # CUDA events (kept out of the timed loop above: recording events costs
    # host time between launches), each span behind a ~75 us device busy-wait
    # so it times the kernels, not the host's launch of them
    n_attr = max(1, min(args.steps, 20))
    with _timing.Recorder(lead_cycles=150_000) as rec:
        for i in range(n_attr):
            step(sets[i % len(sets)])
    barrier()
    per_entry = rec.summary()
    dom_name = max(per_entry, key=lambda k: per_entry[k]["ms_total"]) if per_entry else None
    dom = per_entry.get(dom_name, {"ms_mean": float("nan"), "bytes_mean": 0, "launches": 0})

    e2e = None
    if wl.e2e and sets and sets[0]:
        e2e = _e2e(torch, stream, device, sets, step, max(3, min(args.steps, args.e2e_steps)),
                   barrier)

    vals = torch.tensor([total_ms, dom["ms_mean"], e2e["ms"] if e2e else 0.0,
                         e2e["copy_ms"] if e2e else 0.0], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, dom_ms, e2e_ms, copy_ms = vals.tolist()

    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = dom["bytes_mean"] / (dom_ms * 1e-3) / 1e9 if dom_ms > 0 else None
        step_s = total_ms / args.steps * 1e-3
        line = {
            "metric": METRIC,
            "value": ws * wl.voxels * args.steps / (total_ms * 1e-3),
            "unit": UNIT,
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": wl.dtype,
            "data": "synthetic (seeded per rank; see config)",
            "config": wl.config(),
            "global_batch": ws * wl.elements,
            "parallelism": f"dp{ws} (batch-sharded, no collective on the data path)",
            "roofline": {"bound": "hbm", "entry_point": dom_name,
                         "launches_per_step": dom["launches"] / n_attr,
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": (achieved / peak) if achieved else None,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": DRAM_BYTES_PER_LAUNCH.get(wl.name),
                         "algorithmic_bytes_per_launch": dom["bytes_mean"],
                         "kernel_ms": dom_ms},
            "roofline_step": {"algorithmic_bytes_per_step": wl.alg_bytes,
                              "achieved": wl.alg_bytes / step_s / 1e9,
                              "frac": wl.alg_bytes / step_s / 1e9 / peak,
                              "scope": "whole step (all kernels and host work)"},
            "entry_points": {k: {"launches_per_step": v["launches"] / n_attr,
                                 "ms_mean": v["ms_mean"], "ms_per_step": v["ms_total"] / n_attr}
                             for k, v in per_entry.items()},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if e2e:
            line["e2e"] = {"value": ws * wl.voxels * e2e["steps"] / (e2e_ms * 1e-3), "unit": UNIT,
                           "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                           "steps": e2e["steps"],
                           "copies": "pinned host buffers, upload/download on their own "
                                     "streams, double-buffered",
                           "copy_bound": ws * wl.voxels * e2e["steps"] / (copy_ms * 1e-3),
                           "frac_of_copy_bound": copy_ms / e2e_ms}
        if ws == 1 and not args.no_cpu_baseline and wl.reference is not None:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def _e2e(torch, stream, device, sets, step, n_steps, barrier):
    """The step through the public API from pinned host memory: every step
    uploads its inputs (copy-in stream) and downloads its results
    (copy-out stream), double-buffered so both overlap neighbouring steps."""
    keys = list(sets[0].keys())
    hosts = [{k: sets[i % len(sets)][k].cpu().pin_memory() for k in keys} for i in range(2)]
    devs = [{k: torch.empty_like(sets[0][k]) for k in keys} for _ in range(2)]
    res0 = _outputs(step(sets[0]))
    host_outs = [[torch.empty(r.shape, dtype=r.dtype).pin_memory() for r in res0]
                 for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    barrier()
    h2d = sum(t.numel() * t.element_size() for t in hosts[0].values())
    d2h = sum(r.numel() * r.element_size() for r in res0)
    in_done = [torch.cuda.Event() for _ in range(n_steps)]
    used = [torch.cuda.Event() for _ in range(n_steps)]
    out_done = [torch.cuda.Event() for _ in range(n_steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(n_steps):
        buf = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(used[i - 2])
            for k in keys:
                devs[buf][k].copy_(hosts[buf][k], non_blocking=True)
            in_done[i].record(s_in)
        stream.wait_event(in_done[i])
        outs = _outputs(step(devs[buf]))
        used[i].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(used[i])
            if i >= 2:
                s_out.wait_event(out_done[i - 2])
            for o, h in zip(outs, host_outs[buf]):
                h.copy_(o, non_blocking=True)
                o.record_stream(s_out)
            out_done[i].record(s_out)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    # the same copies with no transform between them
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(n_steps):
        buf = i % 2
        with torch.cuda.stream(s_in):
            for k in keys:
                devs[buf][k].copy_(hosts[buf][k], non_blocking=True)
        with torch.cuda.stream(s_out):
            for o, h in zip(res0, host_outs[buf]):
                h.copy_(o, non_blocking=True)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    c1.record(stream)
    barrier()
    return {"ms": e2e_ms, "copy_ms": c0.elapsed_time(c1), "steps": n_steps, "h2d": h2d,
            "d2h": d2h}


# ---------------------------------------------------------------------------
# CPU legs: the oracle (restated reference path) on the host cores
# ---------------------------------------------------------------------------

def _ref_setup(wl: Workload):
    import oracle
    from oracle import pipelines as P
    oracle.build()
    n = P.cpu_threads()
    rng = np.random.default_rng(0)
    inputs, step = wl.reference(rng, n)
    return inputs, step, rng, n


def cpu_baseline(wl: Workload, seconds: float):
    """Whole steps of the oracle pipeline on the host cores, repeated for
    about ``seconds`` (at least two)."""
    inputs, step, rng, n = _ref_setup(wl)
    step(inputs, rng)  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        step(inputs, rng)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": wl.voxels / med, "unit": UNIT, "cores": n, "kind": "port",
            "sample": f"full {wl.name} steps on one GPU's share ({wl.elements} elements), "
                      f"C oracle restating the reference PyTorch path, {len(times)} "
                      f"repetitions, median {med * 1e3:.1f} ms"}


def run_reference(args, wl: Workload):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    if wl.reference is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"no CPU restatement of workload {wl.name}"}), flush=True)
        return
    inputs, step, rng, n = _ref_setup(wl)
    steps = max(1, args.steps)
    for _ in range(args.warmup):
        step(inputs, rng)
    t0 = time.perf_counter()
    for _ in range(steps):
        step(inputs, rng)
    dt = time.perf_counter() - t0
    value = wl.voxels * steps / dt
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": ws,
        "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded per rank; see config)",
        "config": wl.config(),
        "global_batch": wl.elements, "parallelism": "host CPU, one process",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": n, "kind": "port",
                         "sample": f"{steps} full {wl.name} steps ({wl.elements} elements), C "
                                   f"oracle restating the reference PyTorch path, {n} threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="elements per GPU (default: the workload's own; smaller batches are "
                         "for profiling captures and are reported in config)")
    ap.add_argument("--workload", default=HEADLINE, choices=sorted(WORKLOADS),
                    help=f"{HEADLINE} is the headline; the others time one whole step of that "
                         "configuration or kernel (for profiling and per-config numbers)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.batch:
        wl.elements = args.batch
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_b200(args, wl)


if __name__ == "__main__":
    main()
