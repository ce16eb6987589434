"""Benchmark: augmented voxels/s of batchaug's hot path on B200, and the
fraction of the HBM roofline its dominant kernel reaches.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

Workload (config 2 of the reference's headline set, per GPU):
RandAffine(prob=1, rotate_range=0.785, shear_range=0.3, translate_range=5,
scale_range=0.1), bilinear, border padding, on B=8, C=1, 128^3 fp32; the
volume is uniform [0,1) noise smoothed with sigma=2.  A step is one call of
the transform on the batch — sample_params (host Philox, one pinned upload)
plus the fused resample (one ba_resample3d launch).  Ranks shard the batch
dimension (weak scaling: 8 elements per rank, global element offset
rank*8), with no collective on the data path; NCCL is used only for the
barrier and the max-over-ranks of the timings.

Timing: W untimed warm-up steps, then K steps between barrier +
cuda.synchronize, timed with CUDA events on the launching stream; inputs
rotate over 4 distinct batches (4 x 67 MB > 126 MB L2), so every step reads
its input from HBM.  ``value`` = voxels of all ranks / max-over-ranks time.
``e2e`` is the same step through the public API from pinned host memory:
H2D of the input, the transform, D2H of the augmented volume, every step,
with the two copies on their own streams (double-buffered) so they overlap
the neighbouring steps' work.  ``e2e.copy_bound`` times the same copies with
no transform between them: the host link's concurrent rate, which bounds
``e2e`` (``frac_of_copy_bound`` is e2e over that bound).

--impl reference times the reference algorithm on the host CPU cores (the C
oracle, a restatement of the reference's PyTorch path; the Python reference
cannot be shipped to the GPU host) on the same workload.
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
B, C, S = 8, 1, 128
VOXELS = B * C * S * S * S
BYTES_PER_VOXEL = 4 + 4  # fp32 read once + fp32 written once
CONFIG_TEXT = ("config 2: RandAffine(prob=1, rotate_range=0.785, shear_range=0.3, "
               "translate_range=5, scale_range=0.1), bilinear, border; B=8 C=1 128^3 fp32 per GPU")
AFFINE_KW = dict(prob=1.0, rotate_range=0.785, shear_range=0.3, translate_range=5,
                 scale_range=0.1, mode="bilinear", padding_mode="border")
N_INPUTS = 4


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_per_launch():
    """DRAM bytes (read + write) per launch of the resample kernel from the
    committed ncu summary (profiles/resample3d_config2.md), or None."""
    import re
    p = os.path.join(ROOT, "profiles", "resample3d_config2.md")
    if os.path.exists(p):
        with open(p) as f:
            m = re.search(r"^dram_bytes_per_launch:\s*(\d+)", f.read(), re.M)
        if m:
            return int(m.group(1))
    return None


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


def _make_inputs(torch, ba, device, rank):
    from batchaug_b200 import ops
    xs = []
    g = torch.Generator(device=device)
    for i in range(N_INPUTS):
        g.manual_seed(1000 * rank + i)
        u = torch.rand(B, C, S, S, S, device=device, generator=g)
        K = ops.gauss_taps_len(2.0, 4.0)
        taps = ops.gauss_taps(torch.full((B,), 2.0, device=device), K)
        xs.append(ops.smooth3d(u, taps, taps, taps))
    torch.cuda.synchronize()
    return xs


def run_b200(args):
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
    from batchaug_b200 import ops

    ba.set_shard(rank * B, ws * B)
    torch.manual_seed(1234)  # identical on every rank: same per-call seeds
    xs = _make_inputs(torch, ba, device, rank)
    t = ba.RandAffine(**AFFINE_KW)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        t(xs[i % N_INPUTS])
    barrier()

    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = L.kernel_launches()
    clocks.start()
    start.record(stream)
    for i in range(args.steps):
        x = xs[i % N_INPUTS]
        params = t.sample_params(B, x.shape, device)
        ev[i][0].record(stream)
        t.apply(x, params)
        ev[i][1].record(stream)
    end.record(stream)
    barrier()
    clocks.stop()
    launches = L.kernel_launches() - launches0
    total_ms = start.elapsed_time(end)
    kern_ms = [a.elapsed_time(b) for a, b in ev]

    # e2e: public API from pinned host memory, D2H of the augmented batch.
    # Double-buffered: step i's upload (copy-in stream) and step i-1's
    # download (copy-out stream) overlap step i's transform, as a loader
    # feeding a training loop would run them; every step still moves its own
    # input in and its own result out inside the timed region.
    hosts = [xs[i].cpu().pin_memory() for i in range(2)]
    host_outs = [torch.empty_like(hosts[0]).pin_memory() for _ in range(2)]
    x_devs = [torch.empty_like(xs[0]) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    e2e_steps = max(3, min(args.steps, args.e2e_steps))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    in_done = [torch.cuda.Event() for _ in range(e2e_steps)]
    used = [torch.cuda.Event() for _ in range(e2e_steps)]      # transform read x_devs[i % 2]
    out_done = [torch.cuda.Event() for _ in range(e2e_steps)]  # download of step i finished
    param_bytes = 0
    e0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(e2e_steps):
        buf = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(used[i - 2])
            x_devs[buf].copy_(hosts[buf], non_blocking=True)
            in_done[i].record(s_in)
        # the parameters (their small upload included) before the wait on the
        # volume's upload, so they do not queue behind the next volume's copy
        params = t.sample_params(B, x_devs[buf].shape, device)
        param_bytes = sum(v.numel() * v.element_size() for k, v in params.items()
                          if isinstance(v, torch.Tensor))
        stream.wait_event(in_done[i])
        out = t.apply(x_devs[buf], params)
        used[i].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(used[i])
            if i >= 2:
                s_out.wait_event(out_done[i - 2])
            host_outs[buf].copy_(out, non_blocking=True)
            out.record_stream(s_out)
            out_done[i].record(s_out)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # The e2e roofline: the same double-buffered uploads and downloads with
    # no transform between them (the host link's concurrent copy rate).
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(e2e_steps):
        buf = i % 2
        with torch.cuda.stream(s_in):
            x_devs[buf].copy_(hosts[buf], non_blocking=True)
        with torch.cuda.stream(s_out):
            host_outs[buf].copy_(x_devs[1 - buf], non_blocking=True)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    c1.record(stream)
    barrier()
    copy_ms = c0.elapsed_time(c1)

    # max over ranks
    vals = torch.tensor([total_ms, statistics.mean(kern_ms), e2e_ms, copy_ms], device=device,
                        dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, kern_mean_ms, e2e_ms, copy_ms = vals.tolist()

    if rank == 0:
        peak, peak_kind = _peaks()
        alg_bytes = VOXELS * BYTES_PER_VOXEL
        achieved = alg_bytes / (kern_mean_ms * 1e-3) / 1e9
        traffic = _traffic_per_launch()
        line = {
            "metric": METRIC,
            "value": ws * VOXELS * args.steps / (total_ms * 1e-3),
            "unit": UNIT,
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (uniform noise smoothed with sigma=2, seeded per rank)",
            "config": {"workload": CONFIG_TEXT, "global_batch": ws * B, "elements_per_gpu": B,
                       "volume": [C, S, S, S], "l2": "inputs rotate over 4 distinct 67 MB "
                       "batches (268 MB > 126 MB L2), no flush",
                       "parallelism": f"dp{ws} (batch-sharded, no collective on the data path)"},
            "e2e": {"value": ws * VOXELS * e2e_steps / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": VOXELS * 4 + param_bytes,
                    "d2h_bytes_per_step": VOXELS * 4, "steps": e2e_steps,
                    "copies": "pinned host buffers, upload/download on their own streams, "
                              "double-buffered",
                    "copy_bound": ws * VOXELS * e2e_steps / (copy_ms * 1e-3),
                    "frac_of_copy_bound": copy_ms / e2e_ms},
            "roofline": {"bound": "hbm", "kernel": "resample3d_staged_kernel",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": traffic, "algorithmic_bytes_per_launch": alg_bytes,
                         "kernel_ms": kern_mean_ms},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if ws == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def _oracle_step(oracle, t, xs_np, i, nthreads):
    host = t.sample_host(B, xs_np[0].shape)
    from batchaug_b200.geometric import monai_affine_to_theta
    theta = monai_affine_to_theta(host["affine"], xs_np[0].shape[2:])
    return oracle.resample3d(xs_np[i % len(xs_np)], theta=theta, padding="border",
                             mode="bilinear", mask=host["mask"], nthreads=nthreads)


def _cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(seconds: float):
    """The oracle (restated reference path) on the host cores, full config-2
    steps repeated for about `seconds`."""
    import oracle
    import batchaug_b200 as ba
    oracle.build()
    rng = np.random.default_rng(0)
    xs_np = [rng.random((B, C, S, S, S), dtype=np.float32)]
    t = ba.RandAffine(**AFFINE_KW)
    n = _cpu_threads()
    _oracle_step(oracle, t, xs_np, 0, n)  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        _oracle_step(oracle, t, xs_np, 0, n)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": VOXELS / med, "unit": UNIT, "cores": n, "kind": "port",
            "sample": f"full config-2 step (8x1x128^3 fp32, params + resample), "
                      f"{len(times)} repetitions, median {med * 1e3:.1f} ms"}


def run_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    import oracle
    import batchaug_b200 as ba  # noqa: F401  (host parameter sampler)
    oracle.build()
    rng = np.random.default_rng(0)
    xs_np = [rng.random((B, C, S, S, S), dtype=np.float32) for _ in range(2)]
    t = ba.RandAffine(**AFFINE_KW)
    n = _cpu_threads()
    steps = max(1, args.steps)
    for i in range(args.warmup):
        _oracle_step(oracle, t, xs_np, i, n)
    t0 = time.perf_counter()
    for i in range(steps):
        _oracle_step(oracle, t, xs_np, i, n)
    dt = time.perf_counter() - t0
    value = VOXELS * steps / dt
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": ws,
        "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (uniform noise)",
        "config": {"workload": CONFIG_TEXT, "global_batch": B, "parallelism": "host CPU"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": n, "kind": "port",
                         "sample": f"{steps} full config-2 steps (8x1x128^3), C oracle "
                                   f"restating the reference PyTorch path, {n} threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _secondary(name, torch, ba, device, rank):
    """Other configurations of the reference's benchmark set, for profiling
    and per-config numbers: returns (text, step(i), voxels, bytes) where bytes
    are the algorithmic bytes of a step (every key read once, written once)."""
    g = torch.Generator(device=device)
    g.manual_seed(7 + rank)
    if name == "config3":
        xs = [(0.5 + 0.2 * torch.randn(16, 4, 128, 128, 128, device=device, generator=g))
              .clamp(0, 1).bfloat16() for _ in range(2)]
        c = ba.Compose([ba.RandGaussianNoised(["v"], prob=1.0, std=(0.1, 0.5)),
                        ba.RandAdjustContrastd(["v"], prob=1.0, gamma=(0.5, 2.0)),
                        ba.RandScaleIntensityd(["v"], prob=1.0, factors=0.2),
                        ba.RandShiftIntensityd(["v"], prob=1.0, offsets=0.1),
                        ba.ScaleIntensityd(["v"], minv=0.0, maxv=1.0)], lazy=True)
        n = xs[0].numel()
        return ("config 3 (prob=1 variant): noise -> contrast -> scale -> shift -> "
                "ScaleIntensity, B=16 C=4 128^3 bf16", lambda i: c({"v": xs[i % 2]}), n, n * 4)
    if name == "config4":
        vols = [torch.randn(5, 4, 128, 128, 128, device=device, generator=g) for _ in range(2)]
        segs = [(torch.rand(5, 1, 128, 128, 128, device=device, generator=g) > 0.5).float()
                for _ in range(2)]
        c = ba.Compose([ba.RandRotate90d(["vol", "seg"], prob=0.5, max_k=3),
                        ba.RandAxisFlipd(["vol", "seg"], prob=0.5),
                        ba.RandGaussianNoised(["vol"], std=0.5),
                        ba.RandAffined(["vol", "seg"], prob=0.5, rotate_range=0.785,
                                       shear_range=0.3, translate_range=5),
                        ba.ScaleIntensityd(["vol"])], lazy=True,
                       mode={"vol": "bilinear", "seg": "nearest"})
        n = vols[0].numel() + segs[0].numel()
        return ("config 4: rot90, flip, noise, affine, ScaleIntensity on vol (5x4x128^3 f32) "
                "+ seg (5x1x128^3 f32)", lambda i: c({"vol": vols[i % 2], "seg": segs[i % 2]}),
                n, n * 8)
    if name == "config5":
        vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
        seg = torch.randint(0, 8, (8, 2, 160, 160, 160), device=device, generator=g).float()
        c = ba.Compose([ba.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5, 7),
                                          magnitude_range=(50, 150),
                                          mode={"vol": "bilinear", "seg": "nearest"}),
                        ba.RandAffined(["vol", "seg"], prob=0.1, rotate_range=0.5),
                        ba.RandBiasFieldd(["vol"], prob=0.1),
                        ba.RandGaussianSmoothd(["vol"], prob=0.1, sigma_x=(0.5, 1.5),
                                               sigma_y=(0.5, 1.5), sigma_z=(0.5, 1.5)),
                        ba.ScaleIntensityd(["vol"])], lazy=True,
                       mode={"vol": "bilinear", "seg": "nearest"})
        n = vol.numel() + seg.numel()
        return ("config 5 per-GPU shard: elastic + affine(0.1) -> bias(0.1) -> smooth(0.1) -> "
                "ScaleIntensity, vol 8x2x160^3 bf16 + seg 8x2x160^3 f32",
                lambda i: c({"vol": vol, "seg": seg}), n, vol.numel() * 4 + seg.numel() * 8)
    if name == "config5-fused":
        vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
        seg = torch.randint(0, 8, (8, 2, 160, 160, 160), device=device, generator=g).float()
        c = ba.Compose([ba.Rand3DElasticd(["vol", "seg"], prob=1.0, sigma_range=(5, 7),
                                          magnitude_range=(50, 150),
                                          mode={"vol": "bilinear", "seg": "nearest"}),
                        ba.RandAffined(["vol", "seg"], prob=0.1, rotate_range=0.5),
                        ba.RandBiasFieldd(["vol"], prob=0.1),
                        ba.RandGaussianSmoothd(["vol"], prob=0.1, sigma_x=(0.5, 1.5),
                                               sigma_y=(0.5, 1.5), sigma_z=(0.5, 1.5)),
                        ba.ScaleIntensityd(["vol"])], lazy=True,
                       mode={"vol": "bilinear", "seg": "nearest"}, fuse_elastic=True)
        n = vol.numel() + seg.numel()
        return ("config 5 per-GPU shard with the elastic∘affine single resample "
                "(Compose(fuse_elastic=True), an extension), vol 8x2x160^3 bf16 + seg f32",
                lambda i: c({"vol": vol, "seg": seg}), n, vol.numel() * 4 + seg.numel() * 8)
    if name == "config5-smooth":
        vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
        sm = ba.RandGaussianSmooth(prob=1.0, sigma_x=(0.5, 1.5), sigma_y=(0.5, 1.5),
                                   sigma_z=(0.5, 1.5))
        p = sm.sample_params(8, vol.shape, device)
        n = vol.numel()
        return ("RandGaussianSmooth(prob=1, sigma 0.5..1.5) on config 5's vol shard "
                "(8x2x160^3 bf16)", lambda i: sm.apply(vol, p), n, n * 4)
    if name == "stats":
        xs = [(0.5 + 0.2 * torch.randn(16, 4, 128, 128, 128, device=device, generator=g))
              .clamp(0, 1).bfloat16() for _ in range(2)]
        c = ba.Compose([ba.RandStdShiftIntensityd(["v"], prob=1.0, nonzero=True),
                        ba.RandRicianNoised(["v"], prob=1.0, std=0.1, relative=True),
                        ba.RandScaleIntensityFixedMeand(["v"], prob=1.0, channel_wise=True)],
                       lazy=True)
        n = xs[0].numel()
        return ("std shift (nonzero std) -> relative Rician noise -> fixed-mean scaling "
                "(channel-wise), prob 1, B=16 C=4 128^3 bf16", lambda i: c({"v": xs[i % 2]}),
                n, n * 4)
    if name == "sharpen":
        vol = torch.rand(8, 2, 160, 160, 160, device=device, generator=g).bfloat16()
        sh = ba.RandGaussianSharpen(prob=1.0)
        p = sh.sample_params(8, vol.shape, device)
        n = vol.numel()
        return ("RandGaussianSharpen(prob=1, sigma1 0.5..1, sigma2 0.5..sigma1, alpha 10..30) "
                "on config 5's vol shard (8x2x160^3 bf16)", lambda i: sh.apply(vol, p), n, n * 4)
    if name == "lowres":
        xs = [torch.rand(8, 1, 128, 128, 128, device=device, generator=g) for _ in range(4)]
        lr = ba.RandSimulateLowResolution(prob=1.0, zoom_range=(0.5, 1.0))
        n = xs[0].numel()
        return ("RandSimulateLowResolution(prob=1, zoom 0.5..1, nearest down, trilinear up), "
                "B=8 C=1 128^3 fp32", lambda i: lr(xs[i % 4]), n, n * 8)
    if name == "config5-elastic":
        el = ba.Rand3DElastic(prob=1.0, sigma_range=(5, 7), magnitude_range=(50, 150))
        shape = (8, 2, 160, 160, 160)
        n = 8 * 160 ** 3
        return ("Rand3DElastic.sample_params (sigma 5..7, magnitude 50..150) for config 5's "
                "per-GPU shard: Philox field, separable Gaussian (K=43), grid 8x160^3x3 fp32",
                lambda i: el.sample_params(8, shape, device), n, n * 12)
    raise SystemExit(f"unknown workload {name}")


def run_secondary(args):
    import torch
    import torch.distributed as dist

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    import batchaug_b200 as ba
    from batchaug_b200 import _lib as L

    torch.manual_seed(1234)
    text, step, voxels, alg_bytes = _secondary(args.workload, torch, ba, device, rank)
    stream = torch.cuda.current_stream(device)
    for i in range(args.warmup):
        step(i)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = L.kernel_launches()
    clocks.start()
    start.record(stream)
    for i in range(args.steps):
        step(i)
    end.record(stream)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.stop()
    ms = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    total_ms = float(ms.item())
    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = alg_bytes / (total_ms / args.steps * 1e-3) / 1e9
        print(json.dumps({
            "metric": METRIC, "value": ws * voxels * args.steps / (total_ms * 1e-3), "unit": UNIT,
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "mixed", "data": "synthetic",
            "config": {"workload": text, "l2": "inputs larger than L2 or rotating"},
            "roofline": {"bound": "hbm", "scope": "whole step (all kernels and host work)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_step": alg_bytes},
            "gpu_launches": int(L.kernel_launches() - launches0),
            "clocks": clocks.summary()}), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="config2",
                    choices=["config2", "config3", "config4", "config5", "config5-smooth",
                             "config5-elastic", "config5-fused", "stats", "sharpen", "lowres"],
                    help="config2 is the headline; the others time one whole step of that "
                         "configuration (for profiling and per-config numbers)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "config2":
        run_secondary(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
