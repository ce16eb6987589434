"""Per-entry-point device timing: CUDA events around each C-ABI compute call.

Off by default (one global read per call).  Inside ``with Recorder() as r:``
every ``ops`` entry point records an event pair on the stream it enqueues on,
with the algorithmic bytes of that call (every key's input read once plus its
output written once), so a caller can attribute device time to the library's
kernels without a profiler::

    with Recorder() as rec:
        for _ in range(steps):
            pipeline(batch)
    per_entry = rec.summary()   # {name: {"launches", "ms_total", "ms_mean", "bytes"}}

``lead_cycles`` > 0 puts a GPU busy-wait of that many clock cycles in front
of every span's start event, so the host has enqueued the call's kernels
before the device reaches the start event: the span then measures the
kernels alone, not the host's launch latency (which a host-bound step would
otherwise add to it).
"""
from __future__ import annotations

import torch

_active = None


class Recorder:
    def __init__(self, lead_cycles: int = 0):
        self.spans = []  # (name, algorithmic bytes, start event, end event)
        self.lead_cycles = int(lead_cycles)

    def __enter__(self):
        global _active
        self._prev, _active = _active, self
        return self

    def __exit__(self, *exc):
        global _active
        _active = self._prev
        return False

    def summary(self) -> dict:
        """Per entry point: launches, total and mean device ms, bytes per
        launch (the mean).  Synchronises on the recorded events."""
        out: dict[str, dict] = {}
        for name, nbytes, e0, e1 in self.spans:
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            s = out.setdefault(name, {"launches": 0, "ms_total": 0.0, "bytes_total": 0})
            s["launches"] += 1
            s["ms_total"] += ms
            s["bytes_total"] += int(nbytes)
        for s in out.values():
            s["ms_mean"] = s["ms_total"] / s["launches"]
            s["bytes_mean"] = s["bytes_total"] / s["launches"]
        return out


def begin(name: str, nbytes: int, device):
    """Start a span (None when no recorder is active)."""
    rec = _active
    if rec is None:
        return None
    stream = torch.cuda.current_stream(device)
    if rec.lead_cycles > 0:
        with torch.cuda.device(device):
            torch.cuda._sleep(rec.lead_cycles)
    e0 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    return rec, name, nbytes, e0, stream


def end(token) -> None:
    if token is None:
        return
    rec, name, nbytes, e0, stream = token
    e1 = torch.cuda.Event(enable_timing=True)
    e1.record(stream)
    rec.spans.append((name, nbytes, e0, e1))
