"""Compose with lazy geometric fusion (batchaug/compose.py:9-164).

Same constructor and semantics as the reference:

* eager (``lazy=False``): transforms run in order;
* lazy: consecutive geometric transforms (dict transforms whose
  ``.transform`` has ``to_affine``) accumulate one MONAI affine per key by
  right-multiplication and OR their masks (compose.py:139-151); the pending
  group is materialised before every non-geometric transform and at the end
  (compose.py:153-162), skipping keys whose mask is all false (:84-86).

B200 execution:

* the affines and masks are accumulated on the host from the transforms'
  host parameters, so materialising needs no device read (the reference's
  ``mask.any()`` is a device sync);
* keys that share an accumulated affine and spatial shape are resampled by
  one ``ba_resample3d`` launch (one coordinate computation for all of them,
  per-key mode, padding and dtype);
* a run of consecutive intensity transforms (noise, contrast, scale, shift,
  bias field, ScaleIntensity) becomes one ``ba_intensity_chain`` per key —
  the same ops in the same order as applying them one by one, so results are
  unchanged, in fewer HBM passes.  This applies in eager mode too.

* a key whose tensor the pipeline itself created (its storage shared with
  no input tensor and no other key) is updated in place when a transform
  selects under a third of the elements: the selected elements are gathered,
  transformed and scattered back, and the others are not touched (the
  reference's torch.where copies them).  This covers the geometric materialisation and
  the transforms whose parameters are all per element (Gaussian smoothing
  and sharpening, bias field); a transform that selects no element leaves
  such a key as it is.  Results are unchanged; input tensors are never
  written.

Extension (``fuse_elastic=True``, lazy mode only; off by default, which keeps
the reference's order): a Rand3DElasticd followed by geometric transforms is
resampled once instead of twice.  Pending affines before the elastic
transform are materialised first, as the reference does; the elastic grid is
then held, the affines after it accumulate as usual, and at the next
materialisation ``ba_compose_field`` folds them into the grid
(I(field(A(p))), the displacement extended by clamping) and one
``ba_resample3d`` samples each key with the elastic transform's per-key mode
and padding.  The result differs from the two resamples by the second
interpolation they perform (less blur), not by the geometry.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib as L
from . import ops
from .base import to_device
from .intensity import ScaleIntensity, _FusibleIntensity


def compose_affines(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Batched (B,4,4) fp32 product a @ b rounded as the reference's
    ``per_key_affines[key] @ affine`` (compose.py:145-151) is on torch's CPU
    path: for each entry the four products, each rounded to fp32, summed
    left to right with a rounding after every addition (no fused
    multiply-add).  numpy's matmul rounds differently."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    acc = a[:, :, 0, None] * b[:, None, 0, :]
    for k in range(1, 4):
        acc = acc + a[:, :, k, None] * b[:, None, k, :]
    return acc.astype(np.float32)


def _slice_params(params: dict, b: int, n: int) -> dict:
    """``params`` for elements b .. b+n-1 as a view of the batch: every
    tensor or array whose first dimension is the batch is sliced, the
    element offset of in-kernel random streams (keyed on the global element
    index) advances by b, everything else is kept."""
    B = len(params["_host"]["mask"])

    def cut(v):
        if isinstance(v, (torch.Tensor, np.ndarray)) and v.ndim >= 1 and v.shape[0] == B:
            return v[b:b + n]
        return v

    out = {k: cut(v) for k, v in params.items() if k != "_host"}
    out["_host"] = {k: cut(v) for k, v in params["_host"].items()}
    if "elem_offset" in params:
        out["elem_offset"] = params["elem_offset"] + b
    return out


class Compose:
    def __init__(self, transforms: list, lazy: bool = False, mode="bilinear",
                 padding_mode="zeros", fuse_elastic: bool = False):
        self.transforms = transforms
        self.lazy = lazy
        self.fuse_elastic = fuse_elastic
        self._mode = mode
        self._padding_mode = padding_mode

    # -- helpers (compose.py:51-65) -----------------------------------------
    @staticmethod
    def _is_geometric(t) -> bool:
        inner = getattr(t, "transform", None)
        return inner is not None and hasattr(inner, "to_affine")

    @staticmethod
    def _is_elastic(t) -> bool:
        from .geometric import Rand3DElastic
        return isinstance(getattr(t, "transform", None), Rand3DElastic) and hasattr(t, "_mode")

    @staticmethod
    def _is_fusible(t) -> bool:
        inner = getattr(t, "transform", None)
        return isinstance(inner, _FusibleIntensity) and hasattr(t, "keys")

    @staticmethod
    def _stats_keys(t) -> set:
        """Keys whose materialisation can hand their min/max straight to the
        transform ``t`` that follows it: a ScaleIntensity(d) that rescales
        with per-(element, channel) statistics."""
        inner = getattr(t, "transform", None)
        if isinstance(inner, ScaleIntensity) and inner.takes_stats() and hasattr(t, "keys"):
            return set(t.keys)
        return set()

    def _get_mode(self, key: str) -> str:
        if isinstance(self._mode, dict):
            return self._mode.get(key, "bilinear")
        return self._mode

    def _get_padding_mode(self, key: str) -> str:
        if isinstance(self._padding_mode, dict):
            return self._padding_mode.get(key, "zeros")
        return self._padding_mode

    # -- pipeline-owned keys, updated in place on the selected elements -----
    @staticmethod
    def _storage(x) -> int:
        return x.untyped_storage().data_ptr() if isinstance(x, torch.Tensor) else 0

    def _owned(self, d: dict, keys, inputs: set) -> bool:
        """True when every key's tensor was created by the pipeline: its
        storage is shared with no input tensor and no other key of ``d``."""
        counts: dict[int, int] = {}
        for v in d.values():
            p = self._storage(v)
            counts[p] = counts.get(p, 0) + 1
        for k in keys:
            p = self._storage(d[k])
            if p == 0 or p in inputs or counts[p] != 1:
                return False
        return True

    @staticmethod
    def _subset_index(mask: np.ndarray, device):
        idx = np.flatnonzero(mask)
        # pinned, non-blocking: a pageable upload would synchronise the stream
        return idx, to_device(idx.astype(np.int64), device)

    @staticmethod
    def _runs(idx: np.ndarray):
        """(first element, count) of each run of consecutive indices."""
        runs, i = [], 0
        while i < len(idx):
            j = i
            while j + 1 < len(idx) and idx[j + 1] == idx[j] + 1:
                j += 1
            runs.append((int(idx[i]), j - i + 1))
            i = j + 1
        return runs

    @classmethod
    def _gather(cls, x: torch.Tensor, idx: np.ndarray) -> torch.Tensor:
        """x[idx] by one device copy per run of consecutive elements (an
        element is one contiguous block)."""
        out = torch.empty((len(idx),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        j = 0
        for b, n in cls._runs(idx):
            out[j:j + n].copy_(x[b:b + n])
            j += n
        return out

    @classmethod
    def _scatter(cls, x: torch.Tensor, idx: np.ndarray, y: torch.Tensor) -> None:
        """x[idx] = y in place, one device copy per run."""
        j = 0
        for b, n in cls._runs(idx):
            x[b:b + n].copy_(y[j:j + n])
            j += n

    @staticmethod
    def _sparse(mask: np.ndarray) -> bool:
        """Selected elements few enough that gathering them and scattering the
        results back (two copies of the selection) moves less than copying
        the unselected ones: under a third of the batch."""
        return 3 * int(np.count_nonzero(mask)) < len(mask)

    def _apply_dict(self, d: dict, t, inputs: set, injected: dict | None = None) -> dict:
        """One non-fused dict transform; owned keys of a subsettable
        transform are updated on the selected elements only."""
        inner = getattr(t, "transform", None)
        keys = [k for k in getattr(t, "keys", ()) if k in d]
        if (inputs is None or not getattr(inner, "_subsettable", False) or not keys
                or t.keys[0] not in d or not self._owned(d, keys, inputs)):
            return t(d) if injected is None else t(d, params=injected)
        d = dict(d)
        first = d[t.keys[0]]
        if injected is None:
            params = inner.sample_params(first.shape[0], first.shape, first.device)
        else:
            params = inner.adopt_params(injected)
        mask = np.asarray(params["_host"]["mask"], bool)
        if mask.any() and not self._sparse(mask):
            for k in keys:
                d[k] = inner.apply(d[k], params)
        elif mask.any():
            idx, it = self._subset_index(mask, first.device)
            sub = inner.subset_params(params, idx, it)
            for k in keys:
                self._scatter(d[k], idx, inner.apply(self._gather(d[k], idx), sub))
        return d

    # -- intensity fusion ---------------------------------------------------
    def _run_intensity(self, d: dict, run: list, inputs: set | None = None,
                       injected: list | None = None, stats: dict | None = None) -> dict:
        """Apply consecutive fusible dict transforms as one chain per key.
        ``stats`` (key -> the min/max the preceding materialisation folded)
        serves a ScaleIntensity that opens the run on the full batch."""
        d = dict(d)
        sampled = []
        for i, t in enumerate(run):
            first = d.get(t.keys[0])
            if first is None:  # the reference would raise KeyError here too
                raise KeyError(t.keys[0])
            p = injected[i] if injected is not None else None
            if p is None:
                p = t.transform.chain_params(first.shape[0], first.shape, first.device)
            else:
                p = t.transform.adopt_params(p)
            sampled.append((t, p))
        keys = list(dict.fromkeys(k for t in run for k in t.keys if k in d))
        owned = inputs is not None and bool(keys) and self._owned(d, keys, inputs)
        if owned:
            # pipeline-owned keys: the chain runs in place on the runs of
            # elements some op selects; an element no op selects is left as
            # it is (every op of a chain is the identity on an unselected
            # element, up to the sign of a zero that adds noise * 0)
            sel = np.zeros(len(sampled[0][1]["_host"]["mask"]), bool)
            for _, p in sampled:
                sel |= np.asarray(p["_host"]["mask"], bool)
            if not sel.all():
                for b, n in self._runs(np.flatnonzero(sel)):
                    sub = [(t, _slice_params(p, b, n)) for t, p in sampled]
                    self._chain_keys({k: d[k][b:b + n] for k in keys}, sub, inplace=True)
                return d
        out = self._chain_keys({k: d[k] for k in keys}, sampled, inplace=owned, stats=stats)
        d.update(out)
        return d

    @staticmethod
    def _chain_keys(views: dict, sampled: list, inplace: bool,
                    stats: dict | None = None) -> dict:
        """One ba_intensity_chain per key over the ops that list it; an op
        that selects no element is the identity and is left out.  A key's
        first op takes ``stats[key]`` when it is a ScaleIntensity that can
        (the statistics describe the chain's input)."""
        per_key: dict[str, list] = {}
        for t, params in sampled:
            if not np.asarray(params["_host"]["mask"]).any():
                continue
            for key in t.keys:
                if key in views:
                    chain = per_key.setdefault(key, [])
                    st = stats.get(key) if stats and not chain else None
                    if st is not None and isinstance(t.transform, ScaleIntensity):
                        chain.append(t.transform.chain_op(params, views[key], stats=st))
                    else:
                        chain.append(t.transform.chain_op(params, views[key]))
        out = {}
        for key, chain in per_key.items():
            x = views[key]
            for i in range(0, len(chain), L.BA_MAX_OPS):
                x = ops.intensity_chain(x, chain[i:i + L.BA_MAX_OPS], inplace=inplace)
            out[key] = x
        return out

    def _apply_rest(self, d: dict, transforms: list, inputs: set | None = None,
                    injected: list | None = None) -> dict:
        """Eager pass over ``transforms`` with intensity runs fused."""
        injected = injected if injected is not None else [None] * len(transforms)
        i = 0
        while i < len(transforms):
            t = transforms[i]
            if self._is_fusible(t):
                j = i
                while j < len(transforms) and self._is_fusible(transforms[j]):
                    j += 1
                d = self._run_intensity(d, transforms[i:j], inputs, injected[i:j])
                i = j
            else:
                d = self._apply_dict(d, t, inputs, injected[i])
                i += 1
        return d

    # -- held elastic field composed with the affines after it (extension) ---
    def _materialize_fields(self, d: dict, pending: dict, fields: dict) -> dict:
        from .geometric import monai_affine_to_theta
        groups: dict[tuple, tuple] = {}
        for key, (fstate, _, _) in fields.items():
            if key in d:
                astate = pending.get(key)
                t = d[key]
                gk = (id(fstate), id(astate), t.shape[0], tuple(t.shape[2:]), t.device)
                groups.setdefault(gk, (fstate, astate, []))[2].append(key)
        for fstate, astate, keys in groups.values():
            grid, mask_f = fstate
            B = grid.shape[0]
            spatial = tuple(d[keys[0]].shape[2:])
            if astate is not None:
                affine, mask_a = astate
                theta = monai_affine_to_theta(affine, spatial)
            else:
                mask_a = np.zeros(B, bool)
                theta = np.tile(np.eye(4, dtype=np.float32), (B, 1, 1))
            mask = mask_f | mask_a
            if not mask.any():
                continue
            g = ops.compose_field(grid, theta, mask_field=mask_f, mask_affine=mask_a)
            for i in range(0, len(keys), L.BA_MAX_KEYS):
                chunk = keys[i:i + L.BA_MAX_KEYS]
                outs = ops.resample3d([d[k] for k in chunk], grid=g, mask=mask, align_corners=True,
                                      modes=[fields[k][1] for k in chunk],
                                      paddings=[fields[k][2] for k in chunk])
                for k, o in zip(chunk, outs):
                    d[k] = o
        return d

    # -- lazy materialisation (compose.py:71-110) ---------------------------
    def _materialize(self, d: dict, pending: dict, fields: dict | None = None,
                     inputs: set | None = None, want_stats: set | None = None,
                     stats_out: dict | None = None) -> dict:
        """Resample every pending key (one launch per key group).  Keys in
        ``want_stats`` that a full-batch launch writes also get their output's
        per-(element, channel) min/max in ``stats_out`` (folded by the
        resample as it writes, for the ScaleIntensity that follows)."""
        d = dict(d)
        if fields:
            d = self._materialize_fields(d, pending, fields)
            pending = {k: v for k, v in pending.items() if k not in fields}
        groups: dict[int, tuple] = {}
        for key, state in pending.items():
            if key in d:
                groups.setdefault(id(state), (state, []))[1].append(key)
        for state, keys in groups.values():
            affine, mask = state
            if not mask.any():
                continue  # nothing to resample for these keys (compose.py:85-86)
            by_shape: dict[tuple, list] = {}
            for k in keys:
                t = d[k]
                by_shape.setdefault((t.shape[0], tuple(t.shape[2:]), t.device), []).append(k)
            for ks in by_shape.values():
                for i in range(0, len(ks), L.BA_MAX_KEYS):
                    chunk = ks[i:i + L.BA_MAX_KEYS]
                    modes = [self._get_mode(k) for k in chunk]
                    paddings = [self._get_padding_mode(k) for k in chunk]
                    if (inputs is not None and self._sparse(mask)
                            and self._owned(d, chunk, inputs)):
                        # the selected elements only, written back in place
                        idx = np.flatnonzero(mask)
                        outs = ops.resample3d([self._gather(d[k], idx) for k in chunk],
                                              affine=affine[idx], modes=modes, paddings=paddings)
                        for k, o in zip(chunk, outs):
                            self._scatter(d[k], idx, o)
                        continue
                    mm = None
                    if want_stats and stats_out is not None:
                        mm = [torch.empty((d[k].shape[0], d[k].shape[1], 2), dtype=torch.int32,
                                          device=d[k].device) if k in want_stats else None
                              for k in chunk]
                    outs = ops.resample3d([d[k] for k in chunk], affine=affine, mask=mask,
                                          modes=modes, paddings=paddings, minmax=mm)
                    for i_k, (k, o) in enumerate(zip(chunk, outs)):
                        d[k] = o
                        if mm is not None and mm[i_k] is not None:
                            stats_out[k] = mm[i_k]
        return d

    def __call__(self, data: dict[str, torch.Tensor],
                 params: list | None = None) -> dict[str, torch.Tensor]:
        """Run the pipeline on ``data``.

        ``params`` (optional, an addition to the reference's signature): one
        entry per transform, in order — a params dict as that transform's
        ``sample_params`` returns it (the reference's own params inject
        unchanged: same keys), or None to sample as usual.  Each transform
        samples its params exactly once per call in the reference, so this
        replays a recorded run of the reference's Compose.
        """
        ts = list(self.transforms)
        if params is None:
            injected = [None] * len(ts)
        else:
            injected = list(params)
            if len(injected) != len(ts):
                raise ValueError(f"params has {len(injected)} entries for {len(ts)} transforms")
        # storages of the caller's tensors: never written in place
        inputs = {self._storage(v) for v in data.values()}
        if not self.lazy:
            return self._apply_rest(dict(data), ts, inputs, injected)
        d = dict(data)
        if not d:
            return d
        first = d[next(iter(d))]
        B, shape = first.shape[0], tuple(first.shape)
        # key -> (affine (B,4,4) f32, mask (B,) bool); keys with one history
        # share one state object, so they materialise in one launch.
        pending: dict[str, tuple] = {}
        # key -> ((grid, field mask), mode, padding) of a held elastic field
        fields: dict[str, tuple] = {}
        i = 0
        while i < len(ts):
            t = ts[i]
            if self.fuse_elastic and self._is_elastic(t):
                if pending or fields:
                    d = self._materialize(d, pending, fields, inputs)
                    pending.clear()
                    fields.clear()
                src = d[t.keys[0]]
                if injected[i] is None:
                    p = t.transform.sample_params(src.shape[0], src.shape, src.device)
                else:
                    p = t.transform.adopt_params(injected[i])
                fstate = (p["grid"], np.asarray(p["_host"]["mask"], bool))
                for key in t.keys:
                    if key in d:
                        fields[key] = (fstate, t._mode.get(key, "bilinear"),
                                       t._padding_mode.get(key, t._default_padding))
                i += 1
                continue
            if self._is_geometric(t):
                inner = t.transform
                if injected[i] is None:
                    host = inner.sample_host(B, shape)
                else:
                    host = inner.adopt_params(injected[i])["_host"]
                a_t = inner.host_affine({"_host": host})
                m_t = host["mask"]
                updated: dict[int, tuple] = {}
                for key in t.keys:
                    old = pending.get(key)
                    if old is None:
                        new = updated.setdefault(-1, (a_t.copy(), m_t.copy()))
                    else:
                        new = updated.get(id(old))
                        if new is None:
                            new = (compose_affines(old[0], a_t), old[1] | m_t)
                            updated[id(old)] = new
                    pending[key] = new
                i += 1
                continue
            stats: dict = {}
            if pending or fields:
                want = self._stats_keys(t) if inputs is not None else set()
                d = self._materialize(d, pending, fields, inputs, want, stats)
                pending.clear()
                fields.clear()
            if self._is_fusible(t):
                j = i
                while j < len(ts) and self._is_fusible(ts[j]):
                    j += 1
                d = self._run_intensity(d, ts[i:j], inputs, injected[i:j], stats)
                i = j
            else:
                d = self._apply_dict(d, t, inputs, injected[i])
                i += 1
        if pending or fields:
            d = self._materialize(d, pending, fields, inputs)
        return d
