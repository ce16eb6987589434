"""Transform base classes with the reference's API (batchaug/base.py:6-76).

``BatchTransform.sample_params(batch_size, shape, device) -> dict`` and
``apply(tensor, params) -> tensor`` keep the reference's names, argument
meaning and params keys (``mask`` first).  Parameters are drawn on the host
(see ``_rng``) and uploaded in one copy; the host copies ride along under the
private key ``"_host"`` so ``Compose`` can fuse transforms without reading
anything back from the GPU.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _rng


def to_device(arr: np.ndarray, device) -> torch.Tensor:
    """Asynchronous host-to-device copy of a small numpy array through pinned
    memory (a pageable copy would synchronise the stream).  torch's caching
    host allocator keeps the pinned block until the copy has completed."""
    device = torch.device(device)
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if device.type != "cuda":
        return t.to(device)
    return t.pin_memory().to(device, non_blocking=True)


_TORCH_DTYPES = {np.dtype(np.bool_): torch.bool, np.dtype(np.uint8): torch.uint8,
                 np.dtype(np.float32): torch.float32, np.dtype(np.int64): torch.int64,
                 np.dtype(np.int32): torch.int32}


def upload(arrays: dict, device) -> dict:
    """Copy a dict of small numpy arrays to ``device`` in one transfer: the
    arrays are packed into one byte buffer (floats as float32, each piece
    8-byte aligned) and the returned tensors are typed views of its copy."""
    pieces, off = [], 0
    for k, v in arrays.items():
        v = np.ascontiguousarray(v)
        if v.dtype.kind == "f":
            v = v.astype(np.float32, copy=False)
        if v.dtype not in _TORCH_DTYPES:
            raise ValueError(f"upload: unsupported dtype {v.dtype} for {k!r}")
        off = (off + 7) & ~7
        pieces.append((k, v, off))
        off += v.nbytes
    buf = np.zeros(max(off, 1), np.uint8)
    for _, v, o in pieces:
        buf[o:o + v.nbytes] = v.reshape(-1).view(np.uint8)
    dev = to_device(buf, device)
    out = {}
    for k, v, o in pieces:
        out[k] = dev[o:o + v.nbytes].view(_TORCH_DTYPES[v.dtype]).view(v.shape)
    return out


class BatchTransform:
    """Base class for tensor-level batched transforms on (B, C, H, W, D).

    Random parameters are sampled independently per batch element and shared
    by all channels of an element (batchaug/base.py:6-52).
    """

    _stream = _rng.S_MASK_ONLY
    # True when apply() on a subset of the batch with subset_params() gives
    # those elements' results: every per-element parameter has the batch as
    # its first dimension and nothing else depends on an element's index
    # (in-kernel Philox draws are keyed on the global element index, so
    # noise transforms are not subsettable).
    _subsettable = False

    # keys of injected params that host-side code reads (see adopt_params)
    _host_keys: tuple = ()

    def __init__(self, prob: float = 1.0):
        self.prob = prob

    def adopt_params(self, params: dict) -> dict:
        """Params made elsewhere (the reference's own ``sample_params``, or a
        test's) in this class's form: the same dict plus, under ``"_host"``,
        host copies of the mask and of the other keys that host-side code
        reads (``_host_keys``).  Params from this class's ``sample_params``
        are returned unchanged.  Costs one device read per copied key."""
        if "_host" in params:
            return params
        p = dict(params)
        host = {}
        for k in ("mask",) + tuple(self._host_keys):
            if k in p:
                v = p[k]
                host[k] = v.detach().cpu().numpy() if isinstance(v, torch.Tensor) else np.asarray(v)
        if "mask" not in host:
            raise ValueError("injected params need a 'mask'")
        host["mask"] = np.asarray(host["mask"]).astype(bool).reshape(-1)
        p["_host"] = host
        return p

    def subset_params(self, params: dict, idx: np.ndarray, idx_t: torch.Tensor) -> dict:
        """``params`` restricted to the elements ``idx`` (host) / ``idx_t``
        (device): every tensor or array whose first dimension is the batch is
        indexed, everything else is kept."""
        B = len(params["_host"]["mask"])

        def pick(v):
            if isinstance(v, torch.Tensor) and v.dim() >= 1 and v.shape[0] == B:
                return v.index_select(0, idx_t.to(v.device))
            if isinstance(v, np.ndarray) and v.ndim >= 1 and v.shape[0] == B:
                return v[idx]
            return v

        out = {k: pick(v) for k, v in params.items() if k != "_host"}
        out["_host"] = {k: pick(v) for k, v in params["_host"].items()}
        return out

    # -- parameter sampling ------------------------------------------------
    def _n_uniforms(self, shape) -> int:
        """Uniforms per element this transform draws (the mask's included)."""
        return 1

    def _host_params(self, batch_size: int, shape, u: np.ndarray, seed: int) -> dict:
        """Host parameters from the (batch_size, n) uniforms; column 0 is the
        Bernoulli mask draw (base.py:35: rand < prob)."""
        return {"mask": u[:, 0] < self.prob}

    def sample_host(self, batch_size: int, shape) -> dict:
        seed = _rng.draw_seed()
        u = _rng.uniforms(seed, self._stream, batch_size, self._n_uniforms(shape))
        return self._host_params(batch_size, tuple(shape), u, seed)

    def _device_params(self, host: dict, shape, device) -> dict:
        """Device tensors of the params dict (reference keys)."""
        return upload({"mask": host["mask"]}, device)

    def sample_params(self, batch_size: int, shape, device) -> dict:
        """Sample random parameters; returns at least ``mask`` (B,) bool."""
        host = self.sample_host(batch_size, shape)
        params = self._device_params(host, tuple(shape), device)
        params["_host"] = host
        return params

    def apply(self, tensor: torch.Tensor, params: dict) -> torch.Tensor:
        raise NotImplementedError

    def __call__(self, tensor: torch.Tensor) -> torch.Tensor:
        params = self.sample_params(tensor.shape[0], tensor.shape, tensor.device)
        return self.apply(tensor, params)


class BatchDictTransform:
    """Dict wrapper: samples parameters once from the first key's tensor and
    applies them to every listed key (batchaug/base.py:55-76)."""

    def __init__(self, keys: list[str], transform: BatchTransform):
        self.keys = keys
        self.transform = transform

    def __call__(self, data: dict[str, torch.Tensor], params: dict | None = None
                 ) -> dict[str, torch.Tensor]:
        """``params``: optional injected params (as ``sample_params`` returns
        them, e.g. the reference's own) instead of sampling."""
        d = dict(data)
        if params is None:
            first = d[self.keys[0]]
            params = self.transform.sample_params(first.shape[0], first.shape, first.device)
        else:
            params = self.transform.adopt_params(params)
        for key in self.keys:
            if key in d:
                d[key] = self.transform.apply(d[key], params)
        return d
