"""Per-element random parameters and the batch-shard context.

Every ``sample_params`` call draws one 64-bit seed from torch's default CPU
generator (so ``torch.manual_seed`` makes runs reproducible) and derives each
element's scalars from Philox4x32-10 keyed on (seed, global element index,
parameter stream) with ``ba_host_uniform``.  Large random volumes (Gaussian
noise, the elastic field's uniform draw) are generated on the GPU from the
same (seed, global element index) and are never materialised in HBM.

In a batch-sharded run every rank seeds torch identically and declares its
slice of the global batch with :func:`set_shard`; a rank then derives exactly
the parameters that a single process running the whole global batch would
give those elements, with no communication.  Quantities the reference
computes over the whole batch (the batch-max sigma that sizes Gaussian taps,
smooth.py:24-25) are derived from every global element's scalars.
"""
from __future__ import annotations

import contextlib

import numpy as np
import torch

from . import ops

_state = {"offset": 0, "global_batch": None}

# Parameter stream ids (one per transform family).
S_MASK_ONLY = 1
S_AFFINE = 2
S_FLIP = 3
S_ROT90 = 4
S_ELASTIC = 5
S_NOISE = 6
S_CONTRAST = 7
S_SCALE = 8
S_SHIFT = 9
S_BIAS = 10
S_SMOOTH = 11
S_ZOOM = 12
S_RICIAN = 13
S_STD_SHIFT = 14
S_FIXED_MEAN = 15
S_SHARPEN = 16
S_LOWRES = 17


def set_shard(element_offset: int = 0, global_batch: int | None = None) -> None:
    """Declare that this process's batch holds global elements
    [element_offset, element_offset + B) of a global batch of
    ``global_batch`` elements (None: the local batch is the whole batch)."""
    if element_offset < 0:
        raise ValueError("element_offset must be >= 0")
    _state["offset"] = int(element_offset)
    _state["global_batch"] = None if global_batch is None else int(global_batch)


def get_shard() -> tuple[int, int | None]:
    return _state["offset"], _state["global_batch"]


@contextlib.contextmanager
def shard(element_offset: int, global_batch: int | None = None):
    old = get_shard()
    set_shard(element_offset, global_batch)
    try:
        yield
    finally:
        set_shard(*old)


def draw_seed() -> int:
    """A fresh 63-bit Philox key from torch's default CPU generator."""
    return int(torch.randint(0, 2**63 - 1, (1,), dtype=torch.int64).item())


def uniforms(seed: int, stream: int, batch: int, per_elem: int) -> np.ndarray:
    """(batch, per_elem) uniforms in [0,1) for this process's elements."""
    return ops.host_uniform(seed, stream, _state["offset"], batch, per_elem)


def global_uniforms(seed: int, stream: int, batch: int, per_elem: int) -> tuple[np.ndarray, int]:
    """Uniforms for every element of the global batch and the row index of
    this process's first element."""
    off, gb = _state["offset"], _state["global_batch"]
    if gb is None:
        return ops.host_uniform(seed, stream, off, batch, per_elem), 0
    if off + batch > gb:
        raise ValueError(f"shard [{off}, {off + batch}) exceeds global batch {gb}")
    return ops.host_uniform(seed, stream, 0, gb, per_elem), off


def element_offset() -> int:
    return _state["offset"]
