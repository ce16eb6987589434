"""numpy <-> torch helpers for parity tests (bf16 stored as uint16 bits)."""
from __future__ import annotations

import numpy as np
import torch


def to_dev(a: np.ndarray, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    if a.dtype == np.uint8:
        return torch.from_numpy(a).to(device).bool()
    return torch.from_numpy(a).to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f32(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a


def bf16_ulp_diff(a: np.ndarray, b: np.ndarray) -> int:
    """Max distance in bf16 ulps between two bf16 bit arrays (same sign)."""
    ia = a.astype(np.int32)
    ib = b.astype(np.int32)
    # map sign-magnitude to a monotone integer line
    ia = np.where(ia & 0x8000, -(ia & 0x7FFF), ia)
    ib = np.where(ib & 0x8000, -(ib & 0x7FFF), ib)
    return int(np.abs(ia - ib).max()) if ia.size else 0


def assert_close_dtype(out: np.ndarray, ref: np.ndarray, atol_f32=1e-5, max_bf16_ulp=2,
                       bf16_abs=0.0):
    """The parity bar: fp32 within atol_f32, bf16 within max_bf16_ulp ulps.

    ``bf16_abs`` > 0 also accepts bf16 values within that absolute distance:
    for a bf16 result computed in fp32 and rounded once, a value that
    cancels to near zero (|x| < ~1e-4) has bf16 ulps below the fp32
    arithmetic's own rounding (~1e-7 of the operands), so a reordered fp32
    computation can land several bf16 ulps away while being 1e-8 apart."""
    assert out.shape == ref.shape and out.dtype == ref.dtype
    if out.dtype == np.uint16:
        if bf16_abs > 0:
            near = np.abs(as_f32(out) - as_f32(ref)) <= bf16_abs
            out, ref = out[~near], ref[~near]
        assert bf16_ulp_diff(out, ref) <= max_bf16_ulp
    else:
        np.testing.assert_allclose(out, ref, rtol=0, atol=atol_f32)
