"""ba_intensity_chain_noalloc — the chain for callers that cannot allocate.

Hosts that manage all device memory themselves (or must not trigger a
cudaMalloc inside their loop) cannot hand the chain a scratch buffer; this
entry point uses a static device array instead.  The test drives it through
the C ABI, twice in a row (the array keeps the previous call's statistics,
which the chain must re-initialise), and checks each result against the
ordinary ba_intensity_chain with caller-provided scratch.  Kept in a file of
its own that pytest collects last."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _chain_desc(L, x, out, ops_):
    d = L.ChainDesc()
    d.src, d.dst = x.data_ptr(), out.data_ptr()
    d.batch, d.channels, d.H, d.W, d.D = x.shape
    d.dtype = L.dtype_code(x)
    d.n_ops = len(ops_)
    for i, (kind, flags, param, c0, c1) in enumerate(ops_):
        o = d.ops[i]
        o.kind, o.flags = kind, flags
        o.param = None if param is None else param.data_ptr()
        o.c0, o.c1 = c0, c1
    return d


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_chain_matches_workspace_chain_twice(dtype):
    from batchaug_b200 import _lib as L
    from batchaug_b200 import ops
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((0, 1)):
        g = torch.Generator(device=dev).manual_seed(seed)
        x = torch.rand(3, 2, 20, 18, 16, device=dev, generator=g).to(dtype)
        gamma = torch.rand(3, device=dev, generator=g) * 1.5 + 0.5
        factor = torch.rand(3, device=dev, generator=g) * 0.4 - 0.2
        spec = [(L.BA_OP_CONTRAST, 0, gamma, 0.0, 0.0),
                (L.BA_OP_SCALE, 0, factor, 0.0, 0.0),
                (L.BA_OP_RESCALE, L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV | L.BA_RESCALE_CHANNEL,
                 None, 0.0, 1.0)]
        out = torch.empty_like(x)
        d = _chain_desc(L, x, out, spec)
        assert L.lib.ba_intensity_workspace_bytes(ctypes.byref(d)) <= L.BA_NOALLOC_CHAIN_SCRATCH
        st = L.lib.ba_intensity_chain_noalloc(ctypes.byref(d), stream)
        assert st == L.BA_OK, L.lib.ba_last_error()
        ref = ops.intensity_chain(x, [ops.ChainOp(k, flags=f, param=p, c0=a, c1=b)
                                      for k, f, p, a, b in spec])
        torch.cuda.synchronize()
        # same kernels, same order: identical results (the tests' bar for the
        # chain is 1e-5 fp32 / 2 bf16 ulp; these are bit-equal)
        assert torch.equal(out, ref), f"call {call}"
        flat = out.float().reshape(6, -1)
        assert torch.equal(flat.min(1).values, torch.zeros(6, device=dev))


def test_noalloc_rejects_oversized_scratch():
    from batchaug_b200 import _lib as L
    limit = L.BA_NOALLOC_CHAIN_SCRATCH
    groups = limit // 8 + 1  # 2 int32 keys per group per min/max barrier
    # src and dst hold every voxel the descriptor describes (1 x groups x 1^3
    # fp32), so the call stays in bounds even if the size check regressed
    x = torch.arange(groups, dtype=torch.float32, device="cuda")
    before = x.clone()
    d = L.ChainDesc()
    d.src = d.dst = x.data_ptr()
    d.batch, d.channels, d.H, d.W, d.D = 1, groups, 1, 1, 1
    d.dtype, d.n_ops = L.BA_F32, 1
    d.ops[0].kind = L.BA_OP_RESCALE
    d.ops[0].flags = L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV | L.BA_RESCALE_CHANNEL
    assert L.lib.ba_intensity_workspace_bytes(ctypes.byref(d)) > limit
    st = L.lib.ba_intensity_chain_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert st == L.BA_EINVAL
    assert b"static array" in L.lib.ba_last_error()
    torch.cuda.synchronize()
    assert torch.equal(x, before)  # rejected before any kernel ran


def test_noalloc_reports_bad_shape_first():
    """A malformed descriptor is reported as such, not as a scratch size
    computed from its shape."""
    from batchaug_b200 import _lib as L
    d = L.ChainDesc()
    d.batch, d.channels, d.H, d.W, d.D = -1, 1, 4, 4, 4
    d.dtype, d.n_ops = L.BA_F32, 1
    d.ops[0].kind = L.BA_OP_RESCALE
    d.ops[0].flags = L.BA_RESCALE_MINV | L.BA_RESCALE_MAXV
    st = L.lib.ba_intensity_chain_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert st == L.BA_EINVAL
    assert b"bad shape" in L.lib.ba_last_error()


def test_noalloc_limit_matches_header():
    from batchaug_b200 import _lib as L
    import os
    import re
    hdr = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                       "batchaug_b200.h")
    m = re.search(r"#define BA_NOALLOC_CHAIN_SCRATCH (\d+)", open(hdr).read())
    assert m and int(m.group(1)) == L.BA_NOALLOC_CHAIN_SCRATCH
