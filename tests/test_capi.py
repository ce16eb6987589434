"""C ABI surface, checked without a GPU: the library loads, exports every
function include/batchaug_b200.h declares, and its host-only paths (argument
validation, Gaussian tap sizing, host Philox) behave."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_functions() -> list[str]:
    src = open(os.path.join(ROOT, "include", "batchaug_b200.h")).read()
    return re.findall(r"^BA_API\s+[\w\s\*]+?\b(ba_\w+)\s*\(", src, flags=re.M)


def test_header_symbols_exported(ba):
    from batchaug_b200 import _lib as L
    names = _declared_functions()
    assert len(names) >= 13
    lib = ctypes.CDLL(L.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    assert set(names) == set(L.SIGNATURES), "ctypes binding out of sync with the header"


def test_struct_layouts_match_header(ba, tmp_path):
    """Every ctypes field offset and struct size equals what the C compiler
    gives the header's structs."""
    import shutil
    import subprocess
    from batchaug_b200 import _lib as L
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"ba_resample_key": L.ResampleKey, "ba_resample_desc": L.ResampleDesc,
               "ba_op": L.Op, "ba_chain_desc": L.ChainDesc, "ba_sharpen_desc": L.SharpenDesc,
               "ba_lowres_desc": L.LowresDesc}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "batchaug_b200.h"',
             "int main(void) {"]
    for cname, ct in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in ct._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    seen = 0
    for line in got:
        if not line:
            continue
        cname, what, val = line.split()
        ct = structs[cname]
        expect = ctypes.sizeof(ct) if what == "size" else getattr(ct, what).offset
        assert int(val) == expect, f"{cname}.{what}: C {val} vs ctypes {expect}"
        seen += 1
    assert seen == sum(len(c._fields_) + 1 for c in structs.values())


def test_version_and_error_string(ba):
    from batchaug_b200 import _lib as L
    assert L.lib.ba_version() >> 16 == 1
    st = L.lib.ba_resample3d(None, None)
    assert st == L.BA_EINVAL
    assert b"desc is NULL" in L.lib.ba_last_error()


def test_validation_without_gpu(ba):
    """Bad descriptors are rejected before any CUDA call."""
    from batchaug_b200 import _lib as L
    d = L.ResampleDesc()
    d.batch, d.H, d.W, d.D = 2, 4, 4, 4
    d.n_keys = 0
    assert L.lib.ba_resample3d(ctypes.byref(d), None) == L.BA_EINVAL
    d.n_keys = 1
    d.xform_kind = 7
    assert L.lib.ba_resample3d(ctypes.byref(d), None) == L.BA_EINVAL
    c = L.ChainDesc()
    c.batch, c.channels, c.H, c.W, c.D, c.dtype, c.n_ops = 1, 1, 2, 2, 2, 0, 1
    c.ops[0].kind = L.BA_OP_BIAS_FIELD
    c.ops[0].param = 8  # any non-NULL; rejected on degree first
    c.ops[0].degree = 7
    assert L.lib.ba_intensity_chain(ctypes.byref(c), None, 0, None) == L.BA_EUNSUPPORTED
    assert L.lib.ba_minmax(None, 5, 1, 1, None, None) == L.BA_EINVAL
    assert L.lib.ba_gauss_taps(None, 1, 4, None, None) == L.BA_EINVAL  # even K
    sd = L.SharpenDesc()
    sd.batch, sd.channels, sd.H, sd.W, sd.D, sd.dtype = 2, 3, 5, 6, 7, 1
    for i in range(3):
        sd.K1[i], sd.K2[i] = 9, 5
    # two fp32 scratch volumes (16-byte rounded) plus the first blur in bf16
    n = 2 * 3 * 5 * 6 * 7
    assert L.lib.ba_sharpen_workspace_bytes(ctypes.byref(sd)) == ((8 * n + 15) // 16) * 16 + 2 * n
    assert L.lib.ba_sharpen3d(ctypes.byref(sd), None, 0, None) == L.BA_EINVAL  # NULL src
    sd.K2[1] = 4
    assert L.lib.ba_sharpen3d(ctypes.byref(sd), None, 0, None) == L.BA_EINVAL
    assert b"must be odd" in L.lib.ba_last_error()
    sd.K2[1], sd.padding, sd.K1[0] = 5, 1, 11  # reflect needs K/2 < H
    assert L.lib.ba_sharpen3d(ctypes.byref(sd), None, 0, None) == L.BA_EINVAL
    assert b"reflect" in L.lib.ba_last_error()
    ld = L.LowresDesc()
    ld.batch, ld.channels, ld.H, ld.W, ld.D, ld.dtype, ld.max_zoom = 2, 3, 10, 11, 12, 0, 0.6
    assert L.lib.ba_lowres_workspace_bytes(ctypes.byref(ld)) == 0  # nearest downsample: none
    ld.down_mode = 2  # trilinear: scratch for the largest target, rint(s * 0.6)
    assert L.lib.ba_lowres_workspace_bytes(ctypes.byref(ld)) == 2 * 3 * 6 * 7 * 7 * 4
    ld.up_mode = 9
    assert L.lib.ba_lowres3d(ctypes.byref(ld), None, 0, None) == L.BA_EINVAL
    assert b"mode" in L.lib.ba_last_error()


def test_gauss_taps_len_matches_reference_rule(ba):
    from batchaug_b200 import ops
    # int(max(max_sigma * truncated, 0.5) + 0.5) tail, smooth.py:24-25
    for s, tr in [(7.0, 3.0), (5.2, 3.0), (1.5, 4.0), (0.5, 4.0), (0.01, 4.0), (0.1, 3.0)]:
        tail = int(max(float(np.float32(s)) * tr, 0.5) + 0.5)
        assert ops.gauss_taps_len(s, tr) == 2 * tail + 1


def test_host_uniform_keyed_on_global_element(ba):
    from batchaug_b200 import ops
    full = ops.host_uniform(99, 3, 0, 8, 5)
    part = ops.host_uniform(99, 3, 4, 4, 5)
    assert np.array_equal(full[4:], part)
    assert full.min() >= 0 and full.max() < 1
    other = ops.host_uniform(99, 4, 0, 8, 5)
    assert not np.array_equal(full, other)
    big = ops.host_uniform(1, 1, 0, 1, 200000)[0]
    assert abs(big.mean() - 0.5) < 0.005 and abs(big.var() - 1 / 12) < 0.002


def test_philox_known_answer():
    """Philox4x32-10 known-answer vectors from the Random123 distribution's
    kat_vectors (counter, key -> output), checked through the host path."""
    import batchaug_b200  # noqa: F401
    from batchaug_b200 import _lib as L
    # ba_host_uniform exposes u01(r >> 8); reconstruct the top 24 bits of the
    # first output word for counter {0, elem, elem>>32, stream} ... instead
    # verify via a private re-implementation of the published algorithm.
    def philox(ctr, key):
        M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
        c = list(ctr)
        k0, k1 = key
        for _ in range(10):
            p0, p1 = M0 * c[0], M1 * c[2]
            c = [((p1 >> 32) ^ c[1] ^ k0) & 0xFFFFFFFF, p1 & 0xFFFFFFFF,
                 ((p0 >> 32) ^ c[3] ^ k1) & 0xFFFFFFFF, p0 & 0xFFFFFFFF]
            k0, k1 = (k0 + W0) & 0xFFFFFFFF, (k1 + W1) & 0xFFFFFFFF
        return c
    # Random123 kat_vectors: philox4x32 10 rounds
    assert philox([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6,
                                                           0x6D5451FD]
    assert philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                  [0xA4093822, 0x299F31D0]) == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    # the library's host path uses the same function
    seed, stream, elem = 0x299F31D0A4093822, 5, 0x0000000100000002
    u = np.empty(4, np.float32)
    L.lib.ba_host_uniform(seed, stream, elem, 1, 4, u.ctypes.data)
    w = philox([0, elem & 0xFFFFFFFF, elem >> 32, 0x50410000 | stream],
               [seed & 0xFFFFFFFF, seed >> 32])
    assert np.array_equal(u, np.array([(x >> 8) / 16777216.0 for x in w], np.float32))
