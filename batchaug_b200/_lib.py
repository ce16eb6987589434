"""ctypes binding of libbatchaug_b200.so (the C ABI in include/batchaug_b200.h).

The shared library is built in-tree by ``python batchaug_b200/build.py``.
There is no fallback: if the library is missing or fails to load, importing
``batchaug_b200`` raises ImportError.  Status codes map to exceptions as the
reference does for bad arguments (``ValueError``, batchaug/_backend.py:9-11,
bias_field.py:76-77) and to ``RuntimeError`` for CUDA failures.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbatchaug_b200.so")

BA_OK, BA_EINVAL, BA_EUNSUPPORTED, BA_ECUDA, BA_ETIMEOUT = 0, 1, 2, 3, 4
BA_F32, BA_BF16 = 0, 1
BA_BILINEAR, BA_NEAREST = 0, 1
BA_PAD_ZEROS, BA_PAD_BORDER, BA_PAD_REFLECTION = 0, 1, 2
BA_XFORM_AFFINE, BA_XFORM_THETA, BA_XFORM_GRID = 0, 1, 2
BA_RESAMPLE_EXACT, BA_RESAMPLE_HOST_PARAMS = 0x1, 0x2
BA_MAX_KEYS = 8
BA_MAX_OPS = 8

BA_OP_NOISE, BA_OP_CONTRAST, BA_OP_SCALE, BA_OP_SHIFT, BA_OP_BIAS_FIELD, BA_OP_RESCALE = 1, 2, 3, 4, 5, 6
BA_OP_RICIAN, BA_OP_STD_SHIFT, BA_OP_FIXED_MEAN = 7, 8, 9
BA_NOISE_PHILOX = 0x1
BA_RICIAN_PHILOX, BA_RICIAN_RELATIVE = 0x1, 0x2
BA_STD_NONZERO, BA_STAT_CHANNEL = 0x2, 0x4
BA_SHIFT_SAFE = 0x1
BA_RESCALE_MINV, BA_RESCALE_MAXV, BA_RESCALE_CHANNEL, BA_RESCALE_FACTOR = 0x1, 0x2, 0x4, 0x8
BA_RESCALE_GIVEN = 0x10

BA_SMOOTH_ZEROS, BA_SMOOTH_REFLECT, BA_SMOOTH_REPLICATE = 0, 1, 2

MODES = {"bilinear": BA_BILINEAR, "nearest": BA_NEAREST}
SMOOTH_PADS = {None: BA_SMOOTH_ZEROS, "constant": BA_SMOOTH_ZEROS, "reflect": BA_SMOOTH_REFLECT,
               "replicate": BA_SMOOTH_REPLICATE}
PADDINGS = {"zeros": BA_PAD_ZEROS, "border": BA_PAD_BORDER, "reflection": BA_PAD_REFLECTION}

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64


class ResampleKey(ctypes.Structure):
    _fields_ = [("src", _P), ("dst", _P), ("channels", _I64), ("dtype", _I32), ("mode", _I32),
                ("padding", _I32), ("reserved", _I32), ("minmax", _P)]


class ResampleDesc(ctypes.Structure):
    _fields_ = [("batch", _I64), ("H", _I64), ("W", _I64), ("D", _I64),
                ("xform_kind", _I32), ("align_corners", _I32), ("n_keys", _I32),
                ("flags", _I32), ("xform", _P), ("xform_stride", _I64), ("mask", _P),
                ("keys", ResampleKey * BA_MAX_KEYS)]


class Op(ctypes.Structure):
    _fields_ = [("kind", _I32), ("flags", _I32), ("mask", _P), ("param", _P), ("param2", _P),
                ("noise", _P), ("seed", _U64), ("elem_offset", _U64), ("degree", _I32),
                ("reserved", _I32), ("stats", _P), ("c0", ctypes.c_double),
                ("c1", ctypes.c_double)]


class ChainDesc(ctypes.Structure):
    _fields_ = [("src", _P), ("dst", _P), ("batch", _I64), ("channels", _I64), ("H", _I64),
                ("W", _I64), ("D", _I64), ("dtype", _I32), ("n_ops", _I32),
                ("ops", Op * BA_MAX_OPS)]


class SharpenDesc(ctypes.Structure):
    _fields_ = [("src", _P), ("dst", _P), ("dtype", _I32), ("padding", _I32), ("batch", _I64),
                ("channels", _I64), ("H", _I64), ("W", _I64), ("D", _I64),
                ("taps1", _P * 3), ("K1", _I64 * 3), ("taps2", _P * 3), ("K2", _I64 * 3),
                ("alpha", _P), ("mask", _P)]


class LowresDesc(ctypes.Structure):
    _fields_ = [("src", _P), ("dst", _P), ("dtype", _I32), ("down_mode", _I32),
                ("up_mode", _I32), ("align_corners", _I32), ("batch", _I64), ("channels", _I64),
                ("H", _I64), ("W", _I64), ("D", _I64), ("zoom", _P), ("mask", _P),
                ("max_zoom", ctypes.c_double)]


INTERP_MODES = {"nearest": 0, "nearest-exact": 1, "trilinear": 2, "area": 3}


# Every symbol include/batchaug_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "ba_resample3d": (_I32, [ctypes.POINTER(ResampleDesc), _P]),
    "ba_compose_field": (_I32, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P]),
    "ba_intensity_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(ChainDesc)]),
    "ba_intensity_chain": (_I32, [ctypes.POINTER(ChainDesc), _P, ctypes.c_size_t, _P]),
    "ba_intensity_chain_noalloc": (_I32, [ctypes.POINTER(ChainDesc), _P]),
    "ba_noalloc_chain_scratch_bytes": (ctypes.c_size_t, []),
    "ba_minmax": (_I32, [_P, _I32, _I64, _I64, _P, _P]),
    "ba_gauss_taps_len": (_I64, [ctypes.c_double, ctypes.c_double]),
    "ba_gauss_taps": (_I32, [_P, _I64, _I64, _P, _P]),
    "ba_smooth_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I64]),
    "ba_smooth3d": (_I32, [_P, _P, _I32, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _P,
                           _I64, _I32, _P, _P, ctypes.c_size_t, _P]),
    "ba_sharpen_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SharpenDesc)]),
    "ba_sharpen3d": (_I32, [ctypes.POINTER(SharpenDesc), _P, ctypes.c_size_t, _P]),
    "ba_lowres_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(LowresDesc)]),
    "ba_lowres3d": (_I32, [ctypes.POINTER(LowresDesc), _P, ctypes.c_size_t, _P]),
    "ba_elastic_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I64]),
    "ba_elastic_grid": (_I32, [_P, _U64, _U64, _I64, _I64, _I64, _I64, _P, _I64, _P, _P, _P,
                               ctypes.c_size_t, _P]),
    "ba_host_uniform": (None, [_U64, ctypes.c_uint32, _U64, _I64, _I64, _P]),
    "ba_host_rand_affine": (None, [_P, _I64, _I64, ctypes.c_float, _P, _P, _P, ctypes.c_uint32,
                                   ctypes.c_uint32, _I64, _I64, _I64, _P, _P, _P]),
    "ba_last_error": (ctypes.c_char_p, []),
    "ba_version": (_I32, []),
    "ba_kernel_launches": (ctypes.c_uint64, []),
    "ba_wait_status": (_I32, [_P]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"batchaug_b200: CUDA library {LIB_PATH} is missing; build it with "
            "`python batchaug_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# bytes of the static scratch of ba_intensity_chain_noalloc, from the library
BA_NOALLOC_CHAIN_SCRATCH = int(lib.ba_noalloc_chain_scratch_bytes())


def check(status: int, what: str) -> None:
    if status == BA_OK:
        return
    msg = (lib.ba_last_error() or b"").decode(errors="replace") or what
    if status in (BA_EINVAL, BA_EUNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return BA_F32
    if t.dtype == torch.bfloat16:
        return BA_BF16
    raise ValueError(f"batchaug_b200 supports float32 and bfloat16 tensors, got {t.dtype}")


def kernel_launches() -> int:
    """Kernels the library has enqueued in this process so far."""
    return int(lib.ba_kernel_launches())


def wait_status(device: torch.device | None = None) -> None:
    """Synchronise the current stream and raise if any bounded device wait
    of the library (the TMA-staged resample's mbarrier waits) ran out."""
    dev = torch.device("cuda") if device is None else device
    check(lib.ba_wait_status(stream_ptr(dev)), "ba_wait_status")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(t: torch.Tensor, name: str = "tensor") -> None:
    if not t.is_cuda:
        raise ValueError(f"batchaug_b200 runs on CUDA tensors only; {name} is on {t.device}")
