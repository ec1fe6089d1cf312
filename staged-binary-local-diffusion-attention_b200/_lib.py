"""ctypes binding of the C ABI declared in ``include/sbda_b200.h``.

The library is the in-tree ``libsbda_b200.so`` built by ``build.py``.  There
is no fallback: if it is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIBRARY

SBDA_DTYPE_F32 = 0
SBDA_DTYPE_F16 = 1
SBDA_DTYPE_BF16 = 2

SBDA_OK = 0
SBDA_ERR_INVALID = 1
SBDA_ERR_DTYPE = 2
SBDA_ERR_UNSUPPORTED = 3
SBDA_ERR_CUDA = 4
SBDA_ERR_DEVICE = 5


class SbdaTensor(ctypes.Structure):
    """``sbda_tensor``: element (0,0,0,0) of a [B,H,L,D] view and element strides."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("stride_l", ctypes.c_int64),
        ("stride_d", ctypes.c_int64),
    ]


class SbdaShape(ctypes.Structure):
    """``sbda_shape``."""

    _fields_ = [
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("length", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> str:
    return LIBRARY


def load() -> ctypes.CDLL:
    """Load ``libsbda_b200.so`` (once) and declare the entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIBRARY):
            raise RuntimeError(
                f"SBDA CUDA library not built: {LIBRARY} is missing "
                "(run __graft_entry__.build() or python -m sbda_b200.build)"
            )
        lib = ctypes.CDLL(LIBRARY)
        c_int, c_int32, c_float, c_void_p = ctypes.c_int, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p
        i32p = ctypes.POINTER(ctypes.c_int32)
        lib.sbda_b200_abi_version.restype = c_int
        lib.sbda_b200_abi_version.argtypes = []
        lib.sbda_b200_status_string.restype = ctypes.c_char_p
        lib.sbda_b200_status_string.argtypes = [c_int]
        lib.sbda_b200_forward.restype = c_int
        lib.sbda_b200_forward.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float,
            SbdaTensor, SbdaTensor, SbdaTensor, SbdaTensor, c_void_p, c_void_p,
        ]
        lib.sbda_b200_backward.restype = c_int
        lib.sbda_b200_backward.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float,
            SbdaTensor, SbdaTensor, SbdaTensor, SbdaTensor, c_void_p,
            SbdaTensor, SbdaTensor, SbdaTensor, c_void_p,
        ]
        lib.sbda_b200_forward_masked.restype = c_int
        lib.sbda_b200_forward_masked.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float,
            SbdaTensor, SbdaTensor, SbdaTensor, c_void_p, SbdaTensor, c_void_p, c_void_p,
        ]
        lib.sbda_b200_backward_masked.restype = c_int
        lib.sbda_b200_backward_masked.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float,
            SbdaTensor, SbdaTensor, SbdaTensor, c_void_p, SbdaTensor, c_void_p,
            SbdaTensor, SbdaTensor, SbdaTensor, c_void_p,
        ]
        lib.sbda_b200_forward_paths.restype = c_int
        lib.sbda_b200_forward_paths.argtypes = [
            c_int, SbdaShape, c_int32, c_float, SbdaTensor, SbdaTensor, SbdaTensor, c_void_p, c_void_p,
            SbdaTensor, c_void_p, c_void_p,
        ]
        lib.sbda_b200_paths_workspace_floats.restype = ctypes.c_int64
        lib.sbda_b200_paths_workspace_floats.argtypes = [SbdaShape, c_int32]
        lib.sbda_b200_backward_paths.restype = c_int
        lib.sbda_b200_backward_paths.argtypes = [
            c_int, SbdaShape, c_int32, c_float, SbdaTensor, SbdaTensor, SbdaTensor, c_void_p, c_void_p,
            c_void_p, c_void_p, SbdaTensor, c_void_p, c_void_p, ctypes.c_int64, SbdaTensor, SbdaTensor,
            SbdaTensor, c_void_p,
        ]
        u8p = c_void_p
        lib.sbda_b200_rms_norm_forward.restype = c_int
        lib.sbda_b200_rms_norm_forward.argtypes = [
            c_int, ctypes.c_int64, ctypes.c_int64, c_void_p, c_void_p, u8p, c_void_p, c_float,
            c_void_p, c_void_p, c_void_p, c_void_p,
        ]
        lib.sbda_b200_rms_norm_workspace_floats.restype = ctypes.c_int64
        lib.sbda_b200_rms_norm_workspace_floats.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.sbda_b200_rms_norm_backward.restype = c_int
        lib.sbda_b200_rms_norm_backward.argtypes = [
            c_int, ctypes.c_int64, ctypes.c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, u8p,
            c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_int64, c_void_p,
        ]
        lib.sbda_b200_silu_mul_forward.restype = c_int
        lib.sbda_b200_silu_mul_forward.argtypes = [c_int, ctypes.c_int64, c_void_p, c_void_p, c_void_p, c_void_p]
        lib.sbda_b200_silu_mul_backward.restype = c_int
        lib.sbda_b200_silu_mul_backward.argtypes = [
            c_int, ctypes.c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        ]
        lib.sbda_b200_norm_rope_forward.restype = c_int
        lib.sbda_b200_norm_rope_forward.argtypes = [
            c_int, SbdaShape, SbdaTensor, SbdaTensor, c_void_p, c_float, c_void_p, c_void_p,
            ctypes.c_int64, c_void_p,
        ]
        lib.sbda_b200_norm_rope_workspace_floats.restype = ctypes.c_int64
        lib.sbda_b200_norm_rope_workspace_floats.argtypes = [SbdaShape]
        lib.sbda_b200_norm_rope_backward.restype = c_int
        lib.sbda_b200_norm_rope_backward.argtypes = [
            c_int, SbdaShape, SbdaTensor, SbdaTensor, c_void_p, c_float, c_void_p, c_void_p,
            ctypes.c_int64, SbdaTensor, c_void_p, c_void_p, ctypes.c_int64, c_void_p,
        ]
        lib.sbda_b200_norm_rope_backward_noalloc.restype = c_int
        lib.sbda_b200_norm_rope_backward_noalloc.argtypes = [
            c_int, SbdaShape, SbdaTensor, SbdaTensor, c_void_p, c_float, c_void_p, c_void_p,
            ctypes.c_int64, SbdaTensor, c_void_p, c_void_p,
        ]
        tarr = ctypes.POINTER(SbdaTensor)
        lib.sbda_b200_forward_sharded.restype = c_int
        lib.sbda_b200_forward_sharded.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float, c_int32, c_int32,
            SbdaTensor, tarr, tarr, SbdaTensor, c_void_p, c_void_p,
        ]
        lib.sbda_b200_backward_sharded.restype = c_int
        lib.sbda_b200_backward_sharded.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float, c_int32, c_int32,
            tarr, tarr, tarr, tarr, ctypes.POINTER(c_void_p),
            SbdaTensor, SbdaTensor, SbdaTensor, c_void_p,
        ]
        lib.sbda_b200_normed_supported.restype = c_int
        lib.sbda_b200_normed_supported.argtypes = [c_int, SbdaShape, i32p, c_int32]
        lib.sbda_b200_forward_normed.restype = c_int
        lib.sbda_b200_forward_normed.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float, SbdaTensor, SbdaTensor, SbdaTensor,
            c_void_p, c_float, c_void_p, c_float, c_void_p, c_void_p, ctypes.c_int64, SbdaTensor, c_void_p,
            c_void_p,
        ]
        lib.sbda_b200_backward_normed_workspace_floats.restype = ctypes.c_int64
        lib.sbda_b200_backward_normed_workspace_floats.argtypes = [c_int, SbdaShape, i32p, c_int32]
        lib.sbda_b200_backward_normed.restype = c_int
        lib.sbda_b200_backward_normed.argtypes = [
            c_int, SbdaShape, i32p, c_int32, c_float, SbdaTensor, SbdaTensor, SbdaTensor, SbdaTensor, c_void_p,
            c_void_p, c_float, c_void_p, c_float, c_void_p, c_void_p, ctypes.c_int64, SbdaTensor, SbdaTensor,
            SbdaTensor, c_void_p, c_void_p, c_void_p, ctypes.c_int64, c_void_p,
        ]
        lib.sbda_b200_backward_grouped_workspace_floats.restype = ctypes.c_int64
        lib.sbda_b200_backward_grouped_workspace_floats.argtypes = [SbdaShape]
        lib.sbda_b200_backward_grouped.restype = c_int
        lib.sbda_b200_backward_grouped.argtypes = list(lib.sbda_b200_backward.argtypes[:-1]) + [
            c_void_p, ctypes.c_int64, c_void_p]
        fwd_args = lib.sbda_b200_forward.argtypes
        bwd_args = lib.sbda_b200_backward.argtypes
        lib.sbda_b200_forward_ex.restype = c_int
        lib.sbda_b200_forward_ex.argtypes = [c_int] + list(fwd_args)
        lib.sbda_b200_backward_ex.restype = c_int
        lib.sbda_b200_backward_ex.argtypes = [c_int] + list(bwd_args)
        lib.sbda_b200_forward_sharded_ex.restype = c_int
        lib.sbda_b200_forward_sharded_ex.argtypes = [c_int] + list(lib.sbda_b200_forward_sharded.argtypes)
        lib.sbda_b200_backward_sharded_ex.restype = c_int
        lib.sbda_b200_backward_sharded_ex.argtypes = [c_int] + list(lib.sbda_b200_backward_sharded.argtypes)
        lib.sbda_b200_device_status.restype = c_int
        lib.sbda_b200_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), c_int]
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load().sbda_b200_status_string(int(status)).decode()


def raise_for_status(status: int, what: str) -> None:
    """Map a C status onto the reference's exception types (sbda_triton.py:1295-1303)."""
    if status == SBDA_OK:
        return
    message = f"{what}: {status_string(status)} (status {status})"
    if status == SBDA_ERR_INVALID:
        raise ValueError(message)
    if status == SBDA_ERR_DTYPE:
        raise TypeError(message)
    raise RuntimeError(message)


def offsets_array(offsets: tuple[int, ...]):
    array = (ctypes.c_int32 * 4)()
    for index, offset in enumerate(offsets[:4]):
        array[index] = int(offset)
    return array


KERNEL_FAMILIES = {"auto": 0, "general": 1, "uniform": 2}


def family_code(family: str | int) -> int:
    """Kernel family name (or code) -> the ``family`` argument of the ``*_ex`` entry points."""
    if isinstance(family, str):
        if family not in KERNEL_FAMILIES:
            raise ValueError(f"unknown kernel family {family!r}")
        return KERNEL_FAMILIES[family]
    if int(family) not in KERNEL_FAMILIES.values():
        raise ValueError(f"unknown kernel family {family}")
    return int(family)


def device_status(reset: bool = True) -> int:
    """Fault word of the current device (synchronises the device)."""
    flags = ctypes.c_uint32(0)
    status = load().sbda_b200_device_status(ctypes.byref(flags), 1 if reset else 0)
    if status not in (SBDA_OK, SBDA_ERR_DEVICE):
        raise_for_status(status, "sbda_b200_device_status")
    return int(flags.value)
