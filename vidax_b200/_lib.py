"""ctypes binding of libvidax_cuda.so (the C ABI in include/vidax_cuda.h).

The shared library is the product: every compute call of this package goes
through it. Loading fails loudly when it is missing -- there is no fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

VX_OK, VX_EINVAL, VX_EUNSUPPORTED, VX_ECUDA, VX_ENCCL, VX_ETIMEOUT = range(6)

_ERRNAMES = {
    VX_EINVAL: "VX_EINVAL",
    VX_EUNSUPPORTED: "VX_EUNSUPPORTED",
    VX_ECUDA: "VX_ECUDA",
    VX_ENCCL: "VX_ENCCL",
    VX_ETIMEOUT: "VX_ETIMEOUT",
}

#: Every symbol the public header declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "vx_version",
    "vx_last_error",
    "vx_device_status",
    "vx_attn_fwd",
    "vx_na3d_fwd",
    "vx_na3d_fwd_slab",
    "vx_na3d_window_start",
    "vx_na3d_tiling",
    "vx_ulysses_pack",
    "vx_ulysses_unpack",
    "vx_norm_rope_pack",
    "vx_ln_modulate",
    "vx_gated_residual",
    "vx_memcpy_rows_async",
    "vx_selftest_wait_timeout",
    "vx_comm_get_unique_id",
    "vx_comm_init",
    "vx_comm_wrap",
    "vx_comm_destroy",
    "vx_ulysses_workspace_size",
    "vx_ulysses_attn_fwd",
    "vx_ulysses_attn_fwd_static",
    "vx_ulysses_pack_peers",
    "vx_ulysses_unpack_peers",
    "vx_peer_barrier",
    "vx_ipc_get_handle",
    "vx_ipc_open",
    "vx_ipc_close",
)


class VxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_ERRNAMES.get(code, code)}: {msg}")
        self.code = code


class VxUnsupported(VxError, NotImplementedError):
    """A valid request the CUDA build does not implement (raised, never emulated)."""


class VxInvalid(VxError, ValueError):
    pass


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("batch", ctypes.c_int32),
        ("seq_q", ctypes.c_int32),
        ("seq_k", ctypes.c_int32),
        ("heads_q", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("kv_len", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("schedule", ctypes.c_int32),
    ]


VX_SCHED_STATIC, VX_SCHED_DYNAMIC = 0, 1


_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    """The in-tree library, or VIDAX_B200_LIB when set (an alternative build
    of the same sources, e.g. for tuning)."""
    return os.environ.get("VIDAX_B200_LIB") or _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Loads (building first if absent or stale and nvcc exists) the library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if path == _build.LIB_PATH and build_if_missing and _build.is_stale():
            try:
                _build.build()
            except RuntimeError:
                if not os.path.exists(path):
                    raise
        if not os.path.exists(path):
            raise ImportError(f"libvidax_cuda.so not found at {path}; run python -m vidax_b200.build")
        lib = ctypes.CDLL(path)
        lib.vx_version.restype = ctypes.c_int
        lib.vx_last_error.restype = ctypes.c_char_p
        lib.vx_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
        lib.vx_device_status.restype = ctypes.c_int
        lib.vx_attn_fwd.argtypes = [ctypes.POINTER(AttnArgs), ctypes.c_void_p]
        lib.vx_attn_fwd.restype = ctypes.c_int
        lib.vx_memcpy_rows_async.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_void_p]
        lib.vx_memcpy_rows_async.restype = ctypes.c_int
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc == VX_OK:
        return
    msg = (load().vx_last_error() or b"").decode(errors="replace")
    if rc == VX_EUNSUPPORTED:
        raise VxUnsupported(rc, msg)
    if rc == VX_EINVAL:
        raise VxInvalid(rc, msg)
    raise VxError(rc, msg)


def selftest_wait_timeout(limit_cycles: int = 2_000_000) -> int:
    """Runs the bounded-wait self-test kernel (see vx_selftest_wait_timeout)
    and returns the device status word it left (bit 16 set when the wait gave
    up as designed)."""
    lib = load()
    fn = lib.vx_selftest_wait_timeout
    fn.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_int)]
    fn.restype = ctypes.c_int
    out = ctypes.c_int(0)
    rc = fn(limit_cycles, ctypes.byref(out))
    if rc != VX_ETIMEOUT:
        check(rc if rc != VX_OK else VX_ECUDA)
    return out.value


def device_status(clear: bool = True) -> int:
    """Synchronises the current device and returns its kernel status word."""
    out = ctypes.c_int(0)
    check(load().vx_device_status(ctypes.byref(out), 1 if clear else 0))
    return out.value
