"""C ABI checks that need no GPU: the library loads, exports every symbol the
public header declares, validates arguments before touching the device, and
its host-side window-start helper equals the reference's _window_start."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vidax_cuda.h")


@pytest.fixture(scope="module")
def lib():
    from vidax_b200 import _lib
    return _lib.load()


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(vx_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("vx_attn_fwd", "vx_na3d_fwd", "vx_ulysses_pack", "vx_ulysses_unpack",
              "vx_last_error", "vx_device_status", "vx_version", "vx_na3d_window_start"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    from vidax_b200 import _lib
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in include/vidax_cuda.h but not exported"
    assert set(_lib.EXPORTED_SYMBOLS) <= set(declared_symbols())


def test_version_and_last_error(lib):
    assert lib.vx_version() >= 100
    assert isinstance(lib.vx_last_error(), bytes)


def test_argument_validation_without_device(lib):
    from vidax_b200 import _lib
    assert lib.vx_attn_fwd(None, None) == _lib.VX_EINVAL
    a = _lib.AttnArgs()
    a.batch, a.seq_q, a.seq_k, a.heads_q, a.heads_kv, a.head_dim, a.scale = 1, 8, 8, 2, 2, 96, 0.1
    assert lib.vx_attn_fwd(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED
    assert b"head_dim" in lib.vx_last_error()
    a.head_dim, a.heads_kv = 128, 3
    assert lib.vx_attn_fwd(ctypes.byref(a), None) == _lib.VX_EINVAL
    a.heads_kv, a.scale = 2, -1.0
    assert lib.vx_attn_fwd(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED
    a.scale, a.seq_q = 0.1, 0
    assert lib.vx_attn_fwd(ctypes.byref(a), None) == _lib.VX_OK   # empty problem: no launch


def test_na3d_window_start_matches_reference(lib):
    from vidax_b200.neighborhood import window_start
    g = np.load(os.path.join(ROOT, "tests", "golden", "na3d_reference.npz"))
    for L, k, st in zip(g["ws_length"], g["ws_kernel"], g["ws_start"]):
        assert np.array_equal(window_start(int(L), int(k)), st[:L]), (L, k)


def test_pack_validation(lib):
    from vidax_b200.ulysses import HeadSlabArgs
    from vidax_b200 import _lib
    fn = lib.vx_ulysses_pack
    fn.argtypes = [ctypes.POINTER(HeadSlabArgs), ctypes.c_void_p]
    a = HeadSlabArgs()
    a.num_tensors = 4
    assert fn(ctypes.byref(a), None) == _lib.VX_EINVAL
    a.num_tensors, a.seq, a.heads, a.head_dim, a.groups = 1, 4, 4, 96, 2
    assert fn(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED


def test_norm_rope_pack_validation_without_device(lib):
    from vidax_b200 import _lib
    from vidax_b200.prologue import NormRopePackArgs
    assert lib.vx_norm_rope_pack(None, None) == _lib.VX_EINVAL
    a = NormRopePackArgs()
    a.num_tensors, a.batch, a.seq, a.heads, a.head_dim, a.groups = 1, 1, 4, 2, 96, 1
    assert lib.vx_norm_rope_pack(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED
    a.head_dim = 128
    a.heads = 65   # 8320 features: above the 8192 a warp holds
    assert lib.vx_norm_rope_pack(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED
    a.heads, a.groups, a.num_slices = 5, 2, 2
    a.slice_heads[0], a.slice_heads[1] = 1, 1        # sums to 2, ceil(5 / 2) = 3
    assert lib.vx_norm_rope_pack(ctypes.byref(a), None) == _lib.VX_EINVAL
    assert b"slice_heads" in lib.vx_last_error()
    a.slice_heads[1] = 2
    a.rope_mask = 1                                  # rotation without tables
    assert lib.vx_norm_rope_pack(ctypes.byref(a), None) == _lib.VX_EINVAL
    a.rope_mask = 0
    assert lib.vx_norm_rope_pack(ctypes.byref(a), None) == _lib.VX_EINVAL  # NULL src/dst
    a.seq = 0
    a.src[0] = a.dst[0] = 4096
    assert lib.vx_norm_rope_pack(ctypes.byref(a), None) == _lib.VX_OK     # empty: no launch
