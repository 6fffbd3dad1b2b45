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


def test_na3d_validation_without_device(lib):
    from vidax_b200 import _lib
    from vidax_b200.neighborhood import Na3dArgs, Na3dSlab
    fn = lib.vx_na3d_fwd
    fn.argtypes = [ctypes.POINTER(Na3dArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    slab_fn = lib.vx_na3d_fwd_slab
    slab_fn.argtypes = [ctypes.POINTER(Na3dArgs), ctypes.POINTER(Na3dSlab), ctypes.c_void_p]
    slab_fn.restype = ctypes.c_int
    assert fn(None, None) == _lib.VX_EINVAL
    a = Na3dArgs()
    a.batch, a.T, a.H, a.W, a.heads, a.heads_kv, a.head_dim = 1, 3, 4, 5, 2, 2, 128
    a.kernel_t, a.kernel_h, a.kernel_w, a.scale = 3, 3, 3, 1.0
    a.heads_kv = 3                                   # 2 % 3 != 0
    assert fn(ctypes.byref(a), None) == _lib.VX_EINVAL
    a.heads_kv, a.kernel_h = 2, 0
    assert fn(ctypes.byref(a), None) == _lib.VX_EINVAL
    assert b"kernel" in lib.vx_last_error()
    a.kernel_h, a.head_dim = 3, 96
    assert fn(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED
    a.head_dim, a.scale = 64, 0.0
    assert fn(ctypes.byref(a), None) == _lib.VX_EUNSUPPORTED
    a.scale, a.T = 1.0, 0
    assert fn(ctypes.byref(a), None) == _lib.VX_OK    # empty grid: no launch
    a.T = 3
    assert fn(ctypes.byref(a), None) == _lib.VX_EINVAL  # o is NULL
    assert slab_fn(ctypes.byref(a), None, None) == _lib.VX_EINVAL


def test_glue_and_copy_validation_without_device(lib):
    from vidax_b200 import _lib
    null = ctypes.c_void_p(None)
    i64, i32 = ctypes.c_int64, ctypes.c_int32

    def ln(rows, dim, rpb, x=None, y=None, w=None, b=None):
        return lib.vx_ln_modulate(ctypes.c_void_p(x), ctypes.c_void_p(y), ctypes.c_void_p(w),
                                  ctypes.c_void_p(b), null, null, i64(rows), i32(dim), i32(rpb),
                                  ctypes.c_float(1e-6), null)
    assert ln(8, 6, 8) == _lib.VX_EINVAL            # dim not a multiple of 4
    assert ln(8, 8, 3) == _lib.VX_EINVAL            # rows not a multiple of rows_per_batch
    assert ln(0, 8, 1) == _lib.VX_OK                # empty: no launch
    assert ln(8, 8, 8) == _lib.VX_EINVAL            # x / y NULL
    assert ln(8, 8, 8, x=4096, y=8192, w=4096) == _lib.VX_EINVAL  # w without b
    assert ln(8, 8, 8, x=4100, y=8192) == _lib.VX_EINVAL          # misaligned x

    def gr(rows, dim, rpb, x=None, y=None):
        return lib.vx_gated_residual(ctypes.c_void_p(x), ctypes.c_void_p(y), null, i64(rows),
                                     i32(dim), i32(rpb), null)
    assert gr(8, 12, 8) == _lib.VX_EINVAL           # dim not a multiple of 8
    assert gr(0, 8, 1) == _lib.VX_OK
    assert gr(8, 8, 8) == _lib.VX_EINVAL            # NULL
    assert gr(8, 8, 8, x=4112, y=8192) == _lib.VX_EINVAL  # x not 32-byte aligned

    cp = lib.vx_memcpy_rows_async
    assert cp(None, 0, None, 0, 0, 5, None) == _lib.VX_OK       # nothing to copy
    assert cp(None, 64, None, 64, 64, 5, None) == _lib.VX_EINVAL
    assert cp(4096, 32, 8192, 64, 64, 5, None) == _lib.VX_EINVAL  # dst pitch < row bytes

    st = lib.vx_selftest_wait_timeout
    st.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_int)]
    st.restype = ctypes.c_int
    assert st(0, None) == _lib.VX_EINVAL
    assert st(5_000_000_000, None) == _lib.VX_EINVAL


def test_jax_ffi_shim_declares_every_target_and_fails_clearly_without_jax():
    """The jax.ffi shim: every registered target names a handler the C++
    source defines; without JAX (this image) register() raises ImportError
    with a clear message instead of failing later."""
    import importlib.util
    import re
    from vidax_b200 import jax_ffi
    src = open(jax_ffi.SHIM_SRC).read()
    handlers = set(re.findall(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\((\w+),", src))
    assert set(jax_ffi.TARGETS.values()) == handlers
    for fn in ("vx_attn_fwd", "vx_na3d_fwd", "vx_ulysses_pack", "vx_ulysses_unpack"):
        assert fn + "(" in src
    if importlib.util.find_spec("jax") is None:
        with pytest.raises(ImportError, match="jax"):
            jax_ffi.register()


def test_ulysses_layer_workspace_size_without_device(lib):
    """vx_ulysses_workspace_size is host arithmetic: 256 bytes + 8 slabs of
    world x S_loc x ceil(H / world) x D bf16 (q, k, v sent and received, the
    attention output sent and received), each padded to 256 bytes."""
    from vidax_b200.ulysses_capi import UlyssesArgs
    a = UlyssesArgs()
    a.batch, a.seq_local, a.heads, a.head_dim = 1, 9450, 40, 128
    n = ctypes.c_int64(0)
    f = lib.vx_ulysses_workspace_size
    f.argtypes = [ctypes.POINTER(UlyssesArgs), ctypes.c_int32, ctypes.POINTER(ctypes.c_int64)]
    f.restype = ctypes.c_int
    assert f(ctypes.byref(a), 8, ctypes.byref(n)) == 0
    assert n.value == 256 + 8 * 8 * 9450 * 5 * 128 * 2
    a.heads = 12  # 12 heads on 8 ranks: ceil -> 2 per rank (zero heads)
    assert f(ctypes.byref(a), 8, ctypes.byref(n)) == 0
    assert n.value == 256 + 8 * (-(-(8 * 9450 * 2 * 128 * 2) // 256) * 256)
    assert f(ctypes.byref(a), 0, ctypes.byref(n)) != 0


def test_peer_exchange_validation_without_device(lib):
    """The peer forms of the slab kernels, the flag barrier and the IPC
    helpers reject bad arguments before touching a device."""
    from vidax_b200.ulysses_peer import PeerBarrierArgs, PeerSlabArgs
    f = lib.vx_ulysses_pack_peers
    f.argtypes = [ctypes.POINTER(PeerSlabArgs), ctypes.c_void_p]
    f.restype = ctypes.c_int
    a = PeerSlabArgs()
    a.slab.num_tensors, a.slab.seq, a.slab.heads, a.slab.head_dim = 1, 16, 16, 128
    a.slab.src[0] = 4096
    a.slab.stride[0][0], a.slab.stride[0][1] = 16 * 128, 128
    a.slab.groups = 9
    assert f(ctypes.byref(a), None) == 2            # more than 8 groups: VX_EUNSUPPORTED
    a.slab.groups = 2
    assert f(ctypes.byref(a), None) == 1            # peer addresses missing: VX_EINVAL
    a.peer[0][0], a.peer[0][1] = 4096, 4104         # second one not 16-byte aligned
    assert f(ctypes.byref(a), None) == 1
    a.peer[0][1] = 8192
    a.max_ctas = -1
    assert f(ctypes.byref(a), None) == 1
    b = lib.vx_peer_barrier
    b.argtypes = [ctypes.POINTER(PeerBarrierArgs), ctypes.c_void_p]
    b.restype = ctypes.c_int
    ba = PeerBarrierArgs()
    ba.world, ba.rank = 9, 0
    assert b(ctypes.byref(ba), None) == 1
    ba.world, ba.rank = 2, 2
    assert b(ctypes.byref(ba), None) == 1
    ba.rank = 0
    assert b(ctypes.byref(ba), None) == 1           # NULL flag arrays
    g = lib.vx_ipc_get_handle
    g.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]
    g.restype = ctypes.c_int
    assert g(None, ctypes.create_string_buffer(64), ctypes.byref(ctypes.c_int64())) == 1


def test_na3d_tiling_choices_without_device(lib):
    """vx_na3d_tiling is host arithmetic (the kernel's time model). On these
    shapes its picks were also the fastest of the tilings timed on a B200:
    box pairs along h at head_dim 128 (cfg4), head pairs at head_dim 64 with
    the key tile per window (LTX-2.5 decoder stages)."""
    from vidax_b200.neighborhood import tiling
    assert tiling((21, 30, 52), (5, 9, 9), 128) == {"q_box": (2, 8, 8), "pair": "h",
                                                    "kv_tile": (2, 4, 16)}
    assert tiling((32, 64, 96), (3, 5, 5), 64) == {"q_box": (2, 16, 4), "pair": "heads",
                                                   "kv_tile": (4, 4, 8)}
    assert tiling((16, 32, 48), (3, 7, 7), 64) == {"q_box": (2, 8, 8), "pair": "heads",
                                                   "kv_tile": (4, 2, 16)}
    assert tiling((32, 64, 96), (11, 11, 11), 64) == {"q_box": (8, 4, 4), "pair": "heads",
                                                      "kv_tile": (2, 4, 16)}
    # head_dim 128 never takes head pairs (their K / V stages do not fit)
    assert tiling((32, 64, 96), (3, 5, 5), 128)["pair"] != "heads"
    from vidax_b200._lib import VxError
    with pytest.raises(VxError):
        tiling((0, 4, 4), (3, 3, 3), 64)
    with pytest.raises(VxError):
        tiling((4, 4, 4), (3, 3, 3), 96)
