"""vidax's attention hot path as XLA custom calls (jax.ffi), for a JAX host.

`vidax_ffi.cc` (beside this file) holds XLA FFI handlers over the C ABI of
libvidax_cuda.so; this module compiles it against jaxlib's FFI headers and
registers the handlers, so vidax's JAX code can call the sm_100a kernels
under `jit` / `shard_map`:

    from vidax_b200 import jax_ffi
    jax_ffi.register()                     # builds libvidax_ffi.so on first use
    o = jax_ffi.dot_product_attention(q, k, v)          # (B, S, H, D) bf16 jax.Arrays
    o = jax_ffi.neighborhood_attention_3d(q, k, v, (5, 9, 9))
    o = jax_ffi.sequence_parallel_self_attention(q, k, v, "sp")   # inside shard_map

Targets (platform "CUDA"): vidax_attn_fwd, vidax_na3d_fwd, vidax_ulysses_pack,
vidax_ulysses_unpack. The Ulysses layer is pack -> XLA's all_to_all ->
attention -> all_to_all -> unpack: a JAX host gets the packed layout (the
exchange is one plain equal-split all-to-all per tensor) but not the torch
mirror's head-slice pipelining of the exchange against the kernel, which
needs streams the XLA program does not expose to a custom call.

JAX is not installed in this build image: `register()` raises ImportError
there, and nothing else in vidax_b200 imports this module.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
SHIM_SRC = os.path.join(HERE, "vidax_ffi.cc")
SHIM_LIB = os.path.join(PKG, "lib", "libvidax_ffi.so")
TARGETS = {
    "vidax_attn_fwd": "VidaxAttnFwd",
    "vidax_na3d_fwd": "VidaxNa3dFwd",
    "vidax_ulysses_pack": "VidaxUlyssesPack",
    "vidax_ulysses_unpack": "VidaxUlyssesUnpack",
}

_registered = False


def _jax():
    try:
        import jax  # noqa: F401
        import jax.ffi  # noqa: F401
    except ImportError as e:  # the build image has no JAX
        raise ImportError(
            "vidax_b200.jax_ffi needs jax (with jax.ffi) and jaxlib's FFI headers; "
            f"they are not importable here ({e}). Use the torch mirror (vidax_b200) or the "
            "C ABI (include/vidax_cuda.h) instead.") from e
    return jax


def build(force: bool = False) -> str:
    """Compiles vidax_ffi.cc into lib/libvidax_ffi.so against jax.ffi's
    headers, linked to libvidax_cuda.so (built first if needed)."""
    jax = _jax()
    from .. import build as lib_build
    lib_build.build()
    if (not force and os.path.exists(SHIM_LIB)
            and os.path.getmtime(SHIM_LIB) >= os.path.getmtime(SHIM_SRC)):
        return SHIM_LIB
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("a C++ compiler is needed to build the jax.ffi shim")
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(lib_build.nvcc_path())), "include")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-I" + jax.ffi.include_dir(),
           "-I" + lib_build.INCLUDE, "-I" + cuda_inc, SHIM_SRC, "-o", SHIM_LIB,
           "-L" + lib_build.LIB_DIR, "-lvidax_cuda", "-Wl,-rpath," + lib_build.LIB_DIR]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("building the jax.ffi shim failed:\n" + " ".join(cmd) + "\n"
                           + res.stdout + res.stderr)
    return SHIM_LIB


def register() -> None:
    """Builds (if needed) and registers every handler as a CUDA FFI target."""
    global _registered
    jax = _jax()
    if _registered:
        return
    shim = ctypes.CDLL(build())
    for target, symbol in TARGETS.items():
        jax.ffi.register_ffi_target(target, jax.ffi.pycapsule(getattr(shim, symbol)),
                                    platform="CUDA")
    _registered = True


def dot_product_attention(q, k, v, scale: Optional[float] = None):
    """vidax.core.attention.dot_product_attention without bias / mask
    (src/vidax/core/attention.py:467-533) as one custom call: (B, S, H, D)
    bf16, default scale head_dim^-0.5. Sharded inputs go through shard_map
    (as vidax wraps its Mosaic kernel, attention.py:296-318)."""
    jax = _jax()
    register()
    sm_scale = q.shape[-1] ** -0.5 if scale is None else scale
    return jax.ffi.ffi_call("vidax_attn_fwd", jax.ShapeDtypeStruct(q.shape, q.dtype))(
        q, k, v, scale=float(sm_scale))


local_attention = dot_product_attention


def neighborhood_attention_3d(q, k, v, kernel_size: Sequence[int], round_logits: bool = True):
    """vidax's NA primitive (ltx2_5/diffusion_vae.py:179-234): q pre-scaled
    by the caller, clamped windows; round_logits rounds q.k to bf16 as the
    reference's bf16 einsum does."""
    jax = _jax()
    register()
    import numpy as np
    kt, kh, kw = (int(x) for x in kernel_size)
    return jax.ffi.ffi_call("vidax_na3d_fwd", jax.ShapeDtypeStruct(q.shape, q.dtype))(
        q, k, v, kt=np.int32(kt), kh=np.int32(kh), kw=np.int32(kw),
        round_logits=np.int32(1 if round_logits else 0))


def sequence_parallel_self_attention(q, k, v, sp_axis_name: str, scale: Optional[float] = None):
    """DeepSpeed-Ulysses inside shard_map (attention.py:341-388): per batch
    item, pack -> all_to_all (tokens -> heads) -> attention -> all_to_all
    back -> unpack. Heads must divide the axis size, as in the reference."""
    jax = _jax()
    register()
    import jax.numpy as jnp
    import numpy as np
    axis_size = getattr(jax.lax, "axis_size", None)
    P = int(axis_size(sp_axis_name) if axis_size else jax.lax.psum(1, sp_axis_name))
    B, S_loc, H, D = q.shape
    if H % P:
        raise NotImplementedError("heads must divide the sp axis size (as the reference's tiled all_to_all)")
    Hg = H // P
    sm_scale = D ** -0.5 if scale is None else scale

    def pack(x):  # (S_loc, H, D) -> (P, S_loc, Hg, D)
        return jax.ffi.ffi_call("vidax_ulysses_pack",
                                jax.ShapeDtypeStruct((P, S_loc, Hg, D), x.dtype))(
            x, groups=np.int32(P), heads=np.int32(H))

    def unpack(x):  # (P, S_loc, Hg, D) -> (S_loc, H, D)
        return jax.ffi.ffi_call("vidax_ulysses_unpack",
                                jax.ShapeDtypeStruct((S_loc, H, D), x.dtype))(
            x, groups=np.int32(P), heads=np.int32(H))

    outs = []
    for b in range(B):
        recv = [jax.lax.all_to_all(pack(t[b]), sp_axis_name, 0, 0, tiled=True)
                for t in (q, k, v)]
        qh, kh, vh = (r.reshape(1, P * S_loc, Hg, D) for r in recv)
        o = dot_product_attention(qh, kh, vh, sm_scale).reshape(P, S_loc, Hg, D)
        outs.append(unpack(jax.lax.all_to_all(o, sp_axis_name, 0, 0, tiled=True)))
    return jnp.stack(outs)
