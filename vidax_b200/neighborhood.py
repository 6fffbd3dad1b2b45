"""3-D neighborhood attention on B200 (sm_100a), vidax's NA primitive.

Mirrors `vidax.models.ltx2_5.diffusion_vae.neighborhood_attention_3d(q, k, v,
kernel_size)` (src/vidax/models/ltx2_5/diffusion_vae.py:179-234): q, k, v are
(B, T, H, W, NH, HD), q already scaled by the caller (diffusion_vae.py:265),
windows are NATTEN's clamped ("shifted") windows of `_window_start`
(diffusion_vae.py:152-164). The whole primitive is one launch of the
neighborhood variant of the tcgen05 attention kernel.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib


class Na3dArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 5),
        ("k_stride", ctypes.c_int64 * 5),
        ("v_stride", ctypes.c_int64 * 5),
        ("o_stride", ctypes.c_int64 * 5),
        ("batch", ctypes.c_int32),
        ("T", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("W", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("kernel_t", ctypes.c_int32),
        ("kernel_h", ctypes.c_int32),
        ("kernel_w", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("round_logits", ctypes.c_int32),
        ("q_box", ctypes.c_int32 * 3),
        ("pair_axis", ctypes.c_int32),
        ("kv_tile", ctypes.c_int32 * 3),
    ]


def tiling(grid: Sequence[int], kernel_size: Sequence[int], head_dim: int) -> dict:
    """The tiling the kernel picks for a (T, H, W) grid and window: query
    box, pairing ("t" / "h" / "w" box pairs or "heads") and key tile."""
    qb = (ctypes.c_int32 * 3)()
    kv = (ctypes.c_int32 * 3)()
    pair = ctypes.c_int32(0)
    fn = _lib.load().vx_na3d_tiling
    fn.argtypes = [ctypes.c_int32] * 7 + [ctypes.POINTER(ctypes.c_int32 * 3),
                                          ctypes.POINTER(ctypes.c_int32),
                                          ctypes.POINTER(ctypes.c_int32 * 3)]
    fn.restype = ctypes.c_int
    _lib.check(fn(*[int(x) for x in grid], *[int(x) for x in kernel_size], int(head_dim),
                  ctypes.byref(qb), ctypes.byref(pair), ctypes.byref(kv)))
    return {"q_box": tuple(qb), "pair": ("t", "h", "w", "heads")[pair.value],
            "kv_tile": tuple(kv)}


def window_start(length: int, kernel: int) -> np.ndarray:
    """Per-index window start along one axis, computed by the library
    (the `_window_start` contract, diffusion_vae.py:152-164)."""
    out = (ctypes.c_int32 * length)()
    lib = _lib.load()
    fn = lib.vx_na3d_window_start
    fn.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
    fn.restype = ctypes.c_int
    _lib.check(fn(length, kernel, out))
    return np.frombuffer(out, dtype=np.int32).copy()


def _check6(name: str, t: torch.Tensor) -> None:
    if t.dim() != 6:
        raise ValueError(f"{name} must be (B, T, H, W, NH, HD), got {tuple(t.shape)}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this implementation has no CPU path)")
    if t.dtype != torch.bfloat16:
        raise NotImplementedError(f"{name}.dtype={t.dtype}: the sm_100a kernel takes bfloat16")


def _ready(t: torch.Tensor) -> torch.Tensor:
    st = t.stride()
    ok = (st[5] == 1 and t.data_ptr() % 16 == 0 and all(s > 0 and s % 8 == 0 for s in st[:5])
          and (t.shape[0] == 1 or st[0] == t.shape[1] * st[1]))
    return t if ok else t.contiguous()


def neighborhood_attention_3d(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kernel_size: Sequence[int],
    *, scale: float = 1.0, round_logits: bool = False,
    q_box: Optional[Tuple[int, int, int]] = None, pair_axis: int = 0,
    kv_tile: Optional[Tuple[int, int, int]] = None,
) -> torch.Tensor:
    """3-D neighborhood attention over (B, T, H, W, NH, HD) bf16 tensors.

    Returns (B, T, H, W, NH, HD). `scale` multiplies q.k (vidax pre-scales q,
    hence 1.0). `round_logits=True` rounds each q.k to bf16 before the fp32
    softmax, as the reference's bf16 einsum does (diffusion_vae.py:222).
    `q_box` / `pair_axis` / `kv_tile` override the kernel's tiling (tuning
    only; pair_axis 0-2 pairs two boxes adjacent along t / h / w, 3 pairs two
    heads of one box at head_dim 64; kv_tile is the key tile box, (2, 4, 16)
    unless head pairs take (4, 2, 16), (2, 8, 8) or (4, 4, 8)).
    """
    return _na3d(q, k, v, kernel_size, scale, round_logits, q_box, pair_axis, None, kv_tile)


class Na3dSlab(ctypes.Structure):
    _fields_ = [
        ("T_global", ctypes.c_int32),
        ("q_t0", ctypes.c_int32),
        ("kv_t0", ctypes.c_int32),
        ("T_kv", ctypes.c_int32),
    ]


def neighborhood_attention_3d_slab(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kernel_size: Sequence[int],
    *, t_global: int, q_t0: int, kv_t0: int, scale: float = 1.0, round_logits: bool = False,
) -> torch.Tensor:
    """Neighborhood attention of one time slab: q holds frames
    [q_t0, q_t0 + T) of a `t_global`-frame grid, k / v frames
    [kv_t0, kv_t0 + T_kv), which must cover every window of those queries.
    Windows clamp to the global grid, so the slab's output equals the same
    frames of the unsharded call (`vx_na3d_fwd_slab`)."""
    slab = Na3dSlab()
    slab.T_global, slab.q_t0, slab.kv_t0, slab.T_kv = t_global, q_t0, kv_t0, k.shape[1]
    return _na3d(q, k, v, kernel_size, scale, round_logits, None, 0, slab)


def _na3d(q, k, v, kernel_size, scale, round_logits, q_box, pair_axis, slab, kv_tile=None):
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check6(name, t)
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must live on the same device")
    B, T, H, W, NH, HD = q.shape
    kv_frames = k.shape[1] if slab is not None else T
    if (k.shape[0] != B or k.shape[1] != kv_frames or k.shape[2:4] != q.shape[2:4]
            or v.shape != k.shape or k.shape[5] != HD):
        raise ValueError(f"q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} disagree")
    kt, kh, kw = (int(x) for x in kernel_size)
    q, k, v = _ready(q), _ready(k), _ready(v)
    out = torch.empty((B, T, H, W, NH, HD), dtype=torch.bfloat16, device=q.device)
    a = Na3dArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    for dst, t in ((a.q_stride, q), (a.k_stride, k), (a.v_stride, v), (a.o_stride, out)):
        for i in range(5):
            dst[i] = t.stride(i)
    a.batch, a.T, a.H, a.W = B, T, H, W
    a.heads, a.heads_kv, a.head_dim = NH, k.shape[4], HD
    a.kernel_t, a.kernel_h, a.kernel_w = kt, kh, kw
    a.scale = float(scale)
    a.round_logits = 1 if round_logits else 0
    if q_box is not None:
        a.q_box[0], a.q_box[1], a.q_box[2] = q_box
        a.pair_axis = pair_axis
        if kv_tile is not None:
            a.kv_tile[0], a.kv_tile[1], a.kv_tile[2] = kv_tile
    lib = _lib.load()
    with torch.cuda.device(q.device):
        s = torch.cuda.current_stream(q.device)
        if slab is None:
            fn = lib.vx_na3d_fwd
            fn.argtypes = [ctypes.POINTER(Na3dArgs), ctypes.c_void_p]
            fn.restype = ctypes.c_int
            _lib.check(fn(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)))
        else:
            fn = lib.vx_na3d_fwd_slab
            fn.argtypes = [ctypes.POINTER(Na3dArgs), ctypes.POINTER(Na3dSlab), ctypes.c_void_p]
            fn.restype = ctypes.c_int
            _lib.check(fn(ctypes.byref(a), ctypes.byref(slab), ctypes.c_void_p(s.cuda_stream)))
    return out


def bf16_scalar(x: float) -> float:
    """`x` rounded to bf16 (round to nearest even): what a Python scalar
    becomes when JAX multiplies it into a bf16 array (weak typing)."""
    return float(torch.tensor(x, dtype=torch.float32).bfloat16().float())


def ltx_neighborhood_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kernel_size: Sequence[int], *,
    norm_q: torch.Tensor, norm_k: torch.Tensor, eps: float = 1e-6,
    rope_split: Optional[Sequence[int]] = None, rope_base: float = 10000.0,
    rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
) -> torch.Tensor:
    """LTX-2.5's neighborhood attention between its projections
    (`NeighborhoodAttention3D.__call__`, src/vidax/models/ltx2_5/
    diffusion_vae.py:252-284, from after to_q / to_k / to_v to before
    to_out): per-head RMSNorm of q and k (weights `norm_q` / `norm_k`,
    head_dim floats, src/vidax/core/attention.py:149-162), q scaled by
    head_dim^-0.5 in bf16 (:265; JAX rounds the scalar to bf16 first),
    LTX's absolute split RoPE on q and k (:267-275, tables from
    `ltx_rope_freqs` unless `rope` is given), then the NA primitive (:277).

    q, k, v: (B, T, H, W, NH, HD) bf16 projections. The norms, the scale and
    the rotation of q and k run as one `vx_norm_rope_pack` launch (one HBM
    read and write of q and k), then one `vx_na3d_fwd` launch. Returns
    (B, T, H, W, NH, HD) bf16."""
    from .prologue import ltx_rope_freqs, norm_rope_pack
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check6(name, t)
    if not (q.shape == k.shape == v.shape):
        raise ValueError("q, k, v must have the same (B, T, H, W, NH, HD) shape")
    B, T, H, W, NH, HD = q.shape
    if rope is None:
        rope = ltx_rope_freqs(T, H, W, HD, rope_split, rope_base, device=q.device)
    rows = [t.reshape(B, T * H * W, NH, HD) for t in (q, k)]
    qr, kr = norm_rope_pack(rows, NH, norm_weights=[norm_q, norm_k], per_head=True, eps=eps,
                            post_scale=[bf16_scalar(HD ** -0.5), 1.0], rope=rope,
                            rope_mask=0b11)
    shape = (B, T, H, W, NH, HD)
    return neighborhood_attention_3d(qr.view(shape), kr.view(shape), v, kernel_size)


def na3d_flops(B: int, T: int, H: int, W: int, NH: int, HD: int, kernel_size) -> float:
    """Algorithmic FLOPs, 4 * queries * |window| * HD * NH (window clamped to the grid)."""
    kt, kh, kw = (min(a, b) for a, b in zip(kernel_size, (T, H, W)))
    return 4.0 * B * T * H * W * kt * kh * kw * HD * NH
