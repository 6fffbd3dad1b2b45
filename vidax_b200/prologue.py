"""Fused pre-attention step on B200: QK RMSNorm + 3-D RoPE + head-slab pack.

Mirrors the part of vidax's DiT attention between the q/k/v projections and
the attention primitive:

* `rms_norm` / RMSNorm (src/vidax/core/attention.py:149-162),
* `rope3d_freqs` == `create_rope3d_freqs` (src/vidax/core/rope3d.py:44-86),
* `apply_rope3d` (src/vidax/core/rope3d.py:89-111),
* `attend` == the tail of Wan's attention block
  (src/vidax/models/wan/common/dit_layers.py:131-157 with tp_size 1):
  RMSNorm(dim) on q and k, reshape to heads, RoPE, then
  `sequence_parallel_self_attention` (rope_freqs given, sp axis bound) or
  `dot_product_attention`.

All of norm, reshape, RoPE and (under sequence parallelism) the Ulysses send
packing run as ONE launch of `vx_norm_rope_pack` over q, k and v: a single
HBM read and write per element instead of one per step.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib


class NormRopePackArgs(ctypes.Structure):
    _fields_ = [
        ("num_tensors", ctypes.c_int32),
        ("src", ctypes.c_void_p * 3),
        ("dst", ctypes.c_void_p * 3),
        ("src_stride", (ctypes.c_int64 * 3) * 3),
        ("norm_weight", ctypes.c_void_p * 3),
        ("per_head", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("post_scale", ctypes.c_float * 3),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("rope_stride", ctypes.c_int64),
        ("rope_mask", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("seq", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("groups", ctypes.c_int32),
        ("num_slices", ctypes.c_int32),
        ("slice_heads", ctypes.c_int32 * 8),
    ]


# ------------------------------------------------------------------ tables


def _axis_freqs(seq_len: int, dim: int, theta: float) -> Tuple[np.ndarray, np.ndarray]:
    """Per-position (cos, sin) of one axis in float32 (rope3d.py:33-41):
    inv_freq = 1 / theta^(2i / dim), angle = position * inv_freq. Computed
    with numpy's float32 power / cos / sin, the host math the reference's own
    formulas were pinned with."""
    inv = (np.float32(1.0) / np.power(np.float32(theta),
                                      np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)))
    ang = np.outer(np.arange(seq_len, dtype=np.float32), inv.astype(np.float32))
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope3d_freqs(t: int, h: int, w: int, head_dim: int, theta: float = 10000.0,
                 max_seq_len: int = 1024, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Wan's 3-D RoPE tables for a (t, h, w) token grid (rope3d.py:44-86):
    head_dim // 2 frequency pairs split c - 2*(c//3) / c//3 / c//3 over
    T / H / W. Returns (cos, sin), each (t*h*w, head_dim // 2) float32 in
    row-major (t, h, w) token order -- the reference's (1, S, 1, D/2) arrays
    without the broadcast axes. Built once per sequence on the host. Both are
    views of one (S, D) [cos | sin] buffer, the layout `norm_rope_pack` reads
    with one copy per token block; `pair_tables` gives that layout to other
    tables."""
    if head_dim % 2:
        raise ValueError("head_dim must be even")
    c = head_dim // 2
    dims = (c - 2 * (c // 3), c // 3, c // 3)
    if max(t, h, w) > max_seq_len:
        raise ValueError(f"grid {t}x{h}x{w} exceeds max_seq_len {max_seq_len}")
    tabs = [_axis_freqs(max_seq_len, 2 * d, theta) for d in dims]
    both = np.empty((t * h * w, 2 * c), dtype=np.float32)  # [cos | sin] per token
    for k in range(2):
        ft, fh, fw = (tab[k] for tab in tabs)
        both[:, k * c:(k + 1) * c] = np.concatenate([
            np.broadcast_to(ft[:t, None, None, :], (t, h, w, dims[0])),
            np.broadcast_to(fh[None, :h, None, :], (t, h, w, dims[1])),
            np.broadcast_to(fw[None, None, :w, :], (t, h, w, dims[2])),
        ], axis=-1).reshape(t * h * w, c)
    tab = torch.from_numpy(both)
    if device is not None:
        tab = tab.to(device)
    return tab[:, :c], tab[:, c:]


def ltx_default_rope_split(head_dim: int) -> Tuple[int, int, int]:
    """LTX-2.5's split of head_dim into (T, H, W) RoPE chunks
    (`_default_rope_dim_split`, src/vidax/models/ltx2_5/diffusion_vae.py:
    96-103): T gets (head_dim // 4) rounded down to even, H and W share the
    rest equally, and T gives up 2 more when that share would be odd."""
    d_t = (head_dim // 4) // 2 * 2
    d_hw = (head_dim - d_t) // 2
    if d_hw % 2:
        d_t -= 2
        d_hw = (head_dim - d_t) // 2
    return d_t, d_hw, d_hw


def ltx_rope_freqs(t: int, h: int, w: int, head_dim: int,
                   rope_split: Optional[Sequence[int]] = None, base: float = 10000.0,
                   device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """LTX-2.5's absolute split RoPE as (cos, sin) tables for a (t, h, w)
    token grid (`_rope_inv_freqs` / `_apply_abs_rope`, diffusion_vae.py:
    106-150). head_dim is split into (d_t, d_h, d_w) chunks (default
    `ltx_default_rope_split`); each chunk rotates its interleaved pairs at
    its axis's absolute position with inv_freq = 1 / base^(2i / d) (float64,
    rounded to float32) and angle = float32(position) * inv_freq in float32.
    Returns (cos, sin), each (t*h*w, head_dim // 2) float32, token-major in
    (t, h, w) order: pair p < d_t/2 uses the time position, the next d_h/2
    pairs the row, the last d_w/2 the column -- the interleaved-pair table
    `norm_rope_pack` applies."""
    split = tuple(int(x) for x in (rope_split or ltx_default_rope_split(head_dim)))
    if len(split) != 3 or sum(split) != head_dim or any(d <= 0 or d % 2 for d in split):
        raise ValueError(f"rope_split {split} must be three positive even sizes summing to "
                         f"head_dim {head_dim}")
    c = head_dim // 2
    per_axis = []
    for n, d in zip((t, h, w), split):
        inv = (1.0 / np.power(float(base), np.arange(0, d, 2, dtype=np.float64) / d)).astype(np.float32)
        ang = np.arange(n, dtype=np.float32)[:, None] * inv[None, :]
        per_axis.append((np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)))
    both = np.empty((t * h * w, 2 * c), dtype=np.float32)  # [cos | sin] per token
    dims = [d // 2 for d in split]
    for k in range(2):
        ft, fh, fw = (tab[k] for tab in per_axis)
        both[:, k * c:(k + 1) * c] = np.concatenate([
            np.broadcast_to(ft[:, None, None, :], (t, h, w, dims[0])),
            np.broadcast_to(fh[None, :, None, :], (t, h, w, dims[1])),
            np.broadcast_to(fw[None, None, :, :], (t, h, w, dims[2])),
        ], axis=-1).reshape(t * h * w, c)
    tab = torch.from_numpy(both)
    if device is not None:
        tab = tab.to(device)
    return tab[:, :c], tab[:, c:]


# ------------------------------------------------------------------ launch


def _weight(w: Optional[torch.Tensor], n: int, device) -> Optional[torch.Tensor]:
    if w is None:
        return None
    if w.numel() != n:
        raise ValueError(f"norm weight has {w.numel()} elements, expected {n}")
    return w.detach().reshape(n).to(device=device, dtype=torch.float32).contiguous()


def _rows(t: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    """(B, S, H*D) or (B, S, H, D) -> a (B, S, H, D) view (copy only when the
    feature axis is not contiguous)."""
    if t.dim() == 3:
        if t.stride(-1) != 1:
            t = t.contiguous()
        t = t.unflatten(-1, (heads, head_dim))
    if t.dim() != 4 or t.shape[2] != heads or t.shape[3] != head_dim:
        raise ValueError(f"expected (B, S, {heads}*{head_dim}) or (B, S, {heads}, {head_dim}), "
                         f"got {tuple(t.shape)}")
    if t.stride(-1) != 1 or t.data_ptr() % 16 or any(s % 8 for s in t.stride()[:3]):
        t = t.contiguous()
    return t


def norm_rope_pack(
    tensors: Sequence[torch.Tensor], heads: int, *,
    norm_weights: Sequence[Optional[torch.Tensor]] = (None, None, None),
    per_head: bool = False, eps: float = 1e-6,
    post_scale: Sequence[float] = (1.0, 1.0, 1.0),
    rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, rope_mask: int = 0b011,
    groups: int = 1, slices: Optional[Sequence[int]] = None,
    out: Optional[Sequence[torch.Tensor]] = None,
):
    """One launch over 1-3 tensors of (B, S, H*D) or (B, S, H, D) bf16.

    Returns one contiguous buffer per tensor of shape (B, groups*S*Hg*D) with
    Hg = ceil(heads / groups), laid out slice by slice as
    [slice j][group g][token s][head i < slices[j]][D] (see `slice_views`).
    groups = 1 and no slices gives plain (B, S, H, D) rows."""
    tensors = list(tensors)
    n = len(tensors)
    if not 1 <= n <= 3:
        raise ValueError("1 to 3 tensors")
    x0 = tensors[0]
    if not x0.is_cuda:
        raise ValueError("inputs must be CUDA tensors (this implementation has no CPU path)")
    D = x0.shape[-1] if x0.dim() == 4 else x0.shape[-1] // heads
    rows = [_rows(t, heads, D) for t in tensors]
    B, S = rows[0].shape[:2]
    for r in rows:
        if r.dtype != torch.bfloat16:
            raise NotImplementedError(f"dtype {r.dtype}: the kernel takes bfloat16")
        if r.shape != rows[0].shape or r.device != x0.device:
            raise ValueError("tensors must share shape and device")
    hg = -(-heads // groups)
    if out is None:
        out = [torch.empty((B, groups * S * hg * D), dtype=torch.bfloat16, device=x0.device)
               for _ in range(n)]
    a = NormRopePackArgs()
    a.num_tensors = n
    keep = []
    ncols = D if per_head else heads * D
    for i, (r, o) in enumerate(zip(rows, out)):
        if (not o.is_contiguous() or o.numel() != B * groups * S * hg * D
                or o.dtype != torch.bfloat16 or o.device != x0.device):
            raise ValueError("out buffers must be contiguous bf16 with B*groups*S*Hg*D "
                             "elements on the inputs' device")
        a.src[i], a.dst[i] = r.data_ptr(), o.data_ptr()
        for k in range(3):
            a.src_stride[i][k] = r.stride(k)
        w = _weight(norm_weights[i] if i < len(norm_weights) else None, ncols, x0.device)
        if w is not None:
            keep.append(w)
            a.norm_weight[i] = w.data_ptr()
        a.post_scale[i] = float(post_scale[i]) if i < len(post_scale) else 1.0
    a.per_head = int(bool(per_head))
    a.eps = eps
    if rope is not None and rope_mask:
        cos, sin = pair_tables(*rope, device=x0.device)
        if cos.shape != sin.shape or cos.shape[0] != S or cos.shape[-1] != D // 2:
            raise ValueError(f"rope tables must be ({S}, {D // 2}), got {tuple(cos.shape)}")
        keep += [cos, sin]
        a.rope_cos, a.rope_sin = cos.data_ptr(), sin.data_ptr()
        a.rope_stride = cos.stride(0)
        a.rope_mask = rope_mask
    a.batch, a.seq, a.heads, a.head_dim, a.groups = B, S, heads, D, groups
    if slices is not None:
        a.num_slices = len(slices)
        for j, hs in enumerate(slices):
            a.slice_heads[j] = hs
    lib = _lib.load()
    fn = lib.vx_norm_rope_pack
    fn.argtypes = [ctypes.POINTER(NormRopePackArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    stream = torch.cuda.current_stream(x0.device)
    _lib.check(fn(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)))
    for t in keep:  # tables / converted weights may be freed before the kernel runs
        t.record_stream(stream)
    return out


def pair_tables(cos: torch.Tensor, sin: torch.Tensor, device=None):
    """(cos, sin) as float32 views of one (S, D) [cos | sin] buffer on
    `device`: the kernel then fetches a token block's tables with one copy.
    Tables already in that layout are returned as they are."""
    cos = cos.to(device=device, dtype=torch.float32)
    sin = sin.to(device=device, dtype=torch.float32)
    half = cos.shape[-1]
    paired = (cos.dim() == 2 and cos.shape == sin.shape and cos.stride() == (2 * half, 1)
              and sin.stride() == cos.stride()
              and sin.data_ptr() == cos.data_ptr() + 4 * half and cos.data_ptr() % 16 == 0)
    if paired:
        return cos, sin
    both = torch.cat([cos.reshape(-1, half), sin.reshape(-1, half)], dim=1)
    return both[:, :half], both[:, half:]


def slice_views(buf: torch.Tensor, groups: int, seq: int, head_dim: int,
                slices: Sequence[int]):
    """Views (groups, seq, slices[j], D) of one batch item's packed buffer."""
    views, off = [], 0
    for hs in slices:
        n = groups * seq * hs * head_dim
        views.append(buf[off:off + n].view(groups, seq, hs, head_dim))
        off += n
    return views


def rms_norm_rope(x: torch.Tensor, weight: Optional[torch.Tensor],
                  rope: Optional[Tuple[torch.Tensor, torch.Tensor]], heads: int, *,
                  eps: float = 1e-6, per_head: bool = False, post_scale: float = 1.0) -> torch.Tensor:
    """RMSNorm (whole row or per head) then RoPE of one (B, S, H*D) or
    (B, S, H, D) tensor -> (B, S, H, D) bf16."""
    D = x.shape[-1] if x.dim() == 4 else x.shape[-1] // heads
    (o,) = norm_rope_pack([x], heads, norm_weights=[weight], per_head=per_head, eps=eps,
                          post_scale=[post_scale], rope=rope, rope_mask=1 if rope else 0)
    return o.view(x.shape[0], x.shape[1], heads, D)


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_heads: int, *,
           norm_q: Optional[torch.Tensor] = None, norm_k: Optional[torch.Tensor] = None,
           rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, eps: float = 1e-6,
           sp_axis_name: Optional[str] = None, scale: Optional[float] = None) -> torch.Tensor:
    """Wan self-attention after the q/k/v projections (dit_layers.py:137-157).

    q, k, v: (B, L, dim) projections -- with `sp_axis_name` this rank's
    token chunk (`chunk_by_rank` ownership) and `rope` the tables of those
    tokens' global positions. norm_q / norm_k: RMSNorm(dim) scales (None
    skips the norm, as qk_norm=False). Returns (B, L, dim)."""
    B, L, dim = q.shape
    D = dim // num_heads
    if sp_axis_name is not None:
        from .ulysses import _attend_sp  # local import: ulysses imports this module
        return _attend_sp(q, k, v, num_heads, norm_q, norm_k, rope, eps, sp_axis_name, scale)
    from .attention import flash_attention
    qs, ks, vs = norm_rope_pack([q, k, v], num_heads, norm_weights=[norm_q, norm_k, None],
                                eps=eps, rope=rope, rope_mask=0b011 if rope is not None else 0)
    shape = (B, L, num_heads, D)
    o = flash_attention(qs.view(shape), ks.view(shape), vs.view(shape),
                        D ** -0.5 if scale is None else scale)
    return o.reshape(B, L, dim)
