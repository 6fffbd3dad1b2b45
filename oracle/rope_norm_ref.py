"""CPU restatement of Wan's pre-attention steps -- TEST INFRASTRUCTURE ONLY.

Parity oracle for the fused QK-RMSNorm + 3-D RoPE + head-slab pack kernel.
Restates:

* `RMSNorm.__call__` (src/vidax/core/attention.py:149-162): x in float32,
  var = mean(x^2) over the whole feature axis, normed = x * rsqrt(var + eps),
  cast back to the input dtype (bf16), then multiplied by the weight cast
  to bf16 (a bf16 x bf16 product, rounded to bf16);
* `create_rope3d_freqs` (src/vidax/core/rope3d.py:44-86): head_dim // 2
  frequency pairs split T / H / W as c - 2*(c//3), c//3, c//3; each axis's
  angles are position * theta^(-2i/dim_axis) in float32;
* `apply_rope3d` (src/vidax/core/rope3d.py:89-111): adjacent (even, odd)
  pairs rotated in float32, out = (x1 c - x2 s, x2 c + x1 s), cast to bf16.

Pinned against the reference's own `create_rope3d_freqs` / `apply_rope3d`
executed under the numpy shim (tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np

from .attention_ref import to_bf16


def rms_norm(x, weight, eps=1e-6):
    """x: (..., dim) float32 holding bf16 values; weight (dim,). Returns bf16 values as float32."""
    x = np.asarray(x, np.float32)
    var = np.mean(np.square(x), axis=-1, keepdims=True, dtype=np.float32)
    normed = x * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))
    return to_bf16(to_bf16(normed) * to_bf16(np.asarray(weight, np.float32)))


def _axis_freqs(seq_len, dim, theta=10000.0):
    inv = (1.0 / np.power(np.float32(theta),
                          np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim))).astype(np.float32)
    ang = np.outer(np.arange(seq_len, dtype=np.float32), inv).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope3d_freqs(t, h, w, head_dim, theta=10000.0, max_seq_len=1024):
    """(cos, sin), each (t*h*w, head_dim // 2) float32."""
    c = head_dim // 2
    dt, dh, dw = c - 2 * (c // 3), c // 3, c // 3
    ct, st = _axis_freqs(max_seq_len, 2 * dt, theta)
    ch, sh = _axis_freqs(max_seq_len, 2 * dh, theta)
    cw, sw = _axis_freqs(max_seq_len, 2 * dw, theta)

    def grid(ft, fh, fw):
        gt = np.broadcast_to(ft[:t, None, None, :], (t, h, w, dt))
        gh = np.broadcast_to(fh[None, :h, None, :], (t, h, w, dh))
        gw = np.broadcast_to(fw[None, None, :w, :], (t, h, w, dw))
        return np.concatenate([gt, gh, gw], axis=-1).reshape(t * h * w, c)

    return grid(ct, ch, cw), grid(st, sh, sw)


def apply_rope3d(x, cos, sin):
    """x: (B, S, H, D) float32 holding bf16 values; cos/sin (S, D//2)."""
    x = np.asarray(x, np.float32)
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    x1, x2 = x[..., 0::2], x[..., 1::2]
    o1 = x1 * c - x2 * s
    o2 = x2 * c + x1 * s
    return to_bf16(np.stack([o1, o2], axis=-1).reshape(x.shape))


def norm_rope(x, weight, cos, sin, heads, eps=1e-6):
    """Wan's attend pre-processing for q or k: (B, S, dim) -> (B, S, H, D)."""
    B, S, dim = x.shape
    y = rms_norm(x, weight, eps).reshape(B, S, heads, dim // heads)
    return apply_rope3d(y, cos, sin)


# ---------------------------------------------------------------- LTX-2.5
def ltx_default_rope_split(head_dim):
    """`_default_rope_dim_split` (src/vidax/models/ltx2_5/diffusion_vae.py:96-103)."""
    d_t = (head_dim // 4) // 2 * 2
    d_hw = (head_dim - d_t) // 2
    if d_hw % 2 != 0:
        d_t -= 2
        d_hw = (head_dim - d_t) // 2
    return d_t, d_hw, d_hw


def ltx_inv_freqs(dim, base=10000.0):
    """`_rope_inv_freqs` (diffusion_vae.py:106-109): float64 formula, float32 result."""
    return (1.0 / np.power(float(base), np.arange(0, dim, 2, dtype=np.float64) / dim)).astype(np.float32)


def ltx_abs_rope(x, split=None, base=10000.0):
    """`_apply_abs_rope` (diffusion_vae.py:112-150) on x (B, T, H, W, NH, HD)
    float32 holding bf16 values: head_dim split into (d_t, d_h, d_w) chunks,
    chunk a's interleaved pairs rotated by float32(position_a) * inv_freq in
    float32, (e, o) -> (e c - o s, e s + o c), the result rounded to bf16."""
    x = np.asarray(x, np.float32)
    HD = x.shape[-1]
    split = tuple(split or ltx_default_rope_split(HD))
    outs, off = [], 0
    for axis, d in zip((1, 2, 3), split):
        xc = x[..., off:off + d]
        off += d
        pairs = xc.reshape(xc.shape[:-1] + (d // 2, 2))
        xe, xo = pairs[..., 0], pairs[..., 1]
        pos = np.arange(x.shape[axis], dtype=np.float32)
        ang = pos[:, None] * ltx_inv_freqs(d, base)[None, :]
        bshape = [1] * xc.ndim
        bshape[axis] = pos.shape[0]
        bshape[-1] = d // 2
        c = np.cos(ang).astype(np.float32).reshape(bshape)
        s = np.sin(ang).astype(np.float32).reshape(bshape)
        re = xe * c - xo * s
        ro = xe * s + xo * c
        outs.append(np.stack([re, ro], axis=-1).reshape(xc.shape))
    return to_bf16(np.concatenate(outs, axis=-1))


def ltx_na_prologue(q, k, wq, wk, eps=1e-6, split=None, base=10000.0):
    """The steps of NeighborhoodAttention3D.__call__ between the projections
    and the NA primitive (diffusion_vae.py:263-275): per-head RMSNorm of q and
    k, q * head_dim^-0.5 in bf16 (the scalar rounded to bf16, JAX's weak
    typing), absolute RoPE on both. Returns (q, k) float32 holding bf16."""
    HD = np.asarray(q).shape[-1]
    qn = rms_norm(q, wq, eps)
    kn = rms_norm(k, wk, eps)
    c = np.float32(to_bf16(np.float32(HD ** -0.5)))
    qn = to_bf16(qn * c)
    return ltx_abs_rope(qn, split, base), ltx_abs_rope(kn, split, base)
