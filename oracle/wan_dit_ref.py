"""CPU restatement of vidax's WanDiT forward -- TEST INFRASTRUCTURE ONLY.

Checker for vidax_b200.wan_dit: numpy float32 with bf16 rounding at the
points where vidax casts to the compute dtype (src/vidax/models/wan/wan2_1/
dit.py): the modulated LayerNorm outputs (:108, :131), every Dense output
(bf16 kernels), RMSNorm (src/vidax/core/attention.py:149-162), RoPE
(src/vidax/core/rope3d.py:89-111) and the attention outputs; the residual
stream, modulation, timestep MLP and the head stay float32 (:100-156,
:296-300; dit_layers.py:205-217), the output is cast to bf16. Attention is `sdpa` (fp32 softmax).

Parity unpinned at the block level: flax is absent here, so the
reference's WanDiT cannot run; the structure follows its source line by
line, and the pieces it is built from (RMSNorm, RoPE, attention, Ulysses
layout) are pinned individually against the reference's own functions.
"""
from __future__ import annotations

import numpy as np

from .attention_ref import sdpa, to_bf16
from .rope_norm_ref import apply_rope3d, rms_norm


def _np(t):
    return t.detach().float().cpu().numpy()


def _dense(x, w, b):
    """bf16 Dense: bf16 operands, float32 accumulation, bf16 output."""
    return to_bf16(np.asarray(x, np.float32) @ w.T + b)


def _ln(x, eps, w=None, b=None):
    x = np.asarray(x, np.float32)
    mu = x.mean(-1, keepdims=True)
    var = np.square(x - mu).mean(-1, keepdims=True)
    y = (x - mu) / np.sqrt(var + np.float32(eps))
    if w is not None:
        y = y * w + b
    return y.astype(np.float32)


_SQRT_2_OVER_PI = np.float32((2.0 / np.pi) ** 0.5)


def _gelu_tanh(x):
    """tanh-approximated GELU (flax nn.gelu(approximate=True)), bf16 output."""
    x = np.asarray(x, np.float32)
    return to_bf16(0.5 * x * (1 + np.tanh(_SQRT_2_OVER_PI * (x + np.float32(0.044715) * x ** 3))))


def _silu(x):
    return x / (1 + np.exp(-x))


def wan_dit_forward(params, cfg, latents, t, context, cos, sin):
    """params: the torch tensor dict of vidax_b200.wan_dit.init_params;
    latents (B, T, H, W, C) float32 bf16 values; t (B,); context
    (B, L_text, text_dim); cos / sin (tokens, D/2). Returns (B, T, H, W, out)."""
    p = {k: _np(v) for k, v in params.items()}
    B = latents.shape[0]
    pt, ph, pw = cfg.patch_size
    grid = (B, latents.shape[1] // pt, latents.shape[2] // ph, latents.shape[3] // pw)
    x = latents.reshape(B, grid[1], pt, grid[2], ph, grid[3], pw, -1).transpose(0, 1, 3, 5, 2, 4, 6, 7)
    x = _dense(to_bf16(x.reshape(B, grid[1] * grid[2] * grid[3], -1)), p["patch_w"], p["patch_b"])
    half = cfg.freq_dim // 2
    fr = np.power(np.float32(10000.0), -np.arange(half, dtype=np.float32) / half)
    s = np.outer(np.asarray(t, np.float32), fr)
    t_freq = np.concatenate([np.cos(s), np.sin(s)], axis=1).astype(np.float32)
    e = _silu(t_freq @ p["time_0_w"].T + p["time_0_b"]) @ p["time_2_w"].T + p["time_2_b"]
    e0 = (_silu(e) @ p["time_proj_w"].T + p["time_proj_b"]).reshape(B, 6, cfg.dim)
    ctx = np.pad(to_bf16(context), ((0, 0), (0, cfg.text_len - context.shape[1]), (0, 0)))
    ctx = _dense(_gelu_tanh(_dense(ctx, p["text_0_w"], p["text_0_b"])), p["text_2_w"], p["text_2_b"])
    x = x.astype(np.float32)
    H, D = cfg.num_heads, cfg.head_dim
    L = x.shape[1]
    for i in range(cfg.num_layers):
        b = f"blocks_{i}."
        em = p[b + "modulation"] + e0
        sh_a, sc_a, g_a, sh_m, sc_m, g_m = (em[:, j:j + 1] for j in range(6))
        nx = to_bf16(_ln(x, cfg.eps) * (1 + sc_a) + sh_a)
        q, k, v = (_dense(nx, p[b + f"self_attn_{n}_w"], p[b + f"self_attn_{n}_b"]) for n in "qkv")
        q = apply_rope3d(rms_norm(q, p[b + "self_attn_norm_q"], cfg.eps).reshape(B, L, H, D), cos, sin)
        k = apply_rope3d(rms_norm(k, p[b + "self_attn_norm_k"], cfg.eps).reshape(B, L, H, D), cos, sin)
        o = to_bf16(sdpa(q, k, v.reshape(B, L, H, D))).reshape(B, L, -1)
        x = x + _dense(o, p[b + "self_attn_o_w"], p[b + "self_attn_o_b"]) * g_a
        nc = to_bf16(_ln(x, cfg.eps, p[b + "norm3_w"], p[b + "norm3_b"]))
        q = _dense(nc, p[b + "cross_attn_q_w"], p[b + "cross_attn_q_b"])
        k = _dense(ctx, p[b + "cross_attn_k_w"], p[b + "cross_attn_k_b"])
        v = _dense(ctx, p[b + "cross_attn_v_w"], p[b + "cross_attn_v_b"])
        q = rms_norm(q, p[b + "cross_attn_norm_q"], cfg.eps).reshape(B, L, H, D)
        k = rms_norm(k, p[b + "cross_attn_norm_k"], cfg.eps).reshape(B, -1, H, D)
        o = to_bf16(sdpa(q, k, v.reshape(B, -1, H, D))).reshape(B, L, -1)
        x = x + _dense(o, p[b + "cross_attn_o_w"], p[b + "cross_attn_o_b"])
        nh = to_bf16(_ln(x, cfg.eps) * (1 + sc_m) + sh_m)
        hdn = _dense(_gelu_tanh(_dense(nh, p[b + "ffn_0_w"], p[b + "ffn_0_b"])),
                     p[b + "ffn_2_w"], p[b + "ffn_2_b"])
        x = x + hdn * g_m
    mod = p["head_modulation"] + e[:, None, :]
    y = _ln(x, cfg.eps) * (1 + mod[:, 1:2]) + mod[:, 0:1]   # float32 head (dit_layers.py:212-217)
    y = to_bf16(y @ p["head_w"].T + p["head_b"])
    y = y.reshape(B, grid[1], grid[2], grid[3], pt, ph, pw, cfg.out_dim).transpose(0, 1, 4, 2, 5, 3, 6, 7)
    return y.reshape(B, grid[1] * pt, grid[2] * ph, grid[3] * pw, cfg.out_dim)
