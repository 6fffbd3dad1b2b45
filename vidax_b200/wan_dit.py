"""Wan2.1 DiT denoising step on B200: the driver around the attention hot path.

A torch restatement of vidax's `WanDiT` forward (src/vidax/models/wan/wan2_1/
dit.py) so one step of the model runs end to end on this library:

* `pre_process` (dit.py:270-339): patchify (the stride == kernel Conv3d as a
  GEMM on patch vectors), sinusoidal timestep embedding + MLP, text
  embedding, and under sequence parallelism the `chunk_by_rank` split of the
  tokens and their RoPE angles;
* `WanDiTBlock` (dit.py:78-156): AdaLN-modulated self-attention (Wan's
  `attend`, dit_layers.py:131-157: q/k/v projections, then ONE fused launch
  of RMSNorm(dim) + 3-D RoPE + Ulysses send packing, the all-to-alls and the
  tcgen05 attention kernel), cross-attention to the text (per-device
  attention over the replicated context, q/k RMSNorm), FFN (tanh GELU),
  float32 residual stream;
* `post_process` (dit.py:341-362): AdaLN head (dit_layers.py:195-217), the
  sequence all_gather of every rank's tokens, unpatchify.

The projections and FFN are plain bf16 GEMMs (cuBLAS through torch, the
FFN's bias + tanh-GELU in the cuBLASLt epilogue); the attention, the
pre-attention step, the Ulysses layout and the block's elementwise glue
(LayerNorm + modulation + cast, gated residual adds: one pass each) are this
library's kernels. Weights are random (no checkpoints here), drawn N(0, 0.02) unless
the reference initialises otherwise (modulation tables N(0, dim^-0.5),
norm3's affine and the RMSNorm scales ones / zeros).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib
from .attention import local_attention
from .prologue import attend, rms_norm_rope, rope3d_freqs


@dataclass(frozen=True)
class WanConfig:
    """WanDiT hyperparameters (vidax/models/wan/wan2_1/configs.py)."""
    dim: int = 1536
    ffn_dim: int = 8960
    num_heads: int = 12
    num_layers: int = 30
    patch_size: Tuple[int, int, int] = (1, 2, 2)
    in_dim: int = 16
    out_dim: int = 16
    freq_dim: int = 256
    text_dim: int = 4096
    text_len: int = 512
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


T2V_1_3B = WanConfig()
T2V_14B = WanConfig(dim=5120, ffn_dim=13824, num_heads=40, num_layers=40)


def init_params(cfg: WanConfig, device, seed: int = 0,
                on_device: bool = False) -> Dict[str, torch.Tensor]:
    """Random-init weights with vidax's parameter tree flattened to names;
    Dense kernels stored as torch (out, in) bf16 matrices. The draws come
    from a CPU generator, or with `on_device` from one on `device` (much
    faster for the 1.3B / 14B models; identical on every rank either way)."""
    gen_dev = torch.device(device) if on_device else torch.device("cpu")
    g = torch.Generator(device=gen_dev)
    g.manual_seed(seed)

    def normal(*shape, std=0.02, dtype=torch.bfloat16):
        return (torch.randn(*shape, generator=g, device=gen_dev) * std).to(device=device, dtype=dtype)

    def zeros(*shape, dtype=torch.bfloat16):
        return torch.zeros(*shape, device=device, dtype=dtype)

    d, f = cfg.dim, cfg.ffn_dim
    pt, ph, pw = cfg.patch_size
    p: Dict[str, torch.Tensor] = {}
    p["patch_w"] = normal(d, pt * ph * pw * cfg.in_dim)
    p["patch_b"] = zeros(d)
    for name, (o, i) in {"time_0": (d, cfg.freq_dim), "time_2": (d, d), "time_proj": (6 * d, d)}.items():
        p[f"{name}_w"] = normal(o, i, dtype=torch.float32)  # timestep MLP runs in float32
        p[f"{name}_b"] = zeros(o, dtype=torch.float32)
    p["text_0_w"], p["text_0_b"] = normal(d, cfg.text_dim), zeros(d)
    p["text_2_w"], p["text_2_b"] = normal(d, d), zeros(d)
    for i in range(cfg.num_layers):
        b = f"blocks_{i}."
        p[b + "modulation"] = normal(1, 6, d, std=d ** -0.5, dtype=torch.float32)
        for pre in ("self_attn", "cross_attn"):
            for x in ("q", "k", "v", "o"):
                p[b + f"{pre}_{x}_w"], p[b + f"{pre}_{x}_b"] = normal(d, d), zeros(d)
            p[b + f"{pre}_norm_q"] = torch.ones(d, device=device)
            p[b + f"{pre}_norm_k"] = torch.ones(d, device=device)
        p[b + "norm3_w"] = torch.ones(d, device=device)
        p[b + "norm3_b"] = torch.zeros(d, device=device)
        p[b + "ffn_0_w"], p[b + "ffn_0_b"] = normal(f, d), zeros(f)
        p[b + "ffn_2_w"], p[b + "ffn_2_b"] = normal(d, f), zeros(d)
    p["head_modulation"] = normal(1, 2, d, std=d ** -0.5, dtype=torch.float32)
    p["head_w"] = normal(pt * ph * pw * cfg.out_dim, d)
    p["head_b"] = zeros(pt * ph * pw * cfg.out_dim)
    return p


def sinusoidal_embedding_1d(dim: int, position: torch.Tensor) -> torch.Tensor:
    """[cos, sin] timestep embedding in float32 (vidax/core/rope3d.py:15-30),
    computed on the host with numpy's float32 power / cos / sin (the math the
    reference's formula was pinned with; B values, once per step) and placed
    on `position`'s device."""
    half = dim // 2
    pos = position.detach().float().cpu().numpy()
    freqs = np.power(np.float32(10000.0), -np.arange(half, dtype=np.float32) / np.float32(half))
    s = np.outer(pos, freqs.astype(np.float32)).astype(np.float32)
    emb = np.concatenate([np.cos(s), np.sin(s)], axis=1).astype(np.float32)
    return torch.from_numpy(emb).to(position.device)


def _ln(x: torch.Tensor, eps: float, w=None, b=None) -> torch.Tensor:
    """flax LayerNorm in float32 (use_scale / use_bias as given)."""
    return F.layer_norm(x.float(), (x.shape[-1],), w, b, eps)


def ln_modulate(x: torch.Tensor, eps: float, w=None, b=None, scale=None, shift=None) -> torch.Tensor:
    """bf16((LayerNorm(x) [* w + b]) * (1 + scale) + shift) in one pass
    (`vx_ln_modulate`): x (B, L, dim) float32, scale / shift (B, 1, dim) or
    (B, dim) float32."""
    B, L, d = x.shape
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    y = torch.empty((B, L, d), dtype=torch.bfloat16, device=x.device)
    sc = scale.reshape(B, d).contiguous() if scale is not None else None
    sh = shift.reshape(B, d).contiguous() if shift is not None else None
    lib = _lib.load()
    _lib.check(lib.vx_ln_modulate(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
        ctypes.c_void_p(w.data_ptr() if w is not None else None),
        ctypes.c_void_p(b.data_ptr() if b is not None else None),
        ctypes.c_void_p(sc.data_ptr() if sc is not None else None),
        ctypes.c_void_p(sh.data_ptr() if sh is not None else None),
        ctypes.c_int64(B * L), ctypes.c_int32(d), ctypes.c_int32(L), ctypes.c_float(eps),
        ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)))
    return y


def gated_residual_(x: torch.Tensor, y: torch.Tensor, gate=None) -> torch.Tensor:
    """x += float(y) * gate in place, one pass (`vx_gated_residual`): x
    (B, L, dim) float32, y (B, L, dim) bf16, gate (B, 1, dim) / (B, dim) or None."""
    B, L, d = x.shape
    if not (x.is_contiguous() and y.is_contiguous()) or y.dtype != torch.bfloat16:
        raise ValueError("x (float32) and y (bf16) must be contiguous")
    g = gate.reshape(B, d).contiguous() if gate is not None else None
    lib = _lib.load()
    _lib.check(lib.vx_gated_residual(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
        ctypes.c_void_p(g.data_ptr() if g is not None else None),
        ctypes.c_int64(B * L), ctypes.c_int32(d), ctypes.c_int32(L),
        ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)))
    return x


def _linear_gelu(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """tanh-GELU(x @ w^T + b) with bias and activation in the cuBLASLt GEMM
    epilogue."""
    shape = x.shape
    h = torch._addmm_activation(b, x.reshape(-1, shape[-1]), w.t(), use_gelu=True)
    return h.reshape(*shape[:-1], w.shape[0])


def _gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def patchify(latents: torch.Tensor, patch: Tuple[int, int, int]) -> torch.Tensor:
    """(B, T, H, W, C) -> (B, tokens, pt*ph*pw*C) patch vectors in the
    (pt, ph, pw, C) order of a channels-last Conv kernel."""
    B, T, H, W, C = latents.shape
    pt, ph, pw = patch
    x = latents.reshape(B, T // pt, pt, H // ph, ph, W // pw, pw, C)
    x = x.permute(0, 1, 3, 5, 2, 4, 6, 7)
    return x.reshape(B, (T // pt) * (H // ph) * (W // pw), pt * ph * pw * C)


def unpatchify(x: torch.Tensor, grid, patch, out_dim: int) -> torch.Tensor:
    """dit.py:356-361: (B, tokens, pt*ph*pw*C) -> (B, T, H, W, C)."""
    b, tp, hp, wp = grid
    pt, ph, pw = patch
    x = x.reshape(b, tp, hp, wp, pt, ph, pw, out_dim)
    x = x.permute(0, 1, 4, 2, 5, 3, 6, 7)
    return x.reshape(b, tp * pt, hp * ph, wp * pw, out_dim)


def pre_process(p, cfg: WanConfig, latents, t, context, rope, sp_axis_name: Optional[str] = None):
    """dit.py:270-339. Returns (x f32 (B, L_local, dim), context (B, text_len,
    dim) bf16, e0 (B, 6, dim) f32, rope of the local tokens, e, grid)."""
    B = latents.shape[0]
    grid = (B,) + tuple(latents.shape[1 + i] // cfg.patch_size[i] for i in range(3))
    x = F.linear(patchify(latents.to(torch.bfloat16), cfg.patch_size), p["patch_w"], p["patch_b"])
    t_freq = sinusoidal_embedding_1d(cfg.freq_dim, t)
    e = F.linear(F.silu(F.linear(t_freq, p["time_0_w"], p["time_0_b"])), p["time_2_w"], p["time_2_b"])
    e0 = F.linear(F.silu(e), p["time_proj_w"], p["time_proj_b"]).reshape(B, 6, cfg.dim)
    pad = cfg.text_len - context.shape[1]
    if pad < 0:
        raise ValueError("context length exceeds text_len")
    context = F.pad(context.to(torch.bfloat16), (0, 0, 0, pad))
    context = F.linear(_gelu_tanh(F.linear(context, p["text_0_w"], p["text_0_b"])),
                       p["text_2_w"], p["text_2_b"])
    cos, sin = rope
    if sp_axis_name is not None:
        from .ulysses import _group
        group = _group(sp_axis_name)
        P, r = dist.get_world_size(group), dist.get_rank(group)
        L = x.shape[1]
        if L % P:
            raise ValueError(f"sequence parallelism needs tokens ({L}) divisible by {P}")
        n = L // P
        x = x[:, r * n:(r + 1) * n]
        cos, sin = cos[r * n:(r + 1) * n], sin[r * n:(r + 1) * n]
    return x.float(), context, e0, (cos, sin), e, grid


def block_forward(p, i: int, cfg: WanConfig, x, context, t_mod, rope,
                  sp_axis_name: Optional[str] = None) -> torch.Tensor:
    """WanDiTBlock (dit.py:78-156) on the float32 residual stream x."""
    b = f"blocks_{i}."
    B, L, d = x.shape
    H = cfg.num_heads
    e = p[b + "modulation"] + t_mod.float()
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (e[:, j] for j in range(6))

    nx = ln_modulate(x, cfg.eps, scale=scale_msa, shift=shift_msa)
    q, k, v = (F.linear(nx, p[b + f"self_attn_{n}_w"], p[b + f"self_attn_{n}_b"]) for n in "qkv")
    o = attend(q, k, v, H, norm_q=p[b + "self_attn_norm_q"], norm_k=p[b + "self_attn_norm_k"],
               rope=rope, eps=cfg.eps, sp_axis_name=sp_axis_name)
    gated_residual_(x, F.linear(o, p[b + "self_attn_o_w"], p[b + "self_attn_o_b"]), gate_msa)

    nc = ln_modulate(x, cfg.eps, w=p[b + "norm3_w"], b=p[b + "norm3_b"])
    q = F.linear(nc, p[b + "cross_attn_q_w"], p[b + "cross_attn_q_b"])
    k = F.linear(context, p[b + "cross_attn_k_w"], p[b + "cross_attn_k_b"])
    v = F.linear(context, p[b + "cross_attn_v_w"], p[b + "cross_attn_v_b"])
    qn = rms_norm_rope(q, p[b + "cross_attn_norm_q"], None, H, eps=cfg.eps)
    kn = rms_norm_rope(k, p[b + "cross_attn_norm_k"], None, H, eps=cfg.eps)
    o = local_attention(qn, kn, v.view(B, -1, H, cfg.head_dim))
    gated_residual_(x, F.linear(o.reshape(B, L, d), p[b + "cross_attn_o_w"],
                                p[b + "cross_attn_o_b"]))

    nh = ln_modulate(x, cfg.eps, scale=scale_mlp, shift=shift_mlp)
    h = F.linear(_linear_gelu(nh, p[b + "ffn_0_w"], p[b + "ffn_0_b"]),
                 p[b + "ffn_2_w"], p[b + "ffn_2_b"])
    return gated_residual_(x, h, gate_mlp)


def post_process(p, cfg: WanConfig, x, e, grid, sp_axis_name: Optional[str] = None):
    """WanHead (dit_layers.py:195-217), the sequence all_gather of the ranks'
    token chunks in rank order (dit.py:350-354), unpatchify."""
    mod = p["head_modulation"] + e.float()[:, None, :]
    shift, scale = mod[:, 0:1], mod[:, 1:2]
    # the head runs in float32 (its input keeps e's dtype, dit_layers.py:212-217)
    y = _ln(x, cfg.eps) * (1 + scale) + shift
    y = F.linear(y, p["head_w"].float(), p["head_b"].float()).to(torch.bfloat16)
    if sp_axis_name is not None:
        from .ulysses import _group
        group = _group(sp_axis_name)
        P = dist.get_world_size(group)
        gathered = torch.empty((P,) + tuple(y.shape), dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(gathered, y.contiguous(), group=group)
        y = gathered.permute(1, 0, 2, 3).reshape(y.shape[0], P * y.shape[1], y.shape[2])
    return unpatchify(y, grid, cfg.patch_size, cfg.out_dim)


def wan_dit_forward(p, cfg: WanConfig, latents: torch.Tensor, t: torch.Tensor,
                    context: torch.Tensor, rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                    sp_axis_name: Optional[str] = None) -> torch.Tensor:
    """One WanDiT forward (dit.py:364-394): latents (B, T, H, W, in_dim) on
    every rank, t (B,), context (B, L_text, text_dim); returns
    (B, T, H, W, out_dim) on every rank. `rope`: tables of the whole token
    grid (default: `rope3d_freqs` of the patch grid)."""
    if rope is None:
        tp, hp, wp = (latents.shape[1 + i] // cfg.patch_size[i] for i in range(3))
        rope = rope3d_freqs(tp, hp, wp, cfg.head_dim, device=latents.device)
    x, ctx, e0, rope_l, e, grid = pre_process(p, cfg, latents, t, context, rope, sp_axis_name)
    for i in range(cfg.num_layers):
        x = block_forward(p, i, cfg, x, ctx, e0, rope_l, sp_axis_name)
    return post_process(p, cfg, x, e, grid, sp_axis_name)


def step_flops(cfg: WanConfig, tokens: int, text_len: Optional[int] = None) -> float:
    """Matmul FLOPs of one forward over `tokens` latent tokens (B = 1): per
    block q/k/v/o and cross q/o projections, cross k/v over the text, self-
    and cross-attention cores, FFN; plus patch embedding and head."""
    d, f, L = cfg.dim, cfg.ffn_dim, tokens
    Lt = cfg.text_len if text_len is None else text_len
    per_block = (2 * L * d * d * 4          # self q, k, v, o
                 + 4 * L * L * d            # self-attention core
                 + 2 * L * d * d * 2        # cross q, o
                 + 2 * Lt * d * d * 2       # cross k, v
                 + 4 * L * Lt * d           # cross-attention core
                 + 2 * L * d * f * 2)       # FFN
    pt, ph, pw = cfg.patch_size
    io = 2 * L * d * pt * ph * pw * (cfg.in_dim + cfg.out_dim)
    return float(cfg.num_layers * per_block + io)
