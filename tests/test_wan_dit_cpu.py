"""The DiT-step driver's orchestration (vidax_b200.wan_dit: patchify,
timestep / text embedding, the block's sub-layers, modulation, residuals,
head, unpatchify) on the CPU against the numpy restatement of vidax's WanDiT
(oracle/wan_dit_ref.py). The driver's device-only steps are replaced by
float32 torch / numpy-oracle equivalents of what they compute (LayerNorm +
modulation, gated residual, fused RMSNorm + RoPE + attention, cross-attention
q/k RMSNorm, the attention kernel, the GELU GEMM epilogue); the GPU test
(tests/test_wan_dit_gpu.py) runs the same comparison with the kernels.
Tolerance: relative L2 2e-2."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.attention_ref import to_bf16
from oracle.rope_norm_ref import norm_rope, rms_norm


def _np(t):
    return t.detach().float().cpu().numpy()


def _attention(q, k, v, scale=None):
    sc = q.shape[-1] ** -0.5 if scale is None else scale
    qh, kh, vh = (t.float().transpose(1, 2) for t in (q, k, v))
    p = torch.softmax(qh @ kh.transpose(-1, -2) * sc, dim=-1)
    return (p @ vh).transpose(1, 2).contiguous().bfloat16()


def _ln_modulate(x, eps, w=None, b=None, scale=None, shift=None):
    mean = x.mean(-1, keepdim=True)
    var = ((x * x).mean(-1, keepdim=True) - mean * mean).clamp_min(0)
    y = (x - mean) * torch.rsqrt(var + eps)
    if w is not None:
        y = y * w + b
    if scale is not None:
        B, d = x.shape[0], x.shape[-1]
        y = y * (1 + scale.reshape(B, 1, d)) + shift.reshape(B, 1, d)
    return y.bfloat16()


def _gated_residual(x, y, gate=None):
    g = 1.0 if gate is None else gate.reshape(x.shape[0], 1, x.shape[-1])
    x += y.float() * g
    return x


def _attend(q, k, v, heads, *, norm_q=None, norm_k=None, rope=None, eps=1e-6,
            sp_axis_name=None, scale=None):
    assert sp_axis_name is None
    B, L, dim = q.shape
    cos, sin = (_np(t) for t in rope)
    qn = torch.from_numpy(norm_rope(_np(q), _np(norm_q), cos, sin, heads, eps)).bfloat16()
    kn = torch.from_numpy(norm_rope(_np(k), _np(norm_k), cos, sin, heads, eps)).bfloat16()
    o = _attention(qn, kn, v.view(B, L, heads, dim // heads), scale)
    return o.reshape(B, L, dim)


def _rms_norm_rope(x, weight, rope, heads, *, eps=1e-6, **_):
    assert rope is None
    B, S, dim = x.shape
    y = torch.from_numpy(rms_norm(_np(x), _np(weight), eps)).bfloat16()
    return y.view(B, S, heads, dim // heads)


def _linear_gelu(x, w, b):
    return F.gelu(F.linear(x, w, b).float(), approximate="tanh").bfloat16()


@pytest.mark.parametrize("head_dim,batch", [(64, 1), (32, 2)])
def test_wan_dit_orchestration_matches_oracle(head_dim, batch, monkeypatch):
    from oracle.wan_dit_ref import wan_dit_forward as ref_forward
    from vidax_b200 import wan_dit
    from vidax_b200.prologue import rope3d_freqs
    monkeypatch.setattr(wan_dit, "ln_modulate", _ln_modulate)
    monkeypatch.setattr(wan_dit, "gated_residual_", _gated_residual)
    monkeypatch.setattr(wan_dit, "attend", _attend)
    monkeypatch.setattr(wan_dit, "rms_norm_rope", _rms_norm_rope)
    monkeypatch.setattr(wan_dit, "local_attention", _attention)
    monkeypatch.setattr(wan_dit, "_linear_gelu", _linear_gelu)
    cfg = wan_dit.WanConfig(dim=2 * head_dim, ffn_dim=256, num_heads=2, num_layers=2, in_dim=4,
                            out_dim=4, freq_dim=32, text_dim=64, text_len=16)
    p = wan_dit.init_params(cfg, "cpu", seed=3)
    rng = np.random.Generator(np.random.PCG64(5))
    latents = to_bf16(rng.standard_normal((batch, 2, 8, 16, cfg.in_dim)).astype(np.float32))
    context = to_bf16(rng.standard_normal((batch, 10, cfg.text_dim)).astype(np.float32))
    t = np.array([500.0, 37.0][:batch], np.float32)
    out = wan_dit.wan_dit_forward(p, cfg, torch.from_numpy(latents), torch.from_numpy(t),
                                  torch.from_numpy(context))
    cos, sin = rope3d_freqs(2, 4, 8, cfg.head_dim)
    ref = ref_forward(p, cfg, latents, t, context, cos.numpy(), sin.numpy())
    got = out.float().numpy()
    assert got.shape == ref.shape == (batch, 2, 8, 16, cfg.out_dim)
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert rel <= 2e-2, rel
