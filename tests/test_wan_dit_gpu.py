"""The Wan2.1 DiT-step driver (vidax_b200.wan_dit) on a reduced config
against the numpy restatement of vidax's WanDiT (oracle/wan_dit_ref.py):
the whole forward -- patchify, timestep / text embedding, blocks with the
fused pre-attention step and the attention kernels, head, unpatchify --
within a relative L2 error of 2e-2 (bf16 GEMMs and activations on both
sides, float32 accumulation in different orders)."""
import numpy as np
import pytest
import torch

from oracle.attention_ref import to_bf16


def _tiny(head_dim):
    from vidax_b200.wan_dit import WanConfig
    return WanConfig(dim=2 * head_dim, ffn_dim=512, num_heads=2, num_layers=2, in_dim=4,
                     out_dim=4, freq_dim=32, text_dim=64, text_len=16)


def _inputs(cfg, seed, batch=1):
    rng = np.random.Generator(np.random.PCG64(seed))
    latents = to_bf16(rng.standard_normal((batch, 2, 8, 16, cfg.in_dim)).astype(np.float32))
    context = to_bf16(rng.standard_normal((batch, 10, cfg.text_dim)).astype(np.float32))
    t = np.array([500.0, 37.0][:batch], np.float32)
    return latents, context, t


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim,batch", [(128, 1), (64, 1), (128, 2)])
def test_wan_dit_forward_matches_oracle(head_dim, batch):
    """batch 2 = the classifier-free-guidance batch (two timesteps here)."""
    from oracle.wan_dit_ref import wan_dit_forward as ref_forward
    from vidax_b200 import _lib
    from vidax_b200.wan_dit import init_params, wan_dit_forward
    from vidax_b200.prologue import rope3d_freqs
    cfg = _tiny(head_dim)
    p = init_params(cfg, "cuda", seed=3)
    latents, context, t = _inputs(cfg, 5, batch)
    cos, sin = rope3d_freqs(2, 4, 8, cfg.head_dim)
    out = wan_dit_forward(p, cfg, torch.from_numpy(latents).cuda(), torch.from_numpy(t).cuda(),
                          torch.from_numpy(context).cuda())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = ref_forward(p, cfg, latents, t, context, cos.numpy(), sin.numpy())
    got = out.float().cpu().numpy()
    assert got.shape == ref.shape == (batch, 2, 8, 16, cfg.out_dim)
    assert _rel(got, ref) <= 2e-2, _rel(got, ref)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_wan_dit_two_gpus_nccl():
    """Sequence-parallel forward over 2 GPUs (NCCL) equals the 1-GPU forward."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29615",
           os.path.join(root, "tests", "dist_wan_check.py")]
    res = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "WAN SP OK" in res.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("dim,affine,mod", [(256, False, True), (1536, True, False), (5120, False, True)])
def test_ln_modulate_kernel(dim, affine, mod):
    """vx_ln_modulate against the float32 torch composition it replaces."""
    import torch.nn.functional as F
    from vidax_b200.wan_dit import ln_modulate
    g = torch.Generator(device="cuda").manual_seed(dim)
    x = torch.randn((2, 37, dim), generator=g, device="cuda") * 3 + 0.5
    w = torch.randn(dim, generator=g, device="cuda") if affine else None
    b = torch.randn(dim, generator=g, device="cuda") if affine else None
    sc = torch.randn((2, 1, dim), generator=g, device="cuda") if mod else None
    sh = torch.randn((2, 1, dim), generator=g, device="cuda") if mod else None
    got = ln_modulate(x, 1e-6, w, b, sc, sh).float()
    ref = F.layer_norm(x, (dim,), w, b, 1e-6)
    if mod:
        ref = ref * (1 + sc) + sh
    ref = ref.bfloat16().float()
    diff = (got - ref).abs()
    assert float(diff.max()) <= 2 ** -7 * float(ref.abs().max())  # one bf16 ulp of the scale
    assert float((diff > 0).float().mean()) <= 0.02


@pytest.mark.gpu
@pytest.mark.parametrize("gated", [True, False])
def test_gated_residual_kernel(gated):
    from vidax_b200.wan_dit import gated_residual_
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn((2, 45, 1536), generator=g, device="cuda")
    y = torch.randn((2, 45, 1536), generator=g, device="cuda").bfloat16()
    gate = torch.randn((2, 1, 1536), generator=g, device="cuda") if gated else None
    ref = x + (y.float() * gate if gated else y.float())
    gated_residual_(x, y, gate)
    assert torch.allclose(x, ref, rtol=1e-6, atol=1e-6)
