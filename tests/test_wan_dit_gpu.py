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


def _inputs(cfg, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    latents = to_bf16(rng.standard_normal((1, 2, 8, 16, cfg.in_dim)).astype(np.float32))
    context = to_bf16(rng.standard_normal((1, 10, cfg.text_dim)).astype(np.float32))
    t = np.array([500.0], np.float32)
    return latents, context, t


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim", [128, 64])
def test_wan_dit_forward_matches_oracle(head_dim):
    from oracle.wan_dit_ref import wan_dit_forward as ref_forward
    from vidax_b200 import _lib
    from vidax_b200.wan_dit import init_params, wan_dit_forward
    from vidax_b200.prologue import rope3d_freqs
    cfg = _tiny(head_dim)
    p = init_params(cfg, "cuda", seed=3)
    latents, context, t = _inputs(cfg, 5)
    cos, sin = rope3d_freqs(2, 4, 8, cfg.head_dim)
    out = wan_dit_forward(p, cfg, torch.from_numpy(latents).cuda(), torch.from_numpy(t).cuda(),
                          torch.from_numpy(context).cuda())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = ref_forward(p, cfg, latents, t, context, cos.numpy(), sin.numpy())
    got = out.float().cpu().numpy()
    assert got.shape == ref.shape == (1, 2, 8, 16, cfg.out_dim)
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
