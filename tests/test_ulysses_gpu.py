"""Ulysses data path on one GPU: the pack / unpack kernels and the attention
kernel exactly as sequence_parallel_self_attention uses them, with the NCCL
all-to-all replaced by the equivalent chunk copies between P emulated ranks
(the all-to-all itself is covered by tests/test_ulysses_dist.py on gloo and by
the multi-GPU test below when more than one GPU is visible)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare, sdpa, seeded_qkv

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _emulated_ulysses(q, k, v, P):
    """q, k, v: global (B, S, H, D) float32 numpy; returns the (B, S, H, D)
    output assembled from the P emulated ranks' local outputs."""
    from vidax_b200 import flash_attention
    from vidax_b200.ulysses import pack_heads, unpack_heads
    B, S, H, D = q.shape
    S_loc = S // P
    dev = [[torch.from_numpy(np.ascontiguousarray(x[:, r * S_loc:(r + 1) * S_loc])).cuda().bfloat16()
            for x in (q, k, v)] for r in range(P)]
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device="cuda")
    for b in range(B):
        sends = [pack_heads([t[b] for t in dev[r]], P) for r in range(P)]   # [r][tensor] (P,S_loc,Hg,D)
        Hg = sends[0][0].shape[2]
        outs = []
        for r in range(P):                                                 # rank r's head group
            recv = [torch.stack([sends[src][t][r] for src in range(P)]) for t in range(3)]
            o = flash_attention(*[x.reshape(1, S, Hg, D) for x in recv], D ** -0.5)
            outs.append(o.reshape(P, S_loc, Hg, D))
        for dst in range(P):                                               # heads -> tokens
            recv = torch.stack([outs[src][dst] for src in range(P)])
            unpack_heads([recv], [out[b, dst * S_loc:(dst + 1) * S_loc]], H)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,P", [(1, 512, 4, 2), (1, 768, 8, 4), (2, 1024, 8, 8),
                                     (1, 960, 12, 8), (1, 300, 3, 2)])
def test_ulysses_pack_attention_unpack(B, S, H, P):
    """Includes H % P != 0 (12 heads on 8 ranks, 3 on 2): zero-padded heads."""
    q, k, v = seeded_qkv((B, S, H, 128), 300 + S + H + P)
    got = _emulated_ulysses(q, k, v, P)
    mx, mean = compare(got, sdpa(q, k, v))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_pack_unpack_roundtrip_bit_exact():
    from vidax_b200.ulysses import pack_heads, unpack_heads
    x = torch.randn((2, 257, 10, 128), device="cuda").bfloat16()[:, :, :]
    for P in (1, 2, 4, 8, 3):
        packed = pack_heads([x[0], x[1]], P)
        # packed layout equals the oracle's tiled all_to_all send chunks
        Hg = -(-10 // P)
        ref = torch.zeros((P, 257, Hg, 128), dtype=x.dtype, device="cuda")
        for g in range(P):
            h0, h1 = g * Hg, min(10, (g + 1) * Hg)
            if h1 > h0:
                ref[g, :, : h1 - h0] = x[0, :, h0:h1]
        assert torch.equal(packed[0], ref)
        back = torch.empty_like(x)
        unpack_heads(packed, [back[0], back[1]], 10)
        assert torch.equal(back, x)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_two_gpus_nccl():
    """Real NCCL path: 2 ranks, compared with the oracle of the global sequence."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29611",
           os.path.join(ROOT, "tests", "dist_ulysses_check.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "ULYSSES OK" in res.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("H,P,hs", [(40, 8, 1), (40, 2, 4), (12, 8, 1), (10, 4, 2), (6, 4, 1)])
def test_sub_group_pack_unpack_bit_exact(H, P, hs):
    """Slices of every rank's head group (the pipelined exchange): packed
    layout against direct indexing, and unpacking all slices restores x."""
    from vidax_b200.ulysses import pack_heads, unpack_heads
    S_loc = 96
    x = torch.randn((S_loc, H, 128), device="cuda").bfloat16()
    Hg = -(-H // P)
    back = torch.zeros_like(x)
    for j in range(-(-Hg // hs)):
        valid = min(hs, Hg - j * hs)
        sub = (hs, Hg, j * hs, valid)
        packed, = pack_heads([x], P, sub=sub)
        ref = torch.zeros((P, S_loc, hs, 128), dtype=x.dtype, device="cuda")
        for g in range(P):
            for i in range(valid):
                h = g * Hg + j * hs + i
                if h < H:
                    ref[g, :, i] = x[:, h]
        assert torch.equal(packed, ref)
        unpack_heads([packed], [back], H, sub=sub)
    assert torch.equal(back, x)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_qsplit_two_gpus_nccl():
    """Query-split heads (3, 5, 7 heads on 2 ranks) over NCCL vs the oracle."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29617",
           os.path.join(ROOT, "tests", "dist_qsplit_check.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "QSPLIT OK" in res.stdout
