"""`sequence_parallel_joint_self_attention` (vidax attention.py:391-464) run
as P emulated ranks in one process, against the reference's own per-rank
outputs (tests/golden, written by make_golden.py from vidax's function).

Each rank is a thread; `torch.distributed` inside vidax_b200.ulysses is
replaced by the in-process stand-in of tests/emulated_ranks.py. The product's own orchestration -- text slicing,
packing, exchange, joint attention, reverse exchange, text all-gather --
runs unchanged, with the kernels replaced by float32 torch equivalents
(this pins the orchestration on any host), and on a GPU with the real
kernels (pack, attention, unpack) at the head dims the kernel takes (128,
64). Tolerance: max-abs 2e-2, mean-abs 2e-3."""
import os

import numpy as np
import pytest
import torch

from emulated_ranks import RankGroup, run_ranks
from oracle.attention_ref import compare

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _cpu_attention(q, k, v, scale, **_):
    qh, kh, vh = (t.float().transpose(1, 2) for t in (q, k, v))
    p = torch.softmax(qh @ kh.transpose(-1, -2) * scale, dim=-1)
    return (p @ vh).transpose(1, 2).to(q.dtype).contiguous()  # BSHD, as the kernel writes


def _cpu_pack(strided, groups, out=None, sub=None):
    assert sub is None and out is None
    seq, heads, d = strided[0].shape
    hg = -(-heads // groups)
    res = []
    for t in strided:
        p = torch.zeros((groups, seq, hg, d), dtype=t.dtype)
        for g in range(groups):
            h0, h1 = g * hg, min(heads, (g + 1) * hg)
            if h1 > h0:
                p[g, :, :h1 - h0] = t[:, h0:h1]
        res.append(p)
    return res


def _cpu_unpack(packed, strided_out, heads, sub=None):
    assert sub is None
    for p, o in zip(packed, strided_out):
        groups, _, hg, _ = p.shape
        for g in range(groups):
            h0, h1 = g * hg, min(heads, (g + 1) * hg)
            if h1 > h0:
                o[:, h0:h1] = p[g, :, :h1 - h0]


def _run_joint(tag, monkeypatch, device, dtype, cpu_kernels):
    import vidax_b200 as vx
    from vidax_b200 import ulysses
    g = np.load(os.path.join(GOLDEN, "attention_reference.npz"))
    qg, kg, vg = (g[f"{tag}_{n}"] for n in "qkv")
    T = int(g[f"{tag}_text_len"][0])
    ref = g[f"{tag}_o"]
    P = ref.shape[0]
    S_loc = (qg.shape[1] - T) // P
    fake = RankGroup(P)
    monkeypatch.setattr(ulysses, "dist", fake)
    if cpu_kernels:
        monkeypatch.setattr(ulysses, "flash_attention", _cpu_attention)
        monkeypatch.setattr(ulysses, "pack_heads", _cpu_pack)
        monkeypatch.setattr(ulysses, "unpack_heads", _cpu_unpack)
    vx.register_axis("sp_emulated", None)

    def rank(r):
        loc = [torch.from_numpy(np.ascontiguousarray(np.concatenate(
            [x[:, :T], x[:, T + r * S_loc:T + (r + 1) * S_loc]], axis=1))).to(device, dtype)
            for x in (qg, kg, vg)]
        o = vx.sequence_parallel_joint_self_attention(*loc, T, "sp_emulated")
        return o.float().cpu().numpy()

    try:
        results = run_ranks(P, fake, rank)
    finally:
        vx.unregister_axis("sp_emulated")
    for r in range(P):
        mx, mean = compare(results[r], ref[r])
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (tag, r, mx, mean)


@pytest.mark.parametrize("tag", ["joint2", "joint4", "joint2d128"])
def test_joint_orchestration_matches_reference_code(tag, monkeypatch):
    """CPU: the product's joint Ulysses orchestration with float32 torch
    attention / packing in place of the kernels."""
    _run_joint(tag, monkeypatch, "cpu", torch.float32, cpu_kernels=True)


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["joint2d128", "joint4d128", "joint2d64"])
def test_joint_on_cuda_kernels_matches_reference_code(tag, monkeypatch):
    """GPU: the same orchestration with the CUDA pack / attention / unpack
    kernels, bf16, against the reference's per-rank outputs (P = 2 and 4,
    head_dim 128 and 64)."""
    from vidax_b200 import _lib
    _run_joint(tag, monkeypatch, "cuda", torch.bfloat16, cpu_kernels=False)
    assert _lib.device_status(clear=True) == 0
