"""GPU kernels against outputs of the reference's own code (tests/golden,
written by tests/golden/make_golden.py from vidax's neighborhood_attention_3d,
dot_product_attention, local_attention and sequence_parallel_self_attention).

The reference rounds q.k and the softmax weights to bf16; the kernels keep
them in fp32 (or round q.k too with round_logits=True). Tolerance: max-abs
2e-2, mean-abs 2e-3."""
import os

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


@pytest.mark.gpu
@pytest.mark.parametrize("i", [4, 5, 6, 7])
@pytest.mark.parametrize("round_logits", [False, True])
def test_na3d_kernel_vs_reference_code(i, round_logits):
    import vidax_b200 as vx
    g = np.load(os.path.join(GOLDEN, "na3d_reference.npz"))
    q, k, v = (g[f"na{i}_{n}"] for n in "qkv")
    kernel = tuple(int(x) for x in g[f"na{i}_kernel"])
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), kernel, round_logits=round_logits)
    mx, mean = compare(out.float().cpu().numpy(), g[f"na{i}_o"])
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_attention_kernel_vs_reference_code():
    import vidax_b200 as vx
    g = np.load(os.path.join(GOLDEN, "attention_reference.npz"))
    q, k, v = _dev(g["dpa128_q"]), _dev(g["dpa128_k"]), _dev(g["dpa128_v"])
    mx, mean = compare(vx.dot_product_attention(q, k, v).float().cpu().numpy(), g["dpa128_o"])
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    kx, vx_ = _dev(g["cross128_k"]), _dev(g["cross128_v"])
    mx, mean = compare(vx.local_attention(q, kx, vx_).float().cpu().numpy(), g["cross128_o"])
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_key_padding_vs_reference_code():
    """dot_product_attention with a (B, 1, 1, Sk) 0 / -inf key bias and with
    the boolean mask form, ragged valid lengths (41 and 19 of 41 keys)."""
    import vidax_b200 as vx
    g = np.load(os.path.join(GOLDEN, "attention_reference.npz"))
    q, k, v = _dev(g["keypad_q"]), _dev(g["keypad_k"]), _dev(g["keypad_v"])
    lens = torch.from_numpy(g["keypad_len"]).long()
    valid = torch.arange(k.shape[1])[None, :] < lens[:, None]
    bias = torch.zeros(valid.shape).masked_fill(~valid, float("-inf"))[:, None, None, :]
    for kw, ref in ((dict(bias=bias.cuda()), g["keypad_o_bias"]),
                    (dict(mask=valid[:, None, None, :].cuda()), g["keypad_o_mask"]),
                    (dict(mask=valid[:, None, None, :]), g["keypad_o_mask"])):  # host mask
        out = vx.dot_product_attention(q, k, v, **kw)
        mx, mean = compare(out.float().cpu().numpy(), ref)
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (list(kw), mx, mean)


@pytest.mark.gpu
def test_fully_masked_key_row_vs_reference_code():
    """A batch item with no visible key (valid lengths 41 and 0): the mask
    form gives the reference's mean of v over all keys, the -inf bias form its
    NaN rows; device and host inputs alike."""
    import vidax_b200 as vx
    g = np.load(os.path.join(GOLDEN, "attention_reference.npz"))
    q, k, v = _dev(g["keypad_q"]), _dev(g["keypad_k"]), _dev(g["keypad_v"])
    lens = torch.from_numpy(g["keypad0_len"]).long()
    valid = torch.arange(k.shape[1])[None, :] < lens[:, None]
    bias = torch.zeros(valid.shape).masked_fill(~valid, float("-inf"))[:, None, None, :]
    for host in (False, True):
        args = [t.cpu().pin_memory() for t in (q, k, v)] if host else [q, k, v]
        o_mask = vx.dot_product_attention(*args, mask=valid[:, None, None, :]).float().cpu().numpy()
        mx, mean = compare(o_mask, g["keypad0_o_mask"])
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (host, mx, mean)
        o_bias = vx.dot_product_attention(*args, bias=bias).float().cpu().numpy()
        assert np.isnan(o_bias[1]).all() and not np.isnan(o_bias[0]).any()
        mx, mean = compare(o_bias[0], g["keypad0_o_bias"][0])
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (host, mx, mean)


@pytest.mark.gpu
def test_ulysses_kernels_vs_reference_code():
    """P=8 Ulysses (1, 256, 8, 128): pack -> (chunk copies standing in for the
    NCCL all-to-all) -> attention -> unpack, per emulated rank, against the
    per-rank outputs of the reference's sequence_parallel_self_attention."""
    from vidax_b200 import flash_attention
    from vidax_b200.ulysses import pack_heads, unpack_heads
    g = np.load(os.path.join(GOLDEN, "attention_reference.npz"))
    P = 8
    qg, kg, vg = (g[f"sp{P}_{n}"] for n in "qkv")
    ref = g[f"sp{P}_o"]
    B, S, H, D = qg.shape
    S_loc = S // P
    loc = [[_dev(x[:, r * S_loc:(r + 1) * S_loc]) for x in (qg, kg, vg)] for r in range(P)]
    sends = [pack_heads([t[0] for t in loc[r]], P) for r in range(P)]
    Hg = sends[0][0].shape[2]
    outs = []
    for r in range(P):
        recv = [torch.stack([sends[src][t][r] for src in range(P)]).reshape(1, S, Hg, D)
                for t in range(3)]
        outs.append(flash_attention(*recv, D ** -0.5).reshape(P, S_loc, Hg, D))
    for dst in range(P):
        o = torch.empty((S_loc, H, D), dtype=torch.bfloat16, device="cuda")
        unpack_heads([torch.stack([outs[src][dst] for src in range(P)])], [o], H)
        mx, mean = compare(o.float().cpu().numpy()[None], ref[dst])
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (dst, mx, mean)
