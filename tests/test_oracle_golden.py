"""The CPU oracle against fixtures produced by the reference's own code.

tests/golden/*.npz were written by tests/golden/make_golden.py, which runs
vidax's `_window_start`, `neighborhood_attention_3d`, `dot_product_attention`,
`local_attention` and `sequence_parallel_self_attention` (under a numpy shim
of the jax primitives; JAX itself is not installed). These tests pin the
oracle that every GPU parity test relies on.
"""
import os

import numpy as np
import pytest

from oracle.attention_ref import sdpa, to_bf16
from oracle.na3d_ref import na3d, window_start
from oracle.ulysses_ref import all_to_all_tiled, chunk_by_rank, ulysses_attention

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _assert_bf16_close(got, ref):
    """Same math in a different f32 summation order: the bf16 results agree
    bit for bit almost everywhere and differ by at most a few ulps where a
    rounding boundary (of a logit, a weight or the output) falls between."""
    d = np.abs(np.asarray(got, np.float32) - np.asarray(ref, np.float32))
    assert d.max() <= 2e-3, d.max()
    assert np.mean(d == 0) >= 0.99, np.mean(d == 0)


@pytest.fixture(scope="module")
def na_gold():
    return np.load(os.path.join(GOLDEN, "na3d_reference.npz"))


@pytest.fixture(scope="module")
def attn_gold():
    return np.load(os.path.join(GOLDEN, "attention_reference.npz"))


def test_window_start_bit_exact(na_gold):
    for L, k, st in zip(na_gold["ws_length"], na_gold["ws_kernel"], na_gold["ws_start"]):
        assert np.array_equal(window_start(int(L), int(k)), st[:L]), (L, k)


@pytest.mark.parametrize("i", range(8))
def test_na3d_oracle_matches_reference_code(na_gold, i):
    q, k, v = (na_gold[f"na{i}_{n}"] for n in "qkv")
    kernel = tuple(int(x) for x in na_gold[f"na{i}_kernel"])
    ref = na_gold[f"na{i}_o"]
    got = to_bf16(na3d(q, k, v, kernel, round_logits=True, round_probs=True))
    _assert_bf16_close(got, ref)
    # the fp32-softmax reference used by the GPU tolerance stays within it
    f32 = na3d(q, k, v, kernel)
    assert np.abs(f32 - ref).max() <= 2e-2


def test_dot_product_attention_cpu_path(attn_gold):
    q, k, v = attn_gold["dpa128_q"], attn_gold["dpa128_k"], attn_gold["dpa128_v"]
    _assert_bf16_close(to_bf16(sdpa(q, k, v, round_probs=True)), attn_gold["dpa128_o"])
    kx, vx = attn_gold["cross128_k"], attn_gold["cross128_v"]
    _assert_bf16_close(to_bf16(sdpa(q, kx, vx, round_probs=True)), attn_gold["cross128_o"])
    q, k, v = attn_gold["dpa_q"], attn_gold["dpa_k"], attn_gold["dpa_v"]
    for key, scale in (("dpa_o_default", None), ("dpa_o_scale1", 1.0), ("local_o", None)):
        ref = attn_gold[key]
        got = to_bf16(sdpa(q, k, v, scale=scale, round_probs=True))
        _assert_bf16_close(got, ref)
        assert np.abs(sdpa(q, k, v, scale=scale) - ref).max() <= 2e-2


@pytest.mark.parametrize("P", [2, 4, 8])
def test_ulysses_layout_matches_reference_code(attn_gold, P):
    qg, kg, vg = (attn_gold[f"sp{P}_{n}"] for n in "qkv")
    ref = attn_gold[f"sp{P}_o"]                           # (P, B, S/P, H, D)
    loc = [[chunk_by_rank(x, 1, P, r) for r in range(P)] for x in (qg, kg, vg)]

    def attn(a, b, c):
        return to_bf16(sdpa(a, b, c, round_probs=True))

    outs = ulysses_attention(loc[0], loc[1], loc[2], attn)
    for r in range(P):
        _assert_bf16_close(outs[r], ref[r])
    # and the sequence-parallel result equals attention over the global sequence
    full = to_bf16(sdpa(qg, kg, vg, round_probs=True))
    S_loc = qg.shape[1] // P
    for r in range(P):
        assert np.abs(outs[r] - full[:, r * S_loc:(r + 1) * S_loc]).max() <= 2e-2


def test_all_to_all_tiled_is_inverse_of_itself():
    rng = np.random.default_rng(0)
    P = 4
    xs = [rng.standard_normal((2, 6, 8, 3)) for _ in range(P)]
    there = all_to_all_tiled(xs, 2, 1)
    assert there[0].shape == (2, 24, 2, 3)
    back = all_to_all_tiled(there, 1, 2)
    for a, b in zip(xs, back):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("i", [0, 1])
def test_rope_oracle_matches_reference_code(i):
    from oracle.rope_norm_ref import apply_rope3d, rope3d_freqs
    g = np.load(os.path.join(GOLDEN, "rope_reference.npz"))
    t, h, w, hd = (int(x) for x in g[f"rope{i}_grid"])
    cos, sin = rope3d_freqs(t, h, w, hd)
    assert np.array_equal(cos, g[f"rope{i}_cos"]) and np.array_equal(sin, g[f"rope{i}_sin"])
    y = apply_rope3d(g[f"rope{i}_x"], cos, sin)
    assert np.array_equal(y, g[f"rope{i}_y"])


@pytest.mark.parametrize("i", [0, 1, 2, 3])
def test_rmsnorm_oracle_matches_reference_code(i):
    from oracle.rope_norm_ref import rms_norm
    g = np.load(os.path.join(GOLDEN, "rope_reference.npz"))
    y = rms_norm(g[f"rms{i}_x"], g[f"rms{i}_w"])
    assert np.array_equal(y, g[f"rms{i}_y"])


def test_timestep_embedding_matches_reference_code():
    """The DiT driver's sinusoidal timestep embedding against the reference's
    sinusoidal_embedding_1d run on the same float32 host math: bit-exact."""
    import torch
    from vidax_b200.wan_dit import sinusoidal_embedding_1d
    g = np.load(os.path.join(GOLDEN, "rope_reference.npz"))
    got = sinusoidal_embedding_1d(256, torch.from_numpy(g["sinusoid_t"])).numpy()
    assert got.shape == g["sinusoid_emb"].shape
    assert np.array_equal(got, g["sinusoid_emb"])


def test_patchify_round_trip_and_oracle_order():
    import torch
    from oracle.wan_dit_ref import wan_dit_forward  # noqa: F401  (module imports cleanly)
    from vidax_b200.wan_dit import patchify, unpatchify
    x = torch.randn(2, 4, 6, 10, 3)
    p = patchify(x, (2, 2, 2))
    assert p.shape == (2, 2 * 3 * 5, 8 * 3)
    # patch vector = (pt, ph, pw, C) of one patch
    assert torch.equal(p[1, 3 * 5 + 2 * 5 + 4].reshape(2, 2, 2, 3), x[1, 2:4, 4:6, 8:10])
    assert torch.equal(unpatchify(p, (2, 2, 3, 5), (2, 2, 2), 3), x)


@pytest.mark.parametrize("P", [2, 4])
def test_joint_ulysses_matches_reference_code(attn_gold, P):
    """The reference's joint [text; visual] Ulysses per emulated rank: the
    text rows (all-gathered over heads, identical on every rank) and the
    rank's visual chunk equal attention over the global joint sequence."""
    qg, kg, vg = (attn_gold[f"joint{P}_{n}"] for n in "qkv")
    T = int(attn_gold[f"joint{P}_text_len"][0])
    ref = attn_gold[f"joint{P}_o"]                        # (P, B, T + S/P, H, D)
    full = to_bf16(sdpa(qg, kg, vg, round_probs=True))
    S_loc = (qg.shape[1] - T) // P
    for r in range(P):
        want = np.concatenate([full[:, :T], full[:, T + r * S_loc:T + (r + 1) * S_loc]], axis=1)
        _assert_bf16_close(want, ref[r])
        assert np.array_equal(ref[r][:, :T], ref[0][:, :T])


def test_key_padding_matches_reference_code(attn_gold):
    """dot_product_attention with a 0 / -inf key bias and with the boolean
    mask form, ragged valid lengths: the oracle's kv_len restatement."""
    q, k, v = attn_gold["keypad_q"], attn_gold["keypad_k"], attn_gold["keypad_v"]
    lens = attn_gold["keypad_len"]
    got = to_bf16(sdpa(q, k, v, kv_len=lens, round_probs=True))
    _assert_bf16_close(got, attn_gold["keypad_o_bias"])
    _assert_bf16_close(got, attn_gold["keypad_o_mask"])


@pytest.mark.parametrize("P,tag", [(4, "joint4d128"), (2, "joint2d64")])
def test_joint_ulysses_kernel_sized_fixtures(attn_gold, P, tag):
    """The head_dim-128 / 64 joint fixtures (the sizes the CUDA kernel takes)
    against the oracle, as for the small ones."""
    qg, kg, vg = (attn_gold[f"{tag}_{n}"] for n in "qkv")
    T = int(attn_gold[f"{tag}_text_len"][0])
    ref = attn_gold[f"{tag}_o"]
    full = to_bf16(sdpa(qg, kg, vg, round_probs=True))
    S_loc = (qg.shape[1] - T) // P
    for r in range(P):
        want = np.concatenate([full[:, :T], full[:, T + r * S_loc:T + (r + 1) * S_loc]], axis=1)
        _assert_bf16_close(want, ref[r])


@pytest.fixture(scope="module")
def ltx_gold():
    return np.load(os.path.join(GOLDEN, "ltx_reference.npz"))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_ltx_abs_rope_oracle_matches_reference_code(ltx_gold, i):
    """LTX-2.5's absolute split RoPE (diffusion_vae.py:96-150): the oracle's
    restatement is bit-exact against the reference's own `_apply_abs_rope`."""
    from oracle.rope_norm_ref import ltx_abs_rope, ltx_default_rope_split
    split = tuple(int(x) for x in ltx_gold[f"ltxrope{i}_split"])
    hd = int(ltx_gold[f"ltxrope{i}_grid"][3])
    if i < 2:
        assert ltx_default_rope_split(hd) == split
    y = ltx_abs_rope(ltx_gold[f"ltxrope{i}_x"], split)
    assert np.array_equal(y, ltx_gold[f"ltxrope{i}_y"])


@pytest.mark.parametrize("i", [0, 1, 2])
def test_ltx_rope_tables_match_reference_code(ltx_gold, i):
    """The product's table builder (host numpy, no device needed): every
    token's pair p holds cos / sin of its axis's float32 angle exactly as the
    reference computes it."""
    from vidax_b200.prologue import ltx_default_rope_split, ltx_rope_freqs
    t, h, w, hd = (int(x) for x in ltx_gold[f"ltxrope{i}_grid"])
    split = tuple(int(x) for x in ltx_gold[f"ltxrope{i}_split"])
    if i < 2:
        assert ltx_default_rope_split(hd) == split
    cos, sin = (x.numpy().reshape(t, h, w, hd // 2) for x in ltx_rope_freqs(t, h, w, hd, split))
    d0, d1 = split[0] // 2, (split[0] + split[1]) // 2
    for k, tab in (("cos", cos), ("sin", sin)):
        ref0, ref1, ref2 = (ltx_gold[f"ltxrope{i}_{k}{a}"] for a in range(3))
        assert np.array_equal(tab[..., :d0], np.broadcast_to(ref0[:, None, None, :], (t, h, w, d0)))
        assert np.array_equal(tab[..., d0:d1], np.broadcast_to(ref1[None, :, None, :], (t, h, w, d1 - d0)))
        assert np.array_equal(tab[..., d1:], np.broadcast_to(ref2[None, None, :, :], (t, h, w, hd // 2 - d1)))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_ltx_na_block_oracle_matches_reference_code(ltx_gold, i):
    """NeighborhoodAttention3D.__call__ between its projections (per-head
    RMSNorm, bf16 q scale, abs RoPE, NA): the oracle's q / k after the
    prologue are bit-exact, its output within the bf16 rounding spread."""
    from oracle.rope_norm_ref import ltx_na_prologue
    q, k, v = (ltx_gold[f"ltxna{i}_{n}"] for n in "qkv")
    qr, kr = ltx_na_prologue(q, k, ltx_gold[f"ltxna{i}_wq"], ltx_gold[f"ltxna{i}_wk"])
    assert np.array_equal(qr, ltx_gold[f"ltxna{i}_qr"])
    assert np.array_equal(kr, ltx_gold[f"ltxna{i}_kr"])
    kernel = tuple(int(x) for x in ltx_gold[f"ltxna{i}_kernel"])
    got = to_bf16(na3d(qr, kr, v, kernel, round_logits=True, round_probs=True))
    _assert_bf16_close(got, ltx_gold[f"ltxna{i}_o"])


def test_fully_masked_key_row_matches_reference_code(attn_gold):
    """A batch item with no visible key: jax.nn's mask form gives the mean of
    v over all keys (uniform weights), its -inf bias form gives NaN."""
    q, k, v = attn_gold["keypad_q"], attn_gold["keypad_k"], attn_gold["keypad_v"]
    lens = attn_gold["keypad0_len"]
    valid = np.arange(k.shape[1])[None, :] < lens[:, None]
    got = to_bf16(sdpa(q, k, v, key_mask=valid, round_probs=True))
    _assert_bf16_close(got, attn_gold["keypad0_o_mask"])
    assert np.isnan(attn_gold["keypad0_o_bias"][1]).all()
    bias = np.where(valid, 0.0, -np.inf).astype(np.float32)
    with np.errstate(invalid="ignore"):
        got = to_bf16(sdpa(q, k, v, key_bias=bias, round_probs=True))
    assert np.isnan(got[1]).all()
    _assert_bf16_close(got[0], attn_gold["keypad0_o_bias"][0])
