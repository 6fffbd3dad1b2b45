"""The Ulysses product orchestration on the real CUDA kernels, P ranks
emulated as threads on one GPU (tests/emulated_ranks.py stands in for
torch.distributed; its all-to-alls and all-gathers are device-synchronised
copies). What runs unchanged is the product code a multi-GPU job runs:

* `sequence_parallel_self_attention` -> `_ulysses_one`: the pipelined head
  slices (sub-group `vx_ulysses_pack`, per-slice exchanges, the attention
  kernel on the dynamic schedule, reverse exchange and sub-group unpack on
  the side stream), head padding for H % P != 0, `valid_len` key masking;
* `attend` under sequence parallelism -> `_attend_sp`: one fused RMSNorm +
  RoPE + send-slab launch feeding the same pipeline;
* `sequence_parallel_self_attention_from_host`: host rows copied straight
  into the send slabs and out of the receive slabs;
* `sequence_parallel_self_attention_qsplit`: query-split heads with uneven
  all-to-alls.

References: the per-rank outputs of vidax's own
`sequence_parallel_self_attention` (tests/golden, P = 8) and the oracle of
the global sequence. Tolerance: max-abs 2e-2, mean-abs 2e-3."""
import numpy as np
import pytest
import torch

from emulated_ranks import RankGroup, run_ranks
from oracle.attention_ref import compare, sdpa, seeded_qkv

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


def _setup(monkeypatch, P):
    import vidax_b200 as vx
    from vidax_b200 import ulysses, ulysses_qsplit
    fake = RankGroup(P)
    monkeypatch.setattr(ulysses, "dist", fake)
    monkeypatch.setattr(ulysses_qsplit, "dist", fake)
    vx.register_axis("sp_emul", None)
    return vx, fake


def _teardown(vx):
    vx.unregister_axis("sp_emul")
    from vidax_b200 import _lib
    assert _lib.device_status(clear=True) == 0


def _gathered(results, T_len=0):
    """Per-rank (B, L_loc, H, D) outputs -> the global (B, S, H, D) array."""
    return np.concatenate([r[:, T_len:] for r in results], axis=1)


@pytest.mark.gpu
def test_sp8_vs_reference_code(monkeypatch):
    """P = 8, 8 heads, (1, 256, 8, 128): every rank against the per-rank
    output of vidax's sequence_parallel_self_attention."""
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                             "attention_reference.npz"))
    P = 8
    qg, kg, vg = (g[f"sp{P}_{n}"] for n in "qkv")
    ref = g[f"sp{P}_o"]
    S_loc = qg.shape[1] // P
    vx, fake = _setup(monkeypatch, P)
    try:
        res = run_ranks(P, fake, lambda r: vx.sequence_parallel_self_attention(
            *[_dev(x[:, r * S_loc:(r + 1) * S_loc]) for x in (qg, kg, vg)], "sp_emul"
        ).float().cpu().numpy())
    finally:
        _teardown(vx)
    for r in range(P):
        mx, mean = compare(res[r], ref[r])
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (r, mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,P", [(1, 1024, 10, 2),   # Hg 5: slices 1, 2, 2
                                     (2, 768, 6, 4),     # H % P != 0: zero-padded heads
                                     (1, 2048, 40, 8),   # cfg3's heads on 8 ranks: Hg 5
                                     (1, 960, 12, 8)])   # cfg5's 12 heads on 8 ranks
def test_sliced_pipeline_vs_oracle(monkeypatch, B, S, H, P):
    from vidax_b200.ulysses import _pieces
    assert len(_pieces(-(-H // P))) >= 1
    q, k, v = seeded_qkv((B, S, H, 128), 500 + S + H + P)
    S_loc = S // P
    vx, fake = _setup(monkeypatch, P)
    try:
        res = run_ranks(P, fake, lambda r: vx.sequence_parallel_self_attention(
            *[_dev(x[:, r * S_loc:(r + 1) * S_loc]) for x in (q, k, v)], "sp_emul"
        ).float().cpu().numpy())
    finally:
        _teardown(vx)
    mx, mean = compare(_gathered(res), sdpa(q, k, v))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_valid_len_masks_padding_keys(monkeypatch):
    """A sequence padded to a multiple of P (valid_len < S): pad keys are
    invisible to every query, pad rows are don't-care."""
    B, S, H, P, valid = 1, 1024, 4, 4, 1000
    q, k, v = seeded_qkv((B, S, H, 128), 611)
    S_loc = S // P
    vx, fake = _setup(monkeypatch, P)
    try:
        res = run_ranks(P, fake, lambda r: vx.sequence_parallel_self_attention(
            *[_dev(x[:, r * S_loc:(r + 1) * S_loc]) for x in (q, k, v)], "sp_emul",
            valid_len=valid).float().cpu().numpy())
    finally:
        _teardown(vx)
    ref = sdpa(q[:, :valid], k[:, :valid], v[:, :valid])
    mx, mean = compare(_gathered(res)[:, :valid], ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("grid,H,P", [((4, 8, 16), 8, 2), ((2, 6, 16), 5, 4), ((4, 8, 12), 12, 8)])
def test_attend_fused_prologue_pipeline_vs_oracle(monkeypatch, grid, H, P):
    """Wan's attend under sequence parallelism: per rank one fused RMSNorm(dim)
    + 3-D RoPE + send-slab launch, then the sliced exchange / attention
    pipeline; each rank holds its chunk of the projections and of the RoPE
    tables of its tokens' global positions."""
    from oracle.rope_norm_ref import norm_rope, rope3d_freqs
    t, h, w = grid
    S, D = t * h * w, 128
    S_loc = S // P
    q, k, v = seeded_qkv((1, S, H * D), 700 + S + H + P)
    rng = np.random.Generator(np.random.PCG64(S + H))
    wq, wk = ((1.0 + 0.25 * rng.standard_normal(H * D)).astype(np.float32) for _ in range(2))
    cos, sin = rope3d_freqs(t, h, w, D)
    vx, fake = _setup(monkeypatch, P)
    try:
        dcos, dsin = vx.rope3d_freqs(t, h, w, D, device="cuda")

        def rank(r):
            sl = slice(r * S_loc, (r + 1) * S_loc)
            o = vx.attend(*[_dev(x[:, sl]) for x in (q, k, v)], H, norm_q=torch.from_numpy(wq),
                          norm_k=torch.from_numpy(wk), rope=(dcos[sl], dsin[sl]),
                          sp_axis_name="sp_emul")
            return o.float().cpu().numpy().reshape(1, S_loc, H, D)

        res = run_ranks(P, fake, rank)
    finally:
        _teardown(vx)
    qr, kr = norm_rope(q, wq, cos, sin, H), norm_rope(k, wk, cos, sin, H)
    ref = sdpa(qr, kr, v.reshape(1, S, H, D))
    mx, mean = compare(_gathered(res), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,P", [(1, 1024, 8, 2), (2, 512, 6, 4)])
def test_host_buffer_form_equals_device_form(monkeypatch, B, S, H, P):
    """Pinned host q/k/v through sequence_parallel_self_attention_from_host:
    the same slices and kernels, host rows copied straight into the send
    slabs and out of the receive slabs -- bit-equal to the device form."""
    q, k, v = seeded_qkv((B, S, H, 128), 800 + S + H)
    S_loc = S // P
    vx, fake = _setup(monkeypatch, P)
    try:
        def rank(r):
            mine = [_dev(x[:, r * S_loc:(r + 1) * S_loc]) for x in (q, k, v)]
            dev_out = vx.sequence_parallel_self_attention(*mine, "sp_emul")
            host_out = vx.sequence_parallel_self_attention_from_host(
                *[t.cpu().pin_memory() for t in mine], "sp_emul")
            torch.cuda.synchronize()
            return dev_out.cpu(), host_out.clone()

        res = run_ranks(P, fake, rank)
    finally:
        _teardown(vx)
    for r, (d, h) in enumerate(res):
        assert torch.equal(d, h), r
    mx, mean = compare(_gathered([d.float().numpy() for d, _ in res]), sdpa(q, k, v))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,P", [(1, 1024, 6, 4), (1, 960, 12, 8), (2, 768, 3, 2)])
def test_query_split_heads_vs_oracle(monkeypatch, B, S, H, P):
    """Query-split Ulysses (heads % ranks != 0 without padding): uneven
    all-to-alls around one attention launch over each rank's units."""
    q, k, v = seeded_qkv((B, S, H, 128), 850 + S + H + P)
    S_loc = S // P
    vx, fake = _setup(monkeypatch, P)
    try:
        res = run_ranks(P, fake, lambda r: vx.sequence_parallel_self_attention_qsplit(
            *[_dev(x[:, r * S_loc:(r + 1) * S_loc]) for x in (q, k, v)], "sp_emul"
        ).float().cpu().numpy())
    finally:
        _teardown(vx)
    mx, mean = compare(_gathered(res), sdpa(q, k, v))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
