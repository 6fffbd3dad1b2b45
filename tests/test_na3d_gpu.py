"""GPU parity of the sm_100a 3-D neighborhood-attention kernel.

Window/mask indexing is checked bit-exactly through a one-hot probe (values
that identify each key), outputs against the CPU oracle within max-abs 2e-2
and mean-abs 2e-3 of the fp32-softmax reference.
"""
import numpy as np
import pytest
import torch

from oracle.attention_ref import compare, seeded_qkv, to_bf16
from oracle.na3d_ref import na3d, window_sets

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda").to(torch.bfloat16)


def _status_clean():
    from vidax_b200 import _lib
    return _lib.device_status(clear=True) == 0


CASES = [
    # (B, T, H, W, NH), kernel
    ((1, 3, 5, 7, 2), (3, 3, 5)),
    ((1, 4, 9, 17, 1), (3, 5, 5)),
    ((2, 5, 6, 11, 2), (3, 7, 7)),
    ((1, 2, 3, 4, 1), (5, 9, 9)),       # kernel larger than the grid on every axis
    ((1, 6, 10, 40, 1), (5, 9, 9)),
    ((1, 3, 20, 33, 3), (1, 1, 1)),     # degenerate window: output == v
    ((1, 12, 12, 12, 1), (11, 11, 11)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape,kernel", CASES)
def test_na3d_matches_oracle(shape, kernel):
    import vidax_b200 as vx
    B, T, H, W, NH = shape
    q, k, v = seeded_qkv((B, T, H, W, NH, 128), 500 + T * 7 + W, n=3)
    q = to_bf16(q * np.float32(128 ** -0.5))
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), kernel)
    torch.cuda.synchronize()
    assert _status_clean()
    ref = na3d(q, k, v, kernel)
    mx, mean = compare(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("q_box,pair", [((2, 8, 8), 0), ((1, 8, 16), 2), ((4, 4, 8), 1),
                                        ((1, 2, 64), 0), ((8, 4, 4), 2)])
def test_na3d_every_tiling_agrees(q_box, pair):
    """Every query tiling gives the oracle's result (tiling is a schedule choice only)."""
    import vidax_b200 as vx
    B, T, H, W, NH = 1, 7, 13, 21, 2
    q, k, v = seeded_qkv((B, T, H, W, NH, 128), 77, n=3)
    q = to_bf16(q * np.float32(128 ** -0.5))
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), (5, 9, 9),
                                       q_box=q_box, pair_axis=pair)
    torch.cuda.synchronize()
    assert _status_clean()
    mx, mean = compare(out.float().cpu().numpy(), na3d(q, k, v, (5, 9, 9)))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_na3d_window_sets_bit_exact():
    """Attended key sets are exactly the reference windows: with q = 0 every
    visible key gets equal weight, so v = one-hot(key index bits) makes the
    output the mean of the attended keys' codes; with |window| a power of two
    this mean is exact in bf16 only if the set is exactly right. Instead of
    relying on rounding, each key's code is a distinct small integer and the
    output sum * |window| must equal the exact code sum per query."""
    import vidax_b200 as vx
    B, T, H, W, NH = 1, 5, 7, 11, 1
    kernel = (3, 5, 3)
    q = np.zeros((B, T, H, W, NH, 128), np.float32)
    k = np.zeros_like(q)
    # v[..., c] = bit c of the key's linear index (keys 0..384 need 9 bits)
    v = np.zeros_like(q)
    lin = np.arange(T * H * W).reshape(T, H, W)
    for c in range(9):
        v[0, :, :, :, 0, c] = (lin >> c) & 1
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), kernel).float().cpu().numpy()
    torch.cuda.synchronize()
    (st_t, kt), (st_h, kh), (st_w, kw) = window_sets(T, H, W, kernel)
    n = kt * kh * kw
    for t in range(T):
        for h in range(H):
            for w in range(W):
                keys = lin[st_t[t]:st_t[t] + kt, st_h[h]:st_h[h] + kh, st_w[w]:st_w[w] + kw].ravel()
                expect = np.array([((keys >> c) & 1).sum() for c in range(9)], np.float64) / n
                got = out[0, t, h, w, 0, :9]
                # each channel is a count/n in [0, 1]; bf16 keeps 8 bits, so
                # compare the recovered counts
                assert np.array_equal(np.rint(got * n), np.rint(expect * n)), (t, h, w)


@pytest.mark.gpu
def test_na3d_round_logits_matches_reference_rounding():
    import vidax_b200 as vx
    B, T, H, W, NH = 1, 4, 6, 10, 2
    q, k, v = seeded_qkv((B, T, H, W, NH, 128), 91, n=3)
    q = to_bf16(q * np.float32(128 ** -0.5))
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), (3, 5, 5), round_logits=True)
    torch.cuda.synchronize()
    ref = na3d(q, k, v, (3, 5, 5), round_logits=True)
    mx, mean = compare(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_cfg4_sampled_positions():
    """(1, 21, 30, 52, 24, 128), window 5x9x9, q pre-scaled;
    a seeded sample of query positions (all faces and corners included)."""
    import vidax_b200 as vx
    shape = (1, 21, 30, 52, 24, 128)
    q, k, v = seeded_qkv(shape, 4, n=3)
    q = to_bf16(q * np.float32(128 ** -0.5))
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), (5, 9, 9))
    torch.cuda.synchronize()
    assert _status_clean()
    rng = np.random.default_rng(4)
    pos = np.stack([rng.integers(0, 21, 40), rng.integers(0, 30, 40), rng.integers(0, 52, 40)], 1)
    corners = np.array([[t, h, w] for t in (0, 20) for h in (0, 29) for w in (0, 51)])
    pos = np.concatenate([pos, corners, [[10, 15, 26], [1, 1, 1], [19, 28, 50]]])
    ref = na3d(q, k, v, (5, 9, 9), positions=pos)
    got = out.float().cpu().numpy()[0][pos[:, 0], pos[:, 1], pos[:, 2]][None]
    mx, mean = compare(got, ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,kernel", [
    ((1, 4, 9, 17, 2), (3, 5, 5)),
    ((1, 5, 12, 20, 2), (3, 7, 7)),
    ((1, 12, 13, 14, 1), (11, 11, 11)),   # the LTX-2.5 stage-5 window
    ((2, 3, 6, 9, 2), (3, 3, 3)),
])
def test_na3d_head_dim_64(shape, kernel):
    """The production LTX-2.5 decoder runs neighborhood attention at head_dim 64."""
    import vidax_b200 as vx
    B, T, H, W, NH = shape
    q, k, v = seeded_qkv((B, T, H, W, NH, 64), 700 + T * 7 + W, n=3)
    q = to_bf16(q * np.float32(64 ** -0.5))
    out = vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), kernel)
    torch.cuda.synchronize()
    assert _status_clean()
    mx, mean = compare(out.float().cpu().numpy(), na3d(q, k, v, kernel))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,kernel,q_box,kv_heads,kv_tile", [
    ((1, 4, 9, 17, 2), (3, 5, 5), (2, 8, 8), 2, (2, 4, 16)),
    ((1, 5, 12, 20, 3), (3, 7, 7), (1, 8, 16), 3, (2, 4, 16)),  # odd head count: one head in the last pair
    ((2, 6, 10, 12, 4), (3, 5, 5), (4, 4, 8), 2, (2, 4, 16)),   # grouped K / V heads
    ((1, 12, 13, 14, 2), (11, 11, 11), (8, 4, 4), 2, (2, 4, 16)),
    ((1, 5, 12, 20, 3), (3, 7, 7), (2, 8, 8), 3, (4, 2, 16)),   # the other key tiles
    ((1, 6, 11, 19, 2), (3, 5, 5), (8, 4, 4), 2, (2, 8, 8)),
    ((2, 6, 10, 12, 4), (3, 5, 5), (2, 16, 4), 2, (4, 4, 8)),
    ((1, 9, 13, 14, 2), (11, 11, 11), (8, 4, 4), 1, (2, 8, 8)),
])
def test_na3d_head_pairs_head_dim_64(shape, kernel, q_box, kv_heads, kv_tile):
    """Head-pair tiling (pair_axis 3: the CTA's two query tiles are one box of
    heads h and h + 1, each with its own K / V tiles) against the oracle and
    against the box-pair tiling of the same box."""
    import vidax_b200 as vx
    B, T, H, W, NH = shape
    q, _, _ = seeded_qkv((B, T, H, W, NH, 64), 760 + T * 7 + W, n=3)
    _, k, v = seeded_qkv((B, T, H, W, kv_heads, 64), 761 + T * 7 + W, n=3)
    q = to_bf16(q * np.float32(64 ** -0.5))
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    out = vx.neighborhood_attention_3d(qd, kd, vd, kernel, q_box=q_box, pair_axis=3,
                                       kv_tile=kv_tile)
    boxes = vx.neighborhood_attention_3d(qd, kd, vd, kernel, q_box=q_box, pair_axis=0)
    torch.cuda.synchronize()
    assert _status_clean()
    rep = NH // kv_heads
    ref = na3d(q, np.repeat(k, rep, axis=4), np.repeat(v, rep, axis=4), kernel)
    mx, mean = compare(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    mx2, _ = compare(out.float().cpu().numpy(), boxes.float().cpu().numpy())
    assert mx2 <= MAX_ABS, mx2


@pytest.mark.gpu
def test_na3d_head_pairs_need_head_dim_64():
    import vidax_b200 as vx
    from vidax_b200._lib import VxError
    q, k, v = seeded_qkv((1, 4, 8, 16, 2, 128), 79, n=3)
    with pytest.raises(VxError):
        vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), (3, 5, 5), q_box=(2, 8, 8),
                                     pair_axis=3)
    q, k, v = seeded_qkv((1, 4, 8, 16, 2, 64), 80, n=3)
    with pytest.raises(VxError):   # box pairs read (2, 4, 16) key tiles only
        vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), (3, 5, 5), q_box=(2, 8, 8),
                                     pair_axis=0, kv_tile=(2, 8, 8))
    with pytest.raises(VxError):   # not a key tile of the library
        vx.neighborhood_attention_3d(_dev(q), _dev(k), _dev(v), (3, 5, 5), q_box=(2, 8, 8),
                                     pair_axis=3, kv_tile=(1, 2, 64))


@pytest.mark.gpu
@pytest.mark.parametrize("shape,kernel,world", [
    ((1, 21, 10, 24, 2), (5, 9, 9), 2),
    ((1, 21, 10, 24, 2), (5, 9, 9), 8),      # 2-3 frame slabs: halo from one neighbour
    ((2, 13, 9, 17, 1), (11, 5, 5), 4),      # halo spans several ranks
    ((1, 7, 6, 20, 2), (3, 7, 7), 3),
    ((1, 4, 8, 8, 1), (5, 3, 3), 4),         # one-frame slabs, window wider than a slab
])
def test_na3d_time_slabs_emulated_ranks(shape, kernel, world):
    """Each rank's slab (its frames of q, the key frames it would receive in
    the halo exchange) through vx_na3d_fwd_slab, assembled along T, equals the
    unsharded oracle; windows clamp to the global grid, not the slab."""
    import vidax_b200 as vx
    from vidax_b200.na_parallel import key_ranges, slab_bounds, split_sizes
    B, T, H, W, NH = shape
    q, k, v = seeded_qkv((B, T, H, W, NH, 128), 900 + T + W + world, n=3)
    q = to_bf16(q * np.float32(128 ** -0.5))
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    bounds = slab_bounds(split_sizes(T, world))
    outs = []
    for r, (kv0, kv1) in enumerate(key_ranges(bounds, kernel[0])):
        b0, b1 = bounds[r], bounds[r + 1]
        outs.append(vx.neighborhood_attention_3d_slab(
            qd[:, b0:b1].contiguous(), kd[:, kv0:kv1].contiguous(), vd[:, kv0:kv1].contiguous(),
            kernel, t_global=T, q_t0=b0, kv_t0=kv0))
    got = torch.cat(outs, dim=1)
    full = vx.neighborhood_attention_3d(qd, kd, vd, kernel)
    torch.cuda.synchronize()
    assert _status_clean()
    ref = na3d(q, k, v, kernel)
    mx, mean = compare(got.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    mx2, _ = compare(got.float().cpu().numpy(), full.float().cpu().numpy())
    assert mx2 <= MAX_ABS, mx2


@pytest.mark.gpu
@pytest.mark.parametrize("shape,kernel,world", [((1, 9, 10, 20, 3), (3, 5, 5), 3),
                                               ((1, 8, 12, 16, 2), (3, 7, 7), 4)])
def test_na3d_time_slabs_head_dim_64(shape, kernel, world):
    """Time slabs at head_dim 64, where the tiling chooser picks head pairs:
    the slabs assembled along T equal the unsharded oracle."""
    import vidax_b200 as vx
    from vidax_b200.na_parallel import key_ranges, slab_bounds, split_sizes
    B, T, H, W, NH = shape
    q, k, v = seeded_qkv((B, T, H, W, NH, 64), 930 + T + W + world, n=3)
    q = to_bf16(q * np.float32(64 ** -0.5))
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    bounds = slab_bounds(split_sizes(T, world))
    outs = []
    for r, (kv0, kv1) in enumerate(key_ranges(bounds, kernel[0])):
        b0, b1 = bounds[r], bounds[r + 1]
        outs.append(vx.neighborhood_attention_3d_slab(
            qd[:, b0:b1].contiguous(), kd[:, kv0:kv1].contiguous(), vd[:, kv0:kv1].contiguous(),
            kernel, t_global=T, q_t0=b0, kv_t0=kv0))
    got = torch.cat(outs, dim=1)
    torch.cuda.synchronize()
    assert _status_clean()
    mx, mean = compare(got.float().cpu().numpy(), na3d(q, k, v, kernel))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_na3d_slab_rejects_uncovered_windows():
    import vidax_b200 as vx
    from vidax_b200._lib import VxInvalid
    q, k, v = seeded_qkv((1, 8, 4, 8, 1, 128), 77, n=3)
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    with pytest.raises(VxInvalid):   # frames 2..5 read keys 0..7 with a 5-frame window; 1..6 given
        vx.neighborhood_attention_3d_slab(qd[:, 2:6].contiguous(), kd[:, 1:7].contiguous(),
                                          vd[:, 1:7].contiguous(), (5, 3, 3), t_global=8,
                                          q_t0=2, kv_t0=1)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_na3d_time_sharded_two_gpus_nccl():
    """Real halo exchange: 2 ranks over NCCL vs the oracle of the whole grid."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29613",
           os.path.join(root, "tests", "dist_na_check.py")]
    res = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "NA SP OK" in res.stdout

