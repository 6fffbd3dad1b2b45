"""Fused QK RMSNorm + 3-D RoPE + head-slab pack (vx_norm_rope_pack) against
the oracle restatement of RMSNorm / create_rope3d_freqs / apply_rope3d.

Bit-exactness: given the same mean square, every step is the reference's
float32 formula with the same roundings, so the output is bit-identical.
The mean square itself is a float32 sum whose order the reference leaves to
the backend; inputs with small integer values make every partial sum exact
(order-independent), and those cases are compared bit for bit. Random
normal inputs may differ where the summation order moves the mean square by
an ulp: they must agree bit for bit on >= 99.9 % of elements and within one
bf16 ulp of the rotated pair's magnitude elsewhere."""
import numpy as np
import pytest
import torch

from oracle.attention_ref import compare, sdpa, to_bf16
from oracle.rope_norm_ref import apply_rope3d, rms_norm, rope3d_freqs

ONE_ULP = 2.0 ** -7  # bf16 spacing relative to the value (8 significant bits)


def _seeded(shape, seed, scale=1.0, integer=False):
    rng = np.random.Generator(np.random.PCG64(seed))
    if integer:
        return rng.integers(-4, 5, size=shape).astype(np.float32)
    return to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


def _weight(n, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    return (1.0 + 0.25 * rng.standard_normal(n)).astype(np.float32)


def _cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


def _oracle(x, w, cos, sin, heads, per_head=False, post_scale=1.0):
    B, S, dim = x.shape
    D = dim // heads
    y = x.reshape(B, S, heads, D)
    if w is not None:
        y = rms_norm(y, w) if per_head else rms_norm(x, w).reshape(B, S, heads, D)
    if post_scale != 1.0:
        y = to_bf16(y * np.float32(post_scale))
    if cos is not None:
        y = apply_rope3d(y, cos, sin)
    return y


def _check(got, ref, exact):
    """A last-bit change of a rotated pair's inputs (a, b) moves each output
    by at most ONE_ULP * (|a| + |b|) <= 2 ONE_ULP * |(a, b)| -- the pair's
    magnitude, which the rotation preserves -- plus the output's own
    rounding."""
    if exact:
        assert np.array_equal(got, ref), int(np.sum(got != ref))
        return
    diff = got != ref
    assert diff.mean() <= 1e-3, diff.mean()
    pair = np.sqrt(np.sum(np.square(ref.reshape(ref.shape[:-1] + (-1, 2))), axis=-1))
    pair = np.repeat(pair, 2, axis=-1).reshape(ref.shape)
    tol = 2 * ONE_ULP * pair + ONE_ULP * np.abs(ref) + 1e-30
    assert np.all(np.abs(got - ref)[diff] <= tol[diff]), float(np.max(np.abs(got - ref)))


@pytest.mark.gpu
@pytest.mark.parametrize("integer", [True, False])
@pytest.mark.parametrize("grid,heads,D", [((3, 10, 10), 12, 128), ((2, 6, 9), 40, 128),
                                          ((4, 5, 7), 8, 64)])
def test_wan_full_row_norm_rope(grid, heads, D, integer):
    """Wan: RMSNorm over all H*D features, then 3-D RoPE (dit_layers.py:137-149)."""
    from vidax_b200 import rms_norm_rope, rope3d_freqs as tables
    t, h, w = grid
    S, dim = t * h * w, heads * D
    x = _seeded((2, S, dim), 7 + S + heads, scale=2.0, integer=integer)
    wq = _weight(dim, 11 + heads)
    cos, sin = rope3d_freqs(t, h, w, D)
    dcos, dsin = tables(t, h, w, D, device="cuda")
    assert np.array_equal(dcos.cpu().numpy(), cos) and np.array_equal(dsin.cpu().numpy(), sin)
    got = rms_norm_rope(_cuda(x), torch.from_numpy(wq), (dcos, dsin), heads)
    torch.cuda.synchronize()
    _check(got.float().cpu().numpy(), _oracle(x, wq, cos, sin, heads), integer)


@pytest.mark.gpu
@pytest.mark.parametrize("integer", [True, False])
@pytest.mark.parametrize("heads,D,post", [(8, 64, 0.125), (24, 128, 1.0), (4, 256, 0.5)])
def test_per_head_norm_post_scale_rope(heads, D, post, integer):
    """HunyuanVideo / LTX-2.5: RMSNorm(head_dim), LTX's q scaling, RoPE from
    arbitrary per-token tables (LTX's absolute-position tables)."""
    from vidax_b200 import rms_norm_rope
    S = 333
    x = _seeded((1, S, heads * D), 21 + heads, scale=1.5, integer=integer)
    wq = _weight(D, 23 + D)
    rng = np.random.Generator(np.random.PCG64(5))
    ang = rng.uniform(-10, 10, size=(S, D // 2)).astype(np.float32)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    got = rms_norm_rope(_cuda(x), torch.from_numpy(wq),
                        (torch.from_numpy(cos), torch.from_numpy(sin)), heads,
                        per_head=True, post_scale=post)
    torch.cuda.synchronize()
    _check(got.float().cpu().numpy(), _oracle(x, wq, cos, sin, heads, True, post), integer)


@pytest.mark.gpu
def test_rope_only_and_copy_bit_exact():
    """No norm: RoPE alone is exact; a tensor with nothing to do is a copy."""
    from vidax_b200 import norm_rope_pack
    heads, D, S = 6, 128, 250
    x = _seeded((2, S, heads * D), 31, scale=3.0)
    v = _seeded((2, S, heads * D), 32)
    ang = np.linspace(-50, 50, S * D // 2, dtype=np.float32).reshape(S, D // 2)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    xr, vc = norm_rope_pack([_cuda(x), _cuda(v)], heads,
                            rope=(torch.from_numpy(cos), torch.from_numpy(sin)), rope_mask=0b01)
    torch.cuda.synchronize()
    ref = apply_rope3d(x.reshape(2, S, heads, D), cos, sin).reshape(2, -1)
    assert np.array_equal(xr.float().cpu().numpy(), ref)
    assert np.array_equal(vc.float().cpu().numpy(), v.reshape(2, -1))


@pytest.mark.gpu
@pytest.mark.parametrize("H,P", [(12, 4), (10, 4), (40, 8), (3, 2)])
def test_sp_send_slabs_match_pack(H, P):
    """groups = P with the Ulysses pipeline's slices: each slice equals the
    sub-group pack (vx_ulysses_pack) of the plain normalised/rotated rows,
    bit for bit, including the zero heads of H % P != 0."""
    from vidax_b200 import norm_rope_pack
    from vidax_b200.prologue import slice_views
    from vidax_b200.ulysses import _pieces, pack_heads
    D, S_loc, B = 128, 96, 2
    xs = [_cuda(_seeded((B, S_loc, H * D), 40 + i + H, scale=2.0)) for i in range(3)]
    wq, wk = (torch.from_numpy(_weight(H * D, 50 + i)) for i in range(2))
    ang = np.random.Generator(np.random.PCG64(9)).uniform(0, 30, (S_loc, D // 2)).astype(np.float32)
    rope = (torch.from_numpy(np.cos(ang)), torch.from_numpy(np.sin(ang)))
    Hg = -(-H // P)
    sizes = _pieces(Hg)
    plain = norm_rope_pack(xs, H, norm_weights=[wq, wk, None], rope=rope)
    packed = norm_rope_pack(xs, H, norm_weights=[wq, wk, None], rope=rope, groups=P, slices=sizes)
    offs = [sum(sizes[:j]) for j in range(len(sizes))]
    for b in range(B):
        rows = [p[b].view(S_loc, H, D) for p in plain]
        views = [slice_views(p[b], P, S_loc, D, sizes) for p in packed]
        for j, (hs, off) in enumerate(zip(sizes, offs)):
            ref = pack_heads(rows, P, sub=(hs, Hg, off, hs))
            for t in range(3):
                assert torch.equal(views[t][j], ref[t]), (b, j, t)


@pytest.mark.gpu
def test_attend_matches_oracle():
    """Wan attend without sequence parallelism: norm + RoPE + attention."""
    from vidax_b200 import attend, rope3d_freqs as tables
    t, h, w, heads, D = 4, 8, 12, 4, 128
    S, dim = t * h * w, heads * D
    q, k, v = (_seeded((1, S, dim), 60 + i, scale=2.0) for i in range(3))
    wq, wk = _weight(dim, 70), _weight(dim, 71)
    cos, sin = rope3d_freqs(t, h, w, D)
    got = attend(_cuda(q), _cuda(k), _cuda(v), heads, norm_q=torch.from_numpy(wq),
                 norm_k=torch.from_numpy(wk), rope=tables(t, h, w, D, device="cuda"))
    torch.cuda.synchronize()
    qr = _oracle(q, wq, cos, sin, heads)
    kr = _oracle(k, wk, cos, sin, heads)
    ref = sdpa(qr, kr, v.reshape(1, S, heads, D))
    mx, mean = compare(got.float().cpu().numpy().reshape(1, S, heads, D), ref)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


def _call_raw(srcs, dsts, heads, D, weights, tables, rope_stride, groups=1):
    """vx_norm_rope_pack with explicit table pointers / strides (the Python
    wrapper always pairs the tables)."""
    import ctypes
    from vidax_b200 import _lib
    from vidax_b200.prologue import NormRopePackArgs
    a = NormRopePackArgs()
    a.num_tensors = len(srcs)
    for i, (x, o) in enumerate(zip(srcs, dsts)):
        a.src[i], a.dst[i] = x.data_ptr(), o.data_ptr()
        for k in range(3):
            a.src_stride[i][k] = x.stride(k)
        if weights[i] is not None:
            a.norm_weight[i] = weights[i].data_ptr()
        a.post_scale[i] = 1.0
    a.eps = 1e-6
    a.rope_cos, a.rope_sin = tables[0].data_ptr(), tables[1].data_ptr()
    a.rope_stride = rope_stride
    a.rope_mask = 0b011
    a.batch, a.seq, a.heads, a.head_dim, a.groups = srcs[0].shape[0], srcs[0].shape[1], heads, D, groups
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    _lib.check(lib.vx_norm_rope_pack(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)))


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["fused_qkv", "strided_heads", "plain"])
@pytest.mark.parametrize("tables", ["separate", "paired_padded", "paired"])
def test_source_and_table_layouts(layout, tables):
    """Every source-copy form (tokens adjacent, rows adjacent only, heads
    strided) and table form (separate cos / sin, cos|sin rows with padding,
    packed cos|sin rows) gives the same bits."""
    from vidax_b200 import norm_rope_pack
    H, D, S, B = 6, 128, 77, 2
    base = [_cuda(_seeded((B, S, H, D), 80 + i, scale=2.0)) for i in range(3)]
    w = [torch.from_numpy(_weight(H * D, 90 + i)).cuda() for i in range(2)] + [None]
    ang = np.random.Generator(np.random.PCG64(3)).uniform(-20, 20, (S, D // 2)).astype(np.float32)
    cos, sin = torch.from_numpy(np.cos(ang)).cuda(), torch.from_numpy(np.sin(ang)).cuda()
    want = norm_rope_pack(base, H, norm_weights=w, rope=(cos, sin))
    if layout == "fused_qkv":      # (B, S, 3, H, D) buffer: tokens 3*H*D apart
        buf = torch.stack(base, dim=2)
        srcs = [buf[:, :, i] for i in range(3)]
    elif layout == "strided_heads":  # (B, S, H, 3, D): heads 3*D apart
        buf = torch.stack(base, dim=3)
        srcs = [buf[:, :, :, i] for i in range(3)]
    else:
        srcs = base
    if tables == "separate":
        tabs, stride = (cos.contiguous(), sin.contiguous()), D // 2
    elif tables == "paired_padded":  # rows [cos | sin | pad]
        both = torch.zeros((S, 2 * D), device="cuda")
        both[:, :D // 2], both[:, D // 2:D] = cos, sin
        tabs, stride = (both[:, :D // 2], both[:, D // 2:D]), 2 * D
    else:
        both = torch.cat([cos, sin], dim=1)
        tabs, stride = (both[:, :D // 2], both[:, D // 2:]), D
    got = [torch.empty_like(x) for x in want]
    _call_raw(srcs, got, H, D, w, tabs, stride)
    torch.cuda.synchronize()
    for g_, w_ in zip(got, want):
        assert torch.equal(g_, w_)
