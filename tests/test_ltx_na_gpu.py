"""LTX-2.5's neighborhood-attention caller on the GPU (row a12): the
absolute split RoPE tables, the fused per-head RMSNorm + bf16 q scale + RoPE
launch, and the whole `ltx_neighborhood_attention` (prologue + NA kernel)
against outputs of the reference's own code (tests/golden/ltx_reference.npz,
from `_apply_abs_rope` and `NeighborhoodAttention3D.__call__`,
src/vidax/models/ltx2_5/diffusion_vae.py:96-150, 252-284) and against the
oracle at an LTX-like shape.

Bars: RoPE alone bit-exact; the prologue bit-exact except where the float32
sum of squares of RMSNorm (order left to the backend) moves by an ulp (>=
99.9 % identical, one bf16 ulp of the rotated pair elsewhere); NA outputs
max-abs 2e-2, mean-abs 2e-3."""
import os

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare
from oracle.na3d_ref import na3d
from oracle.rope_norm_ref import ltx_na_prologue

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
ONE_ULP = 2.0 ** -7


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(GOLDEN, "ltx_reference.npz"))


def _cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


def _close_bits(got, ref):
    diff = got != ref
    assert diff.mean() <= 1e-3, diff.mean()
    pair = np.sqrt(np.sum(np.square(ref.reshape(ref.shape[:-1] + (-1, 2))), axis=-1))
    pair = np.repeat(pair, 2, axis=-1).reshape(ref.shape)
    tol = 2 * ONE_ULP * pair + ONE_ULP * np.abs(ref) + 1e-30
    assert np.all(np.abs(got - ref)[diff] <= tol[diff]), float(np.max(np.abs(got - ref)))


@pytest.mark.gpu
@pytest.mark.parametrize("i", [0, 1, 2])
def test_abs_rope_kernel_bit_exact(gold, i):
    """The fused kernel's rotation with `ltx_rope_freqs` tables equals the
    reference's `_apply_abs_rope` bit for bit (head_dim 64 and 128, default
    and custom splits)."""
    from vidax_b200 import ltx_rope_freqs, norm_rope_pack
    t, h, w, hd = (int(x) for x in gold[f"ltxrope{i}_grid"])
    split = tuple(int(x) for x in gold[f"ltxrope{i}_split"])
    x = gold[f"ltxrope{i}_x"]                       # (1, t, h, w, 3, hd)
    nh = x.shape[4]
    rows = _cuda(x.reshape(1, t * h * w, nh, hd))
    (y,) = norm_rope_pack([rows], nh, rope=ltx_rope_freqs(t, h, w, hd, split, device="cuda"),
                          rope_mask=0b1)
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy().reshape(x.shape), gold[f"ltxrope{i}_y"])


@pytest.mark.gpu
@pytest.mark.parametrize("i", [0, 1, 2])
def test_na_block_vs_reference_code(gold, i):
    """ltx_neighborhood_attention on the reference's projections: the q / k
    the NA primitive receives (prologue, one launch) and the block output."""
    import vidax_b200 as vx
    from vidax_b200.neighborhood import bf16_scalar
    q, k, v = (gold[f"ltxna{i}_{n}"] for n in "qkv")
    wq, wk = (torch.from_numpy(gold[f"ltxna{i}_w{n}"]) for n in "qk")
    kernel = tuple(int(x) for x in gold[f"ltxna{i}_kernel"])
    B, T, H, W, NH, HD = q.shape
    qr, kr = vx.norm_rope_pack([_cuda(x.reshape(B, T * H * W, NH, HD)) for x in (q, k)], NH,
                               norm_weights=[wq, wk], per_head=True,
                               post_scale=[bf16_scalar(HD ** -0.5), 1.0],
                               rope=vx.ltx_rope_freqs(T, H, W, HD, device="cuda"), rope_mask=0b11)
    o = vx.ltx_neighborhood_attention(_cuda(q), _cuda(k), _cuda(v), kernel, norm_q=wq, norm_k=wk)
    torch.cuda.synchronize()
    _close_bits(qr.float().cpu().numpy().reshape(q.shape), gold[f"ltxna{i}_qr"])
    _close_bits(kr.float().cpu().numpy().reshape(k.shape), gold[f"ltxna{i}_kr"])
    mx, mean = compare(o.float().cpu().numpy(), gold[f"ltxna{i}_o"])
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,kernel", [((1, 4, 16, 24, 4, 64), (3, 7, 7)),
                                          ((1, 3, 12, 20, 2, 64), (3, 5, 5)),
                                          ((2, 5, 8, 9, 2, 128), (3, 5, 5))])
def test_na_block_vs_oracle(shape, kernel):
    """LTX-like shapes (head_dim 64 with the decoder's 3x7x7 / 3x5x5 windows,
    and head_dim 128): the block against the oracle's prologue + fp32 NA."""
    import vidax_b200 as vx
    rng = np.random.Generator(np.random.PCG64(sum(shape) + sum(kernel)))
    from oracle.attention_ref import to_bf16
    q, k, v = (to_bf16(rng.standard_normal(shape, dtype=np.float32) * 2) for _ in range(3))
    HD = shape[-1]
    wq, wk = ((1.0 + 0.25 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2))
    o = vx.ltx_neighborhood_attention(_cuda(q), _cuda(k), _cuda(v), kernel,
                                      norm_q=torch.from_numpy(wq), norm_k=torch.from_numpy(wk))
    torch.cuda.synchronize()
    qr, kr = ltx_na_prologue(q, k, wq, wk)
    mx, mean = compare(o.float().cpu().numpy(), na3d(qr, kr, v, kernel))
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    from vidax_b200 import _lib
    assert _lib.device_status(clear=True) == 0
