"""CPU restatement of vidax's attention semantics -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle for the CUDA kernels. Only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may
import it; the product (`vidax_b200`) never does.

What it restates
----------------
vidax's CPU/GPU attention path is the third-party `jax.nn.dot_product_attention`
(called at src/vidax/core/attention.py:338, :386, :457, :533; jax>=0.6.2 per
pyproject.toml:40, validated on jax 0.11.0 per docs/benchmarking.md:13). Its
XLA implementation computes, per (batch, head):

    logits = einsum(q, k) in float32            (preferred_element_type=f32)
    logits = logits * scale                     (scale defaults to D**-0.5)
    probs  = softmax(logits, axis=-1) in float32
    probs  = probs.astype(q.dtype)              (bf16 rounding of the weights)
    out    = einsum(probs, v)                   (bf16 operands, f32 accumulate) -> bf16

`sdpa` returns the float32-softmax result without the bf16 rounding of the
weights (the tolerance reference named for this path: max-abs 2e-2, mean-abs
2e-3); `sdpa(..., round_probs=True)` applies the weight rounding exactly as
the jax path does.

Parity status: JAX is not installed in this build environment, so the jax
half of this restatement is *unpinned* against jax itself; the pieces of
vidax's own code on the path (dispatch, default scale, key padding,
neighborhood windows, Ulysses layout) are pinned by executing the reference
functions under a numpy shim of the jax primitives (tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np

try:
    import ml_dtypes

    BF16 = ml_dtypes.bfloat16
except ImportError:  # pragma: no cover - ml_dtypes ships with the image
    BF16 = None


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bfloat16 (round-to-nearest-even), returned as float32."""
    return np.asarray(x, dtype=np.float32).astype(BF16).astype(np.float32)


def seeded_qkv(shape, seed: int, head_scale_range=None, n=3):
    """Seeded synthetic inputs: PCG64(seed) draws N(0,1) in float32, optionally
    multiplied per head (axis -2) by factors drawn U[lo, hi] (separate draws per
    tensor), then rounded to bf16. Returns float32 arrays holding bf16 values."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for _ in range(n):
        x = rng.standard_normal(shape, dtype=np.float32)
        if head_scale_range is not None:
            lo, hi = head_scale_range
            f = rng.uniform(lo, hi, size=shape[-2]).astype(np.float32)
            x = x * f[:, None]
        out.append(to_bf16(x))
    return out


def sdpa(q, k, v, scale=None, kv_len=None, round_probs=False, q_rows=None, chunk=512,
         key_mask=None, key_bias=None):
    """Non-causal attention over BSHD float32 arrays (values bf16-exact).

    q: (B, Sq, H, D); k, v: (B, Sk, Hkv, D), H % Hkv == 0 (head h reads kv
    head h // (H // Hkv)). kv_len: optional per-batch count of visible keys
    (keys >= kv_len[b] are masked, the SegmentIds padding rule of
    attention.py:272-278). q_rows: optional index array of query rows to
    evaluate (returns (B, len(q_rows), H, D)). key_mask (B, Sk) bool /
    key_bias (B, Sk) float: jax.nn.dot_product_attention's mask and additive
    bias restricted to keys -- masked logits become -0.7 * float32 max (so a
    row with no visible key has uniform weights), the bias is added to the
    scaled logits (a row of -inf gives NaN). Returns float32.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, Sq, H, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    if scale is None:
        scale = D ** -0.5
    rows = np.arange(Sq) if q_rows is None else np.asarray(q_rows)
    out = np.zeros((B, len(rows), H, D), np.float32)
    g = H // Hkv
    for b in range(B):
        nk = Sk if kv_len is None else int(min(max(kv_len[b], 0), Sk))
        if nk == 0:
            continue
        for h in range(H):
            kh = k[b, :nk, h // g, :]            # (nk, D)
            vh = v[b, :nk, h // g, :]
            for r0 in range(0, len(rows), chunk):
                rr = rows[r0:r0 + chunk]
                logits = (q[b, rr, h, :] @ kh.T) * np.float32(scale)   # f32
                if key_bias is not None:
                    logits = logits + np.asarray(key_bias, np.float32)[b, None, :nk]
                if key_mask is not None:
                    logits = np.where(np.asarray(key_mask)[b, None, :nk], logits,
                                      np.float32(-0.7 * np.finfo(np.float32).max))
                with np.errstate(invalid="ignore"):
                    logits -= logits.max(axis=1, keepdims=True)
                p = np.exp(logits)
                p /= p.sum(axis=1, keepdims=True)
                if round_probs:
                    p = to_bf16(p)
                out[b, r0:r0 + len(rr), h, :] = p @ vh
    return out


def attention_flops(B, H, Sq, Sk, D):
    """vidax's FLOP convention, 4*B*H*Sq*Sk*D (attention.py:13-16)."""
    return 4.0 * B * H * Sq * Sk * D


def compare(out, ref):
    """(max-abs, mean-abs) error of `out` against `ref` (both float32)."""
    d = np.abs(np.asarray(out, np.float32) - np.asarray(ref, np.float32))
    return float(d.max()) if d.size else 0.0, float(d.mean()) if d.size else 0.0
