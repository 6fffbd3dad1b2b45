"""CPU restatement of vidax's 3-D neighborhood attention -- TEST INFRASTRUCTURE ONLY.

Parity oracle for the sm_100a neighborhood kernel; only tests/, smoke() and
bench.py's baseline legs use it.

Restates src/vidax/models/ltx2_5/diffusion_vae.py:152-234 step by step:

* `window_start` = `_window_start` (:152-164): K = min(kernel, L),
  start(i) = clip(i - K // 2, 0, L - K);
* for each query row (t, h) (the `lax.scan` body, :206-225): gather the
  Kt frames and Kh rows of k/v starting at start_t(t), start_h(h); gather the
  Kw-window along W for every w (the vmapped `_gather_window`, :167-176);
  key order within a window is (t, h) flattened, then w (:216-221);
* logits = einsum(q, k_win) -- bf16 operands with an f32 accumulator whose
  result takes the input dtype, i.e. rounded to bf16 (`round_logits=True`
  reproduces that; False keeps the f32 logits of the fp32-softmax reference);
* softmax in float32; probabilities cast to bf16 (`round_probs=True`) and
  contracted with v_win (:223-224).

Pinned against the reference's own `_window_start` / `neighborhood_attention_3d`
executed under a numpy shim of the jax primitives (tests/golden/make_golden.py
writes the fixtures, tests/test_oracle_golden.py checks them).
"""
from __future__ import annotations

import numpy as np

from .attention_ref import to_bf16


def window_start(length: int, kernel: int) -> np.ndarray:
    k = min(kernel, length)
    idx = np.arange(length)
    return np.clip(idx - k // 2, 0, length - k)


def window_sets(T: int, H: int, W: int, kernel_size):
    """Per-axis (start, size) arrays: query i of an axis attends keys
    [start[i], start[i] + size)."""
    ks = [min(a, b) for a, b in zip(kernel_size, (T, H, W))]
    return [(window_start(L, k), k) for L, k in zip((T, H, W), ks)]


def na3d(q, k, v, kernel_size, round_logits=False, round_probs=False, positions=None,
         rows=None):
    """q, k, v: (B, T, H, W, NH, HD) float32 (bf16-exact values; q pre-scaled).

    Returns float32 (B, T, H, W, NH, HD), or (B, N, NH, HD) for the query
    `positions` (N, 3) of (t, h, w) when given. `rows` ((t, h) pairs)
    computes only those scan steps of the full-grid form (the others stay
    zero): a bounded sample of the reference's per-row work.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, T, H, W, NH, HD = q.shape
    g = NH // k.shape[4]
    if g > 1:
        k = np.repeat(k, g, axis=4)
        v = np.repeat(v, g, axis=4)
    (st_t, kt), (st_h, kh), (st_w, kw) = window_sets(T, H, W, kernel_size)
    w_idx = st_w[:, None] + np.arange(kw)[None, :]                         # (W, Kw)

    def row(t, h, w_sel):
        k_th = k[:, st_t[t]:st_t[t] + kt, st_h[h]:st_h[h] + kh]          # (B,Kt,Kh,W,NH,HD)
        v_th = v[:, st_t[t]:st_t[t] + kt, st_h[h]:st_h[h] + kh]
        k_win = k_th[:, :, :, w_idx[w_sel]]                               # (B,Kt,Kh,n,Kw,NH,HD)
        v_win = v_th[:, :, :, w_idx[w_sel]]
        n = len(w_sel)
        k_win = np.moveaxis(k_win, 3, 1).reshape(B, n, kt * kh * kw, NH, HD)
        v_win = np.moveaxis(v_win, 3, 1).reshape(B, n, kt * kh * kw, NH, HD)
        q_i = q[:, t, h, w_sel]                                            # (B,n,NH,HD)
        logits = np.einsum("bwnd,bwknd->bwnk", q_i, k_win, optimize=True)
        if round_logits:
            logits = to_bf16(logits)
        logits = logits - logits.max(axis=-1, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=-1, keepdims=True)
        if round_probs:
            p = to_bf16(p)
        return np.einsum("bwnk,bwknd->bwnd", p, v_win, optimize=True)

    if positions is None:
        out = np.zeros_like(q)
        all_w = np.arange(W)
        steps = rows if rows is not None else [(t, h) for t in range(T) for h in range(H)]
        for t, h in steps:
            out[:, t, h] = row(int(t), int(h), all_w)
        return out
    positions = np.asarray(positions)
    out = np.zeros((B, len(positions), NH, HD), np.float32)
    for i, (t, h, w) in enumerate(positions):
        out[:, i] = row(int(t), int(h), np.array([int(w)]))[:, 0]
    return out


def na3d_flops(B, T, H, W, NH, HD, kernel_size):
    kt, kh, kw = (min(a, b) for a, b in zip(kernel_size, (T, H, W)))
    return 4.0 * B * T * H * W * kt * kh * kw * HD * NH
