"""CPU restatement of vidax's Ulysses resharding -- TEST INFRASTRUCTURE ONLY.

`jax.lax.all_to_all(x, axis, split_axis, concat_axis, tiled=True)` over a
mesh axis of size P (used at src/vidax/core/attention.py:379-381 and :388):
every rank splits `split_axis` into P equal contiguous chunks, sends chunk j
to rank j, and concatenates the P received chunks along `concat_axis` in
source-rank order. Token ownership follows `chunk_by_rank`
(attention.py:132-146): rank r holds tokens [r*S/P, (r+1)*S/P).

Pinned against the reference's own `sequence_parallel_self_attention`
executed under a thread-per-rank shim of jax.lax.all_to_all
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np


def all_to_all_tiled(xs, split_axis: int, concat_axis: int):
    """xs: list of P per-rank arrays; returns the list of P results."""
    P = len(xs)
    chunks = [np.split(x, P, axis=split_axis) for x in xs]      # chunks[src][dst]
    return [np.concatenate([chunks[src][dst] for src in range(P)], axis=concat_axis)
            for dst in range(P)]


def chunk_by_rank(x, axis: int, sp_size: int, rank: int):
    size = x.shape[axis] // sp_size
    return np.take(x, np.arange(rank * size, (rank + 1) * size), axis=axis)


def ulysses_attention(q_locals, k_locals, v_locals, attn):
    """The reference's data flow with `attn(q, k, v) -> out` as the local
    attention: tokens->heads all_to_all, attention, heads->tokens."""
    qh = all_to_all_tiled(q_locals, 2, 1)
    kh = all_to_all_tiled(k_locals, 2, 1)
    vh = all_to_all_tiled(v_locals, 2, 1)
    outs = [attn(a, b, c) for a, b, c in zip(qh, kh, vh)]
    return all_to_all_tiled(outs, 1, 2)
