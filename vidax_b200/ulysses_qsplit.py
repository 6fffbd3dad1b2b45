"""Ulysses with query-split heads: H % P != 0 without padding.

vidax's `sequence_parallel_self_attention` (src/vidax/core/attention.py:
341-388) needs H % P == 0 (the tiled all_to_all); `vidax_b200.ulysses` pads
the heads up to a multiple of P, so with 12 heads on 8 ranks every rank
computes two heads' attention where 1.5 would do. Here the work unit is a
(head, query part): every head is cut into f = P / gcd(H, P) parts of S / f
query rows, the H * f units are dealt out in (head, part) order, H / gcd(H, P)
per rank -- exactly balanced. A rank receives, per unit, that head's keys and
values for the whole sequence (a head whose parts land on two ranks is sent
to both) and its part's query rows; one kernel launch covers all its units
(units as heads of the launch); the outputs go back to the ranks owning
their rows.

Exchanges are NCCL all-to-alls with per-rank split sizes over flat buffers
laid out as `_send_layout` describes (one each way per call). `attn` can
replace the attention kernel (host-logic tests on CPU).
"""
from __future__ import annotations

from math import gcd
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .ulysses import _group


def unit_plan(heads: int, world: int) -> Tuple[int, List[List[Tuple[int, int]]]]:
    """(f, per-rank list of (head, part) units): each head in f query parts,
    H / gcd(H, P) units per rank in (head, part) order."""
    g = gcd(heads, world)
    f = world // g
    per = heads // g
    units = [(u // f, u % f) for u in range(heads * f)]
    return f, [units[r * per:(r + 1) * per] for r in range(world)]


def _heads_of(units: Sequence[Tuple[int, int]]) -> List[int]:
    out: List[int] = []
    for h, _ in units:
        if h not in out:
            out.append(h)
    return out


def _overlap(a0: int, a1: int, b0: int, b1: int) -> Tuple[int, int]:
    return max(a0, b0), min(a1, b1)


def _send_layout(src: int, dst: int, plan, s_loc: int, rows: int):
    """What rank `src` sends rank `dst` (both directions use it): the keys
    and values of dst's distinct heads over src's tokens, then, per dst
    unit (h, part), src's tokens inside the part: list of
    (kind, head, token0, token1) with global token ranges."""
    t0, t1 = src * s_loc, (src + 1) * s_loc
    out = []
    for h in _heads_of(plan[dst]):
        out.append(("kv", h, t0, t1))
    for h, part in plan[dst]:
        a, b = _overlap(t0, t1, part * rows, (part + 1) * rows)
        if a < b:
            out.append(("q", h, a, b))
    return out


def sequence_parallel_self_attention_qsplit(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sp_axis_name: str,
    scale: Optional[float] = None, *, attn: Optional[Callable] = None,
) -> torch.Tensor:
    """Same contract as `sequence_parallel_self_attention`: q, k, v
    (B, L_local, H, D) with chunk_by_rank token ownership; returns
    (B, L_local, H, D). Needs P * L_local divisible by f = P / gcd(H, P)."""
    group = _group(sp_axis_name)
    P = dist.get_world_size(group)
    r = dist.get_rank(group)
    B, S_loc, H, D = q.shape
    S = P * S_loc
    sm_scale = D ** -0.5 if scale is None else scale
    f, plan = unit_plan(H, P)
    if S % f:
        raise ValueError(f"sequence {S} must divide into {f} query parts")
    rows = S // f
    if attn is None:
        from .attention import flash_attention

        def attn(qq, kk, vv, sc):
            return flash_attention(qq, kk, vv, sc)

    def flat(t):
        return t.reshape(-1)

    # ---- tokens -> units
    sends, send_sizes = [], []
    for d in range(P):
        pieces = []
        for kind, h, a, b in _send_layout(r, d, plan, S_loc, rows):
            la, lb = a - r * S_loc, b - r * S_loc
            if kind == "kv":
                pieces += [flat(k[:, la:lb, h].contiguous()), flat(v[:, la:lb, h].contiguous())]
            else:
                pieces.append(flat(q[:, la:lb, h].contiguous()))
        buf = torch.cat(pieces) if pieces else q.new_empty(0)
        sends.append(buf)
        send_sizes.append(buf.numel())
    recv_sizes = []
    for s in range(P):
        n = 0
        for kind, _, a, b in _send_layout(s, r, plan, S_loc, rows):
            n += B * (b - a) * D * (2 if kind == "kv" else 1)
        recv_sizes.append(n)
    recv = q.new_empty(sum(recv_sizes))
    dist.all_to_all_single(recv, torch.cat(sends), recv_sizes, send_sizes, group=group)

    mine = plan[r]
    heads = _heads_of(mine)
    kfull = q.new_empty((B, S, len(heads), D))
    vfull = q.new_empty((B, S, len(heads), D))
    qunits = q.new_empty((B, rows, len(mine), D))
    off = 0
    for s in range(P):
        for kind, h, a, b in _send_layout(s, r, plan, S_loc, rows):
            n = B * (b - a) * D
            if kind == "kv":
                hi = heads.index(h)
                kfull[:, a:b, hi] = recv[off:off + n].view(B, b - a, D)
                vfull[:, a:b, hi] = recv[off + n:off + 2 * n].view(B, b - a, D)
                off += 2 * n
            else:
                for ui, (uh, part) in enumerate(mine):
                    if uh == h and part * rows <= a < (part + 1) * rows:
                        qunits[:, a - part * rows:b - part * rows, ui] = recv[off:off + n].view(B, b - a, D)
                        break
                off += n
    idx = torch.tensor([heads.index(h) for h, _ in mine], device=q.device)
    o = attn(qunits, kfull.index_select(2, idx).contiguous(),
             vfull.index_select(2, idx).contiguous(), sm_scale)   # (B, rows, units, D)

    # ---- units -> tokens: each unit's rows back to their owners
    sends, send_sizes = [], []
    for d in range(P):
        pieces = []
        for ui, (h, part) in enumerate(mine):
            a, b = _overlap(d * S_loc, (d + 1) * S_loc, part * rows, (part + 1) * rows)
            if a < b:
                pieces.append(flat(o[:, a - part * rows:b - part * rows, ui].contiguous()))
        buf = torch.cat(pieces) if pieces else q.new_empty(0)
        sends.append(buf)
        send_sizes.append(buf.numel())
    recv_sizes, layouts = [], []
    for s in range(P):
        lay, n = [], 0
        for h, part in plan[s]:
            a, b = _overlap(r * S_loc, (r + 1) * S_loc, part * rows, (part + 1) * rows)
            if a < b:
                lay.append((h, a, b))
                n += B * (b - a) * D
        recv_sizes.append(n)
        layouts.append(lay)
    recv = q.new_empty(sum(recv_sizes))
    dist.all_to_all_single(recv, torch.cat(sends), recv_sizes, send_sizes, group=group)
    out = torch.empty_like(q)
    off = 0
    for s in range(P):
        for h, a, b in layouts[s]:
            n = B * (b - a) * D
            out[:, a - r * S_loc:b - r * S_loc, h] = recv[off:off + n].view(B, b - a, D)
            off += n
    return out
