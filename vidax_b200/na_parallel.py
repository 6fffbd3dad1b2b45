"""Sequence (time-axis) sharded 3-D neighborhood attention over torch.distributed.

vidax runs the neighborhood attention of LTX-2.5's video decoder
(src/vidax/models/ltx2_5/diffusion_vae.py:179-284) on one device, or with its
heads Megatron-sharded across the `tp` axis (no collective: every device calls
`neighborhood_attention_3d` on its own heads, which `vidax_b200` does
unchanged). Here the other layout: each rank owns a slab of frames
[b_r, b_{r+1}) of all heads -- the activation memory divides by P and the
channels stay whole for the projections around the attention.

A query at frame t reads key frames [st(t), st(t) + Kt), st clamped to the
whole grid (`_window_start`, diffusion_vae.py:152-164), so rank r needs key
frames [st(b_r), st(b_{r+1} - 1) + Kt): its own plus a halo owned by its
neighbours (several ranks when slabs are thinner than the window). One
batched NCCL send/receive round moves exactly those frames of k and v into a
(T_kv)-frame buffer, then `vx_na3d_fwd_slab` computes the slab with windows
clamped to the global grid: the result equals the same frames of the
unsharded call.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .neighborhood import neighborhood_attention_3d_slab
from .ulysses import _group


def window_start(i: int, length: int, kernel: int) -> int:
    """st(i) = clamp(i - K/2, 0, L - K), K = min(kernel, L) (diffusion_vae.py:152-164)."""
    k = min(kernel, length)
    return min(max(i - k // 2, 0), length - k)


def slab_bounds(sizes: Sequence[int]) -> List[int]:
    """Frame boundaries of the ranks' slabs from their sizes (rank order)."""
    bounds = [0]
    for n in sizes:
        bounds.append(bounds[-1] + int(n))
    return bounds


def split_sizes(t_global: int, world: int) -> List[int]:
    """Slab sizes for `t_global` frames on `world` ranks: the first
    t_global % world ranks take one frame more (numpy.array_split)."""
    base, extra = divmod(t_global, world)
    return [base + (1 if r < extra else 0) for r in range(world)]


def key_ranges(bounds: Sequence[int], kernel_t: int) -> List[Tuple[int, int]]:
    """Per rank, the key frames [kv0, kv1) its queries read."""
    t_global = bounds[-1]
    out = []
    for r in range(len(bounds) - 1):
        lo, hi = bounds[r], bounds[r + 1]
        if hi <= lo:
            out.append((lo, lo))
        else:
            k = min(kernel_t, t_global)
            out.append((window_start(lo, t_global, k), window_start(hi - 1, t_global, k) + k))
    return out


def halo_plan(bounds: Sequence[int], kernel_t: int, rank: int):
    """(recvs, sends) of `rank`: lists of (peer, first frame, last frame + 1)
    in global frames -- what it receives from each peer and sends to each."""
    need = key_ranges(bounds, kernel_t)
    kv0, kv1 = need[rank]
    recvs, sends = [], []
    for s in range(len(bounds) - 1):
        if s == rank:
            continue
        lo, hi = max(kv0, bounds[s]), min(kv1, bounds[s + 1])
        if lo < hi:
            recvs.append((s, lo, hi))
        lo, hi = max(need[s][0], bounds[rank]), min(need[s][1], bounds[rank + 1])
        if lo < hi:
            sends.append((s, lo, hi))
    return recvs, sends


def exchange_halo(tensors: Sequence[torch.Tensor], bounds: Sequence[int], kernel_t: int,
                  group=None) -> List[torch.Tensor]:
    """Each (B, T_loc, ...) slab tensor -> its (B, T_kv, ...) key-frame buffer:
    own frames copied in, halo frames received from their owners (one batched
    send/receive round for all tensors and batch items)."""
    rank = dist.get_rank(group)
    need = key_ranges(bounds, kernel_t)
    kv0, kv1 = need[rank]
    b0 = bounds[rank]
    recvs, sends = halo_plan(bounds, kernel_t, rank)

    def peer(s):
        return dist.get_global_rank(group, s) if group is not None else s

    outs, ops = [], []
    for x in tensors:
        x = x.contiguous()
        ext = torch.empty((x.shape[0], kv1 - kv0) + tuple(x.shape[2:]), dtype=x.dtype,
                          device=x.device)
        own_lo, own_hi = max(kv0, b0), min(kv1, bounds[rank + 1])
        if own_lo < own_hi:
            ext[:, own_lo - kv0:own_hi - kv0].copy_(x[:, own_lo - b0:own_hi - b0])
        for b in range(x.shape[0]):  # per batch item: frame ranges are contiguous
            for s, lo, hi in recvs:
                ops.append(dist.P2POp(dist.irecv, ext[b, lo - kv0:hi - kv0], peer(s), group))
            for s, lo, hi in sends:
                ops.append(dist.P2POp(dist.isend, x[b, lo - b0:hi - b0], peer(s), group))
        outs.append(ext)
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return outs


def neighborhood_attention_3d_sp(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kernel_size: Sequence[int],
    sp_axis_name: str, *, t_global: Optional[int] = None, scale: float = 1.0,
    round_logits: bool = False,
) -> torch.Tensor:
    """Time-sharded `neighborhood_attention_3d`.

    q, k, v: this rank's (B, T_loc, H, W, NH, HD) slab, slabs in rank order
    along T. With `t_global` given, slab sizes follow `split_sizes`; without
    it the sizes are all-gathered (one small collective). Returns this
    rank's (B, T_loc, H, W, NH, HD) output."""
    group = _group(sp_axis_name)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if t_global is not None:
        sizes = split_sizes(t_global, world)
        if sizes[rank] != q.shape[1]:
            raise ValueError(f"rank {rank} holds {q.shape[1]} frames, expected {sizes[rank]} "
                             f"of {t_global} split over {world} ranks")
    else:
        mine = torch.tensor([q.shape[1]], dtype=torch.int64, device=q.device)
        allt = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allt, mine, group=group)
        sizes = [int(t.item()) for t in allt]
    bounds = slab_bounds(sizes)
    kt = int(kernel_size[0])
    k_ext, v_ext = exchange_halo([k, v], bounds, kt, group)
    if q.shape[1] == 0:
        return torch.empty_like(q)
    kv0 = key_ranges(bounds, kt)[rank][0]
    return neighborhood_attention_3d_slab(q, k_ext, v_ext, kernel_size, t_global=bounds[-1],
                                          q_t0=bounds[rank], kv_t0=kv0, scale=scale,
                                          round_logits=round_logits)
