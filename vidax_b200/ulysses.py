"""DeepSpeed-Ulysses sequence-parallel attention on B200 (NCCL over NVLink).

Mirrors the sequence-parallel half of `vidax.core.attention`:

* `sequence_parallel_self_attention(q, k, v, sp_axis_name, scale=None)`
  -- src/vidax/core/attention.py:341-388
* `sequence_parallel_joint_self_attention(q, k, v, text_len, sp_axis_name, scale=None)`
  -- src/vidax/core/attention.py:391-464
* `sequence_parallel_self_attention_from_host(...)`: the same layer on pinned
  host buffers, transfers pipelined against the kernel (end-to-end form)

vidax calls these inside `shard_map` with a bound mesh axis name. Here one
process drives one GPU and the axis name is bound to a `torch.distributed`
process group with `register_axis(name, group)` (the analogue of the mesh
axis; `axis_index` / `axis_size` mirror `jax.lax.axis_index` and the mesh
shape).

Data path per batch item (rank r of P, local tokens S_loc, heads H):

1. `vx_ulysses_pack` (one CUDA launch for q, k, v): strided (S_loc, H, D)
   -> contiguous (P, S_loc, hs, D): a slice of hs heads of every rank's
   head group (Hg = ceil(H / P) heads per rank, zero heads past H).
2. three equal-split NCCL all-to-alls (tokens -> heads): rank r receives
   (P_src, S_loc, hs, D) == the full sequence (S, hs, D) in natural token
   order for its heads -- the tiled all_to_all(split_axis=2, concat_axis=1)
   of attention.py:379-381, one slice at a time.
3. the sm_100a attention kernel over (1, S, hs, D), written as
   (P, S_loc, hs, D) -- already the heads -> tokens send layout.
4. one NCCL all-to-all back (attention.py:388) and `vx_ulysses_unpack`
   into the strided (S_loc, H, D) output, dropping padded heads.

The Hg heads are processed in up to three slices so that the all-to-alls of
one slice (on NCCL's stream) overlap the kernel of another.

Unlike the reference (whose tiled all_to_all requires H % P == 0), head
counts that do not divide P are padded with zero heads.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Dict, Optional

import torch
import torch.distributed as dist

from . import _lib
from .attention import flash_attention

_AXES: Dict[str, Optional["dist.ProcessGroup"]] = {}
_EXCHANGE: Dict[str, str] = {}
_AXES_LOCK = threading.Lock()

#: When set to a list, (start, end) CUDA events bracketing every attention
#: kernel launch of the sequence-parallel path are appended to it (kernel-level
#: timing for benchmarks; the data path is unchanged).
KERNEL_EVENTS: Optional[list] = None


def register_axis(name: str, group=None, exchange: str = "nccl") -> None:
    """Binds mesh axis `name` to a torch.distributed process group (None =
    the default world group). `exchange` selects how the Ulysses layers on
    this axis move the head slabs: "nccl" (all-to-alls; any topology) or
    "peer" (the pack / unpack kernels store into / load from the other
    ranks' slabs over NVLink, vidax_b200.ulysses_peer; ranks of one node)."""
    if exchange not in ("nccl", "peer"):
        raise ValueError(f"exchange must be 'nccl' or 'peer', not {exchange!r}")
    with _AXES_LOCK:
        _AXES[name] = group
        _EXCHANGE[name] = exchange


def unregister_axis(name: str) -> None:
    with _AXES_LOCK:
        _AXES.pop(name, None)
        _EXCHANGE.pop(name, None)


def _exchange(name: str) -> str:
    with _AXES_LOCK:
        return _EXCHANGE.get(name, "nccl")


def _group(name: str):
    with _AXES_LOCK:
        if name in _AXES:
            return _AXES[name]
    raise NameError(
        f"unbound axis name {name!r}: call vidax_b200.register_axis({name!r}, group) first "
        "(the analogue of running inside shard_map over a mesh with that axis)")


def axis_size(name: str) -> int:
    return dist.get_world_size(_group(name))


def axis_index(name: str) -> int:
    """This process's index along axis `name` (jax.lax.axis_index)."""
    return dist.get_rank(_group(name))


# ---------------------------------------------------------------- packing
class HeadSlabArgs(ctypes.Structure):
    _fields_ = [
        ("num_tensors", ctypes.c_int32),
        ("src", ctypes.c_void_p * 3),
        ("dst", ctypes.c_void_p * 3),
        ("stride", (ctypes.c_int64 * 2) * 3),
        ("seq", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("groups", ctypes.c_int32),
        ("slab_heads", ctypes.c_int32),
        ("group_stride", ctypes.c_int32),
        ("head_offset", ctypes.c_int32),
        ("group_valid", ctypes.c_int32),
    ]


def _slab_call(fn_name: str, strided, packed, heads: int, groups: int, sub=None) -> None:
    """strided: list of (S_loc, H, D) views; packed: list of contiguous
    (groups, S_loc, Hg, D) buffers; `sub` = (slab_heads, group_stride,
    head_offset, group_valid) selects a sub-group of every group."""
    a = HeadSlabArgs()
    a.num_tensors = len(strided)
    if not 1 <= len(strided) <= 3 or len(packed) != len(strided):
        raise ValueError("1 to 3 tensors, one packed buffer each")
    seq, _, d = strided[0].shape
    hg = sub[0] if sub is not None and any(sub) else -(-heads // groups)
    want = groups * seq * hg * d   # the kernel writes / reads exactly this many elements
    dev = strided[0].device
    for i, (s_t, p_t) in enumerate(zip(strided, packed)):
        if tuple(s_t.shape) != (seq, heads, d):
            raise ValueError(f"tensor {i}: expected a ({seq}, {heads}, {d}) view, got "
                             f"{tuple(s_t.shape)}")
        if not p_t.is_contiguous() or p_t.numel() != want:
            raise ValueError(f"packed buffer {i} must be contiguous with {groups} x {seq} x "
                             f"{hg} x {d} elements")
        if s_t.element_size() != 2 or p_t.dtype != s_t.dtype:
            raise NotImplementedError("the slab kernels move 16-bit elements (bf16)")
        if not s_t.is_cuda or s_t.device != dev or p_t.device != dev:
            raise ValueError("all tensors must live on the same CUDA device")
        if s_t.stride(-1) != 1:
            raise ValueError("head_dim must be contiguous")
        if fn_name == "vx_ulysses_pack":
            a.src[i], a.dst[i] = s_t.data_ptr(), p_t.data_ptr()
        else:
            a.src[i], a.dst[i] = p_t.data_ptr(), s_t.data_ptr()
        a.stride[i][0], a.stride[i][1] = s_t.stride(0), s_t.stride(1)
    a.seq, a.heads, a.head_dim, a.groups = seq, heads, d, groups
    if sub is not None:
        a.slab_heads, a.group_stride, a.head_offset, a.group_valid = sub
    lib = _lib.load()
    fn = getattr(lib, fn_name)
    fn.argtypes = [ctypes.POINTER(HeadSlabArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    stream = torch.cuda.current_stream(strided[0].device)
    _lib.check(fn(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)))


def pack_heads(strided, groups: int, out=None, sub=None):
    """(S_loc, H, D) strided views (1-3 tensors) -> contiguous (groups, S_loc, Hg, D).
    `sub` = (slab_heads, group_stride, head_offset, group_valid) packs only a
    slice of every group (see vx_head_slab_args)."""
    seq, heads, d = strided[0].shape
    hg = -(-heads // groups) if sub is None else sub[0]
    if out is None:
        out = [torch.empty((groups, seq, hg, d), dtype=t.dtype, device=t.device) for t in strided]
    _slab_call("vx_ulysses_pack", list(strided), list(out), heads, groups, sub)
    return out


def unpack_heads(packed, strided_out, heads: int, sub=None) -> None:
    """contiguous (groups, S_loc, Hg, D) -> strided (S_loc, H, D) views, in place."""
    groups = packed[0].shape[0]
    _slab_call("vx_ulysses_unpack", list(strided_out), list(packed), heads, groups, sub)


# ---------------------------------------------------------------- exchange
def exchange(send: torch.Tensor, group, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Equal-split all-to-all along dim 0 (size P): chunk j of `send` goes to
    rank j; chunk i of the result came from rank i (source-rank order)."""
    recv = torch.empty_like(send) if out is None else out
    dist.all_to_all_single(recv, send, group=group)
    return recv


def _pieces(hg: int):
    """Head counts of the pipelined slices of a rank's hg heads: a small
    first slice (its exchange is the one not hidden behind the kernel), then
    up to two larger ones (fewer, bigger kernel launches keep the GPU full)."""
    if hg <= 1:
        return [hg]
    first = max(1, hg // 5)
    rest = hg - first
    if rest <= 1:
        return [first, rest]
    return [first, rest - rest // 2, rest // 2]


_side: dict = {}


def _side_stream(device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _side:
        _side[idx] = torch.cuda.Stream(device=idx)
    return _side[idx]


def _timed_attention(q, k, v, sm_scale, kv_len, out):
    events = KERNEL_EVENTS
    if events is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    # dynamic schedule: NCCL's all-to-all kernels run concurrently on some SMs
    o = flash_attention(q, k, v, sm_scale, kv_len=kv_len, out=out, dynamic_schedule=True)
    if events is not None:
        e1.record()
        events.append((e0, e1))
    return o


def _ulysses_one(qb, kb, vb, ob, group, P: int, sm_scale: float, kv_valid: Optional[int],
                 sends=None):
    """One batch item: qb/kb/vb/ob are (S_loc, H, D) views.

    The rank's head group (Hg heads after the exchange) is split into slices
    (`_pieces`); slice j+1's three tokens->heads all-to-alls run on NCCL's
    stream while the kernel computes slice j, and slice j's heads->tokens
    all-to-all and unpack (on a side stream) overlap the kernel on slice j+1.
    `sends` (per slice, [q, k, v] of (P, S_loc, hs, D)) replaces the packing
    of qb/kb/vb when the send slabs were already written by the fused
    norm + RoPE + pack kernel."""
    S_loc, H, D = ob.shape
    Hg = -(-H // P)
    S = P * S_loc
    kv_len = None
    if kv_valid is not None and kv_valid < S:
        kv_len = torch.full((1,), kv_valid, dtype=torch.int32, device=ob.device)
    sizes = _pieces(Hg)
    offs = [sum(sizes[:j]) for j in range(len(sizes))]
    subs = [(hs, Hg, off, hs) for hs, off in zip(sizes, offs)]
    n = len(subs)
    if sends is None:
        sends = [pack_heads([qb, kb, vb], P, sub=sub) for sub in subs]   # each (P, S_loc, hs, D)
    else:
        sends = list(sends)
    recvs, works = [None] * n, [None] * n

    def start_in(j):
        recvs[j] = [torch.empty_like(t) for t in sends[j]]
        works[j] = [dist.all_to_all_single(r, t, group=group, async_op=True)
                    for r, t in zip(recvs[j], sends[j])]

    comp = torch.cuda.current_stream(ob.device)
    side = _side_stream(ob.device)
    side.wait_stream(comp)
    start_in(0)
    for j, sub in enumerate(subs):
        hs = sub[0]
        if j + 1 < n:
            start_in(j + 1)
        for w in works[j]:
            w.wait()
        rq, rk, rv = (t.view(1, S, hs, D) for t in recvs[j])
        o = _timed_attention(rq, rk, rv, sm_scale, kv_len, None)
        ro = torch.empty((P, S_loc, hs, D), dtype=o.dtype, device=o.device)
        w_out = dist.all_to_all_single(ro, o.view(P, S_loc, hs, D), group=group, async_op=True)
        sends[j] = None  # release the send buffers of slice j
        with torch.cuda.stream(side):
            w_out.wait()                       # the side stream waits for the exchange
            unpack_heads([ro], [ob], H, sub=sub)
            ro.record_stream(side)
    comp.wait_stream(side)


def _rows_copy(dst_ptr: int, dst_pitch: int, src_ptr: int, src_pitch: int, row_bytes: int,
               rows: int, stream) -> None:
    lib = _lib.load()
    _lib.check(lib.vx_memcpy_rows_async(
        ctypes.c_void_p(dst_ptr), dst_pitch, ctypes.c_void_p(src_ptr), src_pitch, row_bytes, rows,
        ctypes.c_void_p(stream.cuda_stream)))


def _slab_heads(g: int, Hg: int, off: int, hs: int, H: int):
    """Strided heads of group g's slice [off, off + hs): first head, count valid."""
    h0 = g * Hg + off
    return h0, max(0, min(h0 + hs, H) - h0)


def sequence_parallel_self_attention_from_host(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sp_axis_name: str,
    scale: Optional[float] = None, *, out: Optional[torch.Tensor] = None,
    device: Optional[torch.device] = None,
) -> torch.Tensor:
    """`sequence_parallel_self_attention` on host-resident (pinned) q, k, v
    (B, L_local, H, D): returns the host (B, L_local, H, D) output, complete
    once the current CUDA stream has been synchronised (the call enqueues).

    The transfers double as the head-slab layout: for each pipelined slice,
    one 2-D copy per rank group moves that group's heads of every local token
    from host rows straight into the slice's send slab (no pack kernel), and
    after the reverse all-to-all one 2-D copy per group moves the received
    slab straight into the host output rows (no unpack kernel). Uploads of
    slice j+1 and downloads of slice j-1 run on copy streams while the kernel
    computes slice j."""
    from .hostio import _check_host, _side_streams, check_host_out, group_sizes
    if _exchange(sp_axis_name) == "peer":
        from .ulysses_peer import sequence_parallel_self_attention_from_host_peer
        g = _group(sp_axis_name)
        g = g if g is not None else dist.distributed_c10d._get_default_group()
        return sequence_parallel_self_attention_from_host_peer(q, k, v, g, scale, out=out,
                                                               device=device)
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_host(name, t)
    if not (q.shape == k.shape == v.shape):
        raise ValueError("self-attention needs q, k, v of equal shape")
    if out is not None:
        check_host_out(out, q.shape)
    group = _group(sp_axis_name)
    P = dist.get_world_size(group)
    B, S_loc, H, D = q.shape
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    sm_scale = D ** -0.5 if scale is None else scale
    if out is None:
        out = torch.empty((B, S_loc, H, D), dtype=torch.bfloat16).pin_memory()
    Hg = -(-H // P)
    S = P * S_loc
    # slices of 1, 2, 4, ... heads and a last one of 1: only the first
    # slice's upload and the last one's download are not hidden behind a
    # kernel, and each upload fits under the kernels before it
    sizes = group_sizes(Hg, 8)
    offs = [sum(sizes[:j]) for j in range(len(sizes))]
    es = 2
    comp = torch.cuda.current_stream(device)
    h2d, d2h = _side_streams(device)
    side = _side_stream(device)
    h2d.wait_stream(comp)
    d2h.wait_stream(comp)
    side.wait_stream(comp)
    keep = []
    for b in range(B):
        # uploads of every slice, in order, on the copy stream
        sends, ready = [], []
        for hs, off in zip(sizes, offs):
            slab = [torch.empty((P, S_loc, hs, D), dtype=torch.bfloat16, device=device)
                    for _ in range(3)]
            for src, dst in zip((q, k, v), slab):
                for g in range(P):
                    h0, n = _slab_heads(g, Hg, off, hs, H)
                    if n < hs:
                        with torch.cuda.stream(h2d):
                            dst[g, :, n:].zero_()  # head padding (H % P != 0)
                    if n > 0:
                        _rows_copy(dst[g].data_ptr(), hs * D * es,
                                   src.data_ptr() + (b * src.stride(0) + h0 * src.stride(2)) * es,
                                   src.stride(1) * es, n * D * es, S_loc, h2d)
            ev = torch.cuda.Event()
            ev.record(h2d)
            sends.append(slab)
            ready.append(ev)
        recvs, works = [None] * len(sizes), [None] * len(sizes)

        def start_in(j):
            # issued from the side stream so the compute stream never waits
            # for a later slice's upload
            recvs[j] = [torch.empty_like(t) for t in sends[j]]
            with torch.cuda.stream(side):
                side.wait_event(ready[j])
                works[j] = [dist.all_to_all_single(r, t, group=group, async_op=True)
                            for r, t in zip(recvs[j], sends[j])]

        start_in(0)
        for j, (hs, off) in enumerate(zip(sizes, offs)):
            if j + 1 < len(sizes):
                start_in(j + 1)
            for w in works[j]:
                w.wait()
            rq, rk, rv = (t.view(1, S, hs, D) for t in recvs[j])
            o = _timed_attention(rq, rk, rv, sm_scale, None, None)
            ro = torch.empty((P, S_loc, hs, D), dtype=o.dtype, device=o.device)
            w_out = dist.all_to_all_single(ro, o.view(P, S_loc, hs, D), group=group,
                                           async_op=True)
            with torch.cuda.stream(d2h):
                w_out.wait()
                for g in range(P):
                    h0, n = _slab_heads(g, Hg, off, hs, H)
                    if n > 0:
                        _rows_copy(out.data_ptr() + (b * out.stride(0) + h0 * out.stride(2)) * es,
                                   out.stride(1) * es, ro[g].data_ptr(), hs * D * es,
                                   n * D * es, S_loc, d2h)
            keep += [ro, o] + sends[j] + recvs[j]
    comp.wait_stream(d2h)
    comp.wait_stream(side)
    for t in keep:  # device buffers stay allocated until the copies that use them ran
        t.record_stream(h2d)
        t.record_stream(d2h)
        t.record_stream(side)
    return out


def launches_per_layer(heads: int, world: int, batch: int = 1) -> int:
    """CUDA launches of this library per sequence-parallel layer (pack,
    attention and unpack per pipelined slice and batch item)."""
    hg = -(-heads // world)
    return 3 * len(_pieces(hg)) * batch


def sequence_parallel_self_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
    sp_axis_name: str, scale: Optional[float] = None,
    *, valid_len: Optional[int] = None,
) -> torch.Tensor:
    """DeepSpeed-Ulysses self-attention (attention.py:341-388).

    q, k, v: (B, L_local, H, D) -- this rank's contiguous token chunk
    (`chunk_by_rank` ownership: rank r holds tokens [r*L_local, (r+1)*L_local)),
    all heads. Returns (B, L_local, H, D). `valid_len` (extension): number
    of real tokens in the global sequence when the caller padded it to a
    multiple of the axis size; padded keys are then masked.
    """
    group = _group(sp_axis_name)
    P = dist.get_world_size(group)
    head_dim = q.shape[-1]
    sm_scale = head_dim ** -0.5 if scale is None else scale
    if not (q.shape == k.shape == v.shape):
        raise ValueError("self-attention needs q, k, v of equal shape")
    if _exchange(sp_axis_name) == "peer":
        from .ulysses_peer import sequence_parallel_self_attention_peer
        g = group if group is not None else dist.distributed_c10d._get_default_group()
        return sequence_parallel_self_attention_peer(q, k, v, g, sm_scale, valid_len=valid_len)
    out = torch.empty_like(q)
    for b in range(q.shape[0]):
        _ulysses_one(q[b], k[b], v[b], out[b], group, P, sm_scale, valid_len)
    return out


def _attend_sp(q, k, v, num_heads, norm_q, norm_k, rope, eps, sp_axis_name, scale):
    """Wan's attend under sequence parallelism (dit_layers.py:137-151): one
    fused norm + RoPE + pack launch writes every pipelined slice's send slabs
    for all batch items, then the Ulysses exchange / attention pipeline."""
    from .prologue import norm_rope_pack, slice_views
    group = _group(sp_axis_name)
    P = dist.get_world_size(group)
    B, L, dim = q.shape
    H = num_heads
    D = dim // H
    if _exchange(sp_axis_name) == "peer":
        # norm + RoPE in natural (B, L, H, D) rows (the same HBM traffic as
        # the NCCL path: there NCCL reads the packed slabs, here the pack
        # kernel reads these rows and stores them into the peers' slabs)
        from .ulysses_peer import sequence_parallel_self_attention_peer
        rows = norm_rope_pack([q, k, v], H, norm_weights=[norm_q, norm_k, None], eps=eps,
                              rope=rope, rope_mask=0b011 if rope is not None else 0)
        qh, kh, vh = (r.view(B, L, H, D) for r in rows)
        g = group if group is not None else dist.distributed_c10d._get_default_group()
        out = sequence_parallel_self_attention_peer(qh, kh, vh, g, scale)
        return out.reshape(B, L, dim)
    sizes = _pieces(-(-H // P))
    bufs = norm_rope_pack([q, k, v], H, norm_weights=[norm_q, norm_k, None], eps=eps,
                          rope=rope, rope_mask=0b011 if rope is not None else 0,
                          groups=P, slices=sizes)
    out = torch.empty((B, L, H, D), dtype=q.dtype, device=q.device)
    sm_scale = D ** -0.5 if scale is None else scale
    for b in range(B):
        per_t = [slice_views(buf[b], P, L, D, sizes) for buf in bufs]
        sends = [[per_t[t][j] for t in range(3)] for j in range(len(sizes))]
        _ulysses_one(None, None, None, out[b], group, P, sm_scale, None, sends=sends)
    return out.reshape(B, L, dim)


def sequence_parallel_joint_self_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
    text_len: int, sp_axis_name: str, scale: Optional[float] = None,
) -> torch.Tensor:
    """Joint [text; visual] Ulysses attention (attention.py:391-464).

    q, k, v: (B, text_len + L_vis_local, H, D): the text prefix replicated on
    every rank, the visual tokens this rank's chunk. Only visual tokens go
    through the all-to-all; the text q/k/v are sliced to this rank's head
    group, joint attention runs over [text(full); visual(full)] for that
    group, the visual output goes back through the reverse all-to-all and the
    text output is all-gathered over heads.
    """
    group = _group(sp_axis_name)
    if _exchange(sp_axis_name) == "peer":
        from .ulysses_peer import sequence_parallel_joint_self_attention_peer
        g = group if group is not None else dist.distributed_c10d._get_default_group()
        return sequence_parallel_joint_self_attention_peer(q, k, v, text_len, g, scale)
    P = dist.get_world_size(group)
    r = dist.get_rank(group)
    B, L, H, D = q.shape
    sm_scale = D ** -0.5 if scale is None else scale
    S_loc = L - text_len
    Hg = -(-H // P)
    h0, h1 = r * Hg, min((r + 1) * Hg, H)
    out = torch.empty_like(q)
    for b in range(B):
        packed = pack_heads([q[b, text_len:], k[b, text_len:], v[b, text_len:]], P)
        joint = []
        for t_full, t_send in zip((q[b], k[b], v[b]), packed):
            # [text rows of this head group ; received visual rows (P, S_loc, Hg, D)]:
            # the exchange writes every visual row, so only the text rows are
            # filled here (zero heads only past H, when H % P != 0)
            buf = torch.empty((text_len + P * S_loc, Hg, D), dtype=q.dtype, device=q.device)
            nvalid = max(h1 - h0, 0)
            if nvalid > 0:
                buf[:text_len, :nvalid].copy_(t_full[:text_len, h0:h1])
            if nvalid < Hg:
                buf[:text_len, nvalid:].zero_()
            exchange(t_send, group, out=buf[text_len:].view(P, S_loc, Hg, D))
            joint.append(buf.unsqueeze(0))
        o_j = flash_attention(joint[0], joint[1], joint[2], sm_scale)[0]
        ro = exchange(o_j[text_len:].reshape(P, S_loc, Hg, D), group)
        unpack_heads([ro], [out[b, text_len:]], H)
        txt = o_j[:text_len].contiguous()
        gathered = torch.empty((P, text_len, Hg, D), dtype=q.dtype, device=q.device)
        dist.all_gather_into_tensor(gathered, txt, group=group)
        unpack_heads([gathered], [out[b, :text_len]], H)
    return out
