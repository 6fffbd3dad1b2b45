"""DeepSpeed-Ulysses with the exchanges done by the slab kernels over NVLink.

`sequence_parallel_self_attention` (vidax_b200.ulysses) moves the packed
head slabs with NCCL all-to-alls. Here the ranks of one NVLink / NVSwitch
domain map each other's workspace (CUDA IPC, once per process group) and
the exchange becomes part of the slab kernels
(src/vidax/core/attention.py:379-381 and :388):

* tokens -> heads: `vx_ulysses_pack_peers` stores group g's chunk of this
  rank's q / k / v straight into rank g's receive slab (SM stores over
  NVLink; the pack and the all-to-all are one pass);
* attention: the local kernel reads the receive slab and writes its output
  into this rank's output slab, both in its own memory;
* heads -> tokens: `vx_ulysses_unpack_peers` loads this rank's tokens of
  every rank's output slab straight into the strided output rows (the
  all-to-all and the unpack are one pass).

`vx_peer_barrier` (flags in the ranks' workspaces, bounded waits) orders
the steps across GPUs: after each slice's pack (its receive slabs are
complete everywhere), after each slice's attention (the output slabs are),
and at the end of each batch item (the workspace may be reused). The head
group is processed in the same pipelined slices as the NCCL path: slice
j+1's pack (on a side stream, with a small CTA budget) and slice j-1's
unpack (on another) run beside the kernel on slice j, whose dynamic
schedule leaves them SMs. Only ranks whose GPUs can reach each other's
memory (one node) can use it; results are identical to the NCCL path's.

The same workspace serves the host-buffer form (the 2-D host copies
themselves land in the peers' receive slabs and leave from their output
slabs) and the joint [text; visual] layer (the text rows in a prefix of the
receive slab). `vidax_b200.ulysses` dispatches to these functions for an
axis registered with exchange="peer". If the ranks cannot map each other's
memory, the workspace raises PeerUnavailable on every rank alike.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .ulysses import HeadSlabArgs, _pieces, _side_stream, _timed_attention

MAX_GROUPS = 8
CH_IN, CH_OUT, CH_END = 0, 1, 2   # flag arrays: one sequence of barriers each
SLICE_CTAS = 0                    # CTA budget of a pack / unpack beside the kernel (0: none; measured best)
PIPELINED = True                  # head slices pipelined against the kernel (else one slice)
BARRIER_TIMEOUT_NS = 2_000_000_000


class PeerUnavailable(RuntimeError):
    """The ranks of the group cannot map each other's memory (raised on every
    rank alike, so the caller can switch the axis to the NCCL exchange)."""


class PeerSlabArgs(ctypes.Structure):
    _fields_ = [
        ("slab", HeadSlabArgs),
        ("peer", (ctypes.c_void_p * MAX_GROUPS) * 3),
        ("max_ctas", ctypes.c_int32),
    ]


class PeerBarrierArgs(ctypes.Structure):
    _fields_ = [
        ("flags", ctypes.c_void_p * MAX_GROUPS),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("epoch", ctypes.c_uint32),
        ("timeout_ns", ctypes.c_int64),
    ]


def _fn(name, argtypes):
    f = getattr(_lib.load(), name)
    f.argtypes = argtypes
    f.restype = ctypes.c_int
    return f


def ipc_handle(ptr: int) -> Tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding ptr, ptr's offset in it)."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(0)
    _lib.check(_fn("vx_ipc_get_handle", [ctypes.c_void_p, ctypes.c_char_p,
                                         ctypes.POINTER(ctypes.c_int64)])(
        ctypes.c_void_p(ptr), buf, ctypes.byref(off)))
    return buf.raw, off.value


def ipc_open(handle: bytes) -> int:
    base = ctypes.c_void_p()
    _lib.check(_fn("vx_ipc_open", [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)])(
        handle, ctypes.byref(base)))
    return base.value


def ipc_close(base: int) -> None:
    _lib.check(_fn("vx_ipc_close", [ctypes.c_void_p])(ctypes.c_void_p(base)))


def peer_barrier(flags: List[int], rank: int, epoch: int, stream,
                 timeout_ns: int = BARRIER_TIMEOUT_NS) -> None:
    """vx_peer_barrier over the flag arrays `flags` (one address per rank)."""
    a = PeerBarrierArgs()
    for g, f in enumerate(flags):
        a.flags[g] = f
    a.rank, a.world, a.epoch, a.timeout_ns = rank, len(flags), epoch, timeout_ns
    _lib.check(_fn("vx_peer_barrier", [ctypes.POINTER(PeerBarrierArgs), ctypes.c_void_p])(
        ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)))


def slab_peers(pack: bool, strided, peers, heads: int, groups: int, sub, stream,
               max_ctas: int = 0) -> None:
    """vx_ulysses_pack_peers (pack) / vx_ulysses_unpack_peers: `strided` are
    this rank's (S_loc, H, D) views, peers[t][g] the remote chunk addresses."""
    a = PeerSlabArgs()
    s = a.slab
    s.num_tensors = len(strided)
    seq, _, d = strided[0].shape
    for t, x in enumerate(strided):
        if x.stride(-1) != 1 or x.dtype != torch.bfloat16:
            raise ValueError("bf16 views with head_dim contiguous")
        if pack:
            s.src[t] = x.data_ptr()
        else:
            s.dst[t] = x.data_ptr()
        s.stride[t][0], s.stride[t][1] = x.stride(0), x.stride(1)
        for g in range(groups):
            a.peer[t][g] = peers[t][g]
    s.seq, s.heads, s.head_dim, s.groups = seq, heads, d, groups
    s.slab_heads, s.group_stride, s.head_offset, s.group_valid = sub
    a.max_ctas = max_ctas
    name = "vx_ulysses_pack_peers" if pack else "vx_ulysses_unpack_peers"
    _lib.check(_fn(name, [ctypes.POINTER(PeerSlabArgs), ctypes.c_void_p])(
        ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)))


class PeerWorkspace:
    """One rank's receive slabs (q, k, v), output slab and barrier flags,
    with every rank's copy mapped into this process (collective: every rank
    of `group` constructs it with the same sizes, on its own GPU)."""

    def __init__(self, group, seq_local: int, heads: int, head_dim: int, device,
                 prefix: int = 0):
        self.group = group
        self.prefix = prefix   # rows before the received chunks (the joint layout's text)
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.P > MAX_GROUPS:
            raise NotImplementedError(f"the peer exchange spans at most {MAX_GROUPS} GPUs")
        self.seq_local, self.heads, self.head_dim = seq_local, heads, head_dim
        self.Hg = -(-heads // self.P)
        elems = (prefix + self.P * seq_local) * self.Hg * head_dim
        self.slab_bytes = (elems * 2 + 255) // 256 * 256
        self.flag_off = 4 * self.slab_bytes
        self.device = torch.device(device)
        self.buf = torch.empty(self.flag_off + 256, dtype=torch.uint8, device=self.device)
        # zeroed once: the flags, and the padded heads (H % P != 0) the
        # host-buffer form never writes (the slab kernels write them as zeros)
        self.buf.zero_()
        torch.cuda.synchronize(self.device)
        why = ""
        try:
            info = ipc_handle(self.buf.data_ptr())
        except _lib.VxError as e:   # e.g. an allocator without cudaMalloc'd segments
            info, why = None, str(e)
        infos: List = [None] * self.P
        dist.all_gather_object(infos, info, group=group)
        self._opened: List[int] = []
        self.base: List[int] = []
        if all(i is not None for i in infos):
            for g, (handle, off) in enumerate(infos):
                if g == self.rank:
                    self.base.append(self.buf.data_ptr())
                    continue
                try:
                    b = ipc_open(handle)
                except _lib.VxError as e:   # no peer access between these GPUs
                    why = str(e)
                    break
                self._opened.append(b)
                self.base.append(b + off)
        else:
            why = why or "another rank could not export its workspace"
        # every rank learns whether all of them mapped all the others
        ok = torch.tensor([0 if why else 1], device=self.device, dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if ok.item() == 0:
            for b in self._opened:
                ipc_close(b)
            self._opened, self.buf = [], None
            raise PeerUnavailable("the peer-memory exchange cannot map the ranks' memory "
                                  f"({why or 'failed on another rank'}); use exchange='nccl'")
        self.epoch = [0, 0, 0]
        # every rank has zeroed its flags and mapped the others' before any barrier
        dist.barrier(group=group)

    def fits(self, seq_local: int, heads: int, head_dim: int, prefix: int = 0) -> bool:
        return ((seq_local, heads, head_dim, prefix) ==
                (self.seq_local, self.heads, self.head_dim, self.prefix))

    def rows(self) -> int:
        return self.prefix + self.P * self.seq_local

    def slice_off(self, off: int) -> int:
        """byte offset of a slice (first head `off` of the group) in a slab"""
        return 2 * self.rows() * off * self.head_dim

    def local_view(self, slab: int, off: int, hs: int) -> torch.Tensor:
        """(1, prefix + S, hs, D) view of this rank's slab `slab` (0-2 q/k/v
        received, 3 output)."""
        start = slab * self.slab_bytes + self.slice_off(off)
        n = self.rows() * hs * self.head_dim
        return self.buf[start:start + 2 * n].view(torch.bfloat16).view(
            1, self.rows(), hs, self.head_dim)

    def remote(self, g: int, slab: int, off: int, hs: int) -> int:
        """address of this rank's chunk of slice (off, hs) in rank g's slab"""
        row = self.prefix + self.rank * self.seq_local
        return (self.base[g] + slab * self.slab_bytes + self.slice_off(off) +
                2 * row * hs * self.head_dim)

    def remote_prefix(self, g: int, slab: int, off: int) -> int:
        """address of the prefix rows of slice `off` in rank g's slab"""
        return self.base[g] + slab * self.slab_bytes + self.slice_off(off)

    def barrier(self, channel: int, stream) -> None:
        self.epoch[channel] += 1
        flags = [b + self.flag_off + channel * MAX_GROUPS * 4 for b in self.base]
        peer_barrier(flags, self.rank, self.epoch[channel] & 0xFFFFFFFF, stream)

    def close(self) -> None:
        """Collective: unmaps the other ranks' workspaces once all are done."""
        if self.buf is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for b in self._opened:
            ipc_close(b)
        self._opened = []
        self.buf = None


_WORKSPACES: Dict[Tuple[int, int], PeerWorkspace] = {}


def workspace(group, seq_local: int, heads: int, head_dim: int, device,
              prefix: int = 0) -> PeerWorkspace:
    """The cached workspace of `group` on `device`, (re)made collectively when
    the shapes change."""
    key = (id(group), torch.device(device).index)
    ws = _WORKSPACES.get(key)
    if ws is not None and not ws.fits(seq_local, heads, head_dim, prefix):
        ws.close()
        ws = None
    if ws is None:
        ws = PeerWorkspace(group, seq_local, heads, head_dim, device, prefix)
        _WORKSPACES[key] = ws
    return ws


def release_workspaces() -> None:
    """Collective: closes every cached workspace (before destroy_process_group)."""
    for ws in _WORKSPACES.values():
        ws.close()
    _WORKSPACES.clear()


def _ret_stream(device):
    dev = torch.device(device).index
    s = _RET_STREAMS.get(dev)
    if s is None:
        s = torch.cuda.Stream(device=dev)
        _RET_STREAMS[dev] = s
    return s


_RET_STREAMS: Dict[int, "torch.cuda.Stream"] = {}


def sequence_parallel_self_attention_peer(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group=None,
    scale: Optional[float] = None, *, valid_len: Optional[int] = None,
) -> torch.Tensor:
    """sequence_parallel_self_attention (attention.py:341-388) with the
    exchanges over peer memory: q, k, v (B, L_local, H, D) bf16, this rank's
    token chunk; returns (B, L_local, H, D). `group`: a process group whose
    ranks are GPUs of one NVLink domain (default: the default group)."""
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    if not (q.shape == k.shape == v.shape):
        raise ValueError("self-attention needs q, k, v of equal shape")
    B, S_loc, H, D = q.shape
    ws = workspace(group, S_loc, H, D, q.device)
    P, r, Hg = ws.P, ws.rank, ws.Hg
    S = P * S_loc
    sm_scale = D ** -0.5 if scale is None else scale
    kv_len = None
    if valid_len is not None and valid_len < S:
        kv_len = torch.full((1,), valid_len, dtype=torch.int32, device=q.device)
    sizes = _pieces(Hg) if PIPELINED else [Hg]
    offs = [sum(sizes[:j]) for j in range(len(sizes))]
    n = len(sizes)
    out = torch.empty_like(q)
    comp = torch.cuda.current_stream(q.device)
    side = _side_stream(q.device)
    ret = _ret_stream(q.device)
    for b in range(B):
        side.wait_stream(comp)
        ret.wait_stream(comp)
        ev_in = []
        with torch.cuda.stream(side):
            for j, (hs, off) in enumerate(zip(sizes, offs)):
                peers = [[ws.remote(g, t, off, hs) for g in range(P)] for t in range(3)]
                slab_peers(True, [q[b], k[b], v[b]], peers, H, P, (hs, Hg, off, hs), side,
                           0 if j == 0 else SLICE_CTAS)
                ws.barrier(CH_IN, side)
                ev = torch.cuda.Event()
                ev.record(side)
                ev_in.append(ev)
        for j, (hs, off) in enumerate(zip(sizes, offs)):
            comp.wait_event(ev_in[j])
            rq, rk, rv = (ws.local_view(t, off, hs) for t in range(3))
            _timed_attention(rq, rk, rv, sm_scale, kv_len, ws.local_view(3, off, hs))
            ev = torch.cuda.Event()
            ev.record(comp)
            with torch.cuda.stream(ret):
                ret.wait_event(ev)
                ws.barrier(CH_OUT, ret)
                peers = [[ws.remote(g, 3, off, hs) for g in range(P)]]
                slab_peers(False, [out[b]], peers, H, P, (hs, Hg, off, hs), ret,
                           0 if j == n - 1 else SLICE_CTAS)
        comp.wait_stream(ret)
        ws.barrier(CH_END, comp)
    return out


def launches_per_layer(heads: int, world: int, batch: int = 1) -> int:
    """Kernel launches of one sequence_parallel_self_attention_peer call: per
    batch item and head slice a pack, a barrier, the attention kernel, a
    barrier and an unpack, and one closing barrier."""
    n = len(_pieces(-(-heads // world))) if PIPELINED else 1
    return batch * (5 * n + 1)


def measure_exchange(x: torch.Tensor, reps: int = 10, group=None) -> dict:
    """One q-sized tokens->heads exchange of the peer path on its own: the
    pack-to-peers of x's whole head group (x: this rank's (S_loc, H, D)) and
    its barrier, timed `reps` times after 3 warm-up runs (device time, max
    over ranks). Uses the layer's cached workspace (call the layer first)."""
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    S_loc, H, D = x.shape
    ws = workspace(group, S_loc, H, D, x.device)
    P, Hg = ws.P, ws.Hg
    peers = [[ws.remote(g, 0, 0, Hg) for g in range(P)]]
    stream = torch.cuda.current_stream(x.device)

    def once():
        slab_peers(True, [x], peers, H, P, (Hg, Hg, 0, Hg), stream)
        ws.barrier(CH_IN, stream)

    for _ in range(3):
        once()
    torch.cuda.synchronize(x.device)
    dist.barrier(group=group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        once()
    e1.record(stream)
    torch.cuda.synchronize(x.device)
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=x.device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    ms = float(t.item())
    cross = S_loc * Hg * D * 2 * (P - 1)   # bytes this rank sends to the others
    return {"buffer_bytes_per_gpu": P * S_loc * Hg * D * 2, "bytes_per_gpu_per_direction": cross,
            "ms": round(ms, 4), "gbs_per_direction": round(cross / ms / 1e6, 1),
            "what": "pack-to-peers kernel + flag barrier (SM stores over NVLink)"}


def sequence_parallel_self_attention_from_host_peer(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group=None,
    scale: Optional[float] = None, *, out: Optional[torch.Tensor] = None,
    device: Optional[torch.device] = None,
) -> torch.Tensor:
    """The host-buffer form (pinned q, k, v (B, L_local, H, D) in, pinned
    output back; complete once the current stream is synchronised) with the
    exchanges over peer memory: per slice, one 2-D copy per rank group moves
    that group's heads of every local token from host rows straight into
    rank g's receive slab, and after every rank's kernel one 2-D copy per
    group moves this rank's tokens of rank g's output slab straight into
    the host output rows -- the copies are the all-to-alls. Uploads of slice
    j+1 and downloads of slice j-1 run on copy streams beside the kernel on
    slice j; flag barriers order them across GPUs."""
    from .hostio import _check_host, _side_streams, check_host_out, group_sizes
    from .ulysses import _rows_copy, _slab_heads
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_host(name, t)
    if not (q.shape == k.shape == v.shape):
        raise ValueError("self-attention needs q, k, v of equal shape")
    if out is not None:
        check_host_out(out, q.shape)
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    B, S_loc, H, D = q.shape
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    sm_scale = D ** -0.5 if scale is None else scale
    if out is None:
        out = torch.empty((B, S_loc, H, D), dtype=torch.bfloat16).pin_memory()
    ws = workspace(group, S_loc, H, D, device)
    P, Hg = ws.P, ws.Hg
    sizes = group_sizes(Hg, 8)
    offs = [sum(sizes[:j]) for j in range(len(sizes))]
    es = 2
    comp = torch.cuda.current_stream(device)
    h2d, d2h = _side_streams(device)
    h2d.wait_stream(comp)
    d2h.wait_stream(comp)
    for b in range(B):
        ready = []
        for hs, off in zip(sizes, offs):
            for t, src in enumerate((q, k, v)):
                for g in range(P):
                    h0, n = _slab_heads(g, Hg, off, hs, H)
                    if n > 0:
                        _rows_copy(ws.remote(g, t, off, hs), hs * D * es,
                                   src.data_ptr() + (b * src.stride(0) + h0 * src.stride(2)) * es,
                                   src.stride(1) * es, n * D * es, S_loc, h2d)
            ws.barrier(CH_IN, h2d)   # every rank's uploads of this slice landed
            ev = torch.cuda.Event()
            ev.record(h2d)
            ready.append(ev)
        for j, (hs, off) in enumerate(zip(sizes, offs)):
            comp.wait_event(ready[j])
            rq, rk, rv = (ws.local_view(t, off, hs) for t in range(3))
            _timed_attention(rq, rk, rv, sm_scale, None, ws.local_view(3, off, hs))
            ev = torch.cuda.Event()
            ev.record(comp)
            d2h.wait_event(ev)
            ws.barrier(CH_OUT, d2h)  # every rank's kernel on this slice finished
            for g in range(P):
                h0, n = _slab_heads(g, Hg, off, hs, H)
                if n > 0:
                    _rows_copy(out.data_ptr() + (b * out.stride(0) + h0 * out.stride(2)) * es,
                               out.stride(1) * es, ws.remote(g, 3, off, hs), hs * D * es,
                               n * D * es, S_loc, d2h)
        ws.barrier(CH_END, d2h)      # every rank's downloads done: the workspace is free
        h2d.wait_stream(d2h)
    comp.wait_stream(d2h)
    return out


def sequence_parallel_joint_self_attention_peer(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, text_len: int, group=None,
    scale: Optional[float] = None,
) -> torch.Tensor:
    """Joint [text; visual] Ulysses attention (attention.py:391-464) with the
    exchanges over peer memory. q, k, v (B, text_len + L_vis_local, H, D):
    the text prefix replicated on every rank, the visual rows this rank's
    chunk. The text rows of this rank's head group are packed into its own
    receive slab's prefix, the visual rows stored straight into every rank's
    slab; after the joint kernel the visual output is loaded back from every
    rank's output slab and the text output gathered over heads the same way
    (the all_gather of attention.py:463 as loads of each rank's prefix rows)."""
    from .ulysses import pack_heads
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    if not (q.shape == k.shape == v.shape):
        raise ValueError("self-attention needs q, k, v of equal shape")
    B, L, H, D = q.shape
    S_loc = L - text_len
    ws = workspace(group, S_loc, H, D, q.device, prefix=text_len)
    P, r, Hg = ws.P, ws.rank, ws.Hg
    sm_scale = D ** -0.5 if scale is None else scale
    h0 = r * Hg
    nvalid = max(0, min(h0 + Hg, H) - h0)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(q.device)
    sub = (Hg, Hg, 0, Hg)
    for b in range(B):
        # this rank's text heads -> its own slabs' prefix rows (zero heads past H)
        for t, x in enumerate((q, k, v)):
            prefix = ws.local_view(t, 0, Hg)[0, :text_len]
            pack_heads([x[b, :text_len]], 1, out=[prefix.unsqueeze(0)],
                       sub=(Hg, 0, h0, nvalid))
        peers = [[ws.remote(g, t, 0, Hg) for g in range(P)] for t in range(3)]
        slab_peers(True, [q[b, text_len:], k[b, text_len:], v[b, text_len:]], peers, H, P, sub,
                   stream)
        ws.barrier(CH_IN, stream)
        rq, rk, rv = (ws.local_view(t, 0, Hg) for t in range(3))
        _timed_attention(rq, rk, rv, sm_scale, None, ws.local_view(3, 0, Hg))
        ws.barrier(CH_OUT, stream)
        # visual rows: this rank's tokens of every rank's head group
        slab_peers(False, [out[b, text_len:]], [[ws.remote(g, 3, 0, Hg) for g in range(P)]],
                   H, P, sub, stream)
        # text rows: every rank's head group of the text (the all_gather)
        slab_peers(False, [out[b, :text_len]], [[ws.remote_prefix(g, 3, 0) for g in range(P)]],
                   H, P, sub, stream)
        ws.barrier(CH_END, stream)
    return out
