"""The Ulysses layer through the C ABI (`vx_ulysses_attn_fwd`), for callers
that hold an NCCL communicator rather than a torch process group.

`sequence_parallel_self_attention` in `vidax_b200.ulysses` runs the same
pipeline from Python (pack -> NCCL all-to-alls -> attention kernel ->
all-to-all -> unpack, pipelined by head slices). Here the whole layer
(src/vidax/core/attention.py:341-388) is one C call, with the exchanges on
the library's own stream, so any host that can lend the library an NCCL
communicator (`Comm.wrap`) -- or create one from a unique id passed around
by its own means (`unique_id`, `Comm.init`) -- gets the overlapped layer.
Torch callers can lend their process group's communicator
(`Comm.from_process_group`).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib


class UlyssesArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("batch", ctypes.c_int32),
        ("seq_local", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("valid_len", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
    ]


def _fn(name, argtypes):
    f = getattr(_lib.load(), name)
    f.argtypes = argtypes
    f.restype = ctypes.c_int
    return f


def unique_id() -> bytes:
    """An NCCL unique id (128 bytes) for `Comm.init`; make it on one rank
    and send it to the others."""
    buf = ctypes.create_string_buffer(128)
    _lib.check(_fn("vx_comm_get_unique_id", [ctypes.c_char_p])(buf))
    return buf.raw


class Comm:
    """A library communicator handle (`vx_comm`) for the current device."""

    def __init__(self, handle: ctypes.c_void_p, world: int, keep=None):
        self.handle = handle
        self.world = world
        self._keep = keep  # the lent process group stays alive as long as this handle

    @classmethod
    def init(cls, rank: int, world: int, uid: bytes) -> "Comm":
        """Creates this rank's communicator (every rank calls it on its own GPU)."""
        h = ctypes.c_void_p()
        f = _fn("vx_comm_init", [ctypes.c_int32, ctypes.c_int32, ctypes.c_char_p,
                                 ctypes.POINTER(ctypes.c_void_p)])
        _lib.check(f(rank, world, uid, ctypes.byref(h)))
        return cls(h, world)

    @classmethod
    def wrap(cls, nccl_comm_ptr: int, world: int, keep=None) -> "Comm":
        """Borrows an existing ncclComm_t of the current device."""
        h = ctypes.c_void_p()
        f = _fn("vx_comm_wrap", [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)])
        _lib.check(f(ctypes.c_void_p(nccl_comm_ptr), ctypes.byref(h)))
        return cls(h, world, keep)

    @classmethod
    def from_process_group(cls, group=None) -> "Comm":
        """Borrows the NCCL communicator of a torch process group (backend
        nccl, created with a device id so the communicator exists)."""
        pg = group if group is not None else dist.distributed_c10d._get_default_group()
        backend = pg._get_backend(torch.device("cuda", torch.cuda.current_device()))
        return cls.wrap(backend._comm_ptr(), dist.get_world_size(pg), keep=pg)

    def close(self) -> None:
        if self.handle:
            _lib.check(_fn("vx_comm_destroy", [ctypes.c_void_p])(self.handle))
            self.handle = None

    def __del__(self):  # best effort; close() reports errors
        try:
            self.close()
        except Exception:
            pass


def workspace_bytes(q: torch.Tensor, world: int) -> int:
    a = UlyssesArgs()
    a.batch, a.seq_local, a.heads, a.head_dim = q.shape
    n = ctypes.c_int64(0)
    _lib.check(_fn("vx_ulysses_workspace_size", [ctypes.POINTER(UlyssesArgs), ctypes.c_int32,
                                                  ctypes.POINTER(ctypes.c_int64)])(
        ctypes.byref(a), world, ctypes.byref(n)))
    return n.value


def sequence_parallel_self_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, comm: Comm,
    scale: Optional[float] = None, *, valid_len: Optional[int] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """DeepSpeed-Ulysses self-attention in one C call: q, k, v (B, L_local,
    H, D) bf16, this rank's token chunk (chunk_by_rank ownership). Returns
    (B, L_local, H, D). `valid_len`: real tokens of the global sequence when
    it was padded to a multiple of the axis size (padding keys masked)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dtype != torch.bfloat16 or t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a (B, L, H, D) bf16 CUDA tensor, head_dim contiguous")
    if not (q.shape == k.shape == v.shape):
        raise ValueError("self-attention needs q, k, v of equal shape")
    B, S_loc, H, D = q.shape
    out = torch.empty_like(q)
    need = workspace_bytes(q, comm.world)
    if workspace is None or workspace.numel() < need or not workspace.is_cuda:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    a = UlyssesArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    for f, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", out)):
        getattr(a, f)[:] = t.stride()[:3]
    a.batch, a.seq_local, a.heads, a.head_dim = B, S_loc, H, D
    a.scale = float(D ** -0.5 if scale is None else scale)
    a.valid_len = int(valid_len or 0)
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    stream = torch.cuda.current_stream(q.device)
    f = _fn("vx_ulysses_attn_fwd", [ctypes.POINTER(UlyssesArgs), ctypes.c_void_p, ctypes.c_void_p])
    _lib.check(f(ctypes.byref(a), comm.handle, ctypes.c_void_p(stream.cuda_stream)))
    workspace.record_stream(stream)
    return out
