"""Attention on host-resident (pinned) tensors with overlapped transfers.

A caller whose q/k/v live in host memory (the end-to-end path of a plugin
that hands over host buffers) would otherwise pay copy-in, compute and
copy-out back to back. Here the heads are split into groups: the copy stream
moves group g+1's q/k/v to the device (one strided 2-D copy per tensor,
`vx_memcpy_rows_async`) while the compute stream runs the attention kernel
on group g (in place on head-sliced views -- the kernel takes arbitrary BSHD
strides) and a second copy stream brings group g-1's output back. PCIe
traffic in both directions hides behind the kernel except for the first
group's upload and the last group's download.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_streams: Dict[int, Tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}
_lock = threading.Lock()


def _side_streams(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        if idx not in _streams:
            _streams[idx] = (torch.cuda.Stream(device=idx), torch.cuda.Stream(device=idx))
        return _streams[idx]


def copy_heads(dst: torch.Tensor, src: torch.Tensor, h0: int, h1: int,
               stream: torch.cuda.Stream) -> None:
    """Copies heads [h0, h1) of a (B, S, H, D) tensor between host and device
    (either direction), stream-ordered: one 2-D copy per batch item (rows are
    tokens, pitch = the token stride)."""
    B, S, H, D = src.shape
    es = src.element_size()
    row_bytes = (h1 - h0) * D * es
    lib = _lib.load()
    for b in range(B):
        s_ptr = src.data_ptr() + (b * src.stride(0) + h0 * src.stride(2)) * es
        d_ptr = dst.data_ptr() + (b * dst.stride(0) + h0 * dst.stride(2)) * es
        _lib.check(lib.vx_memcpy_rows_async(
            ctypes.c_void_p(d_ptr), dst.stride(1) * es, ctypes.c_void_p(s_ptr), src.stride(1) * es,
            row_bytes, S, ctypes.c_void_p(stream.cuda_stream)))


def group_sizes(hkv: int, cap: int) -> list:
    """KV heads per pipeline group: 1, 2, 4, ... up to `cap`, then a last
    group of 1. Only the first group's upload and the last group's download
    are exposed, so both are one head; doubling keeps each upload (about
    0.4x a head's kernel time at Wan 14B lengths over PCIe 5) shorter than
    the kernels of the groups before it, so the compute stream never waits."""
    body = hkv - 1 if hkv > 1 else hkv
    sizes, n = [], 1
    while sum(sizes) < body:
        sizes.append(min(n, cap, body - sum(sizes)))
        n *= 2
    if hkv > 1:
        sizes.append(1)
    return sizes


def _check_host(name: str, t: torch.Tensor) -> None:
    if t.device.type != "cpu":
        raise ValueError(f"{name} must be a host tensor on this path")
    if t.dtype != torch.bfloat16:
        raise NotImplementedError(f"{name}.dtype={t.dtype}: the sm_100a kernels take bfloat16")
    if t.dim() != 4 or t.stride(-1) != 1 or t.stride(2) != t.shape[3]:
        raise ValueError(f"{name} must be (B, S, H, D) with contiguous (H, D) rows")


def check_host_out(out: torch.Tensor, shape) -> None:
    """`out` receives row copies straight from the device: it must be a host
    bf16 tensor of exactly `shape` with contiguous (H, D) rows."""
    _check_host("out", out)
    if tuple(out.shape) != tuple(shape):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {tuple(shape)}")


def attention_from_host(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
    kv_len: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
    heads_per_group: Optional[int] = None, device: Optional[torch.device] = None,
) -> torch.Tensor:
    """softmax(scale * q k^T) v for host (B, S, H, D) bf16 tensors (pinned for
    overlap), computed on `device` (default: the current CUDA device) with
    transfers pipelined against the kernel by head groups. Returns a host
    tensor (`out` if given, else a new pinned tensor) whose contents are
    complete once the current CUDA stream has been synchronised (the call
    only enqueues, like a device kernel)."""
    from .attention import flash_attention

    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_host(name, t)
    B, Sq, H, D = q.shape
    _, Sk, Hkv, _ = k.shape
    if H % Hkv != 0:
        raise ValueError("heads_q must be a multiple of heads_kv")
    group = H // Hkv
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if heads_per_group is None:
        sizes = group_sizes(Hkv, max(1, min(Hkv, 8 // group if group < 8 else 1)))
    else:
        n = max(1, heads_per_group // group)
        sizes = [min(n, Hkv - i) for i in range(0, Hkv, n)]
    if out is None:
        out = torch.empty((B, Sq, H, D), dtype=torch.bfloat16).pin_memory()
    else:
        check_host_out(out, (B, Sq, H, D))
    qd = torch.empty((B, Sq, H, D), dtype=torch.bfloat16, device=device)
    kd = torch.empty((B, Sk, Hkv, D), dtype=torch.bfloat16, device=device)
    vd = torch.empty_like(kd)
    od = torch.empty_like(qd)
    if kv_len is not None:
        kv_len = kv_len.to(device=device, dtype=torch.int32)
    comp = torch.cuda.current_stream(device)
    h2d, d2h = _side_streams(device)
    h2d.wait_stream(comp)   # device buffers may reuse memory the compute stream just freed
    d2h.wait_stream(comp)
    groups = []
    for n in sizes:
        g0 = groups[-1][1] if groups else 0
        groups.append((g0, g0 + n))
    ready = []
    for k0, k1 in groups:
        q0, q1 = k0 * group, k1 * group
        copy_heads(qd, q, q0, q1, h2d)
        copy_heads(kd, k, k0, k1, h2d)
        copy_heads(vd, v, k0, k1, h2d)
        ev = torch.cuda.Event()
        ev.record(h2d)
        ready.append(ev)
    for (k0, k1), ev in zip(groups, ready):
        q0, q1 = k0 * group, k1 * group
        comp.wait_event(ev)
        flash_attention(qd[:, :, q0:q1], kd[:, :, k0:k1], vd[:, :, k0:k1], scale, kv_len=kv_len,
                        out=od[:, :, q0:q1], stream=comp)
        done = torch.cuda.Event()
        done.record(comp)
        d2h.wait_event(done)
        copy_heads(out, od, q0, q1, d2h)
    comp.wait_stream(d2h)
    # keep the device buffers alive until the copies that use them finished
    for t in (qd, kd, vd, od):
        t.record_stream(h2d)
        t.record_stream(d2h)
    return out
