"""vidax's attention-function API on B200, backed by libvidax_cuda.so.

Mirrors `vidax.core.attention` (src/vidax/core/attention.py) name for name and
argument for argument, with torch CUDA tensors in vidax's BSHD layout in place
of `jax.Array`s:

* `dot_product_attention`  -- attention.py:467-533
* `local_attention`        -- attention.py:321-338
* `chunk_by_rank`          -- attention.py:132-146

The sequence-parallel entry points live in `vidax_b200.ulysses` and are
re-exported from the package. Every call runs the sm_100a kernel through the
C ABI; requests the kernel does not implement raise `NotImplementedError`
(there is no CPU or library fallback).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


#: When set to a list, (start, end) CUDA events bracketing every attention
#: kernel launch of `flash_attention` are appended to it (kernel-level timing
#: for benchmarks; the data path is unchanged).
KERNEL_EVENTS: Optional[list] = None


def _check_bshd(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dim() != 4:
        raise ValueError(f"{name} must be (B, S, H, D), got shape {tuple(t.shape)}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this implementation has no CPU path)")
    if t.dtype != torch.bfloat16:
        raise NotImplementedError(f"{name}.dtype={t.dtype}: the sm_100a kernels take bfloat16")
    if t.numel() > 0 and t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous head_dim (stride(-1) == 1)")


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """Returns `t` if its strides/base satisfy the TMA rules, else a contiguous copy."""
    if t.numel() == 0:
        return t
    ok = t.data_ptr() % 16 == 0 and all(s > 0 and s % 8 == 0 for s in t.stride()[:3])
    return t if ok else t.contiguous()


def _strides3(t: torch.Tensor):
    return (ctypes.c_int64 * 3)(*t.stride()[:3])


def flash_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
    kv_len: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
    return_lse: bool = False, stream: Optional[torch.cuda.Stream] = None,
    dynamic_schedule: bool = False,
):
    """Runs the sm_100a attention kernel: softmax(scale * q k^T) v, per (b, h).

    q: (B, Sq, Hq, D), k/v: (B, Sk, Hkv, D) with Hq % Hkv == 0, bf16 on one
    CUDA device. `kv_len` (int32 [B], device) hides keys at index >= kv_len[b]
    -- the key-side SegmentIds padding mask of attention.py:272-278.
    `dynamic_schedule` distributes work at run time (for launches that share
    the GPU with concurrent kernels such as NCCL collectives).
    Returns o (B, Sq, Hq, D) bf16 [and lse (B, Hq, Sq) fp32].
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_bshd(name, t)
    B, Sq, Hq, D = q.shape
    Bk, Sk, Hkv, Dk = k.shape
    if v.shape != k.shape:
        raise ValueError(f"k {tuple(k.shape)} and v {tuple(v.shape)} must match")
    if Bk != B or Dk != D:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree on batch/head_dim")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must live on the same device")
    q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    if out is None:
        out = torch.empty((B, Sq, Hq, D), dtype=torch.bfloat16, device=q.device)
    elif (out.shape != (B, Sq, Hq, D) or out.dtype != torch.bfloat16 or out.stride(-1) != 1
          or out.device != q.device):
        raise ValueError("out must be a bf16 (B, Sq, Hq, D) tensor with contiguous head_dim "
                         "on q's device")
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device) if return_lse else None
    if kv_len is not None:
        if kv_len.dtype != torch.int32 or kv_len.numel() != B or kv_len.device != q.device:
            raise ValueError("kv_len must be an int32 tensor with B elements on q's device")
        kv_len = kv_len.contiguous()

    a = _lib.AttnArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    a.q_stride, a.k_stride = _strides3(q), _strides3(k)
    a.v_stride, a.o_stride = _strides3(v), _strides3(out)
    a.batch, a.seq_q, a.seq_k = B, Sq, Sk
    a.heads_q, a.heads_kv, a.head_dim = Hq, Hkv, D
    a.scale = float(scale)
    a.kv_len = kv_len.data_ptr() if kv_len is not None else None
    a.lse = lse.data_ptr() if lse is not None else None
    a.schedule = _lib.VX_SCHED_DYNAMIC if dynamic_schedule else _lib.VX_SCHED_STATIC
    lib = _lib.load()
    events = KERNEL_EVENTS
    with torch.cuda.device(q.device):
        s = stream if stream is not None else torch.cuda.current_stream(q.device)
        if events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
        _lib.check(lib.vx_attn_fwd(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)))
        if events is not None:
            e1.record(s)
            events.append((e0, e1))
    return (out, lse) if return_lse else out


def _key_lengths_from_mask(mask: torch.Tensor, B: int, Sk: int) -> torch.Tensor:
    """Converts a key-only boolean mask (True = attend) that marks a valid key
    prefix per batch row into per-batch lengths; anything else is rejected."""
    m = mask
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.shape[1] != 1 or m.shape[2] != 1 or m.shape[3] != Sk or m.shape[0] not in (1, B):
        raise NotImplementedError(
            "only key-padding masks broadcastable as (B, 1, 1, Sk) are supported by the CUDA "
            f"kernel; got mask of shape {tuple(mask.shape)}")
    m = m.reshape(m.shape[0], Sk).expand(B, Sk).to(torch.bool)
    lens = m.sum(dim=1, dtype=torch.int32)
    prefix = torch.arange(Sk, device=m.device)[None, :] < lens[:, None]
    if not bool(torch.equal(prefix, m)):
        raise NotImplementedError("key mask is not a valid-prefix mask; general masks are unsupported")
    return lens.to(torch.int32)


def _key_lengths_from_bias(bias: torch.Tensor, B: int, Sk: int) -> torch.Tensor:
    """Accepts the additive key-padding bias idiom (0 for valid keys, -inf or a
    large negative for padding, shape (B, 1, 1, Sk)); rejects dense biases."""
    b = bias
    while b.dim() < 4:
        b = b.unsqueeze(0)
    if b.shape[1] != 1 or b.shape[2] != 1:
        raise NotImplementedError(
            "dense additive attention bias (e.g. T5 relative position bias) is not implemented "
            f"by the CUDA kernel; got bias of shape {tuple(bias.shape)}")
    bf = b.float()
    valid = bf == 0
    pad = bf <= -1e9
    if not bool((valid | pad).all()):
        raise NotImplementedError("only 0 / -inf key-padding biases are supported")
    return _key_lengths_from_mask(valid, B, Sk)


def _fully_masked_rows(bias: Optional[torch.Tensor], mask: Optional[torch.Tensor],
                       lens: torch.Tensor, B: int, Sk: int):
    """Batch items whose every key is masked, and what the reference gives
    for them (jax.nn.dot_product_attention, attention.py:533): with a boolean
    mask the masked logits become one large negative number, so the weights
    are uniform and each output row is the mean of v over all Sk keys
    ("mean"); with an additive bias of -inf the softmax is 0/0 ("nan"); a
    row of one finite large negative value is uniform again ("mean").
    Returns [(b, mode)]."""
    empty = [int(b) for b in torch.nonzero(lens.cpu() == 0).flatten()]
    if not empty or Sk == 0:
        return []
    if mask is not None:
        return [(b, "mean") for b in empty]
    bb = bias
    while bb.dim() < 4:
        bb = bb.unsqueeze(0)
    rows = bb.reshape(bb.shape[0], Sk).expand(B, Sk).float().cpu()
    out = []
    for b in empty:
        r = rows[b]
        if bool(torch.isneginf(r).all()):
            out.append((b, "nan"))
        elif bool((r == r[0]).all()):
            out.append((b, "mean"))
        else:
            raise NotImplementedError(
                "a fully masked key row with unequal padding-bias values is not supported")
    return out


def _fill_fully_masked(out: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows, scale: float):
    """Writes the reference's result for fully masked batch items into `out`
    (device or host): NaN, or the mean of v over all keys, computed by the
    attention kernel with a zero query (all logits 0: uniform weights)."""
    for b, mode in rows:
        if mode == "nan":
            out[b].fill_(float("nan"))
            continue
        dev = out.device if out.is_cuda else torch.device("cuda", torch.cuda.current_device())
        kb, vb = k[b:b + 1].to(dev), v[b:b + 1].to(dev)
        zq = torch.zeros((1, 1, out.shape[2], out.shape[3]), dtype=torch.bfloat16, device=dev)
        m = flash_attention(zq, kb, vb, scale)
        out[b].copy_(m[0].expand(out.shape[1], -1, -1))


def local_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
) -> torch.Tensor:
    """Plain attention as one local call (attention.py:321-338): always this
    device's kernel, no cross-device communication. Default scale D^-0.5."""
    head_dim = q.shape[-1]
    sm_scale = head_dim ** -0.5 if scale is None else scale
    if q.device.type == "cpu":
        from .hostio import attention_from_host
        return attention_from_host(q, k, v, sm_scale)
    return flash_attention(q, k, v, sm_scale)


def dot_product_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    mask: Optional[torch.Tensor] = None,
    scale: Optional[float] = None,
    mesh=None,
) -> torch.Tensor:
    """Full (non-causal) attention (attention.py:467-533).

    q, k, v: (B, S, num_heads, head_dim); k/v may have another sequence
    length (cross-attention). `scale` defaults to head_dim ** -0.5. CUDA
    tensors run in place; host (pinned) tensors take the pipelined
    host-buffer path and return a host tensor.
    `bias` / `mask` are accepted only in their key-padding forms ((B,1,1,Sk)
    0/-inf bias or boolean valid-prefix mask), which become per-batch key
    lengths for the kernel; dense biases and general masks raise
    NotImplementedError. A batch item with no visible key gets what the
    reference gives it: the mean of v over all keys (mask form, or a row of
    one finite padding value) or NaN (a row of -inf biases); the C ABI's
    kv_len = 0 itself writes zero rows. `mesh` marks q/k/v as this rank's Megatron head
    shard (`P('dp', None, 'tp', None)`, attention.py:293-318): heads are
    independent, so the local kernel runs with no communication.
    """
    del mesh  # head-sharded inputs are already local in one-process-per-GPU
    B, Sk = q.shape[0], k.shape[1]
    head_dim = q.shape[-1]
    sm_scale = head_dim ** -0.5 if scale is None else scale
    kv_len = None
    empty = []
    if mask is not None and bias is not None:
        raise NotImplementedError("bias and mask together are not supported")
    if mask is not None:
        kv_len = _key_lengths_from_mask(mask, B, Sk)
    elif bias is not None:
        kv_len = _key_lengths_from_bias(bias, B, Sk)
    if kv_len is not None:
        empty = _fully_masked_rows(bias, mask, kv_len, B, Sk)
    if q.device.type == "cpu":
        # host tensors: transfers pipelined against the kernel (vidax_b200.hostio)
        from .hostio import attention_from_host
        out = attention_from_host(q, k, v, sm_scale, kv_len=kv_len)
    else:
        if kv_len is not None:
            kv_len = kv_len.to(device=q.device)  # the mask / bias may live on the host
        out = flash_attention(q, k, v, sm_scale, kv_len=kv_len)
    if empty:
        _fill_fully_masked(out, k, v, empty, sm_scale)
    return out


def chunk_by_rank(x: torch.Tensor, axis: int, sp_size: int, rank: int) -> torch.Tensor:
    """This rank's contiguous 1/sp_size share of `x` along `axis`
    (attention.py:132-146): rank r owns [r*n, (r+1)*n), n = len // sp_size."""
    size = x.shape[axis] // sp_size
    return x.narrow(axis, rank * size, size)


def attention_flops(batch: int, heads: int, seq_q: int, seq_k: int, head_dim: int) -> float:
    """FLOPs of one attention forward, vidax's convention 4*B*H*Sq*Sk*D."""
    return 4.0 * batch * heads * seq_q * seq_k * head_dim
