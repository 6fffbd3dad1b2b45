"""`sequence_parallel_joint_self_attention` (vidax attention.py:391-464) run
as P emulated ranks in one process, against the reference's own per-rank
outputs (tests/golden, written by make_golden.py from vidax's function).

Each rank is a thread; `torch.distributed` inside vidax_b200.ulysses is
replaced by an in-process stand-in whose all_to_all_single /
all_gather_into_tensor exchange the ranks' tensors through shared memory
behind a barrier (with a timeout: a failing rank breaks the barrier instead
of hanging the others). The product's own orchestration -- text slicing,
packing, exchange, joint attention, reverse exchange, text all-gather --
runs unchanged, with the kernels replaced by float32 torch equivalents
(this pins the orchestration; the kernels themselves are pinned by
tests/test_golden_gpu.py and the 2-GPU NCCL test). `_run_joint` also takes
the CUDA device and the real kernels. Tolerance: max-abs 2e-2, mean-abs
2e-3."""
import os
import threading

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


class _Done:
    def wait(self):
        return True


class _RankGroup:
    """The collectives the joint path calls, for P threads of one process."""

    def __init__(self, P: int):
        self.P = P
        self.barrier = threading.Barrier(P, timeout=120)
        self.local = threading.local()
        self.slots = [None] * P

    def get_world_size(self, group=None):
        return self.P

    def get_rank(self, group=None):
        return self.local.rank

    @staticmethod
    def _settle(t):
        if t.is_cuda:
            torch.cuda.synchronize(t.device)

    def _publish(self, t):
        self._settle(t)
        self.slots[self.local.rank] = t
        self.barrier.wait()

    def _done(self, t):
        self._settle(t)
        self.barrier.wait()  # every rank has read the slots

    def all_to_all_single(self, output, input, output_split_sizes=None, input_split_sizes=None,
                          group=None, async_op=False):
        assert output_split_sizes is None and input_split_sizes is None
        self._publish(input)
        r = self.local.rank
        output.view(self.P, -1).copy_(
            torch.stack([self.slots[s].reshape(self.P, -1)[r] for s in range(self.P)]))
        self._done(output)
        return _Done() if async_op else None

    def all_gather_into_tensor(self, output, input, group=None, async_op=False):
        self._publish(input)
        output.view(self.P, -1).copy_(
            torch.stack([self.slots[s].reshape(-1) for s in range(self.P)]))
        self._done(output)
        return _Done() if async_op else None


def _cpu_attention(q, k, v, scale, **_):
    qh, kh, vh = (t.float().transpose(1, 2) for t in (q, k, v))
    p = torch.softmax(qh @ kh.transpose(-1, -2) * scale, dim=-1)
    return (p @ vh).transpose(1, 2).to(q.dtype).contiguous()  # BSHD, as the kernel writes


def _cpu_pack(strided, groups, out=None, sub=None):
    assert sub is None and out is None
    seq, heads, d = strided[0].shape
    hg = -(-heads // groups)
    res = []
    for t in strided:
        p = torch.zeros((groups, seq, hg, d), dtype=t.dtype)
        for g in range(groups):
            h0, h1 = g * hg, min(heads, (g + 1) * hg)
            if h1 > h0:
                p[g, :, :h1 - h0] = t[:, h0:h1]
        res.append(p)
    return res


def _cpu_unpack(packed, strided_out, heads, sub=None):
    assert sub is None
    for p, o in zip(packed, strided_out):
        groups, _, hg, _ = p.shape
        for g in range(groups):
            h0, h1 = g * hg, min(heads, (g + 1) * hg)
            if h1 > h0:
                o[:, h0:h1] = p[g, :, :h1 - h0]


def _run_joint(tag, monkeypatch, device, dtype, cpu_kernels):
    import vidax_b200 as vx
    from vidax_b200 import ulysses
    g = np.load(os.path.join(GOLDEN, "attention_reference.npz"))
    qg, kg, vg = (g[f"{tag}_{n}"] for n in "qkv")
    T = int(g[f"{tag}_text_len"][0])
    ref = g[f"{tag}_o"]
    P = ref.shape[0]
    S_loc = (qg.shape[1] - T) // P
    fake = _RankGroup(P)
    monkeypatch.setattr(ulysses, "dist", fake)
    if cpu_kernels:
        monkeypatch.setattr(ulysses, "flash_attention", _cpu_attention)
        monkeypatch.setattr(ulysses, "pack_heads", _cpu_pack)
        monkeypatch.setattr(ulysses, "unpack_heads", _cpu_unpack)
    vx.register_axis("sp_emulated", None)
    results, errors = [None] * P, []

    def rank(r):
        try:
            fake.local.rank = r
            loc = [torch.from_numpy(np.ascontiguousarray(np.concatenate(
                [x[:, :T], x[:, T + r * S_loc:T + (r + 1) * S_loc]], axis=1))).to(device, dtype)
                for x in (qg, kg, vg)]
            o = vx.sequence_parallel_joint_self_attention(*loc, T, "sp_emulated")
            results[r] = o.float().cpu().numpy()
        except BaseException as e:  # noqa: BLE001 -- reported below
            errors.append(f"rank {r}: {type(e).__name__}: {e}")
            fake.barrier.abort()

    threads = [threading.Thread(target=rank, args=(r,)) for r in range(P)]
    try:
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=300)
    finally:
        vx.unregister_axis("sp_emulated")
    assert not errors, errors
    for r in range(P):
        mx, mean = compare(results[r], ref[r])
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (tag, r, mx, mean)


@pytest.mark.parametrize("tag", ["joint2", "joint4", "joint2d128"])
def test_joint_orchestration_matches_reference_code(tag, monkeypatch):
    """CPU: the product's joint Ulysses orchestration with float32 torch
    attention / packing in place of the kernels."""
    _run_joint(tag, monkeypatch, "cpu", torch.float32, cpu_kernels=True)
