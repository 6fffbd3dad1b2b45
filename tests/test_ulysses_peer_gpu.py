"""The Ulysses exchange done by the slab kernels over peer memory
(vx_ulysses_pack_peers / vx_ulysses_unpack_peers, vx_peer_barrier, vx_ipc_*;
the all_to_all pair of sequence_parallel_self_attention,
src/vidax/core/attention.py:379-388).

On one GPU, P ranks are emulated by P workspaces on the device: the pack of
every rank stores into the other ranks' receive slabs, each rank's
attention runs on its own slab, and the unpack of every rank loads from the
other ranks' output slabs -- the same addressing as across GPUs, ordered
here by the single stream. The result must equal the unsharded kernel bit
for bit and the oracle within max-abs 2e-2 / mean-abs 2e-3. The barrier is
tested with flags that another rank would set (set here by the test) and
with a flag that nothing sets (its bounded wait expires and reports).
With two GPUs a torchrun worker compares the layer with the NCCL path."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare, sdpa, seeded_qkv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


@pytest.mark.gpu
@pytest.mark.parametrize("S,H,D,P,ctas", [(1024, 8, 128, 2, 0), (1536, 12, 128, 8, 6),
                                          (960, 10, 64, 4, 0), (512, 3, 128, 2, 1)])
def test_emulated_ranks_peer_exchange(S, H, D, P, ctas):
    from vidax_b200 import _lib
    from vidax_b200.attention import flash_attention
    from vidax_b200.ulysses import _pieces
    from vidax_b200.ulysses_peer import slab_peers
    q, k, v = seeded_qkv((1, S, H, D), 1800 + S + H + P)
    tq, tk, tv = _dev(q), _dev(k), _dev(v)
    S_loc, Hg = S // P, -(-H // P)
    sizes = _pieces(Hg)
    offs = [sum(sizes[:j]) for j in range(len(sizes))]
    slab = P * S_loc * Hg * D
    ws = [torch.full((4 * slab,), float("nan"), device="cuda").bfloat16() for _ in range(P)]

    def remote(g, s, off, hs, r):  # rank r's chunk of slice (off, hs) in rank g's slab s
        return ws[g].data_ptr() + 2 * (s * slab + P * S_loc * off * D + r * S_loc * hs * D)

    def local(r, s, off, hs):
        start = s * slab + P * S_loc * off * D
        return ws[r][start:start + P * S_loc * hs * D].view(1, P * S_loc, hs, D)

    stream = torch.cuda.current_stream()
    mine = [[t[0, r * S_loc:(r + 1) * S_loc] for t in (tq, tk, tv)] for r in range(P)]
    outs = [torch.full((S_loc, H, D), float("nan"), device="cuda").bfloat16() for _ in range(P)]
    for r in range(P):
        for off, hs in zip(offs, sizes):
            peers = [[remote(g, t, off, hs, r) for g in range(P)] for t in range(3)]
            slab_peers(True, mine[r], peers, H, P, (hs, Hg, off, hs), stream, ctas)
    for r in range(P):
        for off, hs in zip(offs, sizes):
            flash_attention(local(r, 0, off, hs), local(r, 1, off, hs), local(r, 2, off, hs),
                            D ** -0.5, out=local(r, 3, off, hs), dynamic_schedule=True)
    for r in range(P):
        for off, hs in zip(offs, sizes):
            peers = [[remote(g, 3, off, hs, r) for g in range(P)]]
            slab_peers(False, [outs[r]], peers, H, P, (hs, Hg, off, hs), stream, ctas)
    full = torch.cat(outs, dim=0).unsqueeze(0)
    direct = flash_attention(tq, tk, tv, D ** -0.5)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    assert torch.equal(full, direct)
    mx, mean = compare(full.float().cpu().numpy(), sdpa(q, k, v))
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


@pytest.mark.gpu
def test_peer_barrier_passes_once_every_rank_arrived():
    from vidax_b200 import _lib
    from vidax_b200.ulysses_peer import peer_barrier
    mine = torch.zeros(8, dtype=torch.int32, device="cuda")
    theirs = torch.zeros(8, dtype=torch.int32, device="cuda")
    mine[1] = 5            # rank 1 already arrived (at a later epoch: epochs only grow)
    peer_barrier([mine.data_ptr(), theirs.data_ptr()], 0, 3, torch.cuda.current_stream(),
                 timeout_ns=1_000_000_000)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    assert mine[0].item() == 3 and theirs[0].item() == 3   # rank 0's arrival in both arrays


@pytest.mark.gpu
def test_peer_barrier_wait_expires_and_reports():
    """A rank that never arrives: the bounded wait gives up and sets the
    barrier bit of the status word; the context stays usable."""
    from vidax_b200 import _lib
    from vidax_b200.ulysses_peer import peer_barrier
    _lib.device_status(clear=True)
    mine = torch.zeros(8, dtype=torch.int32, device="cuda")
    theirs = torch.zeros(8, dtype=torch.int32, device="cuda")
    peer_barrier([mine.data_ptr(), theirs.data_ptr()], 0, 1, torch.cuda.current_stream(),
                 timeout_ns=2_000_000)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & 32
    x = torch.ones(4, device="cuda")
    assert (x * 2).sum().item() == 8.0


@pytest.mark.gpu
def test_ipc_handle_offsets():
    from vidax_b200.ulysses_peer import ipc_handle
    t = torch.empty(1 << 22, dtype=torch.uint8, device="cuda")
    h0, o0 = ipc_handle(t.data_ptr())
    h1, o1 = ipc_handle(t[4096:].data_ptr())
    assert h0 == h1 and len(h0) == 64 and o1 - o0 == 4096


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_peer_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29631",
           os.path.join(ROOT, "tests", "dist_ulysses_peer_check.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "PEER OK" in res.stdout
