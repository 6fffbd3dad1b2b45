"""The Ulysses layer through the C ABI (`vx_ulysses_attn_fwd`, the pipeline
of sequence_parallel_self_attention, src/vidax/core/attention.py:341-388, in
one C call over an NCCL communicator).

One GPU runs a one-rank communicator: the whole C++ pipeline -- sub-group
packing per head slice, the NCCL exchanges (to itself) on the library's
stream, the attention kernel per slice, the reverse exchange, unpacking --
against the oracle, through a communicator made from a unique id and one
borrowed from a torch process group. With two GPUs a torchrun check compares
it bit for bit with the torch mirror's pipeline and with the oracle.
Tolerance: max-abs 2e-2, mean-abs 2e-3."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare, sdpa, seeded_qkv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,D,valid", [(2, 512, 10, 128, None),   # slices of 2, 4, 4 heads
                                           (1, 777, 5, 64, 700),      # padded keys masked
                                           (1, 300, 1, 128, None)])
def test_capi_layer_one_rank_vs_oracle(B, S, H, D, valid):
    from vidax_b200 import _lib
    from vidax_b200.ulysses_capi import Comm, sequence_parallel_self_attention, unique_id
    q, k, v = seeded_qkv((B, S, H, D), 1200 + S + H)
    comm = Comm.init(0, 1, unique_id())
    try:
        out = sequence_parallel_self_attention(_dev(q), _dev(k), _dev(v), comm, valid_len=valid)
        again = sequence_parallel_self_attention(_dev(q), _dev(k), _dev(v), comm, valid_len=valid)
        torch.cuda.synchronize()
    finally:
        comm.close()
    assert _lib.device_status(clear=True) == 0
    assert torch.equal(out, again)
    if valid:
        ref = sdpa(q, k, v, kv_len=np.full(B, valid))
    else:
        ref = sdpa(q, k, v)
    mx, mean = compare(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.gpu
def test_capi_layer_borrows_a_torch_communicator():
    """A torch process group's NCCL communicator lent to the library gives
    the same bits as a communicator the library made itself."""
    import torch.distributed as dist
    from vidax_b200.ulysses_capi import Comm, sequence_parallel_self_attention, unique_id
    q, k, v = seeded_qkv((1, 640, 6, 128), 1301)
    tq, tk, tv = _dev(q), _dev(k), _dev(v)
    own = Comm.init(0, 1, unique_id())
    ref = sequence_parallel_self_attention(tq, tk, tv, own)
    torch.cuda.synchronize()
    own.close()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        lent = Comm.from_process_group()
        out = sequence_parallel_self_attention(tq, tk, tv, lent)
        torch.cuda.synchronize()
        lent.close()
    finally:
        dist.destroy_process_group()
    assert torch.equal(out, ref)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_capi_layer_two_gpus_matches_torch_mirror():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29619",
           os.path.join(ROOT, "tests", "dist_ulysses_capi_check.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "CAPI ULYSSES OK" in res.stdout
