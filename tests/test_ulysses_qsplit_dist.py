"""Query-split Ulysses (heads % ranks != 0 without padding), host logic on
CPU: the unit plan is balanced and covers every (head, query row) once, and
on gloo (world 2, 3, 4) the two uneven all-to-alls around a float32 CPU
attention reproduce the unsharded attention on every rank."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("heads,world", [(12, 8), (3, 2), (6, 4), (4, 3), (40, 8), (5, 5)])
def test_unit_plan_balanced_and_complete(heads, world):
    from vidax_b200.ulysses_qsplit import unit_plan
    f, plan = unit_plan(heads, world)
    sizes = {len(p) for p in plan}
    assert len(sizes) == 1 and sizes.pop() * world == heads * f
    units = [u for p in plan for u in p]
    assert sorted(units) == [(h, part) for h in range(heads) for part in range(f)]
    assert f * heads % world == 0
    if heads % world == 0:
        assert f == 1  # divisible: plain head groups


def _cpu_attention(q, k, v, scale):
    qh, kh, vh = (t.float().transpose(1, 2) for t in (q, k, v))
    p = torch.softmax(qh @ kh.transpose(-1, -2) * scale, dim=-1)
    return (p @ vh).transpose(1, 2).to(q.dtype)


def _worker(rank, world, port, H, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import vidax_b200 as vx
        from vidax_b200.ulysses_qsplit import sequence_parallel_self_attention_qsplit
        vx.register_axis("sp", None)
        B, S_loc, D = 2, 6, 8
        S = world * S_loc
        g = torch.Generator().manual_seed(3)
        q, k, v = (torch.randn((B, S, H, D), generator=g) for _ in range(3))
        sl = slice(rank * S_loc, (rank + 1) * S_loc)
        out = sequence_parallel_self_attention_qsplit(q[:, sl], k[:, sl], v[:, sl], "sp",
                                                      attn=_cpu_attention)
        ref = _cpu_attention(q, k, v, D ** -0.5)[:, sl]
        assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5), float((out - ref).abs().max())
        vx.unregister_axis("sp")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,H", [(2, 3), (3, 4), (4, 6), (2, 4)])
def test_qsplit_matches_unsharded_attention(world, H):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, H, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
