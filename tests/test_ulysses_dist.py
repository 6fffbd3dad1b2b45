"""Multi-process host logic of the Ulysses path on CPU (gloo, world size 2
and 4): axis registration, axis_index / axis_size, and the equal-split
exchange that carries the tokens->heads and heads->tokens reshards. The
packed send layout comes from the oracle's restatement of the tiled
all_to_all (the CUDA pack kernel is covered by the GPU tests); the result
must equal jax.lax.all_to_all(tiled=True) semantics on every rank."""
import os
import socket
import sys

import numpy as np
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


def _pack_ref(x, P):
    """(S_loc, H, D) -> (P, S_loc, Hg, D): head group g of every token, zero
    heads past H (the layout vx_ulysses_pack produces)."""
    S_loc, H, D = x.shape
    Hg = -(-H // P)
    out = np.zeros((P, S_loc, Hg, D), x.dtype)
    for g in range(P):
        h0, h1 = g * Hg, min(H, (g + 1) * Hg)
        if h1 > h0:
            out[g, :, : h1 - h0] = x[:, h0:h1]
    return out


def _worker(rank, world, port, H, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import vidax_b200 as vx
        from vidax_b200.ulysses import exchange
        from oracle.ulysses_ref import all_to_all_tiled, chunk_by_rank
        vx.register_axis("sp", None)
        assert vx.axis_size("sp") == world and vx.axis_index("sp") == rank
        B, S, D = 1, 8 * world, 4
        rng = np.random.default_rng(5)
        xg = rng.standard_normal((B, S, H, D)).astype(np.float32)
        locs = [chunk_by_rank(xg, 1, world, r)[0] for r in range(world)]     # (S_loc, H, D)
        Hg = -(-H // world)
        # tokens -> heads
        recv = exchange(torch.from_numpy(_pack_ref(locs[rank], world)), None).numpy()
        pad = [np.pad(x, ((0, 0), (0, Hg * world - H), (0, 0))) for x in locs]
        expect = all_to_all_tiled([p[None] for p in pad], 2, 1)[rank][0]      # (S, Hg, D)
        assert np.array_equal(recv.reshape(S, Hg, D), expect)
        # heads -> tokens: send this rank's (S, Hg, D) back as (P, S_loc, Hg, D)
        back = exchange(torch.from_numpy(recv.copy()), None).numpy()          # (P_src, S_loc, Hg, D)
        mine = np.concatenate([back[g] for g in range(world)], axis=1)[:, :H]  # (S_loc, H, D)
        assert np.array_equal(mine, locs[rank])
        vx.unregister_axis("sp")
        try:
            vx.axis_size("sp")
            raise AssertionError("unbound axis accepted")
        except NameError:
            pass
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,H", [(2, 4), (2, 3), (4, 8), (4, 6)])
def test_exchange_matches_tiled_all_to_all(world, H):
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


def _a2a_worker(rank, world, port, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from bench import measure_all_to_all
        r = measure_all_to_all(1 << 20 | 3, 2, torch.device("cpu"), torch.bfloat16)
        n = (1 << 20 | 3) - (1 << 20 | 3) % world
        assert r["buffer_bytes_per_gpu"] == 2 * n
        assert r["bytes_per_gpu_per_direction"] == (world - 1) / world * 2 * n
        assert r["ms"] > 0 and r["gbs_per_direction"] > 0
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_bench_all_to_all_measurement_on_gloo():
    """bench.py's NVLink figure for N > 1: the same collective sequence on
    every rank, byte accounting of an equal-split exchange."""
    world = 2
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_a2a_worker, args=(r, world, port, errq)) for r in range(world)]
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
