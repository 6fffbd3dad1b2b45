"""Time-sharded neighborhood attention, host side on CPU: the halo plan
(which key frames each rank needs and from whom) against a brute-force
restatement of the window-start contract, and the batched send/receive round
on gloo (world 2, 3, 4): every rank must end with exactly the global key
frames its queries read."""
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


@pytest.mark.parametrize("T", [1, 2, 5, 8, 21, 33])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("kt", [1, 2, 3, 5, 11])
def test_key_ranges_cover_exactly_the_windows(T, world, kt):
    from oracle.na3d_ref import window_start
    from vidax_b200.na_parallel import halo_plan, key_ranges, slab_bounds, split_sizes
    sizes = split_sizes(T, world)
    assert sum(sizes) == T and max(sizes) - min(sizes) <= 1
    bounds = slab_bounds(sizes)
    st = window_start(T, kt)
    k = min(kt, T)
    for r, (kv0, kv1) in enumerate(key_ranges(bounds, kt)):
        frames = set()
        for t in range(bounds[r], bounds[r + 1]):
            frames |= set(range(st[t], st[t] + k))
        if frames:
            assert (kv0, kv1) == (min(frames), max(frames) + 1)
            assert frames == set(range(kv0, kv1))  # windows of consecutive frames overlap
        recvs, sends = halo_plan(bounds, kt, r)
        got = set(range(max(kv0, bounds[r]), min(kv1, bounds[r + 1])))
        for s, lo, hi in recvs:
            assert bounds[s] <= lo < hi <= bounds[s + 1]
            got |= set(range(lo, hi))
        assert got == frames
        for s, lo, hi in sends:  # symmetric: s receives exactly this range from r
            assert (r, lo, hi) in halo_plan(bounds, kt, s)[0]


def _worker(rank, world, port, T, kt, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from vidax_b200.na_parallel import exchange_halo, key_ranges, slab_bounds, split_sizes
        bounds = slab_bounds(split_sizes(T, world))
        rng = np.random.default_rng(11)
        kg = torch.from_numpy(rng.standard_normal((2, T, 3, 4, 2, 8)).astype(np.float32))
        vg = torch.from_numpy(rng.standard_normal((2, T, 3, 4, 2, 8)).astype(np.float32))
        mine = [x[:, bounds[rank]:bounds[rank + 1]] for x in (kg, vg)]
        k_ext, v_ext = exchange_halo(mine, bounds, kt, None)
        kv0, kv1 = key_ranges(bounds, kt)[rank]
        assert torch.equal(k_ext, kg[:, kv0:kv1]) and torch.equal(v_ext, vg[:, kv0:kv1])
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,T,kt", [(2, 21, 5), (3, 21, 11), (4, 8, 5), (4, 21, 3), (3, 5, 2)])
def test_exchange_halo_delivers_the_key_frames(world, T, kt):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, kt, errq)) for r in range(world)]
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


def _oracle_slab(q, k_ext, v_ext, kernel_size, *, t_global, q_t0, kv_t0, scale=1.0,
                 round_logits=False):
    """The slab kernel's contract restated with the oracle: the slab's rows
    of the unsharded call, its key frames placed at their global offset
    (frames outside them must never be read: left as NaN)."""
    from oracle.na3d_ref import na3d
    B, T, H, W, NH, HD = q.shape
    shape = (B, t_global, H, W, NH, HD)
    qg = np.zeros(shape, np.float32)
    kg = np.full(shape, np.nan, np.float32)
    vg = np.full(shape, np.nan, np.float32)
    qg[:, q_t0:q_t0 + T] = (q * scale).numpy()
    kg[:, kv_t0:kv_t0 + k_ext.shape[1]] = k_ext.numpy()
    vg[:, kv_t0:kv_t0 + v_ext.shape[1]] = v_ext.numpy()
    rows = [(t, h) for t in range(q_t0, q_t0 + T) for h in range(H)]
    out = na3d(qg, kg, vg, kernel_size, rows=rows)
    return torch.from_numpy(out[:, q_t0:q_t0 + T].copy())


def _sp_worker(rank, world, port, sizes, kernel, pass_t, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import vidax_b200 as vx
        from vidax_b200 import na_parallel
        from oracle.na3d_ref import na3d
        na_parallel.neighborhood_attention_3d_slab = _oracle_slab
        vx.register_axis("sp", None)
        T = sum(sizes)
        rng = np.random.default_rng(13)
        qg, kg, vg = (rng.standard_normal((1, T, 4, 6, 2, 8)).astype(np.float32) for _ in range(3))
        b0 = sum(sizes[:rank])
        mine = [torch.from_numpy(x[:, b0:b0 + sizes[rank]].copy()) for x in (qg, kg, vg)]
        out = na_parallel.neighborhood_attention_3d_sp(
            *mine, kernel, "sp", t_global=T if pass_t else None)
        ref = na3d(qg, kg, vg, kernel)[:, b0:b0 + sizes[rank]]
        assert out.shape == ref.shape
        assert np.isfinite(out.numpy()).all(), "read a key frame outside the exchanged range"
        assert np.allclose(out.numpy(), ref, atol=1e-5), float(np.abs(out.numpy() - ref).max())
        vx.unregister_axis("sp")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("sizes,kernel,pass_t", [
    ((4, 4, 3), (5, 3, 3), True),      # split_sizes(11, 3)
    ((2, 5, 0, 4), (3, 3, 5), False),  # uneven, one rank without frames: sizes all-gathered
    ((1, 1, 1, 1), (5, 3, 3), False),  # slabs thinner than the window
])
def test_time_sharded_na_matches_unsharded(sizes, kernel, pass_t):
    """neighborhood_attention_3d_sp end to end on gloo (the slab kernel
    replaced by the oracle's rows of the global grid): every rank's output
    equals the same frames of the unsharded attention."""
    world = len(sizes)
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_worker, args=(r, world, port, list(sizes), kernel, pass_t,
                                                  errq)) for r in range(world)]
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
