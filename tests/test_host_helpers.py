"""Host-side helpers that shape the device work, checked on CPU: the
pipelined Ulysses slice sizes, the send-slab views of the fused pre-step,
and the head groups of the host-buffer attention path."""
import pytest
import torch


@pytest.mark.parametrize("hg", [1, 2, 3, 5, 6, 10, 20, 40])
def test_ulysses_pieces_cover_the_head_group(hg):
    from vidax_b200.ulysses import _pieces
    sizes = _pieces(hg)
    assert sum(sizes) == hg and all(s >= 1 for s in sizes) and len(sizes) <= 3
    assert sizes[0] == min(sizes)  # the exposed first exchange is the smallest


def test_slice_views_tile_the_packed_buffer():
    from vidax_b200.prologue import slice_views
    P, S, D, sizes = 4, 5, 8, [1, 2, 2]
    buf = torch.arange(P * S * sum(sizes) * D)
    views = slice_views(buf, P, S, D, sizes)
    assert [tuple(v.shape) for v in views] == [(P, S, n, D) for n in sizes]
    flat = torch.cat([v.reshape(-1) for v in views])
    assert torch.equal(flat, buf)  # back to back, no gaps or overlaps


@pytest.mark.parametrize("B,H,Hkv", [(1, 40, 40), (1, 12, 12), (2, 8, 4), (1, 1, 1), (1, 24, 8)])
def test_host_attention_head_groups(B, H, Hkv, monkeypatch):
    """attention_from_host visits every head exactly once, in order, in
    groups of whole KV heads (captured by replacing the copy and the kernel)."""
    import vidax_b200.hostio as hostio
    import vidax_b200.attention as attention
    seen = []
    monkeypatch.setattr(hostio, "copy_heads", lambda dst, src, h0, h1, stream: None)
    monkeypatch.setattr(attention, "flash_attention",
                        lambda q, k, v, scale, **kw: seen.append((q.shape[2], k.shape[2])))

    class FakeStream:
        def wait_stream(self, s):
            pass

        def wait_event(self, e):
            pass

    class FakeEvent:
        def record(self, s=None):
            pass

    monkeypatch.setattr(hostio, "_side_streams", lambda device: (FakeStream(), FakeStream()))
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: FakeStream())
    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.Tensor, "record_stream", lambda self, s: None)
    q = torch.zeros((B, 16, H, 8), dtype=torch.bfloat16)
    k = torch.zeros((B, 16, Hkv, 8), dtype=torch.bfloat16)
    hostio.attention_from_host(q, k, k.clone(), 0.1, out=torch.empty_like(q), device="cpu")
    assert sum(h for h, _ in seen) == H and sum(g for _, g in seen) == Hkv
    assert all(h == g * (H // Hkv) for h, g in seen)


@pytest.mark.parametrize("hkv,cap", [(40, 8), (20, 8), (12, 8), (5, 8), (2, 8), (1, 8), (8, 2), (7, 1)])
def test_host_group_sizes_ramp(hkv, cap):
    """Host-buffer pipeline groups: cover every head once, start and end with
    one head (the exposed upload and download), double up to the cap."""
    from vidax_b200.hostio import group_sizes
    sizes = group_sizes(hkv, cap)
    assert sum(sizes) == hkv and all(1 <= s <= cap for s in sizes)
    assert sizes[0] == 1 and sizes[-1] == 1
    body = sizes[:-1] if hkv > 1 else sizes
    for a, b in zip(body, body[1:]):
        assert b <= 2 * a  # each upload fits under the kernels before it


def test_key_lengths_from_mask_and_bias():
    """The key-padding forms dot_product_attention accepts become per-batch
    valid lengths; anything that is not a valid-prefix key mask is refused."""
    from vidax_b200.attention import _key_lengths_from_bias, _key_lengths_from_mask
    B, Sk = 3, 7
    lens = torch.tensor([7, 3, 0])
    valid = torch.arange(Sk)[None, :] < lens[:, None]
    for m in (valid[:, None, None, :], valid[:, None, None, :].int()):
        assert torch.equal(_key_lengths_from_mask(m, B, Sk), lens.int())
    # one row broadcast over the batch
    assert torch.equal(_key_lengths_from_mask(valid[1][None, None, None, :], B, Sk),
                       torch.tensor([3, 3, 3], dtype=torch.int32))
    bias = torch.zeros(B, 1, 1, Sk).masked_fill(~valid[:, None, None, :], float("-inf"))
    assert torch.equal(_key_lengths_from_bias(bias, B, Sk), lens.int())
    big_neg = torch.zeros(B, 1, 1, Sk).masked_fill(~valid[:, None, None, :], -1e30)
    assert torch.equal(_key_lengths_from_bias(big_neg, B, Sk), lens.int())
    holes = valid.clone()
    holes[0, 2] = False  # a hole inside the prefix
    with pytest.raises(NotImplementedError):
        _key_lengths_from_mask(holes[:, None, None, :], B, Sk)
    with pytest.raises(NotImplementedError):  # per-query (dense) mask
        _key_lengths_from_mask(torch.ones(B, 1, 5, Sk, dtype=torch.bool), B, Sk)
    with pytest.raises(NotImplementedError):  # dense additive bias (T5-style)
        _key_lengths_from_bias(torch.zeros(B, 2, 5, Sk), B, Sk)
    with pytest.raises(NotImplementedError):  # values other than 0 / -inf
        _key_lengths_from_bias(torch.full((B, 1, 1, Sk), -3.0), B, Sk)


def test_host_paths_reject_a_wrong_out_buffer():
    """The host-buffer paths copy device rows straight into `out`: a buffer of
    another shape, dtype or row layout is refused before any device work."""
    from vidax_b200.hostio import attention_from_host
    from vidax_b200.ulysses import sequence_parallel_self_attention_from_host
    q = torch.zeros(1, 8, 2, 64, dtype=torch.bfloat16)
    dev = torch.device("cuda", 0)  # never reached: validation comes first
    for bad, err in ((torch.zeros(1, 4, 2, 64, dtype=torch.bfloat16), ValueError),
                     (torch.zeros(1, 8, 2, 64), NotImplementedError),
                     (torch.zeros(1, 8, 64, 2, dtype=torch.bfloat16).transpose(2, 3), ValueError)):
        with pytest.raises(err):
            attention_from_host(q, q, q, 0.125, out=bad, device=dev)
        with pytest.raises(err):
            sequence_parallel_self_attention_from_host(q, q, q, "sp", out=bad, device=dev)


def test_slab_calls_check_buffers_before_the_kernel():
    """pack / unpack refuse packed buffers of the wrong size (the kernel would
    write past them) and views of the wrong shape, before any launch."""
    from vidax_b200.ulysses import pack_heads, unpack_heads
    x = torch.zeros(6, 10, 64, dtype=torch.bfloat16)     # (S_loc, H, D)
    with pytest.raises(ValueError, match="packed buffer"):
        pack_heads([x], 4, out=[torch.zeros(4, 6, 2, 64, dtype=torch.bfloat16)])  # Hg = 3
    with pytest.raises(ValueError, match="packed buffer"):
        unpack_heads([torch.zeros(4, 6, 3, 64, dtype=torch.bfloat16)], [x], 10, sub=(2, 3, 0, 2))
    with pytest.raises(ValueError, match="view"):
        unpack_heads([torch.zeros(4, 6, 3, 64, dtype=torch.bfloat16)], [x], 12)
    with pytest.raises(ValueError, match="CUDA"):        # right sizes, host memory
        pack_heads([x], 4, out=[torch.zeros(4, 6, 3, 64, dtype=torch.bfloat16)])


def test_bench_na_cpu_line():
    """bench.py's CPU leg for cfg4: the oracle's scan timed on row steps, the
    JSON fields the bench line carries."""
    import json
    import bench
    sec = {"cfg4": {"ms": 1.2}}
    bench.add_na_cpu_line(sec, 0.5)
    line = sec["cfg4_cpu_scan"]
    assert line["rows"] >= 1 and line["est_full_ms"] > 0 and line["cores"] >= 1
    assert line["est_full_over_kernel"] == round(line["est_full_ms"] / 1.2)
    json.dumps(sec)


def test_bench_host_cpu_record():
    import bench
    h = bench.host_cpu()
    assert set(h) == {"cpu_model", "logical_cpus"} and h["logical_cpus"] >= 1


def test_fully_masked_rows_modes():
    """Which batch items have no visible key, and what the reference gives
    them: mask form -> mean of v, -inf bias -> NaN, one finite padding value
    -> mean; unequal finite padding values are refused."""
    import pytest
    import torch
    from vidax_b200.attention import _fully_masked_rows, _key_lengths_from_bias, _key_lengths_from_mask
    B, Sk = 3, 5
    valid = torch.tensor([[1, 1, 0, 0, 0], [0, 0, 0, 0, 0], [1, 1, 1, 1, 1]], dtype=torch.bool)
    lens = _key_lengths_from_mask(valid[:, None, None, :], B, Sk)
    assert lens.tolist() == [2, 0, 5]
    assert _fully_masked_rows(None, valid[:, None, None, :], lens, B, Sk) == [(1, "mean")]
    bias = torch.where(valid, 0.0, float("-inf"))[:, None, None, :]
    lens = _key_lengths_from_bias(bias, B, Sk)
    assert _fully_masked_rows(bias, None, lens, B, Sk) == [(1, "nan")]
    bias2 = torch.where(valid, 0.0, -1e9)[:, None, None, :]
    assert _fully_masked_rows(bias2, None, _key_lengths_from_bias(bias2, B, Sk), B, Sk) == [(1, "mean")]
    bias3 = bias2.clone()
    bias3[1, 0, 0, 0] = -2e9
    with pytest.raises(NotImplementedError):
        _fully_masked_rows(bias3, None, _key_lengths_from_bias(bias3, B, Sk), B, Sk)


def _parity_worker(rank, world, port, errq):
    import os
    import torch
    import torch.distributed as dist
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import bench
        g = torch.Generator().manual_seed(5)
        S_loc, H, D = 40, 3, 16
        q, k, v = (torch.randn((world, S_loc, H, D), generator=g).bfloat16() for _ in range(3))
        # the global sequence is the ranks' chunks in rank order
        qg, kg, vg = (t.reshape(1, world * S_loc, H, D) for t in (q, k, v))
        p = torch.softmax(torch.einsum("bqhd,bkhd->bhqk", qg.float(), kg.float()) * D ** -0.5, -1)
        o = torch.einsum("bhqk,bkhd->bqhd", p, vg.float()).bfloat16()
        sl = slice(rank * S_loc, (rank + 1) * S_loc)
        rec = bench.parity_sample(o[:, sl], qg[:, sl], kg[:, sl], vg[:, sl], world,
                                  torch.device("cpu"), rows_per_rank=8)
        assert rec["pass"] and rec["max_abs"] < 2e-2, rec
        # a wrong output on one rank fails every rank's verdict (max over ranks)
        bad = o[:, sl].clone()
        if rank == 1:
            bad += 0.5
        rec = bench.parity_sample(bad, qg[:, sl], kg[:, sl], vg[:, sl], world,
                                  torch.device("cpu"), rows_per_rank=8)
        assert not rec["pass"], rec
        dist.destroy_process_group()
    except BaseException as e:  # noqa: BLE001
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")


def test_bench_parity_sample_over_ranks():
    """bench.py's parity self-check at N > 1 (gloo on CPU): each rank checks
    its rows against the ranks' gathered keys / values, the verdict is the
    max over ranks."""
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    procs = [ctx.Process(target=_parity_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs)


def test_axis_exchange_mode():
    """register_axis records how the Ulysses layers on the axis exchange
    (NCCL all-to-alls by default, or the peer-memory slab kernels)."""
    import pytest
    from vidax_b200 import ulysses
    ulysses.register_axis("xchg_test", None)
    assert ulysses._exchange("xchg_test") == "nccl"
    ulysses.register_axis("xchg_test", None, exchange="peer")
    assert ulysses._exchange("xchg_test") == "peer"
    with pytest.raises(ValueError):
        ulysses.register_axis("xchg_test", None, exchange="mpi")
    ulysses.unregister_axis("xchg_test")
    assert ulysses._exchange("xchg_test") == "nccl"


def test_peer_workspace_layout():
    """The peer exchange's slab layout: slice j of a slab is a contiguous
    block of (prefix + P * S_loc) rows x hs heads; in it, rank r's chunk
    starts at row prefix + r * S_loc; the chunks of all ranks and slices
    tile the slab exactly once (so no two ranks' stores overlap)."""
    from vidax_b200.ulysses import _pieces
    from vidax_b200.ulysses_peer import PeerWorkspace
    for P, S_loc, H, D, prefix in [(2, 96, 5, 64, 0), (8, 40, 12, 128, 0), (4, 24, 6, 128, 17)]:
        Hg = -(-H // P)
        owners = {}
        for r in range(P):
            ws = object.__new__(PeerWorkspace)
            ws.P, ws.rank, ws.seq_local, ws.heads, ws.head_dim = P, r, S_loc, H, D
            ws.prefix, ws.Hg = prefix, Hg
            ws.slab_bytes = ((prefix + P * S_loc) * Hg * D * 2 + 255) // 256 * 256
            ws.base = [g * 10 ** 9 for g in range(P)]
            sizes = _pieces(Hg)
            offs = [sum(sizes[:j]) for j in range(len(sizes))]
            for hs, off in zip(sizes, offs):
                for g in range(P):
                    addr = ws.remote(g, 1, off, hs)
                    rel = addr - ws.base[g] - ws.slab_bytes
                    assert rel % (hs * D * 2) == 0
                    start = rel // 2
                    for e in range(start, start + S_loc * hs * D, D):
                        assert (g, e) not in owners, (P, r, g, e)
                        owners[(g, e)] = r
                    assert ws.remote_prefix(g, 1, off) == ws.base[g] + ws.slab_bytes + 2 * (
                        prefix + P * S_loc) * off * D
        # every rank-g slab row-head vector outside the prefix has exactly one writer
        for g in range(P):
            mine = sorted(e for (gg, e) in owners if gg == g)
            assert len(mine) == P * S_loc * Hg, (len(mine), P * S_loc * Hg)
