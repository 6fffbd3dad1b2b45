"""Worker for test_ulysses_peer_two_gpus (run under torch.distributed.run):
each rank feeds its chunk_by_rank share of a seeded global sequence through
the peer-memory Ulysses layer and through the NCCL one; the two must agree
bit for bit (same kernels on the same data), and rank 0 compares the
gathered result with the oracle. Covers padded heads (H % P != 0), B = 2,
a masked padded sequence and repeated calls on one workspace."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import vidax_b200 as vx  # noqa: E402
from vidax_b200 import _lib  # noqa: E402
from vidax_b200.ulysses_peer import release_workspaces, sequence_parallel_self_attention_peer  # noqa: E402
from oracle.attention_ref import compare, sdpa, seeded_qkv  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    vx.register_axis("sp", None)
    ok = True
    cases = [(1, 1024, 8, 128, None), (2, 768, 6, 128, None), (1, 512, 3, 128, None),
             (1, 1024, 8, 64, 1000), (1, 1024, 8, 128, None)]   # last: the first shape again
    for (B, S, H, D, valid) in cases:
        q, k, v = seeded_qkv((B, S, H, D), 1700 + S + H + D)
        sl = S // world
        mine = [torch.from_numpy(np.ascontiguousarray(x[:, rank * sl:(rank + 1) * sl])).cuda().bfloat16()
                for x in (q, k, v)]
        for rep in range(2):
            out = sequence_parallel_self_attention_peer(*mine, valid_len=valid)
            ref = vx.sequence_parallel_self_attention(*mine, "sp", valid_len=valid)
            torch.cuda.synchronize()
            same = torch.equal(out, ref)
            ok = ok and same
            if not same:
                print(f"rank {rank}: peer path differs from NCCL for B={B} S={S} H={H} D={D} "
                      f"(rep {rep}): max {(out.float() - ref.float()).abs().max().item():.3g}",
                      flush=True)
        status = _lib.device_status(clear=True)
        ok = ok and status == 0
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            got = torch.cat(gathered, dim=1).float().cpu().numpy()
            ref_np = sdpa(q, k, v, kv_len=np.full(B, valid)) if valid else sdpa(q, k, v)
            mx, mean = compare(got, ref_np)
            print(f"B={B} S={S} H={H} D={D} valid={valid}: max {mx:.3g} mean {mean:.3g} "
                  f"status {status}", flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3
    # Wan's attend (fused norm + RoPE, then the layer) with the axis in peer
    # mode against the same call in NCCL mode: B = 2, 12 heads (padded when
    # they do not divide the ranks), this rank's tokens' RoPE rows
    from vidax_b200.prologue import rope3d_freqs
    B, T, Hh, W, heads, D = 2, 4, 8, 16, 12, 128
    L = T * Hh * W
    sl = L // world
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1750)
    x = [torch.randn((B, L, heads * D), generator=gen, device="cuda").bfloat16() for _ in range(3)]
    nq, nk = (1.0 + 0.1 * torch.randn(heads * D, generator=gen, device="cuda") for _ in range(2))
    cos, sin = rope3d_freqs(T, Hh, W, D, device="cuda")
    mine = [t[:, rank * sl:(rank + 1) * sl].contiguous() for t in x]
    rope = (cos[rank * sl:(rank + 1) * sl].contiguous(), sin[rank * sl:(rank + 1) * sl].contiguous())
    outs = {}
    for mode in ("peer", "nccl"):
        vx.register_axis("sp", None, exchange=mode)
        outs[mode] = vx.attend(*mine, heads, norm_q=nq, norm_k=nk, rope=rope, sp_axis_name="sp")
    torch.cuda.synchronize()
    same = torch.equal(outs["peer"], outs["nccl"])
    ok = ok and same and _lib.device_status(clear=True) == 0
    print(f"rank {rank}: attend peer == nccl: {same}", flush=True)
    # joint [text; visual] layout (CogVideoX) in peer mode against NCCL mode
    for (B, T_len, S, H) in [(1, 226, 1024, 8), (2, 77, 512, 6), (1, 64, 512, 3)]:
        q, k, v = seeded_qkv((B, T_len + S, H, 128), 1950 + T_len + S + H)
        sl = S // world

        def rank_rows(x):
            return np.concatenate([x[:, :T_len], x[:, T_len + rank * sl:T_len + (rank + 1) * sl]],
                                  axis=1)
        mine = [torch.from_numpy(np.ascontiguousarray(rank_rows(x))).cuda().bfloat16()
                for x in (q, k, v)]
        res = {}
        for mode in ("peer", "nccl"):
            vx.register_axis("sp", None, exchange=mode)
            res[mode] = vx.sequence_parallel_joint_self_attention(*mine, T_len, "sp")
        torch.cuda.synchronize()
        same = torch.equal(res["peer"], res["nccl"])
        ok = ok and same and _lib.device_status(clear=True) == 0
        print(f"rank {rank}: joint peer == nccl for B={B} T={T_len} S={S} H={H}: {same}", flush=True)
    # host-buffer form in peer mode: uploads straight into the peers' receive
    # slabs, downloads straight from their output slabs; equal to the device
    # form bit for bit (padded heads included)
    vx.register_axis("sp", None, exchange="peer")
    for (B, S, H) in [(2, 768, 6), (1, 512, 3), (1, 1024, 8)]:
        q, k, v = seeded_qkv((B, S, H, 128), 1900 + S + H)
        sl = S // world
        mine = [torch.from_numpy(np.ascontiguousarray(x[:, rank * sl:(rank + 1) * sl])).cuda().bfloat16()
                for x in (q, k, v)]
        dev_out = vx.sequence_parallel_self_attention(*mine, "sp")
        host = vx.sequence_parallel_self_attention_from_host(
            *[t.cpu().pin_memory() for t in mine], "sp")
        torch.cuda.synchronize()
        same = torch.equal(host, dev_out.cpu())
        ok = ok and same and _lib.device_status(clear=True) == 0
        print(f"rank {rank}: host path (peer) == device path for B={B} S={S} H={H}: {same}",
              flush=True)
    vx.register_axis("sp", None)
    # a rank that never arrives: rank 0's barrier wait is bounded (50 ms
    # here), expires, sets the status bit and returns; rank 1 stays alive
    # and mapped meanwhile, then both close the workspace together
    from vidax_b200.ulysses_peer import CH_END, MAX_GROUPS, PeerWorkspace, peer_barrier
    ws = PeerWorkspace(dist.distributed_c10d._get_default_group(), 64, 2 * world, 64,
                       torch.device("cuda", local))
    _lib.device_status(clear=True)
    if rank == 0:
        flags = [b + ws.flag_off + CH_END * MAX_GROUPS * 4 for b in ws.base]
        peer_barrier(flags, 0, 1, torch.cuda.current_stream(), timeout_ns=50_000_000)
        torch.cuda.synchronize()
        expired = bool(_lib.device_status(clear=True) & 32)
        ok = ok and expired
        print(f"rank 0: barrier without rank 1 expired and reported: {expired}", flush=True)
    dist.barrier()
    ws.close()
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    release_workspaces()
    dist.destroy_process_group()
    if rank == 0:
        print("PEER OK" if flag.item() == 1 else "PEER FAILED", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
