"""Worker for test_ulysses_two_gpus_nccl (run under torch.distributed.run):
each rank feeds its chunk_by_rank share of a seeded global sequence through
sequence_parallel_self_attention over NCCL; rank 0 gathers and compares with
the oracle."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import vidax_b200 as vx  # noqa: E402
from oracle.attention_ref import compare, sdpa, seeded_qkv  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    vx.register_axis("sp", None)
    ok = True
    for (B, S, H) in [(1, 1024, 8), (2, 768, 6), (1, 512, 3)]:
        q, k, v = seeded_qkv((B, S, H, 128), 900 + S + H)
        sl = S // world
        mine = [torch.from_numpy(np.ascontiguousarray(x[:, rank * sl:(rank + 1) * sl])).cuda().bfloat16()
                for x in (q, k, v)]
        out = vx.sequence_parallel_self_attention(*mine, "sp")
        # host-buffer form: same slices and kernels, transfers as the layout
        host = vx.sequence_parallel_self_attention_from_host(
            *[t.cpu().pin_memory() for t in mine], "sp")
        torch.cuda.synchronize()
        same_host = torch.equal(host, out.cpu())
        ok = ok and same_host
        if not same_host:
            print(f"rank {rank}: host path differs for B={B} S={S} H={H}", flush=True)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            got = torch.cat(gathered, dim=1).float().cpu().numpy()
            mx, mean = compare(got, sdpa(q, k, v))
            print(f"B={B} S={S} H={H}: max {mx:.3g} mean {mean:.3g}", flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3
    # joint [text; visual] layout (CogVideoX): text replicated, visual chunked
    for (B, T_len, S, H) in [(1, 226, 1024, 8), (2, 77, 512, 6)]:
        seed = 950 + T_len + S
        q, k, v = seeded_qkv((B, T_len + S, H, 128), seed)
        sl = S // world
        def local(x):
            return np.concatenate([x[:, :T_len], x[:, T_len + rank * sl:T_len + (rank + 1) * sl]], axis=1)
        mine = [torch.from_numpy(np.ascontiguousarray(local(x))).cuda().bfloat16() for x in (q, k, v)]
        out = vx.sequence_parallel_joint_self_attention(*mine, T_len, "sp")
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            ref = sdpa(q, k, v)
            txt = gathered[0][:, :T_len].float().cpu().numpy()
            vis = torch.cat([g[:, T_len:] for g in gathered], dim=1).float().cpu().numpy()
            got = np.concatenate([txt, vis], axis=1)
            mx, mean = compare(got, ref)
            same_txt = all(torch.equal(gathered[0][:, :T_len], g[:, :T_len]) for g in gathered)
            print(f"joint B={B} T={T_len} S={S} H={H}: max {mx:.3g} mean {mean:.3g} txt-replicated {same_txt}", flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3 and same_txt
    # Wan attend: fused RMSNorm + RoPE + pack, then the Ulysses pipeline; each
    # rank holds its chunk of the projections and of the RoPE tables
    for (t, h, w, H) in [(4, 8, 16, 8), (2, 6, 16, 5)]:
        S, D = t * h * w, 128
        sl = S // world
        q, k, v = seeded_qkv((1, S, H * D), 970 + S + H, head_scale_range=None)
        rng = np.random.Generator(np.random.PCG64(S + H))
        wq, wk = ((1.0 + 0.25 * rng.standard_normal(H * D)).astype(np.float32) for _ in range(2))
        cos, sin = vx.rope3d_freqs(t, h, w, D)
        full = [torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16() for x in (q, k, v)]
        mine = [x[:, rank * sl:(rank + 1) * sl] for x in full]
        rope_mine = (cos[rank * sl:(rank + 1) * sl], sin[rank * sl:(rank + 1) * sl])
        out = vx.attend(*mine, H, norm_q=torch.from_numpy(wq), norm_k=torch.from_numpy(wk),
                        rope=rope_mine, sp_axis_name="sp")
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            got = torch.cat(gathered, dim=1)
            single = vx.attend(*full, H, norm_q=torch.from_numpy(wq), norm_k=torch.from_numpy(wk),
                               rope=(cos, sin))
            same = torch.equal(got, single)
            from oracle.rope_norm_ref import norm_rope
            qr = norm_rope(q, wq, cos.numpy(), sin.numpy(), H)
            kr = norm_rope(k, wk, cos.numpy(), sin.numpy(), H)
            ref = sdpa(qr, kr, v.reshape(1, S, H, D))
            mx, mean = compare(got.float().cpu().numpy().reshape(1, S, H, D), ref)
            print(f"attend S={S} H={H}: max {mx:.3g} mean {mean:.3g} equals-single-gpu {same}",
                  flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3 and same
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)  # every rank's checks count
    vx.unregister_axis("sp")
    dist.destroy_process_group()
    if rank == 0:
        print("ULYSSES OK" if flag.item() else "ULYSSES FAIL", flush=True)
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
