"""Worker for test_ulysses_qsplit_two_gpus_nccl (run under
torch.distributed.run): the query-split Ulysses path over NCCL against the
oracle of the global sequence, with heads % ranks != 0. With `--time`, also
times it against the padded-head path on a larger shape (rank 0 prints)."""
import datetime
import json
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
    from vidax_b200.ulysses_qsplit import sequence_parallel_self_attention_qsplit
    ok = True
    for (B, S, H) in [(1, 1024, 3), (2, 768, 5), (1, 512, 7)]:
        q, k, v = seeded_qkv((B, S, H, 128), 990 + S + H)
        sl = S // world
        mine = [torch.from_numpy(np.ascontiguousarray(x[:, rank * sl:(rank + 1) * sl])).cuda().bfloat16()
                for x in (q, k, v)]
        out = sequence_parallel_self_attention_qsplit(*mine, "sp")
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            got = torch.cat(gathered, dim=1).float().cpu().numpy()
            mx, mean = compare(got, sdpa(q, k, v))
            print(f"qsplit B={B} S={S} H={H}: max {mx:.3g} mean {mean:.3g}", flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3
    if "--time" in sys.argv:
        H, S = 3 * world // 2, 16384 * world  # 1.5 heads per rank
        g = torch.Generator(device="cuda").manual_seed(rank)
        t = [torch.randn((1, S // world, H, 128), generator=g, device="cuda").bfloat16() for _ in range(3)]
        res = {}
        for name, fn in (("pad", lambda: vx.sequence_parallel_self_attention(*t, "sp")),
                         ("qsplit", lambda: sequence_parallel_self_attention_qsplit(*t, "sp"))):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / 5], device="cuda")
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            res[name] = round(float(ms.item()), 3)
        if rank == 0:
            print(json.dumps({"world": world, "heads": H, "seq": S, "ms": res}), flush=True)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    vx.unregister_axis("sp")
    dist.destroy_process_group()
    if rank == 0:
        print("QSPLIT OK" if flag.item() else "QSPLIT FAIL", flush=True)
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
