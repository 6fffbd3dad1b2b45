"""Worker for test_capi_layer_two_gpus_matches_torch_mirror (under
torch.distributed.run): the C-ABI Ulysses layer over the ranks' NCCL
communicator against the torch mirror's pipeline (same slices and kernels:
identical bits) and, on rank 0, against the oracle of the global sequence."""
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
from vidax_b200.ulysses_capi import Comm, sequence_parallel_self_attention  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    vx.register_axis("sp", None)
    comm = Comm.from_process_group()
    ok = True
    for (B, S, H) in [(1, 1024, 10), (2, 768, 6), (1, 512, 3)]:
        q, k, v = seeded_qkv((B, S, H, 128), 1400 + S + H)
        sl = S // world
        mine = [torch.from_numpy(np.ascontiguousarray(x[:, rank * sl:(rank + 1) * sl])).cuda().bfloat16()
                for x in (q, k, v)]
        out = sequence_parallel_self_attention(*mine, comm)
        mirror = vx.sequence_parallel_self_attention(*mine, "sp")
        torch.cuda.synchronize()
        same = torch.equal(out, mirror)
        ok = ok and same
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            mx, mean = compare(torch.cat(gathered, dim=1).float().cpu().numpy(), sdpa(q, k, v))
            print(f"B={B} S={S} H={H}: max {mx:.3g} mean {mean:.3g} same-as-mirror {same}", flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3
    comm.close()
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    vx.unregister_axis("sp")
    dist.destroy_process_group()
    if rank == 0:
        print("CAPI ULYSSES OK" if flag.item() == 1 else "CAPI ULYSSES FAILED", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
