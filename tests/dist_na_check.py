"""Worker for test_na3d_time_sharded_two_gpus_nccl (run under
torch.distributed.run): each rank holds its frames of a seeded global grid,
neighborhood_attention_3d_sp exchanges the halo over NCCL and computes its
slab; rank 0 gathers and compares with the oracle of the whole grid."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import vidax_b200 as vx  # noqa: E402
from oracle.attention_ref import compare, seeded_qkv, to_bf16  # noqa: E402
from oracle.na3d_ref import na3d  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    vx.register_axis("sp", None)
    from vidax_b200.na_parallel import slab_bounds, split_sizes
    ok = True
    for (B, T, H, W, NH), kernel, pass_t in [((1, 21, 10, 24, 2), (5, 9, 9), True),
                                             ((2, 9, 8, 16, 1), (11, 5, 5), False),
                                             ((1, 3, 6, 8, 2), (3, 3, 3), True)]:
        q, k, v = seeded_qkv((B, T, H, W, NH, 128), 950 + T + W, n=3)
        q = to_bf16(q * np.float32(128 ** -0.5))
        bounds = slab_bounds(split_sizes(T, world))
        mine = [torch.from_numpy(np.ascontiguousarray(x[:, bounds[rank]:bounds[rank + 1]]))
                .cuda().bfloat16() for x in (q, k, v)]
        out = vx.neighborhood_attention_3d_sp(*mine, kernel, "sp",
                                              t_global=T if pass_t else None)
        sizes = [bounds[r + 1] - bounds[r] for r in range(world)]
        pad = torch.zeros((B, max(sizes), H, W, NH, 128), dtype=out.dtype, device=out.device)
        pad[:, :out.shape[1]] = out
        gathered = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(gathered, pad)  # equal sizes; slabs may differ by a frame
        if rank == 0:
            got = torch.cat([g[:, :n] for g, n in zip(gathered, sizes)], dim=1).float().cpu().numpy()
            mx, mean = compare(got, na3d(q, k, v, kernel))
            print(f"T={T} kernel={kernel}: max {mx:.3g} mean {mean:.3g}", flush=True)
            ok = ok and mx <= 2e-2 and mean <= 2e-3
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.broadcast(flag, 0)
    vx.unregister_axis("sp")
    dist.destroy_process_group()
    if rank == 0:
        print("NA SP OK" if flag.item() else "NA SP FAIL", flush=True)
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
