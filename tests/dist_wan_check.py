"""Worker for test_wan_dit_two_gpus_nccl (run under torch.distributed.run):
every rank runs the reduced Wan DiT forward with sequence parallelism (its
token chunk, Ulysses self-attention, the sequence all_gather after the head)
on the same inputs; each rank's output must match the single-GPU forward."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import vidax_b200 as vx  # noqa: E402
from test_wan_dit_gpu import _inputs, _rel, _tiny  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    vx.register_axis("sp", None)
    from vidax_b200.wan_dit import init_params, wan_dit_forward
    ok = True
    for head_dim in (128, 64):
        cfg = _tiny(head_dim)
        p = init_params(cfg, "cuda", seed=3)
        lat, ctx, t = (torch.from_numpy(x).cuda() for x in _inputs(cfg, 5))
        sp = wan_dit_forward(p, cfg, lat, t, ctx, sp_axis_name="sp").float().cpu().numpy()
        single = wan_dit_forward(p, cfg, lat, t, ctx).float().cpu().numpy()
        err = _rel(sp, single)
        print(f"rank {rank} head_dim {head_dim}: rel err vs single GPU {err:.3g}", flush=True)
        ok = ok and err <= 1e-2
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    vx.unregister_axis("sp")
    dist.destroy_process_group()
    if rank == 0:
        print("WAN SP OK" if flag.item() else "WAN SP FAIL", flush=True)
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
