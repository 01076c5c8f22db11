"""torchrun job for tests/test_gpu_ep.py: the expert-parallel layer over NCCL
on N GPUs against chalot_moe_layer on rank 0's GPU. Prints EP_NCCL_OK."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from chalot_c1_b200 import ep, moe  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    ok = True
    try:
        layer = moe.synthetic_moe_layer(896, 4864, 8, 2, 32, seed=3)
        T = 512 * world
        x = torch.from_numpy(np.random.default_rng(3).standard_normal((T, 896), dtype=np.float32)).cuda()
        cuts = [int(T * k / world) for k in range(world + 1)]
        out, sel = ep.ep_forward(ep.GpuBackend(layer, world, rank), x[cuts[rank]:cuts[rank + 1]].contiguous(),
                                 ep.dist_all_to_all(), world)
        outs = [torch.empty((cuts[r + 1] - cuts[r], 896), device="cuda") for r in range(world)]
        dist.all_gather(outs, out)
        if rank == 0:
            ref, _, _ = moe.MoeLayer(layer, T)(x)
            ok = torch.equal(torch.cat(outs).view(torch.int32), ref.view(torch.int32))
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.broadcast(flag, 0)
        torch.cuda.synchronize()
        if rank == 0:
            print("EP_NCCL_OK" if ok else "EP_NCCL_MISMATCH", flush=True)
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
