"""torchrun job for tests/test_gpu_ep.py: chalot_moe_layer_ep (the
expert-parallel layer over NVLink peer memory) on N GPUs against
chalot_moe_layer on one GPU, bit for bit, over several calls in a row of
different sizes (one rank with no tokens in one of them). Prints EP_P2P_OK."""
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
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=datetime.timedelta(seconds=120))
    ok = True
    pl = None
    try:
        layer = moe.synthetic_moe_layer(896, 4864, 8, 2, 32, seed=3)
        pl = ep.PeerExpertLayer(layer, rank, world, max_tokens=1024)
        for call, per_rank in enumerate([512, 37, 1024, 300]):
            T = per_rank * world
            x = torch.from_numpy(np.random.default_rng(10 + call).standard_normal((T, 896), dtype=np.float32)).cuda()
            cuts = [int(T * k / world) for k in range(world + 1)]
            if call == 1:  # the last rank brings no tokens
                cuts = cuts[:-1] + [cuts[-2]] if world > 1 else cuts
                T = cuts[-1]
                x = x[:T]
            mine = x[cuts[rank]:cuts[rank + 1]].contiguous()
            out, sel = pl(mine)
            outs = [torch.empty((cuts[r + 1] - cuts[r], 896), device="cuda") for r in range(world)]
            dist.all_gather(outs, out)
            if rank == 0:
                ref, _, _ = moe.MoeLayer(layer, T)(x)
                good = torch.equal(torch.cat(outs).view(torch.int32), ref.view(torch.int32))
                print(f"call {call}: {T} tokens {'bit-exact' if good else 'MISMATCH'}", flush=True)
                ok = ok and good
        from chalot_c1_b200 import ops
        ops.device_status()  # no bounded wait gave up
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.broadcast(flag, 0)
        ok = bool(flag.item())
        torch.cuda.synchronize()
        if rank == 0:
            print("EP_P2P_OK" if ok else "EP_P2P_MISMATCH", flush=True)
    finally:
        if pl is not None:
            pl.close()
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
