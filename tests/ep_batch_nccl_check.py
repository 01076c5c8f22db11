"""torchrun job for tests/test_gpu_ep_batch.py: expert-parallel batched decode
over NCCL, one engine per GPU, each rank decoding its own sequences of the
1B-class shape. Every rank compares its tokens with a second engine on its GPU
that decodes the same sequences alone. Prints EP_BATCH_NCCL_OK on rank 0."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import chalot_c1_b200 as cb  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    ok = True
    try:
        d = os.environ.get("CHALOT_MODEL_DIR", "/tmp/chalot_models")
        if rank == 0:
            cb.ensure_shape(d, "1b")  # written once, by rank 0
        dist.barrier()
        path = cb.ensure_shape(d, "1b")
        rng = np.random.default_rng(40 + rank)
        prompts = [rng.integers(0, 32000, n).tolist() for n in (9, 4, 13)]
        max_new = 6
        steps = torch.tensor([cb.Engine.batch_steps(prompts, max_new)])
        dist.all_reduce(steps, op=dist.ReduceOp.MAX)
        e = cb.Engine.load(path, device=local)
        try:
            e.attach_ep_nccl(rank, world)
            got = e.generate_batch(prompts, max_new, reserve=4, steps=int(steps))
            e.detach_ep()
        finally:
            e.close()
        a = cb.Engine.load(path, device=local)
        try:
            want = a.generate_batch(prompts, max_new)
        finally:
            a.close()
        ok = got == want
        flag = torch.tensor([1 if ok else 0])
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
        if rank == 0:
            print("EP_BATCH_NCCL_OK" if ok else "EP_BATCH_NCCL_MISMATCH", flush=True)
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
