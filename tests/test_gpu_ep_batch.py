"""Expert-parallel batched decode: chalot_forward_batch with the experts spread
over a group of engines (expert e on rank e % world), every rank decoding its
own sequences.

On one GPU the ranks are engines on threads of this process, exchanging
through an in-process hub; with two or more GPUs a torchrun job exchanges over
NCCL. Either way every rank's greedy tokens must equal what the same
sequences give through one engine alone: the rows travel as int8 and the
outputs are combined in selection order, so the distribution changes no
arithmetic."""
import os
import subprocess
import sys
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).tolist() for n in lens]


def _run_group(chalot, path, per_rank, max_new, reserve):
    """Decodes per_rank[r] on engine r of an in-process group; returns the
    new tokens per rank."""
    world = len(per_rank)
    hub = chalot.EpHub(world)
    engines = [chalot.Engine.load(path) for _ in range(world)]
    steps = max(chalot.Engine.batch_steps(p, max_new) for p in per_rank)
    out, errs = [None] * world, []

    def run(r):
        try:
            engines[r].attach_ep_hub(hub, r)
            out[r] = engines[r].generate_batch(per_rank[r], max_new, reserve=reserve, steps=steps)
        except Exception as e:  # surfaced below
            errs.append(e)

    try:
        th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
        for t in th:
            t.start()
        for t in th:
            t.join(timeout=600)
        assert not any(t.is_alive() for t in th), "a rank did not finish"
        if errs:
            raise errs[0]
        return out
    finally:
        for e in engines:
            e.close()
        hub.close()


def _alone(chalot, path, prompts, max_new):
    e = chalot.Engine.load(path)
    try:
        return e.generate_batch(prompts, max_new)
    finally:
        e.close()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_batch_hub_matches_one_engine(chalot, tiny_model, world):
    per_rank = [_prompts(4096, [5 + 3 * r, 9, 2 + r][: 1 + (r % 3)], seed=10 + r) for r in range(world)]
    got = _run_group(chalot, tiny_model, per_rank, 6, reserve=4)
    for r in range(world):
        assert got[r] == _alone(chalot, tiny_model, per_rank[r], 6), f"rank {r}"


def test_ep_batch_hub_empty_rank(chalot, tiny_model):
    """A rank without sequences still takes every exchange; the others decode
    as alone."""
    per_rank = [_prompts(4096, [7, 4, 11], seed=21), []]
    got = _run_group(chalot, tiny_model, per_rank, 5, reserve=3)
    assert got[1] == []
    assert got[0] == _alone(chalot, tiny_model, per_rank[0], 5)


def test_ep_batch_hub_1b_shape(chalot, model_dir):
    """The 1B-class shape: 16 experts, 4 per rank at world 4, a few
    sequences per rank."""
    path = chalot.ensure_shape(model_dir, "1b")
    per_rank = [_prompts(32000, [6, 3], seed=30 + r) for r in range(4)]
    got = _run_group(chalot, path, per_rank, 4, reserve=2)
    for r in range(4):
        assert got[r] == _alone(chalot, path, per_rank[r], 4), f"rank {r}"


def test_ep_attach_errors(chalot, tiny_model):
    from chalot_c1_b200._capi import ChalotError
    e = chalot.Engine.load(tiny_model)
    hub3 = chalot.EpHub(3)  # 8 experts do not split over 3 ranks
    hub2 = chalot.EpHub(2)
    try:
        with pytest.raises(ChalotError, match="world dividing n_experts"):
            e.attach_ep_hub(hub3, 0)
        with pytest.raises(ChalotError, match="rank < world"):
            e.attach_ep_hub(hub2, 2)
        e.attach_ep_hub(hub2, 0)
        with pytest.raises(ChalotError, match="already attached"):
            e.attach_ep_hub(hub2, 1)
        e.detach_ep()
    finally:
        e.close()
        hub3.close()
        hub2.close()


def test_ep_batch_nccl_two_gpus(chalot):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29541", os.path.join(ROOT, "tests", "ep_batch_nccl_check.py")]
    r = subprocess.run(["timeout", "-k", "30", "900"] + cmd, capture_output=True, text=True, cwd=ROOT,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "EP_BATCH_NCCL_OK" in r.stdout
