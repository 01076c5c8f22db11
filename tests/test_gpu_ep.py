"""Expert-parallel MoE layer on the GPU building blocks (route, plan,
gather, experts, combine through the C ABI).

On one GPU the ranks are emulated in one process (an in-process all-to-all);
with two or more GPUs a torchrun job exchanges over NCCL. Either way the
gathered outputs must equal chalot_moe_layer's bit for bit."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _single(layer, x):
    from chalot_c1_b200 import moe
    out, sel, _ = moe.MoeLayer(layer, x.shape[0])(x)
    return out, sel


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("path", ["simt", "tc"])
def test_ep_emulated_matches_single_gpu(chalot, monkeypatch, world, path):
    import torch
    from chalot_c1_b200 import ep, moe
    monkeypatch.setenv("CHALOT_MOE_PATH", path)
    layer = moe.synthetic_moe_layer(896, 4864, 8, 2, 32, seed=3)
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((600, 896), dtype=np.float32)).cuda()
    ref, ref_sel = _single(layer, x)
    cuts = [int(600 * k / world) for k in range(world + 1)]
    backends = [ep.GpuBackend(layer, world, r) for r in range(world)]
    res = ep.emulated_forward(backends, [x[cuts[r]:cuts[r + 1]].contiguous() for r in range(world)])
    from chalot_c1_b200 import ops
    ops.device_status()  # no tensor-core wait gave up
    out = torch.cat([o for o, _ in res])
    sel = torch.cat([s for _, s in res])
    assert torch.equal(sel, ref_sel)
    assert torch.equal(out.view(torch.int32), ref.view(torch.int32))


def test_ep_nccl_two_gpus(chalot):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(ROOT, "tests", "ep_nccl_check.py")]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, cwd=ROOT,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "EP_NCCL_OK" in r.stdout


def test_ep_peer_memory_two_gpus(chalot):
    """chalot_moe_layer_ep over NVLink peer memory on two GPUs, bit-identical
    to the single-GPU layer (tests/ep_p2p_check.py)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29537", os.path.join(ROOT, "tests", "ep_p2p_check.py")]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, cwd=ROOT,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "EP_P2P_OK" in r.stdout
