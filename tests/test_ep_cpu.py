"""Expert-parallel layer on CPU ranks (gloo, world size 2 and 4): the
exchange logic of chalot_c1_b200.ep (plans, counts, splits, the return trip,
the combine) with every compute step restated by the oracle. The gathered
outputs must equal the oracle's single-process expert block bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shards(T, world, skew):
    if skew:  # rank 0 gets nothing, the rest split the tokens
        cuts = [0, 0] + [int(T * k / (world - 1)) for k in range(1, world)]
        return [(cuts[r], cuts[r + 1]) for r in range(world)]
    cuts = [int(T * k / world) for k in range(world + 1)]
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def _worker(rank, world, port, case, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist
    from chalot_c1_b200 import ep, moe
    from oracle import oracle as orc
    from tests.ep_oracle_backend import OracleBackend
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        dim, hidden, E, K, T, seed, bias, skew = case
        layer = moe.synthetic_moe_layer(dim, hidden, E, K, 32, seed=seed)
        for e, b in bias.items():
            layer.router_b[e] = b
        x = np.random.default_rng(seed).standard_normal((T, dim), dtype=np.float32)
        a, b = _shards(T, world, skew)[rank]
        out, sel = ep.ep_forward(OracleBackend(layer, world, rank, orc), torch.from_numpy(x[a:b].copy()),
                                 ep.dist_all_to_all(), world)
        q.put((rank, out.numpy(), sel.numpy()))
    finally:
        dist.destroy_process_group()


CASES = {
    "balanced": (256, 256, 8, 2, 40, 1, {}, False),
    "skewed": (256, 256, 8, 2, 33, 2, {0: 40.0, 4: 30.0}, False),  # experts 0 and 4: both on rank 0 of 2/4
    "empty_rank": (256, 256, 4, 2, 17, 3, {}, True),
}


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("name", list(CASES))
def test_ep_gloo_matches_single_process(oracle_lib, world, name):
    case = CASES[name]
    dim, hidden, E, K, T, seed, bias, skew = case
    if E % world:
        pytest.skip("experts must divide among the ranks")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = {}
        for _ in range(world):
            r, out, sel = q.get(timeout=240)
            got[r] = (out, sel)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    from chalot_c1_b200 import moe
    layer = moe.synthetic_moe_layer(dim, hidden, E, K, 32, seed=seed)
    for e, b in bias.items():
        layer.router_b[e] = b
    x = np.random.default_rng(seed).standard_normal((T, dim), dtype=np.float32)
    ref, ref_sel = oracle_lib.moe_forward(x, layer.layer_bytes(), dim, hidden, E, K, 32)
    out = np.concatenate([got[r][0] for r in range(world)])
    sel = np.concatenate([got[r][1] for r in range(world)])
    assert (sel == ref_sel).all()
    assert (out.view(np.uint32) == ref.view(np.uint32)).all()
