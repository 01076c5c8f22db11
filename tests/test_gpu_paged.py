"""Paged int8 KV cache (long-context format): the page store against the
oracle's quantizer (bit-exact), and decode-step attention against the oracle's
attention over the dequantized pages (float tolerance: the GPU splits the
pages and merges online-softmax partials, which reorders the sums)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3


@pytest.fixture(scope="module")
def paged(chalot):
    from chalot_c1_b200 import paged
    return paged


def _pool(paged, n_pages, P, H, hd, seed):
    import torch
    pool = paged.PagedKVPool(n_pages, P, H, hd)
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((n_pages, P, H, hd), dtype=np.float32)
    v = rng.standard_normal((n_pages, P, H, hd), dtype=np.float32)
    ids = rng.permutation(n_pages).astype(np.int32)
    pool.store(torch.from_numpy(ids).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    return pool, ids, k, v


@pytest.mark.parametrize("P,H,hd", [(16, 14, 64), (8, 3, 128), (32, 2, 64)])
def test_store_bit_exact(paged, oracle_lib, P, H, hd):
    pool, ids, k, v = _pool(paged, 7, P, H, hd, seed=P + H)
    data = np.zeros((7, 2, H, P, hd), np.int8)
    sc = np.zeros((7, 2, H), np.float32)
    oracle_lib.paged_store(data, sc, ids, P, H, hd, k, v)
    assert np.array_equal(pool.data.cpu().numpy(), data)
    assert np.array_equal(pool.scales.cpu().numpy().view(np.uint32), sc.view(np.uint32))


@pytest.mark.parametrize("P,H,hd,lens", [(16, 14, 64, [1, 37, 300]), (8, 3, 128, [64, 5]),
                                         (32, 2, 64, [1000, 31, 32, 33]), (16, 14, 64, [2048])])
def test_attention_matches_oracle(paged, oracle_lib, P, H, hd, lens):
    import torch
    max_pages = max((n + P - 1) // P for n in lens)
    n_pages = max_pages * len(lens) + 3
    pool, _, _, _ = _pool(paged, n_pages, P, H, hd, seed=len(lens) * 11 + P)
    rng = np.random.default_rng(5)
    table = rng.permutation(n_pages)[: max_pages * len(lens)].reshape(len(lens), max_pages).astype(np.int32)
    q = rng.standard_normal((len(lens), H, hd), dtype=np.float32)
    out = pool.attention(torch.from_numpy(q).cuda(), torch.from_numpy(table).cuda(),
                         torch.from_numpy(np.array(lens, np.int32)).cuda())
    torch.cuda.synchronize()
    ref = oracle_lib.paged_attention(pool.data.cpu().numpy(), pool.scales.cpu().numpy(), table, lens, P, H, hd, q,
                                     threads=oracle_lib.hw_threads())
    got = out.cpu().numpy()
    tol = RTOL * np.abs(ref).max(axis=-1, keepdims=True)
    assert (np.abs(got - ref) <= tol).all(), np.abs(got - ref).max()


def test_attention_reports_bad_page(paged):
    """No environment switch: the bad id is reported by chalot_device_status,
    or by the next operator call once the work finished, and then cleared."""
    import torch

    from chalot_c1_b200 import ops
    from chalot_c1_b200._capi import ChalotError
    pool, _, _, _ = _pool(paged, 4, 16, 2, 64, seed=1)
    table = torch.tensor([[0, 1, 99]], dtype=torch.int32, device="cuda")  # 99 is outside the pool
    good = torch.tensor([[0, 1, 2]], dtype=torch.int32, device="cuda")
    q = torch.zeros((1, 2, 64), device="cuda")
    lens = torch.tensor([40], dtype=torch.int32, device="cuda")
    pool.attention(q, table, lens)  # asynchronous: returns before the check
    with pytest.raises(ChalotError, match="outside"):
        ops.device_status()
    ops.device_status()  # reported once
    pool.attention(q, table, lens)
    torch.cuda.synchronize()
    with pytest.raises(ChalotError, match="outside"):
        pool.attention(q, good, lens)  # the next call reports the earlier failure
    pool.attention(q, good, lens)
    ops.device_status()


def test_store_reports_bad_page(paged):
    import torch

    from chalot_c1_b200 import ops
    from chalot_c1_b200._capi import ChalotError
    pool = paged.PagedKVPool(2, 16, 2, 64)
    k = torch.zeros((1, 16, 2, 64), device="cuda")
    pool.store(torch.tensor([5], dtype=torch.int32, device="cuda"), k, k)
    with pytest.raises(ChalotError, match="outside"):
        ops.device_status()
    pool.store(torch.tensor([1], dtype=torch.int32, device="cuda"), k, k)
    ops.device_status()
