"""The device PagedKVCache against the oracle's restatement of the reference
(src/model/memory.rs:100-201): the same sequence of writes, batched writes,
reads and clears must leave the same pages (bit-exact rows, the same found
flags, the same active page count), evictions included."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def paged(chalot):
    from chalot_c1_b200 import paged
    return paged


def _rows(rng, n, dim):
    x = rng.standard_normal((n, dim), dtype=np.float32) * rng.uniform(0.1, 10.0, (n, 1)).astype(np.float32)
    x[rng.random(n) < 0.1] = 0.0  # all-zero rows keep scale 1.0
    return x


def _check_all(ref, dev, n_layers, positions, dim):
    for layer in range(n_layers):
        for p in positions:
            ok, k, v = ref.read(layer, p)
            k2 = np.full(dim, 7.0, np.float32)
            v2 = np.full(dim, 7.0, np.float32)
            found = dev.read(layer, p, k2, v2)
            assert found == ok, (layer, p)
            if ok:
                assert (k2.view(np.uint32) == k.view(np.uint32)).all(), (layer, p)
                assert (v2.view(np.uint32) == v.view(np.uint32)).all(), (layer, p)
            else:
                assert (k2 == 7.0).all()  # untouched, as the reference leaves them


def test_reference_kats_on_device(paged):
    # memory.rs tests: round trip, page 1 at position 300, LRU bound
    c = paged.PagedKVCache.new(64, 4)
    c.write(0, 300, np.ones(64, np.float32), np.full(64, 2.0, np.float32))
    k, v = np.zeros(64, np.float32), np.zeros(64, np.float32)
    assert c.read(0, 300, k, v) and abs(k[0] - 1.0) < 0.1 and abs(v[0] - 2.0) < 0.1
    assert not c.read(0, 0, k, v)
    c1 = paged.PagedKVCache.new(32, 1)
    for i in range(16 + 5):
        c1.write(0, i * 256, np.ones(32, np.float32), np.full(32, 2.0, np.float32))
    assert c1.active_pages() <= 16
    assert c.memory_mb() == pytest.approx(1 * (256 * 64 * 2 + 256 * 8) / 1e6)


@pytest.mark.parametrize("dim,n_layers,max_pages,seed", [(64, 2, 3, 0), (896, 3, 2, 1), (40, 1, 1, 2)])
def test_random_ops_match_reference(paged, oracle_lib, dim, n_layers, max_pages, seed):
    import torch
    rng = np.random.default_rng(seed)
    ref = oracle_lib.RefPagedKVCache(dim, n_layers, max_pages)
    dev = paged.PagedKVCache(dim, n_layers, max_pages)
    touched = set()
    for step in range(60):
        op = rng.random()
        layer = int(rng.integers(0, n_layers))
        if op < 0.45:  # one write
            p = int(rng.integers(0, 256 * 6))
            k, v = _rows(rng, 2, dim)
            if rng.random() < 0.05:
                k[0] = np.nan
            ref.write(layer, p, k, v)
            dev.write(layer, p, k, v)
            touched.add(p)
        elif op < 0.8:  # a batch: repeated positions and several pages
            n = int(rng.integers(1, 40))
            pos = rng.integers(0, 256 * 6, n).astype(np.uint32)
            pos[rng.random(n) < 0.2] = pos[0]
            k, v = _rows(rng, n, dim), _rows(rng, n, dim)
            for i in range(n):
                ref.write(layer, int(pos[i]), k[i], v[i])
            dev.write_batch(layer, pos, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
            touched.update(int(p) for p in pos)
        elif op < 0.95:  # batched reads
            pos = np.array(sorted(touched) or [0], np.uint32)[: 50]
            k_out = torch.zeros((pos.size, dim), device="cuda")
            v_out = torch.zeros((pos.size, dim), device="cuda")
            found = dev.gather(layer, pos, k_out, v_out)
            for i, p in enumerate(pos):
                ok, k, v = ref.read(layer, int(p))
                assert found[i] == ok
                if ok:
                    assert (k_out[i].cpu().numpy().view(np.uint32) == k.view(np.uint32)).all()
                    assert (v_out[i].cpu().numpy().view(np.uint32) == v.view(np.uint32)).all()
        else:
            ref.clear()
            dev.clear()
        assert dev.active_pages() == ref.active_pages(), step
    _check_all(ref, dev, n_layers, sorted(touched), dim)
