"""Paged batch K/V (chalot_batch_reserve_paged) and continuous batching
(chalot_sched_*): sequences that share the engine's slots, are admitted while
others run, prefill in chunks and leave when done must each produce exactly
the greedy tokens of a single-sequence generate (the oracle's Engine::generate,
engine.rs:497-548), and every page must return to the pool."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).tolist() for n in lens]


def test_paged_batch_matches_oracle(chalot, oracle_lib, tiny_model):
    prompts = _prompts(4096, [5, 40, 1, 17], seed=21)
    e = chalot.Engine.load(tiny_model)
    try:
        e.reserve_batch_paged(4, n_pages=64, page_tokens=16)
        got = e.generate_batch(prompts, 12)
        for i in range(4):
            e.release_slot(i)
        assert e.kv_pages() == {"free": 64, "total": 64, "page_tokens": 16}
    finally:
        e.close()
    o = oracle_lib.OracleEngine(tiny_model, threads=oracle_lib.hw_threads())
    try:
        for p, g in zip(prompts, got):
            assert g == o.generate(p, 12)
    finally:
        o.close()


def test_scheduler_continuous_batching(chalot, oracle_lib, tiny_model):
    # 9 sequences through 3 slots (3 rows per forward): admitted as slots
    # free up, a second wave submitted while the first runs
    first = _prompts(4096, [7, 23, 2, 11, 30], seed=3)
    second = _prompts(4096, [9, 4, 16, 1], seed=4)
    new = [6, 3, 9, 1, 5, 8, 4, 2, 7]
    e = chalot.Engine.load(tiny_model)
    try:
        e.reserve_batch_paged(3, n_pages=20, page_tokens=16)
        sch = e.scheduler(max_rows=3)
        ids = [sch.submit(p, n) for p, n in zip(first, new)]
        for _ in range(4):
            sch.step()
        ids += [sch.submit(p, n) for p, n in zip(second, new[5:])]
        sch.run()
        got = []
        for i in ids:
            toks, done = sch.poll(i)
            assert done
            got.append(toks)
        sch.close()
        assert e.kv_pages()["free"] == 20
    finally:
        e.close()
    o = oracle_lib.OracleEngine(tiny_model, threads=oracle_lib.hw_threads())
    try:
        for p, n, g in zip(first + second, new, got):
            assert g == o.generate(p, n)
    finally:
        o.close()


def test_scheduler_stop_tokens_and_page_pressure(chalot, tiny_model):
    # a pool that holds two generations at a time: admission waits for pages;
    # a stop token ends a sequence early without being returned
    prompts = _prompts(4096, [20, 20, 20, 20], seed=8)
    e = chalot.Engine.load(tiny_model)
    try:
        ref = [e.generate(p, 12) for p in prompts]
        e.reserve_batch_paged(4, n_pages=4, page_tokens=16)  # 31 positions = 2 pages per generation
        sch = e.scheduler()
        stop = ref[1][5]
        ids = [sch.submit(p, 12, stop=[stop] if i == 1 else []) for i, p in enumerate(prompts)]
        st = sch.step()
        assert st["running"] == 2 and st["waiting"] == 2
        sch.run()
        outs = [sch.poll(i)[0] for i in ids]
        assert outs[0] == ref[0] and outs[2] == ref[2] and outs[3] == ref[3]
        assert outs[1] == ref[1][: ref[1].index(stop)]
        assert e.kv_pages()["free"] == 4
        sch.close()
    finally:
        e.close()


def test_scheduler_errors(chalot, tiny_model):
    from chalot_c1_b200._capi import ChalotError
    e = chalot.Engine.load(tiny_model)
    try:
        with pytest.raises(ChalotError, match="reserve"):
            e.scheduler(max_rows=1)
        e.reserve_batch_paged(2, n_pages=2, page_tokens=16)
        sch = e.scheduler()
        with pytest.raises(ChalotError, match="max_new"):
            sch.submit([1, 2], 0)
        with pytest.raises(ChalotError, match="max_seq_len"):
            sch.submit([1] * 500, 100)
        with pytest.raises(ChalotError, match="pages"):
            sch.submit([1] * 40, 1)  # 40 positions > 2 pages of 16
        with pytest.raises(ChalotError, match="unknown"):
            sch.poll(12345)
        sch.close()
        with pytest.raises(ChalotError, match="page_tokens"):
            e2 = chalot.Engine.load(tiny_model)
            try:
                e2.reserve_batch_paged(2, n_pages=4, page_tokens=12)
            finally:
                e2.close()
    finally:
        e.close()
