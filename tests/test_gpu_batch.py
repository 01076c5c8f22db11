"""Batched decode (chalot_forward_batch): several sequences through one
engine, each in its own KV slot and at its own position. Every sequence must
decode exactly as the oracle's single-sequence Engine does (identical greedy
tokens; logits within 1e-3 relative), on the tensor-core and the tile-GEMM
paths of the MoE layer."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).tolist() for n in lens]


@pytest.mark.parametrize("path", ["simt", "tc"])
def test_batch_tiny_matches_single_sequences(chalot, oracle_lib, tiny_model, monkeypatch, path):
    monkeypatch.setenv("CHALOT_MOE_PATH", path)
    prompts = _prompts(4096, [5, 12, 1, 30, 7], seed=11)
    e = chalot.Engine.load(tiny_model)
    try:
        got = e.generate_batch(prompts, 16)
    finally:
        e.close()
    o = oracle_lib.OracleEngine(tiny_model, threads=oracle_lib.hw_threads())
    try:
        for p, g in zip(prompts, got):
            assert g == o.generate(p, 16)
    finally:
        o.close()


def test_batch_logits_match_single_forward(chalot, oracle_lib, tiny_model):
    # one batched forward at mixed positions against the oracle's forwards
    prompts = _prompts(4096, [3, 9], seed=5)
    e = chalot.Engine.load(tiny_model)
    o = oracle_lib.OracleEngine(tiny_model, threads=1)
    try:
        e.reserve_batch(2)
        for t in range(3):  # both sequences advance together for 3 tokens
            e.forward_batch([0, 1], [prompts[0][t], prompts[1][t]], [t, t])
        for t in range(3, 9):  # then the second alone
            e.forward_batch([1], [prompts[1][t]], [t])
        e.forward_batch([1, 0], [7, 8], [9, 3])
        # the oracle replays each history from position 0 (rewriting its KV rows)
        for i, (slot, hist) in enumerate([(1, prompts[1] + [7]), (0, prompts[0][:3] + [8])]):
            for pos, tok in enumerate(hist):
                o.forward(tok, pos)
            ref = o.logits()
            got = e.batch_logits(i)
            assert float(np.max(np.abs(got - ref)) / np.max(np.abs(ref))) <= 1e-3
    finally:
        e.close()
        o.close()


def test_batch_qwen_shape(chalot, oracle_lib, model_dir):
    path = chalot.ensure_shape(model_dir, "qwen")
    prompts = _prompts(151936, [20, 9, 33], seed=2)
    e = chalot.Engine.load(path)
    try:
        got = e.generate_batch(prompts, 8)
    finally:
        e.close()
    o = oracle_lib.OracleEngine(path, threads=oracle_lib.hw_threads())
    try:
        for p, g in zip(prompts, got):
            assert g == o.generate(p, 8)
    finally:
        o.close()


def test_batch_argument_errors(chalot, tiny_model):
    from chalot_c1_b200._capi import ChalotError
    e = chalot.Engine.load(tiny_model)
    try:
        with pytest.raises(ChalotError, match="batch_reserve"):
            e.forward_batch([0], [1], [0])
        e.reserve_batch(2)
        with pytest.raises(ChalotError, match="slot"):
            e.forward_batch([0, 0], [1, 2], [0, 0])
        with pytest.raises(ChalotError, match="slot out of range"):
            e.forward_batch([2], [1], [0])
    finally:
        e.close()
