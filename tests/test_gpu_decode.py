"""End-to-end decode parity on the tiny synthetic model through the C ABI.

Bars (stated in the hot-path contract): greedy tokens identical to the
oracle's; f32 logits within 1e-3 relative (max |gpu - cpu| / max |cpu|). The
int8/int4 paths are exact, so in practice the logits differ only where libm
(tanhf/expf in the attention softmax tail) rounds differently on the device.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LOGIT_RTOL = 1e-3


@pytest.fixture(scope="module")
def golden():
    return json.load(open(os.path.join(HERE, "golden", "tiny_greedy.json")))


@pytest.fixture(scope="module")
def engine(chalot, tiny_model):
    e = chalot.Engine.load(tiny_model)
    yield e
    e.close()


@pytest.fixture(scope="module")
def oracle_engine(oracle_lib, tiny_model):
    return oracle_lib.OracleEngine(tiny_model, threads=0)


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def test_greedy_tokens_identical(engine, golden):
    assert engine.generate(golden["prompt"], golden["max_new"]) == golden["tokens"]


def test_greedy_with_penalty_identical(chalot, engine, golden):
    sp = chalot.SamplingConfig(repetition_penalty=1.15, repetition_window=64)
    assert engine.generate(golden["prompt"], golden["max_new"], sp) == golden["tokens_penalty_1_15"]


def test_forward_sequence_and_logits(engine, oracle_engine, golden):
    worst = 0.0
    for pos, tok in enumerate(golden["prompt"][:24]):
        g = engine.forward(tok, pos)
        c = oracle_engine.forward(tok, pos)
        assert g == c, f"argmax differs at pos {pos}"
        worst = max(worst, rel_err(engine.logits(), oracle_engine.logits()))
    assert worst <= LOGIT_RTOL, worst


def test_logits_bitwise_first_position(engine, oracle_engine):
    # at pos 0 the softmax has one element (tail path: exp(0) = 1 exactly), so
    # the whole forward is libm-free except tanh of one score per head
    engine.forward(7, 0)
    oracle_engine.forward(7, 0)
    a, b = engine.logits(), oracle_engine.logits()
    assert rel_err(a, b) <= LOGIT_RTOL
    assert np.mean(a.view(np.uint32) == b.view(np.uint32)) > 0.99


def test_stop_tokens_truncate(chalot, engine, golden):
    stop = golden["tokens"][5]
    first = golden["tokens"].index(stop)
    sp = chalot.SamplingConfig(stop_tokens=[stop])
    assert engine.generate(golden["prompt"], 40, sp) == golden["tokens"][:first]


def test_empty_prompt_starts_from_bos(engine, oracle_engine):
    # engine.rs:520-524: no prompt -> next token is 1 (BOS)
    assert engine.generate([], 16) == oracle_engine.generate([], 16)


def test_prefill_clamped_to_room(engine, oracle_engine):
    # engine.rs:509: n_prefill = min(len, max(max_seq - max_new, 1)); max_seq 512
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, 4096, 500).tolist()
    assert engine.generate(prompt, 20) == oracle_engine.generate(prompt, 20)


def test_out_of_vocab_prompt_ids_are_clamped(engine, oracle_engine):
    # engine.rs:512: prompt ids are clamped to vocab-1
    prompt = [5, 9999, 100000, 3]
    assert engine.generate(prompt, 8) == oracle_engine.generate(prompt, 8)


def test_sample_from_logits_penalty(chalot, engine, oracle_engine):
    engine.forward(11, 0)
    oracle_engine.forward(11, 0)
    hist = list(range(0, 4096, 7))
    sp = chalot.SamplingConfig(repetition_penalty=1.3, repetition_window=64)
    g = engine.sample_from_logits(sp, hist)
    from oracle import oracle as orc
    lg = orc.repetition_penalty(oracle_engine.logits(), hist[-64:], 1.3)
    assert g == orc.argmax(lg)


def test_forward_rejects_bad_input(chalot, engine):
    with pytest.raises(chalot.ChalotError):
        engine.forward(4096, 0)
    with pytest.raises(chalot.ChalotError):
        engine.forward(1, 512)


def test_eager_and_graph_agree(chalot, tiny_model, golden):
    e = chalot.Engine.load(tiny_model, use_cuda_graph=False)
    try:
        assert e.generate(golden["prompt"], 32) == golden["tokens"][:32]
    finally:
        e.close()


def test_dense_ffn_model(chalot, oracle_lib, tmp_path):
    # n_experts < 2 takes the dense FFN path (engine.rs:402-442)
    p = chalot.write_shape(str(tmp_path / "dense.myai"), "tiny", n_experts=1, top_k=1, n_layers=2)
    e = chalot.Engine.load(p)
    o = oracle_lib.OracleEngine(p, threads=0)
    prompt = list(range(1, 17))
    assert e.generate(prompt, 24) == o.generate(prompt, 24)
    e.close()


def test_group64_model(chalot, oracle_lib, tmp_path):
    p = chalot.write_shape(str(tmp_path / "g64.myai"), "tiny", int4_group_size=64, n_layers=2)
    e = chalot.Engine.load(p)
    o = oracle_lib.OracleEngine(p, threads=0)
    prompt = list(range(100, 140))
    assert e.generate(prompt, 24) == o.generate(prompt, 24)
    e.close()


def test_timing_reported(engine, golden):
    engine.generate(golden["prompt"], 32)
    t = engine.last_timing()
    assert t["n_prefill"] == 32 and t["n_decode"] == 32
    assert t["prefill_ms"] > 0 and t["decode_ms"] > 0
