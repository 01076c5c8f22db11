"""Decode parity at the Qwen2.5-0.5B shape (d896, 24 layers, 14 heads,
vocab 151936, 8 experts top-2, int4 group 32, rope theta 1e6) through the
C ABI: greedy tokens identical to the oracle's and logits within 1e-3
relative. A 64-token prompt and 32 new tokens keep the oracle's CPU time to
seconds; the full 512 + 512 run is the benchmark's workload.
"""
import numpy as np
import pytest
from parity import near_tie_report

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qwen_model(chalot, model_dir):
    return chalot.ensure_shape(model_dir, "qwen")


def test_qwen_greedy_identical(chalot, oracle_lib, qwen_model):
    prompt = np.random.default_rng(1).integers(0, 151936, 64).tolist()
    e = chalot.Engine.load(qwen_model)
    o = oracle_lib.OracleEngine(qwen_model, threads=oracle_lib.hw_threads())
    try:
        g = e.generate(prompt, 32)
        c = o.generate(prompt, 32)
        assert g == c, near_tie_report(oracle_lib, qwen_model, prompt, g, c)
        a, b = e.logits(), o.logits()
        assert float(np.max(np.abs(a - b)) / np.max(np.abs(b))) <= 1e-3
    finally:
        e.close()
        o.close()


def test_1b_shape_greedy_identical(chalot, oracle_lib, model_dir):
    """The 1B-class shape (d2048, 16 layers, 16 experts top-2, hidden 5632):
    two 32-column chunks per lane in the gate/up kernel and six in the down
    kernel. Greedy tokens identical to the oracle's, logits within 1e-3."""
    path = chalot.ensure_shape(model_dir, "1b")
    prompt = np.random.default_rng(3).integers(0, 32000, 12).tolist()
    e = chalot.Engine.load(path)
    o = oracle_lib.OracleEngine(path, threads=oracle_lib.hw_threads())
    try:
        g = e.generate(prompt, 8)
        c = o.generate(prompt, 8)
        assert g == c, near_tie_report(oracle_lib, path, prompt, g, c)
        a, b = e.logits(), o.logits()
        assert float(np.max(np.abs(a - b)) / np.max(np.abs(b))) <= 1e-3
    finally:
        e.close()
        o.close()
