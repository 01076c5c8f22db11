"""The int8 tensor-core peak probe (the MoE prefill's roofline denominator)
runs, reports a plausible figure and is repeatable."""
import pytest

pytestmark = pytest.mark.gpu


def test_int8_mma_probe(chalot):
    from chalot_c1_b200 import ops
    a = ops.probe_int8_mma(4000)
    b = ops.probe_int8_mma(4000)
    for r in (a, b):
        assert r["ms"] > 0
        assert 500.0 < r["tops"] < 10000.0  # B200 dense int8 is 4.5 POPS nominal
    assert abs(a["tops"] - b["tops"]) / a["tops"] < 0.2
