"""The near-tie diagnostic of the greedy parity tests, on the oracle alone
(CPU): a planted difference in the token sequence is located and the two
tokens' oracle logits are reported."""
from parity import near_tie_report


def test_near_tie_report_locates_planted_difference(chalot, oracle_lib, tiny_model):
    prompt = [11, 22, 33, 44]
    o = oracle_lib.OracleEngine(tiny_model, threads=1)
    try:
        want = o.generate(prompt, 6)
    finally:
        o.close()
    got = list(want)
    got[3] = (got[3] + 1) % 4096  # planted in the checker's input, not in any kernel
    msg = near_tie_report(oracle_lib, tiny_model, prompt, got, want)
    assert "first difference at new token 3" in msg
    assert f"oracle {want[3]}" in msg and "gap" in msg
    assert "lengths differ" in near_tie_report(oracle_lib, tiny_model, prompt, want[:4], want)
