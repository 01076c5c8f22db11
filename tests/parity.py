"""Near-tie diagnostic for greedy parity checks: when two token sequences
differ, replay the oracle to the first differing step and report how far
apart the two candidate tokens' logits were (a gap within float rounding
means a near tie rather than an arithmetic difference)."""
import numpy as np


def near_tie_report(oracle_lib, path, prompt, got, want) -> str:
    i = next((k for k, (a, b) in enumerate(zip(got, want)) if a != b), min(len(got), len(want)))
    if i >= len(got) or i >= len(want):
        return f"lengths differ: {len(got)} vs {len(want)} tokens (equal up to {i})"
    o = oracle_lib.OracleEngine(path, threads=oracle_lib.hw_threads())
    try:
        seq = list(prompt) or [0]
        for pos, tok in enumerate(seq + list(want[:i])):
            o.forward(int(tok), pos)
        lg = o.logits()
    finally:
        o.close()
    top = np.sort(lg)[::-1]
    return (f"first difference at new token {i}: got {got[i]}, oracle {want[i]}; oracle logits "
            f"{lg[want[i]]:.6g} vs {lg[got[i]]:.6g} (gap {lg[want[i]] - lg[got[i]]:.3g}), "
            f"top-2 gap {top[0] - top[1]:.3g}")
