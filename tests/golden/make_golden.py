"""Regenerates tests/golden/tiny_greedy.json.

The reference (Rust) cannot run in this environment, so this fixture records
the CPU oracle's output on the tiny synthetic model (dim 256, 4 layers,
8 experts top-2, int4 group 32, seed 0) for a 32-token prompt drawn with
numpy default_rng(0).integers(0, 4096, 32) and 128 greedy tokens, with and
without the CLI's repetition penalty (1.15 over 64 tokens). It guards the
oracle and the synthetic writer against silent changes; parity with the
reference itself is pinned by the known-answer tests in tests/test_oracle.py.

    python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

import chalot_c1_b200 as cb  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def main():
    with tempfile.TemporaryDirectory() as d:
        path = cb.write_shape(os.path.join(d, "tiny.myai"), "tiny")
        prompt = np.random.default_rng(0).integers(0, 4096, 32).tolist()
        e = orc.OracleEngine(path, threads=0)
        toks = e.generate(prompt, 128)
        pen = e.generate(prompt, 128, repetition_penalty=1.15, repetition_window=64)
        out = {
            "shape": "tiny", "prompt": prompt, "max_new": 128, "tokens": toks,
            "tokens_penalty_1_15": pen, "file_bytes": os.path.getsize(path),
            "file_sha256": hashlib.sha256(open(path, "rb").read()).hexdigest(),
        }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tiny_greedy.json")
    with open(dst, "w") as f:
        json.dump(out, f)
    print(dst, len(toks), len(pen))


if __name__ == "__main__":
    main()
