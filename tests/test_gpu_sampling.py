"""Sampling strategies on the device (chalot_sample, and through
Engine.generate) against the oracle's restatement of sampling.rs for the
same draw r. The GPU sums probability mass in another order than the
reference's sequential sums, so a draw that lies within rounding of a
running-sum boundary may pick a neighbour; for those draws (margin below
2e-4) the pick must lie close to the oracle's in the order the strategy
walks. Every other draw must pick the same token."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
MARGIN = 2e-4


def _sample_gpu(logits_dev, V, cfg, r):
    from chalot_c1_b200._capi import check, lib
    out = C.c_uint32()
    s, _keep = cfg._c()
    check(lib().chalot_sample(logits_dev.data_ptr(), V, C.byref(s), r, C.byref(out), None))
    return out.value


CASES = [
    # V, logit scale, strategy, temperature, top_k, top_p, min_p
    (1000, 1.0, 1, 0.7, 40, 0.9, 0.05),
    (1000, 3.0, 1, 1.0, 1, 0.9, 0.05),
    (4096, 0.5, 1, 1.3, 500, 0.9, 0.05),
    (1000, 1.0, 2, 0.7, 40, 0.9, 0.05),
    (4096, 3.0, 2, 1.0, 40, 0.1, 0.05),
    (151936, 2.0, 2, 0.7, 40, 0.9, 0.05),
    (1000, 1.0, 3, 0.7, 40, 0.9, 0.05),
    (4096, 2.0, 3, 1.0, 40, 0.9, 0.5),
    (151936, 1.0, 3, 1.3, 40, 0.9, 0.05),
    (151936, 2.0, 1, 0.7, 40, 0.9, 0.05),
]


@pytest.mark.parametrize("V,scale,strategy,temp,top_k,top_p,min_p", CASES)
def test_sample_matches_oracle(chalot, oracle_lib, V, scale, strategy, temp, top_k, top_p, min_p):
    import torch
    from chalot_c1_b200.engine import SamplingConfig
    rng = np.random.default_rng(V + strategy * 7 + int(scale * 10))
    logits = (rng.standard_normal(V) * scale).astype(np.float32)
    dev = torch.from_numpy(logits).cuda()
    cfg = SamplingConfig(strategy=strategy, temperature=temp, top_k=top_k, top_p=top_p, min_p=min_p)
    # position of each token in the order the strategy walks: descending
    # logits for top-k/top-p (ties lower index first), index order for min-p
    order = np.argsort(-logits, kind="stable") if strategy in (1, 2) else np.arange(V)
    where = np.empty(V, np.int64)
    where[order] = np.arange(V)
    near = max(8, V // 200)
    checked = 0
    for r in rng.random(40).astype(np.float32):
        tok, margin = oracle_lib.sample(logits, strategy, temp, top_k, top_p, min_p, float(r))
        got = _sample_gpu(dev, V, cfg, float(r))
        if margin < MARGIN:  # within rounding of a boundary: a close neighbour in that order
            assert abs(int(where[got]) - int(where[tok])) <= near, (float(r), got, tok, margin)
            continue
        checked += 1
        assert got == tok, (float(r), got, tok, margin)
    if V <= 4096:  # over a large flat vocabulary nearly every draw sits within rounding
        assert checked >= 10


def test_greedy_limits(chalot, oracle_lib):
    # top-k 1 and min-p 1 keep only the argmax; greedy is the argmax
    import torch
    from chalot_c1_b200.engine import SamplingConfig
    logits = np.random.default_rng(3).standard_normal(5000).astype(np.float32)
    dev = torch.from_numpy(logits).cuda()
    best = int(np.argmax(logits))
    for cfg in (SamplingConfig(strategy=0), SamplingConfig(strategy=1, top_k=1),
                SamplingConfig(strategy=3, min_p=1.0)):
        for r in (0.0, 0.5, 0.999):
            assert _sample_gpu(dev, 5000, cfg, r) == best


def test_generate_with_strategies(chalot, tiny_model):
    from chalot_c1_b200.engine import GREEDY, MIN_P, TOP_K, TOP_P, SamplingConfig
    prompt = np.random.default_rng(0).integers(0, 4096, 16).tolist()
    e = chalot.Engine.load(tiny_model)
    try:
        greedy = e.generate(prompt, 24)
        assert e.generate(prompt, 24, SamplingConfig(strategy=TOP_K, top_k=1, seed=5)) == greedy
        for st in (TOP_K, TOP_P, MIN_P):
            cfg = SamplingConfig(strategy=st, temperature=1.3, seed=1234)
            a = e.generate(prompt, 24, cfg)
            b = e.generate(prompt, 24, cfg)
            assert a == b and len(a) == 24  # the seed fixes the draws
            assert all(0 <= t < 4096 for t in a)
        c = e.generate(prompt, 24, SamplingConfig(strategy=TOP_P, temperature=1.3, seed=99))
        assert c != e.generate(prompt, 24, SamplingConfig(strategy=TOP_P, temperature=1.3, seed=1234))
        assert e.generate(prompt, 24, SamplingConfig(strategy=GREEDY)) == greedy
    finally:
        e.close()
