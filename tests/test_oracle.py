"""Pins the CPU oracle (oracle/oracle.cpp) before it is trusted as the checker.

1. The reference's own known-answer tests (src/tensor/tests.rs,
   src/model/memory.rs tests, src/model/mod.rs tests) run against the oracle,
   with the exact values where the reference asserts exact values.
2. A second restatement written separately (tests/refpy.py, numpy float32
   scalar code) must agree with the oracle bit for bit on seeded inputs.
3. The committed golden fixture (tests/golden/tiny_greedy.json) pins the
   oracle's end-to-end greedy output on the tiny synthetic model.
"""
import json
import os

import numpy as np
import pytest

from tests import refpy

HERE = os.path.dirname(os.path.abspath(__file__))


# ---- 1. the reference's known-answer tests ------------------------------------

def test_quantize_i8_roundtrip(oracle_lib):
    # src/tensor/tests.rs:22-31
    q, s = oracle_lib.quantize_i8(np.array([1.0, 0.5, -0.5, 0.0, -1.0], np.float32))
    assert q[0] == 127 and q[4] == -127 and s > 0


def test_matmul_int8_identity_like(oracle_lib):
    # src/tensor/tests.rs:34-49 (in_dim 3: the whole row is the scalar tail)
    w = np.array([127, 0, 0, 0, 127, 0], np.int8)
    out = oracle_lib.matmul_i8(w, np.full(2, 1 / 127, np.float32), [1.0, 2.0, 3.0], 2, 3)
    assert abs(out[0] - 1.0) < 0.1 and abs(out[1] - 2.0) < 0.1
    # exact value: x=[1,2,3] -> scale 3/127, q=[42,85,127] (tail rounds half away)
    assert out.tolist() == refpy.matmul_i8(w, np.full(2, 1 / 127, np.float32),
                                           [1.0, 2.0, 3.0], 2, 3).tolist()


def test_rmsnorm_kat(oracle_lib):
    # src/tensor/tests.rs:52-60
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    out = oracle_lib.rmsnorm(x, np.ones(4, np.float32))
    rms = np.sqrt((x * x).sum() / 4 + 1e-5)
    assert abs(out[0] - 1 / rms) < 1e-4


def test_softmax_kat(oracle_lib):
    # src/tensor/tests.rs:63-69
    x = oracle_lib.softmax([1.0, 2.0, 3.0])
    assert abs(x.sum() - 1.0) < 1e-5 and x[2] > x[1] > x[0]


def test_sample_argmax_kat(oracle_lib):
    # src/tensor/tests.rs:72-75
    assert oracle_lib.argmax([0.1, 0.9, 0.5, 0.3]) == 1


def test_argmax_ties_take_last(oracle_lib):
    # Iterator::max_by returns the last of equal maxima (sampling.rs:34-41);
    # the dummy model (all logits equal) therefore yields vocab-1 (mod.rs:120-132)
    assert oracle_lib.argmax([0.5, 0.9, 0.9, 0.1]) == 2
    assert oracle_lib.argmax(np.zeros(256, np.float32)) == 255


def test_int4_pack_unpack_exhaustive(oracle_lib):
    # src/tensor/tests.rs:78-87
    for lo in range(-8, 8):
        for hi in range(-8, 8):
            assert oracle_lib.unpack_int4(oracle_lib.pack_int4(lo, hi)) == (lo, hi)
    assert oracle_lib.pack_int4(0, 0) == 0x88  # tests.rs:117


def test_quantize_i4_roundtrip(oracle_lib):
    # src/tensor/tests.rs:90-102
    packed, scales = oracle_lib.quantize_i4([1.0, -0.5, 0.0, 0.25, -1.0, 0.7, -0.3, 0.9])
    assert scales[0] > 0
    lo, _ = oracle_lib.unpack_int4(int(packed[0]))
    assert lo > 0 and lo == 7


def test_matmul_int4_basic(oracle_lib):
    # src/tensor/tests.rs:105-127, plus its exact value: x=1 quantizes to 127,
    # so row 0 = ((64*7*127 as f32) * (1/7)) * (1/127), row 1 = 0.
    pk = oracle_lib.pack_int4(7, 7)
    z = oracle_lib.pack_int4(0, 0)
    w = np.array([pk] * 32 + [z] * 32, np.uint8)
    s = np.full(2, np.float32(1.0) / np.float32(7.0), np.float32)
    out = oracle_lib.matmul_i4(w, s, np.ones(64, np.float32), 2, 64, 64)
    assert out[0] > 10 and abs(out[1]) < 1.0
    xs = np.float32(1.0) / np.float32(127.0)
    assert out[0] == np.float32(np.float32(np.float32(56896) * s[0]) * xs)
    assert out[1] == 0.0


def test_softmax_top_k_kat(oracle_lib):
    # src/tensor/tests.rs:130-138
    idx, w = oracle_lib.softmax_top_k([1.0, 3.0, 2.0, 0.5], 2)
    assert idx.tolist() == [1, 2] and abs(w.sum() - 1.0) < 1e-5


def test_repetition_penalty(oracle_lib):
    # src/tensor/sampling.rs:168-178: divide positive, multiply non-positive,
    # repeated ids penalised repeatedly, out-of-range ids ignored
    out = oracle_lib.repetition_penalty([2.0, -1.0, 0.0, 4.0], [0, 1, 0, 9], 2.0)
    assert out.tolist() == [0.5, -2.0, 0.0, 4.0]


def test_fast_exp_values(oracle_lib):
    # exact by construction at 0; elsewhere the degree-5 Taylor polynomial on
    # r in [0, ln2) of the reference is within ~1.5e-4 of exp
    assert oracle_lib.fast_exp(0.0) == 1.0
    for v in np.linspace(-60, 10, 141):
        assert abs(oracle_lib.fast_exp(v) / np.exp(v) - 1) < 2e-4


# ---- 2. independent restatement agrees bit for bit ---------------------------------

def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("seed", range(4))
def test_oracle_matches_refpy_float_paths(oracle_lib, seed):
    rng = np.random.default_rng(seed)
    for n in (7, 8, 16, 24, 64, 100, 896):
        x = rng.standard_normal(n).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        assert (_bits(oracle_lib.rmsnorm(x, w)) == _bits(refpy.rmsnorm(x, w))).all()
        y = rng.standard_normal(n).astype(np.float32)
        assert _bits(oracle_lib.dot_f32(x, y)) == _bits(refpy.dot_f32(x, y))
        q1, s1 = oracle_lib.quantize_i8(x)
        q2, s2 = refpy.quantize_i8(x)
        assert (q1 == q2).all() and _bits(s1) == _bits(s2)
    for v in rng.uniform(-80, 20, 2000).astype(np.float32):
        assert _bits(oracle_lib.fast_exp(v)) == _bits(refpy.fast_exp(v))
    for n in (8, 16, 64, 256):  # whole 8-chunks: no libm term
        x = (rng.standard_normal(n) * 5).astype(np.float32)
        assert (_bits(oracle_lib.softmax(x)) == _bits(refpy.softmax(x))).all()


@pytest.mark.parametrize("in_dim,group", [(64, 32), (96, 32), (128, 64), (100, 32), (33, 32)])
def test_oracle_matmuls_match_refpy(oracle_lib, in_dim, group):
    rng = np.random.default_rng(in_dim)
    out_dim = 5
    x = rng.standard_normal(in_dim).astype(np.float32)
    w8 = rng.integers(-127, 128, out_dim * in_dim).astype(np.int8)
    ws = rng.uniform(0.001, 0.01, out_dim).astype(np.float32)
    assert (_bits(oracle_lib.matmul_i8(w8, ws, x, out_dim, in_dim))
            == _bits(refpy.matmul_i8(w8, ws, x, out_dim, in_dim))).all()
    prow, ng = (in_dim + 1) // 2, (in_dim + group - 1) // group
    wp = rng.integers(0, 256, out_dim * prow).astype(np.uint8)
    s4 = rng.uniform(0.001, 0.01, out_dim * ng).astype(np.float32)
    assert (_bits(oracle_lib.matmul_i4(wp, s4, x, out_dim, in_dim, group))
            == _bits(refpy.matmul_i4(wp, s4, x, out_dim, in_dim, group))).all()


def test_topk_stable_order(oracle_lib):
    # equal probabilities keep index order (insertion sort below 20 elements)
    idx, w = oracle_lib.softmax_top_k([0.0, 1.0, 1.0, 1.0], 2)
    assert idx.tolist() == [1, 2] and w[0] == w[1]


# ---- 3. golden end-to-end fixture --------------------------------------------------

def test_golden_tiny_greedy(oracle_lib, tiny_model):
    g = json.load(open(os.path.join(HERE, "golden", "tiny_greedy.json")))
    assert os.path.getsize(tiny_model) == g["file_bytes"]
    import hashlib
    h = hashlib.sha256(open(tiny_model, "rb").read()).hexdigest()
    assert h == g["file_sha256"], "synthetic writer output changed"
    e = oracle_lib.OracleEngine(tiny_model, threads=0)
    assert e.generate(g["prompt"], g["max_new"]) == g["tokens"]
    pen = e.generate(g["prompt"], g["max_new"], repetition_penalty=1.15, repetition_window=64)
    assert pen == g["tokens_penalty_1_15"]


def test_oracle_paged_attention_matches_f32_attention(oracle_lib):
    # the paged oracle over dequantized pages equals the plain attention
    # restatement (engine.rs:283-309) run on those dequantized rows
    P, H, hd, L = 16, 2, 64, 40
    rng = np.random.default_rng(0)
    k = rng.standard_normal((3, P, H, hd), dtype=np.float32)
    v = rng.standard_normal((3, P, H, hd), dtype=np.float32)
    data = np.zeros((3, 2, H, P, hd), np.int8)
    sc = np.zeros((3, 2, H), np.float32)
    oracle_lib.paged_store(data, sc, [0, 1, 2], P, H, hd, k, v)
    q = rng.standard_normal((1, H, hd), dtype=np.float32)
    out = oracle_lib.paged_attention(data, sc, np.array([[0, 1, 2]], np.int32), [L], P, H, hd, q)
    for h in range(H):
        kd = (data[:, 0, h].astype(np.float32) * sc[:, 0, h, None, None]).reshape(-1, hd)[:L]
        vd = (data[:, 1, h].reshape(3, hd, P).transpose(0, 2, 1).astype(np.float32)
              * sc[:, 1, h, None, None]).reshape(-1, hd)[:L]
        s = np.array([oracle_lib.soft_cap(oracle_lib.dot_f32(q[0, h], kd[t]) * np.float32(1 / np.sqrt(np.float32(hd))), 30.0)
                      for t in range(L)], np.float32)
        w = oracle_lib.softmax(s)
        ref = np.zeros(hd, np.float32)
        for t in range(L):
            ref = (ref + (w[t] * vd[t]).astype(np.float32)).astype(np.float32)
        assert np.allclose(out[0, h], ref, rtol=1e-5, atol=1e-6)


# ---- PagedKVCache (src/model/memory.rs tests) ---------------------------------

def test_kvcache_quantization_kat(oracle_lib):
    # memory.rs:210-225: a row round-trips within 0.1
    c = oracle_lib.RefPagedKVCache(4, 1)
    row = np.array([0.5, -1.2, 3.4, 0.0], np.float32)
    c.write(0, 0, row, row)
    ok, k, v = c.read(0, 0)
    assert ok and np.all(np.abs(k - row) < 0.1) and np.all(np.abs(v - row) < 0.1)


def test_kvcache_paging_kat(oracle_lib):
    # memory.rs:227-243: position 300 lives in page 1
    c = oracle_lib.RefPagedKVCache(64, 4)
    c.write(0, 300, np.ones(64, np.float32), np.full(64, 2.0, np.float32))
    ok, k, v = c.read(0, 300)
    assert ok and abs(k[0] - 1.0) < 0.1 and abs(v[0] - 2.0) < 0.1
    assert not c.read(0, 0)[0] and not c.read(1, 300)[0]


def test_kvcache_lru_eviction_kat(oracle_lib):
    # memory.rs:245-260: 21 pages into a 1-layer cache keep at most 16
    c = oracle_lib.RefPagedKVCache(32, 1)
    for i in range(16 + 5):
        c.write(0, i * 256, np.ones(32, np.float32), np.full(32, 2.0, np.float32))
    assert c.active_pages() <= 16
    assert not c.read(0, 0)[0] and c.read(0, 20 * 256)[0]


def test_kvcache_truncating_quantizer(oracle_lib):
    # (val / scale).clamp(-128, 127) as i8 truncates toward zero: 0.9 * 127 -> 114
    c = oracle_lib.RefPagedKVCache(2, 1)
    c.write(0, 0, np.array([1.0, 0.9], np.float32), np.zeros(2, np.float32))
    ok, k, v = c.read(0, 0)
    s = np.float32(1.0) / np.float32(127.0)
    assert k[1] == np.float32(np.float32(int(np.float32(0.9) / s)) * s)
    assert (v == 0).all()  # an all-zero row keeps scale 1.0 and zeros


def test_oracle_writer_matches_library_writer(tmp_path):
    """The oracle's copy of the synthetic writer (compiled from the library's
    writer sources, used by the CPU reference arm) writes the same bytes."""
    import filecmp

    import chalot_c1_b200 as cb
    from oracle import oracle as orc
    shape = dict(cb.SHAPES["tiny"], n_layers=1, vocab_size=512)
    a = cb.write_synthetic(str(tmp_path / "lib.myai"), **shape)
    b = orc.write_synthetic(str(tmp_path / "orc.myai"), **shape)
    assert filecmp.cmp(a, b, shallow=False)
