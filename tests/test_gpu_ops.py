"""Operator parity: the sm_100a kernels behind the C ABI against the CPU oracle.

Bar: bit-exact. The int8/int4 dots are exact int32 sums and every float
epilogue rounds in the reference's order, so outputs must match to the bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def ops(chalot):
    from chalot_c1_b200 import ops
    return ops


@pytest.mark.parametrize("out_dim,in_dim", [(2, 3), (7, 64), (5, 100), (3, 33), (2688, 896),
                                            (896, 896), (4096, 256), (1031, 2048)])
def test_matmul_i8_bit_exact(ops, oracle_lib, out_dim, in_dim):
    import torch
    rng = np.random.default_rng(out_dim * 7 + in_dim)
    w = rng.integers(-127, 128, out_dim * in_dim).astype(np.int8)
    ws = rng.uniform(1e-4, 1e-2, out_dim).astype(np.float32)
    x = rng.standard_normal(in_dim).astype(np.float32)
    ref = oracle_lib.matmul_i8(w, ws, x, out_dim, in_dim)
    out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    ops.matmul_int8(out, _t(w), _t(ws), _t(x), out_dim, in_dim)
    torch.cuda.synchronize()
    assert (_bits(out.cpu().numpy()) == _bits(ref)).all()


def test_matmul_i8_reference_kat(ops):
    # src/tensor/tests.rs:34-49
    import torch
    w = np.array([127, 0, 0, 0, 127, 0], np.int8)
    out = torch.empty(2, dtype=torch.float32, device="cuda")
    ops.matmul_int8(out, _t(w), _t(np.full(2, 1 / 127, np.float32)),
                    _t(np.array([1.0, 2.0, 3.0], np.float32)), 2, 3)
    o = out.cpu().numpy()
    assert abs(o[0] - 1.0) < 0.1 and abs(o[1] - 2.0) < 0.1


@pytest.mark.parametrize("out_dim,in_dim,group", [(2, 64, 64), (9728, 896, 32), (896, 4864, 32),
                                                  (100, 128, 64), (7, 100, 32), (5, 33, 32),
                                                  (64, 2048, 32), (33, 5632, 32), (16, 256, 128)])
def test_matmul_i4_bit_exact(ops, oracle_lib, out_dim, in_dim, group):
    import torch
    rng = np.random.default_rng(out_dim + in_dim + group)
    prow, ng = (in_dim + 1) // 2, (in_dim + group - 1) // group
    wp = rng.integers(0, 256, out_dim * prow).astype(np.uint8)
    s = rng.uniform(1e-3, 1e-2, out_dim * ng).astype(np.float32)
    x = rng.standard_normal(in_dim).astype(np.float32)
    ref = oracle_lib.matmul_i4(wp, s, x, out_dim, in_dim, group)
    out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    ops.matmul_int4(out, _t(wp), _t(s), _t(x), out_dim, in_dim, group)
    torch.cuda.synchronize()
    assert (_bits(out.cpu().numpy()) == _bits(ref)).all()


def test_matmul_i4_reference_kat(ops, oracle_lib):
    # src/tensor/tests.rs:105-127 with its exact value
    import torch
    pk, z = oracle_lib.pack_int4(7, 7), oracle_lib.pack_int4(0, 0)
    w = np.array([pk] * 32 + [z] * 32, np.uint8)
    s = np.full(2, np.float32(1) / np.float32(7), np.float32)
    out = torch.empty(2, dtype=torch.float32, device="cuda")
    ops.matmul_int4(out, _t(w), _t(s), _t(np.ones(64, np.float32)), 2, 64, 64)
    o = out.cpu().numpy()
    assert o[0] == np.float32(np.float32(np.float32(56896) * s[0]) * (np.float32(1) / np.float32(127)))
    assert o[1] == 0.0


@pytest.mark.parametrize("n", [1, 5, 8, 13, 64, 896, 4864])
def test_quantize_i8_bit_exact(ops, oracle_lib, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((3, n)) * rng.uniform(0.1, 10)).astype(np.float32)
    q, s = ops.quantize_f32_to_i8(_t(x))
    q, s = q.cpu().numpy(), s.cpu().numpy()
    for v in range(3):
        rq, rs = oracle_lib.quantize_i8(x[v])
        assert (q[v] == rq).all() and _bits(s[v]) == _bits(rs)


def test_quantize_i8_reference_kat(ops):
    q, s = ops.quantize_f32_to_i8(_t(np.array([[1.0, 0.5, -0.5, 0.0, -1.0]], np.float32)))
    q = q.cpu().numpy()[0]
    assert q[0] == 127 and q[4] == -127  # src/tensor/tests.rs:22-31


@pytest.mark.parametrize("E,dim,k", [(8, 896, 2), (16, 2048, 2), (8, 256, 2), (4, 64, 2), (8, 200, 3)])
def test_router_topk_bit_exact(ops, oracle_lib, E, dim, k):
    rng = np.random.default_rng(E * dim)
    T = 64
    x = rng.standard_normal((T, dim)).astype(np.float32)
    w = (rng.standard_normal((E, dim)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(E) * 0.01).astype(np.float32)
    idx, wt = ops.router_top_k(_t(x), _t(w), _t(b), k)
    idx, wt = idx.cpu().numpy(), wt.cpu().numpy()
    for t in range(T):
        logits = np.array([b[e] + oracle_lib.dot_f32(w[e], x[t]) for e in range(E)], np.float32)
        ri, rw = oracle_lib.softmax_top_k(logits, k)
        assert idx[t].tolist() == ri.tolist()
        # fast_exp on whole 8-chunks, the restated glibc expf on the tail: bit-exact
        assert (_bits(wt[t]) == _bits(rw)).all()


def test_router_topk_reference_kat(ops):
    # src/tensor/tests.rs:130-138 via a router whose logits are the scores
    x = np.ones((1, 16), np.float32)
    w = np.zeros((4, 16), np.float32)
    b = np.array([1.0, 3.0, 2.0, 0.5], np.float32)
    idx, wt = ops.router_top_k(_t(x), _t(w), _t(b), 2)
    assert idx.cpu().numpy()[0].tolist() == [1, 2]
    assert abs(float(wt.sum()) - 1.0) < 1e-5


def test_bad_arguments_raise(chalot, ops):
    import torch
    out = torch.empty(2, dtype=torch.float32, device="cuda")
    w = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = torch.ones(4, dtype=torch.float32, device="cuda")
    x = torch.ones(64, dtype=torch.float32, device="cuda")
    with pytest.raises(chalot.ChalotError):
        ops.matmul_int4(out, w, s, x, 2, 64, 33)  # odd group
    with pytest.raises(ValueError):
        ops.matmul_int8(out, torch.zeros(3, dtype=torch.int8, device="cuda"), s, x, 2, 64)


def test_device_division_is_ieee_exact(chalot):
    """The kernels' fast division (reciprocal approximation + Newton step + two
    fma remainder corrections) against the compiler's IEEE division, bit for
    bit, on 2^30 pairs over 80 binades and the decode path's divisors."""
    import ctypes as C

    from chalot_c1_b200._capi import check, lib
    bad = C.c_uint64()
    ex = (C.c_float * 2)()
    check(lib().chalot_selftest_division(1 << 30, 12345, C.byref(bad), ex))
    assert bad.value == 0, (bad.value, ex[0], ex[1])
