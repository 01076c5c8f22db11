"""chalot_moe_layer (router + dispatch + int4 SwiGLU experts + combine for T
tokens) against the oracle's per-token expert block (engine.rs:334-401).

Bar: bit-exact outputs and identical router choices. Every int32 group dot is
exact and each f32 epilogue keeps the reference's order, so the batched,
expert-sorted GPU path must reproduce the per-token CPU arithmetic to the bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # dim, hidden, E, K, group, T
    (256, 1024, 8, 2, 32, 1),
    (256, 1024, 8, 2, 32, 7),
    (256, 1024, 8, 2, 32, 100),
    (256, 512, 4, 1, 64, 33),
    (256, 512, 6, 3, 128, 65),
    (896, 4864, 8, 2, 32, 64),
    (2048, 5632, 16, 2, 32, 24),
]


@pytest.fixture(scope="module")
def moe(chalot):
    from chalot_c1_b200 import moe
    return moe


def _run(moe, oracle_lib, dim, hidden, E, K, group, T, seed):
    import torch
    layer = moe.synthetic_moe_layer(dim, hidden, E, K, group, seed=seed)
    x = np.random.default_rng(seed + 100).standard_normal((T, dim), dtype=np.float32)
    ref, ref_sel = oracle_lib.moe_forward(x, layer.layer_bytes(), dim, hidden, E, K, group,
                                          threads=oracle_lib.hw_threads())
    dev = moe.MoeLayer(layer, max_tokens=T)
    out, sel, selw = dev(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    return ref, ref_sel, out.cpu().numpy(), sel.cpu().numpy(), selw.cpu().numpy()


@pytest.mark.parametrize("dim,hidden,E,K,group,T", CASES)
def test_moe_layer_bit_exact(moe, oracle_lib, dim, hidden, E, K, group, T):
    ref, ref_sel, out, sel, selw = _run(moe, oracle_lib, dim, hidden, E, K, group, T, seed=T + E)
    assert (sel == ref_sel).all()
    assert (selw > 0).all() and np.allclose(selw.sum(1), 1.0, atol=1e-5)
    assert (out.view(np.uint32) == ref.view(np.uint32)).all()


def test_moe_layer_skewed_routing(moe, oracle_lib):
    # a router bias that sends every token to experts 3 and 5: one expert holds
    # all slots, the others none (empty experts, many 32-slot blocks per expert)
    import torch
    dim, hidden, E, K, T = 256, 512, 8, 2, 300
    layer = moe.synthetic_moe_layer(dim, hidden, E, K, 32, seed=9)
    layer.router_b[:] = 0
    layer.router_b[3], layer.router_b[5] = 50.0, 40.0
    x = np.random.default_rng(1).standard_normal((T, dim), dtype=np.float32)
    ref, ref_sel = oracle_lib.moe_forward(x, layer.layer_bytes(), dim, hidden, E, K, 32,
                                          threads=oracle_lib.hw_threads())
    out, sel, _ = moe.MoeLayer(layer, T)(torch.from_numpy(x).cuda())
    assert (sel.cpu().numpy() == ref_sel).all()
    assert (ref_sel[:, 0] == 3).all()
    assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()


def test_moe_layer_repeat_and_fewer_tokens(moe, oracle_lib):
    # the workspace is reused across calls of different sizes
    import torch
    dim, hidden, E, K = 256, 1024, 8, 2
    layer = moe.synthetic_moe_layer(dim, hidden, E, K, 32, seed=4)
    dev = moe.MoeLayer(layer, 64)
    for T in (64, 5, 64, 1):
        x = np.random.default_rng(T).standard_normal((T, dim), dtype=np.float32)
        ref, _ = oracle_lib.moe_forward(x, layer.layer_bytes(), dim, hidden, E, K, 32, threads=4)
        out, _, _ = dev(torch.from_numpy(x).cuda())
        assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all(), T


def test_moe_layer_argument_errors(moe, chalot):
    import ctypes as C
    import torch
    from chalot_c1_b200._capi import ChalotError, check, lib
    layer = moe.synthetic_moe_layer(256, 512, 4, 2, 32, seed=0)
    dev = moe.MoeLayer(layer, 8)
    x = torch.zeros((8, 256), device="cuda")
    out = torch.empty((8, 256), device="cuda")
    need = dev.workspace_size(8)
    with pytest.raises(ChalotError, match="workspace too small"):
        check(lib().chalot_moe_layer(C.byref(dev.desc), x.data_ptr(), 8, out.data_ptr(), None, None,
                                     dev.workspace.data_ptr(), need - 1, None))
    bad = type(dev.desc).from_buffer_copy(dev.desc)
    bad.group = 48
    with pytest.raises(ChalotError, match="group"):
        check(lib().chalot_moe_layer(C.byref(bad), x.data_ptr(), 8, out.data_ptr(), None, None,
                                     dev.workspace.data_ptr(), need, None))


# ---- tensor-core path (tcgen05 kind::i8 group dots + f32 group epilogue) ----

TC_CASES = [
    # dim, hidden, E, K, T
    (256, 1024, 8, 2, 1),
    (256, 1024, 8, 2, 100),
    (256, 1024, 8, 2, 700),
    (256, 512, 4, 1, 260),
    (896, 4864, 8, 2, 300),
    (2048, 5632, 16, 2, 64),
]


@pytest.fixture
def tc_path(monkeypatch):
    from chalot_c1_b200 import ops
    monkeypatch.setenv("CHALOT_MOE_PATH", "tc")
    yield
    ops.device_status()  # no tensor-core wait gave up


@pytest.mark.parametrize("dim,hidden,E,K,T", TC_CASES)
def test_moe_layer_tensor_core_bit_exact(moe, oracle_lib, tc_path, dim, hidden, E, K, T):
    ref, ref_sel, out, sel, _ = _run(moe, oracle_lib, dim, hidden, E, K, 32, T, seed=T + 7 * E)
    assert (sel == ref_sel).all()
    assert (out.view(np.uint32) == ref.view(np.uint32)).all()


def test_moe_layer_tensor_core_skewed(moe, oracle_lib, tc_path):
    # every token on experts 3 and 5: several 128-slot blocks of one expert,
    # a partial last block, and experts with no slots at all
    import torch
    dim, hidden, E, K, T = 256, 512, 8, 2, 333
    layer = moe.synthetic_moe_layer(dim, hidden, E, K, 32, seed=19)
    layer.router_b[3], layer.router_b[5] = 50.0, 40.0
    x = np.random.default_rng(3).standard_normal((T, dim), dtype=np.float32)
    ref, ref_sel = oracle_lib.moe_forward(x, layer.layer_bytes(), dim, hidden, E, K, 32,
                                          threads=oracle_lib.hw_threads())
    out, sel, _ = moe.MoeLayer(layer, T)(torch.from_numpy(x).cuda())
    assert (sel.cpu().numpy() == ref_sel).all()
    assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()


def test_moe_layer_paths_agree_at_prefill_size(moe, monkeypatch):
    # 4096 tokens of the Qwen-shaped layer: the tensor-core path against the
    # tile-GEMM path (both bit-exact restatements of the same arithmetic)
    import torch
    layer = moe.synthetic_moe_layer(896, 4864, 8, 2, 32, seed=3)
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((4096, 896), dtype=np.float32)).cuda()
    monkeypatch.setenv("CHALOT_MOE_PATH", "simt")
    a, sa, _ = moe.MoeLayer(layer, 4096)(x)
    monkeypatch.setenv("CHALOT_MOE_PATH", "tc")
    b, sb, _ = moe.MoeLayer(layer, 4096)(x)
    from chalot_c1_b200 import ops
    ops.device_status()
    assert torch.equal(sa, sb)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
