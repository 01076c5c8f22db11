"""chalot_moe_layer_noalloc: the MoE layer entry point that allocates nothing.

It serves callers that cannot hand the library device memory for scratch (a
host whose allocator owns the whole device budget, or an FFI host that binds
only plain pointers): its scratch is a fixed array inside the library. These
tests call it through the C ABI and check it against chalot_moe_layer, the
entry point that takes a caller workspace, to the bit (the tolerance of every
MoE layer test), on two calls in a row whose sizes and inputs differ, so
leftovers of the first call in the shared array cannot leak into the second.

The file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DIM, HIDDEN, E, K = 896, 4864, 8, 2


def _noalloc(desc, x, out, sel, selw):
    import torch
    from chalot_c1_b200._capi import check, lib
    check(lib().chalot_moe_layer_noalloc(C.byref(desc), x.data_ptr(), x.shape[0], out.data_ptr(),
                                         sel.data_ptr(), selw.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_workspace_entry_point(chalot):
    import torch
    from chalot_c1_b200 import moe
    layer = moe.synthetic_moe_layer(DIM, HIDDEN, E, K, 32, seed=11)
    dev = moe.MoeLayer(layer, max_tokens=64)
    assert dev.workspace_size(64) <= 4 << 20
    rng = np.random.default_rng(12)
    for T in (64, 17):  # two calls in a row
        x = torch.from_numpy(rng.standard_normal((T, DIM), dtype=np.float32)).cuda()
        ref_out, ref_sel, ref_w = dev(x)
        out = torch.full_like(ref_out, float("nan"))
        sel = torch.full_like(ref_sel, -1)
        selw = torch.full_like(ref_w, float("nan"))
        _noalloc(dev.desc, x, out, sel, selw)
        torch.cuda.synchronize()
        assert torch.equal(sel, ref_sel), T
        assert torch.equal(selw.view(torch.int32), ref_w.view(torch.int32)), T
        assert torch.equal(out.view(torch.int32), ref_out.view(torch.int32)), T


def test_noalloc_sized_by_its_own_path_when_tc_is_forced(chalot, monkeypatch):
    """CHALOT_MOE_PATH=tc makes chalot_moe_layer's workspace include the
    tensor-core buffers; this entry point runs the tile-GEMM path only, so a
    1-token call still fits its scratch and matches."""
    import torch
    from chalot_c1_b200 import moe
    layer = moe.synthetic_moe_layer(DIM, HIDDEN, E, K, 32, seed=14)
    dev = moe.MoeLayer(layer, max_tokens=8)
    x = torch.from_numpy(np.random.default_rng(15).standard_normal((1, DIM), dtype=np.float32)).cuda()
    ref_out, ref_sel, ref_w = dev(x)
    monkeypatch.setenv("CHALOT_MOE_PATH", "tc")
    out = torch.full_like(ref_out, float("nan"))
    sel = torch.full_like(ref_sel, -1)
    selw = torch.full_like(ref_w, float("nan"))
    _noalloc(dev.desc, x, out, sel, selw)
    torch.cuda.synchronize()
    assert torch.equal(sel, ref_sel)
    assert torch.equal(out.view(torch.int32), ref_out.view(torch.int32))


def test_noalloc_rejects_sizes_beyond_its_scratch(chalot):
    import torch
    from chalot_c1_b200 import moe
    from chalot_c1_b200._capi import ChalotError
    layer = moe.synthetic_moe_layer(DIM, HIDDEN, E, K, 32, seed=13)
    dev = moe.MoeLayer(layer, max_tokens=1)
    T = 4096  # needs ~230 MB of scratch
    x = torch.zeros((T, DIM), device="cuda")
    out = torch.empty((T, DIM), device="cuda")
    sel = torch.empty((T, K), dtype=torch.int32, device="cuda")
    selw = torch.empty((T, K), device="cuda")
    with pytest.raises(ChalotError, match="scratch"):
        _noalloc(dev.desc, x, out, sel, selw)
