"""Host-side pieces of the batched MoE layer: the synthetic layer quantizer,
the workspace-size query and descriptor checks (no GPU needed)."""
import ctypes as C
import math

import numpy as np
import pytest


def _scalar_i4(row, group):
    # quantize_f32_to_i4's rule per group (src/tensor/quantization.rs:131-162)
    q, s = [], []
    for g0 in range(0, len(row), group):
        blk = row[g0:g0 + group]
        amax = max(float(np.max(np.abs(blk))), float(np.float32(1e-12)))
        sc = np.float32(np.float32(amax) / np.float32(7))
        inv = np.float32(np.float32(1) / sc)
        s.append(sc)
        for v in blk:
            p = float(np.float32(np.float32(v) * inv))
            r = math.floor(abs(p) + 0.5) * (1 if p >= 0 else -1)
            q.append(min(max(r, -8), 7))
    return q, s


def test_quantize_i4_rows_matches_scalar_rule(chalot):
    from chalot_c1_b200.moe import quantize_i4_rows
    rng = np.random.default_rng(0)
    w = rng.standard_normal((5, 128), dtype=np.float32)
    w[0, :32] = np.arange(32, dtype=np.float32) * np.float32(0.5) - 8  # ties at .5 after scaling
    w[1, :32] = 0.0                                                     # all-zero group
    packed, scales = quantize_i4_rows(w, 32)
    for r in range(w.shape[0]):
        q, s = _scalar_i4(w[r], 32)
        assert np.array_equal(scales[r], np.array(s, np.float32))
        lo = (packed[r] & 0x0F).astype(int) - 8
        hi = (packed[r] >> 4).astype(int) - 8
        got = np.empty(128, int)
        got[0::2], got[1::2] = lo, hi
        assert got.tolist() == q


def test_synthetic_layer_layout(chalot):
    from chalot_c1_b200.moe import synthetic_moe_layer
    L = synthetic_moe_layer(256, 1024, 8, 2, 32, seed=0)
    # weight_index.rs:211-246 arithmetic: 491,520 bytes per tiny expert
    assert L.expert_bytes == 491520
    assert L.experts.size == 8 * L.expert_bytes
    assert L.layer_bytes().size == 8 * 256 * 4 + 8 * 4 + 8 * 491520


def test_workspace_size_and_checks(chalot):
    from chalot_c1_b200._capi import MoeDesc, lib
    d = MoeDesc(896, 4864, 8, 2, 32, 16, 16, 16)
    n = lib().chalot_moe_workspace_size(C.byref(d), 4096)
    # at least h f32, h int8 and y f32 for every (token, choice) slot
    assert n >= 4096 * 2 * (4864 * 5 + 896 * 4)
    assert lib().chalot_moe_workspace_size(C.byref(d), 1) < n
    for field, val in (("group", 48), ("n_experts", 1), ("top_k", 9), ("dim", 900)):
        bad = MoeDesc.from_buffer_copy(d)
        setattr(bad, field, val)
        assert lib().chalot_moe_workspace_size(C.byref(bad), 16) == 0
        assert b"moe_layer" in lib().chalot_last_error()
    bad = MoeDesc.from_buffer_copy(d)
    bad.experts = 8  # not 16-byte aligned
    assert lib().chalot_moe_workspace_size(C.byref(bad), 16) == 0


def test_oracle_moe_forward_routes_like_router(oracle_lib):
    from chalot_c1_b200.moe import synthetic_moe_layer
    L = synthetic_moe_layer(256, 256, 4, 2, 32, seed=1)
    x = np.random.default_rng(2).standard_normal((3, 256), dtype=np.float32)
    out, sel = oracle_lib.moe_forward(x, L.layer_bytes(), 256, 256, 4, 2, 32)
    for t in range(3):
        logits = np.array([L.router_b[e] + oracle_lib.dot_f32(L.router_w[e], x[t]) for e in range(4)],
                          np.float32)
        idx, _ = oracle_lib.softmax_top_k(logits, 2)
        assert list(sel[t]) == list(idx)
    assert np.isfinite(out).all()
