"""Batched MoE layer: synthetic layer weights in the .myai layout and the
``chalot_moe_layer`` entry point on CUDA tensors.

A layer is stored as a .myai file stores it (src/model/weight_index.rs:126-160):
router W [E][dim] f32, b [E] f32, then E experts back to back, each
{gate+up packed int4 [2H][dim/2], scales [2H][dim/group], down packed
[dim][H/2], scales [dim][H/group]}.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._capi import MoeDesc, check, lib


def quantize_i4_rows(w: np.ndarray, group: int):
    """Per-row, per-group int4 quantization (scale = absmax/7, round half away
    from zero, clamp [-8, 7]; the rule of quantize_f32_to_i4,
    src/tensor/quantization.rs:131-162, applied per group), packed two per byte
    with the even column in the low nibble (quantization.rs:114-126)."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    assert cols % group == 0 and cols % 2 == 0
    g = w.reshape(rows, cols // group, group)
    amax = np.maximum(np.abs(g).max(axis=2), np.float32(1e-12)).astype(np.float32)
    scale = (amax / np.float32(7)).astype(np.float32)
    inv = (np.float32(1) / scale).astype(np.float32)
    v = (g * inv[:, :, None]).astype(np.float32).astype(np.float64)
    q = np.clip(np.trunc(v + np.copysign(0.5, v)), -8, 7).astype(np.int16).reshape(rows, cols)
    nib = (q + 8).astype(np.uint8) & 0x0F
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    return packed, scale.reshape(rows, cols // group)


@dataclass
class SyntheticMoeLayer:
    dim: int
    hidden: int
    n_experts: int
    top_k: int
    group: int
    router_w: np.ndarray   # [E][dim] f32
    router_b: np.ndarray   # [E] f32
    experts: np.ndarray    # uint8, E experts back to back

    @property
    def expert_bytes(self) -> int:
        d, h, g = self.dim, self.hidden, self.group
        return 2 * h * (d // 2) + 2 * h * (d // g) * 4 + d * (h // 2) + d * (h // g) * 4

    def layer_bytes(self) -> np.ndarray:
        """Router weights followed by the experts, as one .myai layer region."""
        return np.concatenate([self.router_w.reshape(-1).view(np.uint8),
                               self.router_b.view(np.uint8), self.experts])


def synthetic_moe_layer(dim: int, hidden: int, n_experts: int, top_k: int = 2, group: int = 32,
                        seed: int = 3, std: float = 0.02) -> SyntheticMoeLayer:
    """Router W ~ N(0, std), b = 0; expert weights ~ N(0, std) quantized to int4."""
    rng = np.random.default_rng(seed)
    rw = (rng.standard_normal((n_experts, dim), dtype=np.float32) * np.float32(std)).astype(np.float32)
    rb = np.zeros(n_experts, np.float32)
    parts = []
    for _ in range(n_experts):
        gu = rng.standard_normal((2 * hidden, dim), dtype=np.float32) * np.float32(std)
        gp, gs = quantize_i4_rows(gu, group)
        dn = rng.standard_normal((dim, hidden), dtype=np.float32) * np.float32(std)
        dp, ds = quantize_i4_rows(dn, group)
        parts += [gp.reshape(-1), gs.reshape(-1).view(np.uint8), dp.reshape(-1),
                  ds.reshape(-1).view(np.uint8)]
    return SyntheticMoeLayer(dim, hidden, n_experts, top_k, group, rw, rb, np.concatenate(parts))


class MoeLayer:
    """Device copy of one MoE layer plus a workspace sized for up to
    ``max_tokens`` tokens; ``__call__`` runs chalot_moe_layer on the current
    torch stream."""

    def __init__(self, layer: SyntheticMoeLayer, max_tokens: int, device="cuda"):
        import torch
        self.layer = layer
        self.router_w = torch.from_numpy(layer.router_w).to(device)
        self.router_b = torch.from_numpy(layer.router_b).to(device)
        self.experts = torch.from_numpy(layer.experts).to(device)
        self.desc = MoeDesc(layer.dim, layer.hidden, layer.n_experts, layer.top_k, layer.group,
                            self.router_w.data_ptr(), self.router_b.data_ptr(),
                            self.experts.data_ptr())
        self.max_tokens = max_tokens
        n = self.workspace_size(max_tokens)
        self.workspace = torch.empty(n, dtype=torch.uint8, device=device)

    def workspace_size(self, n_tok: int) -> int:
        n = lib().chalot_moe_workspace_size(C.byref(self.desc), n_tok)
        if n == 0:
            check(-1)
        return n

    def __call__(self, x, out=None, sel=None, selw=None):
        import torch
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > workspace capacity {self.max_tokens}")
        if out is None:
            out = torch.empty((T, self.layer.dim), dtype=torch.float32, device=x.device)
        if sel is None:
            sel = torch.empty((T, self.layer.top_k), dtype=torch.int32, device=x.device)
        if selw is None:
            selw = torch.empty((T, self.layer.top_k), dtype=torch.float32, device=x.device)
        check(lib().chalot_moe_layer(C.byref(self.desc), x.data_ptr(), T, out.data_ptr(),
                                     sel.data_ptr(), selw.data_ptr(), self.workspace.data_ptr(),
                                     self.workspace.numel(),
                                     torch.cuda.current_stream().cuda_stream))
        return out, sel, selw
