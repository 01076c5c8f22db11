"""Operator entry points over caller-owned device memory.

Python mirrors of the reference's tensor API (src/tensor/mod.rs re-exports):
``matmul_int8`` (matmul.rs:47), ``matmul_int4`` (matmul.rs:363),
``quantize_f32_to_i8`` (quantization.rs:26) and the MoE router's
``softmax_top_k`` (normalization.rs:203 with engine.rs:334-341). Arguments are
CUDA torch tensors; the work runs in the B200 library on the current stream.
"""
from __future__ import annotations

import torch

from ._capi import check, lib


def _ptr(t: torch.Tensor):
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def matmul_int8(out: torch.Tensor, w: torch.Tensor, w_scales: torch.Tensor, x: torch.Tensor,
                out_dim: int, in_dim: int) -> None:
    if w.numel() < out_dim * in_dim or w_scales.numel() < out_dim or x.numel() < in_dim \
            or out.numel() < out_dim:
        raise ValueError("matmul_int8: buffer shorter than its dimensions")  # matmul.rs:55-58
    check(lib().chalot_matmul_i8(_ptr(out), _ptr(w), _ptr(w_scales), _ptr(x), out_dim, in_dim,
                                 _stream()))


def matmul_int4(out: torch.Tensor, w_packed: torch.Tensor, w_scales: torch.Tensor,
                x: torch.Tensor, out_dim: int, in_dim: int, group_size: int) -> None:
    g = group_size or 64
    ng, prow = (in_dim + g - 1) // g, (in_dim + 1) // 2
    if w_packed.numel() < out_dim * prow or w_scales.numel() < out_dim * ng \
            or x.numel() < in_dim or out.numel() < out_dim:
        raise ValueError("matmul_int4: buffer shorter than its dimensions")  # matmul.rs:376-379
    check(lib().chalot_matmul_i4(_ptr(out), _ptr(w_packed), _ptr(w_scales), _ptr(x), out_dim,
                                 in_dim, group_size, _stream()))


def quantize_f32_to_i8(x: torch.Tensor):
    """Per-vector (last dimension) quantization; returns (q int8, scale f32)."""
    n = x.shape[-1]
    nv = x.numel() // max(n, 1)
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(nv, dtype=torch.float32, device=x.device)
    check(lib().chalot_quantize_i8(_ptr(q), _ptr(s), _ptr(x), nv, n, _stream()))
    return q, s


def router_top_k(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, top_k: int):
    """Router logits b + W x per token and softmax_top_k: (idx int32, weight f32)."""
    T, dim = x.shape
    E = w.shape[0]
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    wt = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    check(lib().chalot_router_topk(_ptr(idx), _ptr(wt), _ptr(x), _ptr(w), _ptr(b), T, dim, E,
                                   top_k, _stream()))
    return idx, wt


def probe_int8_mma(iters: int = 20000) -> dict:
    """Measured int8 tensor-core peak of the current device (chalot_probe_int8_mma):
    one CTA per SM streams tcgen05.mma.kind::i8 out of shared memory."""
    import ctypes as C
    tops, ms = C.c_double(), C.c_double()
    check(lib().chalot_probe_int8_mma(iters, C.byref(tops), C.byref(ms)))
    return {"tops": tops.value, "ms": ms.value, "iters": iters}


def device_status(stream=None) -> None:
    """chalot_device_status: synchronises `stream` (default: the current
    stream) and raises ChalotError if a device-side check of earlier operator
    work failed (a bounded wait that gave up, a page id outside a pool). The
    next operator call on the device raises the same error once that work has
    finished, without this call."""
    s = _stream() if stream is None else stream
    check(lib().chalot_device_status(s))
