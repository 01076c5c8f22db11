"""Paged int8 KV cache for long-context decode, on CUDA tensors.

``PagedKVPool`` owns a device page pool in the format of
``chalot_paged_kv`` (include/chalot_b200.h): pages of ``page_tokens`` tokens,
K and V blocks of each head int8 with one scale per (page, K|V, head).
``store`` quantizes whole pages; ``attention`` runs the decode-step attention
of Engine::forward (src/model/engine.rs:283-309) over the pages.
"""
from __future__ import annotations

import ctypes as C

from ._capi import PagedKV, check, lib


class PagedKVPool:
    def __init__(self, n_pages: int, page_tokens: int = 16, n_heads: int = 14, head_dim: int = 64,
                 device="cuda"):
        import torch
        self.P, self.H, self.hd = page_tokens, n_heads, head_dim
        self.data = torch.zeros((n_pages, 2, n_heads, page_tokens, head_dim), dtype=torch.int8, device=device)
        self.scales = torch.ones((n_pages, 2, n_heads), dtype=torch.float32, device=device)
        self.desc = PagedKV(n_pages, page_tokens, n_heads, head_dim, self.data.data_ptr(),
                            self.scales.data_ptr())
        self._ws = None

    @property
    def page_bytes(self) -> int:
        return 2 * self.H * self.P * self.hd

    def store(self, page_ids, k, v) -> None:
        """k, v: f32 [n][page_tokens][n_heads][head_dim] CUDA tensors; page_ids int32 CUDA."""
        import torch
        check(lib().chalot_paged_kv_store(C.byref(self.desc), page_ids.data_ptr(), page_ids.numel(),
                                          k.data_ptr(), v.data_ptr(), torch.cuda.current_stream().cuda_stream))

    def workspace(self, n_seq: int, max_pages: int):
        import torch
        n = lib().chalot_paged_attention_workspace_size(C.byref(self.desc), n_seq, max_pages)
        if n == 0:
            check(-1)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.data.device)
        return self._ws

    def attention(self, q, page_table, seq_lens, out=None):
        """q: f32 [n_seq][n_heads][head_dim]; page_table int32 [n_seq][max_pages]; seq_lens int32 [n_seq]."""
        import torch
        n_seq, max_pages = page_table.shape
        if out is None:
            out = torch.empty_like(q)
        ws = self.workspace(n_seq, max_pages)
        check(lib().chalot_paged_attention(C.byref(self.desc), q.data_ptr(), n_seq, page_table.data_ptr(),
                                           max_pages, seq_lens.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                           ws.numel(), torch.cuda.current_stream().cuda_stream))
        return out
