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


class PagedKVCache:
    """PagedKVCache (src/model/memory.rs:100-201) on the device: ``new``,
    ``write``, ``read``, ``clear``, ``active_pages``, ``memory_mb`` with the
    reference's page size, quantization and LRU eviction; ``write_batch`` and
    ``gather`` move many rows of device memory at once."""

    def __init__(self, kv_dim: int, n_layers: int, max_pages_per_layer: int = 16, device: int = 0):
        from ._capi import check, lib
        self.dim = kv_dim
        h = C.c_void_p()
        check(lib().chalot_kv_create(kv_dim, n_layers, max_pages_per_layer, device, C.byref(h)))
        self._h = h

    @classmethod
    def new(cls, kv_dim: int, n_layers: int) -> "PagedKVCache":
        return cls(kv_dim, n_layers)

    def write(self, layer: int, pos: int, k, v) -> None:
        import numpy as np
        from ._capi import check, lib
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        if k.size < self.dim or v.size < self.dim:
            raise ValueError("k and v must hold kv_dim values")
        check(lib().chalot_kv_write(self._h, layer, pos, k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p)))

    def read(self, layer: int, pos: int, k_out, v_out) -> bool:
        from ._capi import check, lib
        f = C.c_int()
        check(lib().chalot_kv_read(self._h, layer, pos, k_out.ctypes.data_as(C.c_void_p),
                                   v_out.ctypes.data_as(C.c_void_p), C.byref(f)))
        return bool(f.value)

    def write_batch(self, layer: int, pos, k, v) -> None:
        import numpy as np
        import torch
        from ._capi import check, lib
        p = np.ascontiguousarray(pos, np.uint32)
        check(lib().chalot_kv_write_batch(self._h, layer, p.ctypes.data_as(C.c_void_p), p.size, k.data_ptr(),
                                          v.data_ptr(), torch.cuda.current_stream().cuda_stream))

    def gather(self, layer: int, pos, k_out, v_out):
        import numpy as np
        import torch
        from ._capi import check, lib
        p = np.ascontiguousarray(pos, np.uint32)
        found = np.zeros(p.size, np.uint8)
        check(lib().chalot_kv_gather(self._h, layer, p.ctypes.data_as(C.c_void_p), p.size, k_out.data_ptr(),
                                     v_out.data_ptr(), found.ctypes.data_as(C.c_void_p),
                                     torch.cuda.current_stream().cuda_stream))
        return found.astype(bool)

    def clear(self) -> None:
        from ._capi import check, lib
        check(lib().chalot_kv_clear(self._h))

    def active_pages(self) -> int:
        from ._capi import lib
        return int(lib().chalot_kv_active_pages(self._h))

    def memory_mb(self) -> float:
        from ._capi import lib
        return float(lib().chalot_kv_memory_mb(self._h))

    def close(self) -> None:
        from ._capi import lib
        if getattr(self, "_h", None):
            lib().chalot_kv_free(self._h)
            self._h = None

    def __del__(self):
        self.close()
