"""ctypes binding of ``libchalot_b200.so`` (declarations: include/chalot_b200.h).

The library is the product: there is no Python or CPU fallback. Importing this
module raises if the library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("CHALOT_LIB") or os.path.join(_PKG, "_lib", "libchalot_b200.so")

CHALOT_OK = 0
ERRORS = {-1: "CHALOT_ERR_ARG", -2: "CHALOT_ERR_IO", -3: "CHALOT_ERR_FORMAT",
          -4: "CHALOT_ERR_OOM", -5: "CHALOT_ERR_CUDA", -6: "CHALOT_ERR_NCCL",
          -7: "CHALOT_ERR_TIMEOUT", -8: "CHALOT_ERR_STATE"}


class ChalotError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class SynthSpec(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("hidden_dim", C.c_uint32), ("n_layers", C.c_uint32),
                ("n_heads", C.c_uint32), ("vocab_size", C.c_uint32), ("n_experts", C.c_uint32),
                ("top_k", C.c_uint32), ("int4_group_size", C.c_uint32),
                ("max_seq_len", C.c_uint32), ("rope_theta_x100", C.c_uint32),
                ("weight_std", C.c_float), ("seed", C.c_uint64), ("n_threads", C.c_int)]


class ModelConfig(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("hidden_dim", C.c_uint32), ("n_layers", C.c_uint32),
                ("n_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab_size", C.c_uint32),
                ("max_seq_len", C.c_uint32), ("n_experts", C.c_uint32), ("top_k", C.c_uint32),
                ("int4_group_size", C.c_uint32), ("depth_router_layer", C.c_uint32),
                ("rope_theta", C.c_float), ("total_bytes", C.c_uint64),
                ("expert_bytes", C.c_uint64)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class Opts(C.Structure):
    _fields_ = [("device", C.c_int), ("use_cuda_graph", C.c_int)]


class Sampling(C.Structure):
    _fields_ = [("strategy", C.c_int), ("temperature", C.c_float), ("top_k", C.c_uint32),
                ("top_p", C.c_float), ("min_p", C.c_float), ("repetition_penalty", C.c_float),
                ("repetition_window", C.c_uint32), ("stop_tokens", C.POINTER(C.c_uint32)),
                ("n_stop_tokens", C.c_uint32), ("seed", C.c_uint64)]


class MoeDesc(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("hidden_dim", C.c_uint32), ("n_experts", C.c_uint32),
                ("top_k", C.c_uint32), ("group", C.c_uint32), ("router_w", C.c_void_p),
                ("router_b", C.c_void_p), ("experts", C.c_void_p)]


class PagedKV(C.Structure):
    _fields_ = [("n_pages", C.c_uint32), ("page_tokens", C.c_uint32), ("n_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("data", C.c_void_p), ("scales", C.c_void_p)]


# name -> (restype, argtypes); every function include/chalot_b200.h declares
P = C.c_void_p
SIGNATURES = {
    "chalot_last_error": (C.c_char_p, []),
    "chalot_abi_version": (C.c_int, []),
    "chalot_device_status": (C.c_int, [C.c_void_p]),
    "chalot_ep_comm_create": (C.c_int, [C.c_uint32, C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]),
    "chalot_ep_comm_connect": (C.c_int, [C.c_void_p, C.c_void_p]),
    "chalot_ep_comm_free": (None, [C.c_void_p]),
    "chalot_moe_layer_ep": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p]),
    "chalot_selftest_division": (C.c_int, [C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p]),
    "chalot_decode_trace": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "chalot_myai_write_synthetic": (C.c_int, [C.c_char_p, C.POINTER(SynthSpec)]),
    "chalot_myai_inspect": (C.c_int, [C.c_char_p, C.POINTER(ModelConfig)]),
    "chalot_load": (C.c_int, [C.c_char_p, C.POINTER(Opts), C.POINTER(P)]),
    "chalot_free": (None, [P]),
    "chalot_get_config": (C.c_int, [P, C.POINTER(ModelConfig)]),
    "chalot_forward": (C.c_int, [P, C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32)]),
    "chalot_generate": (C.c_int, [P, P, C.c_size_t, C.c_size_t, C.POINTER(Sampling), P,
                                  C.POINTER(C.c_size_t)]),
    "chalot_sample_from_logits": (C.c_int, [P, C.POINTER(Sampling), P, C.c_size_t,
                                            C.POINTER(C.c_uint32)]),
    "chalot_get_logits": (C.c_int, [P, P, C.c_size_t]),
    "chalot_sample": (C.c_int, [P, C.c_size_t, C.POINTER(Sampling), C.c_float, C.POINTER(C.c_uint32), P]),
    "chalot_batch_reserve": (C.c_int, [P, C.c_uint32]),
    "chalot_forward_batch": (C.c_int, [P, P, P, P, C.c_uint32, P]),
    "chalot_get_batch_logits": (C.c_int, [P, C.c_uint32, P, C.c_size_t]),
    "chalot_batch_reserve_paged": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32]),
    "chalot_batch_release": (C.c_int, [P, C.c_uint32]),
    "chalot_batch_capacity": (C.c_int, [P, C.POINTER(C.c_uint32)]),
    "chalot_batch_kv_pages": (C.c_int, [P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "chalot_sched_create": (C.c_int, [P, C.c_uint32, C.POINTER(P)]),
    "chalot_sched_free": (None, [P]),
    "chalot_sched_submit": (C.c_int, [P, P, C.c_size_t, C.c_uint32, P, C.c_size_t, C.POINTER(C.c_uint64)]),
    "chalot_sched_step": (C.c_int, [P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "chalot_sched_poll": (C.c_int, [P, C.c_uint64, P, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(C.c_int)]),
    "chalot_probe_int8_mma": (C.c_int, [C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "chalot_myai_validate": (C.c_int, [C.c_char_p, C.c_char_p, C.c_size_t]),
    "chalot_ep_nccl_id": (C.c_int, [P]),
    "chalot_ep_attach_nccl": (C.c_int, [P, C.c_uint32, C.c_uint32, P]),
    "chalot_ep_hub_create": (P, [C.c_uint32]),
    "chalot_ep_hub_free": (None, [P]),
    "chalot_ep_attach_hub": (C.c_int, [P, P, C.c_uint32]),
    "chalot_ep_detach": (C.c_int, [P]),
    "chalot_last_timing": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                     C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "chalot_bench_moe_layers": (C.c_int, [P, C.c_int, C.POINTER(C.c_double),
                                          C.POINTER(C.c_double)]),
    "chalot_profile_forward": (C.c_int, [P, C.c_uint32, C.c_uint32, P, C.c_int,
                                         C.POINTER(C.c_int)]),
    "chalot_matmul_i8": (C.c_int, [P, P, P, P, C.c_size_t, C.c_size_t, P]),
    "chalot_matmul_i4": (C.c_int, [P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, P]),
    "chalot_quantize_i8": (C.c_int, [P, P, P, C.c_size_t, C.c_size_t, P]),
    "chalot_router_topk": (C.c_int, [P, P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t,
                                     C.c_size_t, P]),
    "chalot_moe_workspace_size": (C.c_size_t, [C.POINTER(MoeDesc), C.c_size_t]),
    "chalot_moe_layer": (C.c_int, [C.POINTER(MoeDesc), P, C.c_size_t, P, P, P, P, C.c_size_t, P]),
    "chalot_moe_layer_noalloc": (C.c_int, [C.POINTER(MoeDesc), P, C.c_size_t, P, P, P, P]),
    "chalot_moe_route": (C.c_int, [C.POINTER(MoeDesc), P, C.c_size_t, P, P, P, P, P]),
    "chalot_moe_plan": (C.c_int, [P, C.c_size_t, C.c_uint32, C.c_uint32, P, P, P, P]),
    "chalot_moe_gather": (C.c_int, [P, P, P, C.c_size_t, C.c_uint32, C.c_size_t, P, P, P]),
    "chalot_moe_experts_workspace_size": (C.c_size_t, [C.POINTER(MoeDesc), C.c_size_t]),
    "chalot_moe_experts": (C.c_int, [C.POINTER(MoeDesc), P, P, P, C.c_size_t, P, P, C.c_size_t, P]),
    "chalot_moe_combine": (C.c_int, [P, P, P, C.c_size_t, C.c_uint32, C.c_size_t, P, P]),
    "chalot_kv_create": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.POINTER(P)]),
    "chalot_kv_free": (None, [P]),
    "chalot_kv_write": (C.c_int, [P, C.c_uint32, C.c_uint32, P, P]),
    "chalot_kv_read": (C.c_int, [P, C.c_uint32, C.c_uint32, P, P, C.POINTER(C.c_int)]),
    "chalot_kv_write_batch": (C.c_int, [P, C.c_uint32, P, C.c_size_t, P, P, P]),
    "chalot_kv_gather": (C.c_int, [P, C.c_uint32, P, C.c_size_t, P, P, P, P]),
    "chalot_kv_clear": (C.c_int, [P]),
    "chalot_kv_active_pages": (C.c_size_t, [P]),
    "chalot_kv_memory_mb": (C.c_float, [P]),
    "chalot_paged_kv_store": (C.c_int, [C.POINTER(PagedKV), P, C.c_size_t, P, P, P]),
    "chalot_paged_attention_workspace_size": (C.c_size_t, [C.POINTER(PagedKV), C.c_size_t, C.c_size_t]),
    "chalot_paged_attention": (C.c_int, [C.POINTER(PagedKV), P, C.c_size_t, P, C.c_size_t, P, P, P,
                                         C.c_size_t, P]),
}

_lib = None


def lib():
    """Loads the library once; raises when it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with "
                              f"`python -m chalot_c1_b200.build` (there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != CHALOT_OK:
        raise ChalotError(rc, lib().chalot_last_error().decode())
