"""ctypes binding of the CPU oracle (``oracle/liboracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference arm, never by the product package.
The library restates chalot_C1's AVX2 CPU path (see ``oracle.cpp``'s header
for the function-by-function citations).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compiles liboracle.so with the committed Makefile (g++, AVX2, no FMA)."""
    csrc = os.path.join(os.path.dirname(_HERE), "chalot_c1_b200", "csrc")
    srcs = [os.path.join(_HERE, f) for f in ("oracle.cpp", "synth_entry.cpp", "Makefile")] + \
        [os.path.join(csrc, f) for f in ("myai.cpp", "myai_synth.cpp", "myai.h")]
    newest = max(os.path.getmtime(p) for p in srcs if os.path.exists(p))
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < newest:
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        L.orc_error.restype = C.c_char_p
        L.orc_load.restype = P
        L.orc_load.argtypes = [C.c_char_p, C.c_int]
        L.orc_free.argtypes = [P]
        L.orc_set_trace.argtypes = [P, C.c_int]
        L.orc_get_trace.restype = C.c_size_t
        L.orc_get_trace.argtypes = [P, C.c_int, P, C.c_size_t]
        L.orc_forward.restype = C.c_long
        L.orc_forward.argtypes = [P, C.c_uint32, C.c_uint32]
        L.orc_sample_greedy.restype = C.c_long
        L.orc_sample_greedy.argtypes = [P, P, C.c_size_t, C.c_float, C.c_uint32]
        L.orc_generate.restype = C.c_int
        L.orc_generate.argtypes = [P, P, C.c_size_t, C.c_size_t, C.c_float, C.c_uint32, P,
                                   C.c_size_t, P, C.POINTER(C.c_size_t)]
        L.orc_get_logits.restype = C.c_size_t
        L.orc_get_logits.argtypes = [P, P, C.c_size_t]
        L.orc_config.argtypes = [P, P]
        L.orc_quantize_i8.restype = C.c_float
        L.orc_quantize_i8.argtypes = [P, P, C.c_size_t]
        L.orc_matmul_i8.argtypes = [P, P, P, P, C.c_size_t, C.c_size_t]
        L.orc_matmul_i8_dots.argtypes = [P, P, P, C.c_size_t, C.c_size_t]
        L.orc_matmul_i4.argtypes = [P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t]
        L.orc_matmul_i4_gdots.argtypes = [P, P, P, C.c_size_t, C.c_size_t, C.c_size_t]
        L.orc_rmsnorm.argtypes = [P, P, P, C.c_size_t]
        L.orc_softmax.argtypes = [P, C.c_size_t]
        L.orc_fast_exp.restype = C.c_float
        L.orc_fast_exp.argtypes = [C.c_float]
        L.orc_dot_f32.restype = C.c_float
        L.orc_dot_f32.argtypes = [P, P, C.c_size_t]
        L.orc_swiglu.argtypes = [P, P, C.c_size_t]
        L.orc_soft_cap.restype = C.c_float
        L.orc_soft_cap.argtypes = [C.c_float, C.c_float]
        L.orc_argmax.restype = C.c_long
        L.orc_argmax.argtypes = [P, C.c_size_t]
        L.orc_repetition_penalty.argtypes = [P, C.c_size_t, P, C.c_size_t, C.c_float]
        L.orc_softmax_top_k.restype = C.c_size_t
        L.orc_softmax_top_k.argtypes = [P, C.c_size_t, C.c_size_t, P, P]
        L.orc_pack_int4.restype = C.c_uint8
        L.orc_pack_int4.argtypes = [C.c_int8, C.c_int8]
        L.orc_unpack_int4.argtypes = [C.c_uint8, C.POINTER(C.c_int8), C.POINTER(C.c_int8)]
        L.orc_quantize_i4.argtypes = [P, C.c_size_t, P, P]
        L.orc_moe_forward.restype = C.c_int
        L.orc_moe_forward.argtypes = [P, C.c_size_t, P, C.c_size_t, C.c_size_t, C.c_size_t,
                                      C.c_size_t, C.c_size_t, P, P, C.c_int]
        L.orc_expert_rows.argtypes = [P, P, P, C.c_size_t, P, C.c_size_t, C.c_size_t, C.c_size_t, P, C.c_int]
        L.orc_sample.restype = C.c_long
        L.orc_sample.argtypes = [P, C.c_size_t, C.c_int, C.c_float, C.c_size_t, C.c_float, C.c_float, C.c_float,
                                 C.POINTER(C.c_float)]
        L.orc_kvc_create.restype = P
        L.orc_kvc_create.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t]
        L.orc_kvc_free.argtypes = [P]
        L.orc_kvc_write.argtypes = [P, C.c_size_t, C.c_size_t, P, P]
        L.orc_kvc_read.restype = C.c_int
        L.orc_kvc_read.argtypes = [P, C.c_size_t, C.c_size_t, P, P]
        L.orc_kvc_clear.argtypes = [P]
        L.orc_kvc_active_pages.restype = C.c_size_t
        L.orc_kvc_active_pages.argtypes = [P]
        L.orc_paged_store.argtypes = [P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, P, P]
        L.orc_paged_attention.argtypes = [P, P, P, C.c_size_t, P, C.c_size_t, C.c_size_t, C.c_size_t,
                                          C.c_size_t, P, P, C.c_int]
        L.orc_hw_threads.restype = C.c_int
        L.orc_fill_kv_random.argtypes = [P, C.c_size_t, C.c_uint64]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- operators -------------------------------------------------------------

def quantize_i8(x):
    x = _f32(x)
    q = np.empty(x.shape[-1], np.int8)
    s = lib().orc_quantize_i8(_p(x), _p(q), x.size)
    return q, np.float32(s)


def matmul_i8(w, w_scales, x, out_dim, in_dim):
    out = np.empty(out_dim, np.float32)
    w = np.ascontiguousarray(w, np.int8)
    lib().orc_matmul_i8(_p(out), _p(w), _p(_f32(w_scales)), _p(_f32(x)), out_dim, in_dim)
    return out


def matmul_i8_dots(w, xq, out_dim, in_dim):
    d = np.empty(out_dim, np.int32)
    lib().orc_matmul_i8_dots(_p(d), _p(np.ascontiguousarray(w, np.int8)),
                             _p(np.ascontiguousarray(xq, np.int8)), out_dim, in_dim)
    return d


def matmul_i4(w_packed, w_scales, x, out_dim, in_dim, group):
    out = np.empty(out_dim, np.float32)
    lib().orc_matmul_i4(_p(out), _p(np.ascontiguousarray(w_packed, np.uint8)),
                        _p(_f32(w_scales)), _p(_f32(x)), out_dim, in_dim, group)
    return out


def matmul_i4_gdots(w_packed, xq, out_dim, in_dim, group):
    ng = (in_dim + group - 1) // group
    g = np.empty((out_dim, ng), np.int32)
    lib().orc_matmul_i4_gdots(_p(g), _p(np.ascontiguousarray(w_packed, np.uint8)),
                              _p(np.ascontiguousarray(xq, np.int8)), out_dim, in_dim, group)
    return g


def rmsnorm(x, w):
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(out), _p(x), _p(w), x.size)
    return out


def softmax(x):
    x = _f32(x).copy()
    lib().orc_softmax(_p(x), x.size)
    return x


def fast_exp(v: float) -> np.float32:
    return np.float32(lib().orc_fast_exp(float(v)))


def dot_f32(a, b):
    a, b = _f32(a), _f32(b)
    return np.float32(lib().orc_dot_f32(_p(a), _p(b), a.size))


def swiglu(g, u):
    g = _f32(g).copy()
    lib().orc_swiglu(_p(g), _p(_f32(u)), g.size)
    return g


def soft_cap(x, cap=30.0):
    return np.float32(lib().orc_soft_cap(float(x), float(cap)))


def argmax(x):
    x = _f32(x)
    return int(lib().orc_argmax(_p(x), x.size))


def repetition_penalty(logits, history, penalty):
    logits = _f32(logits).copy()
    h = np.ascontiguousarray(history, np.uint32)
    lib().orc_repetition_penalty(_p(logits), logits.size, _p(h), h.size, float(penalty))
    return logits


def softmax_top_k(scores, k):
    s = _f32(scores).copy()
    idx = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    n = lib().orc_softmax_top_k(_p(s), s.size, k, _p(idx), _p(w))
    return idx[:n], w[:n]


def pack_int4(lo: int, hi: int) -> int:
    return int(lib().orc_pack_int4(lo, hi))


def unpack_int4(b: int):
    lo, hi = C.c_int8(), C.c_int8()
    lib().orc_unpack_int4(b, C.byref(lo), C.byref(hi))
    return lo.value, hi.value


def quantize_i4(x):
    x = _f32(x)
    out = np.zeros((x.size + 1) // 2, np.uint8)
    sc = np.zeros((x.size + 63) // 64, np.float32)
    lib().orc_quantize_i4(_p(x), x.size, _p(out), _p(sc))
    return out, sc


def moe_forward(x, layer_bytes, dim, hidden, n_experts, top_k, group, threads=1):
    """MoE sub-block for T tokens; `layer_bytes` starts at the router weights."""
    x = _f32(x)
    T = x.shape[0]
    out = np.empty((T, dim), np.float32)
    sel = np.full((T, top_k), -1, np.int32)
    lb = np.ascontiguousarray(layer_bytes, np.uint8)
    lib().orc_moe_forward(_p(x), T, _p(lb), dim, hidden, n_experts, top_k, group, _p(out),
                          _p(sel), threads)
    return out, sel


def expert_rows(xq, xs, expert, experts, dim, hidden, group, threads=1):
    """Expert outputs y [n][dim] of already-quantized rows (xq int8 [n][dim], xs [n])."""
    xq = np.ascontiguousarray(xq, np.int8)
    n = xq.shape[0]
    y = np.zeros((n, dim), np.float32)
    lib().orc_expert_rows(_p(xq), _p(_f32(xs)), _p(np.ascontiguousarray(expert, np.int32)), n,
                          _p(np.ascontiguousarray(experts, np.uint8)), dim, hidden, group, _p(y), threads)
    return y


def sample(logits, strategy, temperature=0.7, top_k=40, top_p=0.9, min_p=0.05, r=0.5):
    """sampling.rs's strategies for the draw r; returns (token, margin)."""
    lg = _f32(logits)
    m = C.c_float()
    t = lib().orc_sample(_p(lg), lg.size, strategy, temperature, top_k, top_p, min_p, r, C.byref(m))
    return int(t), float(m.value)


class RefPagedKVCache:
    """PagedKVCache (src/model/memory.rs:100-201) restated: write/read/clear."""

    def __init__(self, kv_dim: int, n_layers: int, max_pages_per_layer: int = 16):
        self.dim = kv_dim
        self.h = lib().orc_kvc_create(kv_dim, n_layers, max_pages_per_layer)

    def write(self, layer, pos, k, v):
        lib().orc_kvc_write(self.h, layer, pos, _p(_f32(k)), _p(_f32(v)))

    def read(self, layer, pos):
        k = np.zeros(self.dim, np.float32)
        v = np.zeros(self.dim, np.float32)
        ok = lib().orc_kvc_read(self.h, layer, pos, _p(k), _p(v))
        return bool(ok), k, v

    def clear(self):
        lib().orc_kvc_clear(self.h)

    def active_pages(self) -> int:
        return int(lib().orc_kvc_active_pages(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_kvc_free(self.h)
            self.h = None


def paged_store(data, scales, page_ids, P, H, hd, k, v):
    """Quantizes whole pages into data [pages][2][H][P][hd] / scales [pages][2][H]."""
    pid = np.ascontiguousarray(page_ids, np.int32)
    lib().orc_paged_store(_p(data), _p(scales), _p(pid), pid.size, P, H, hd, _p(_f32(k)), _p(_f32(v)))


def paged_attention(data, scales, page_table, lens, P, H, hd, q, threads=1):
    pt = np.ascontiguousarray(page_table, np.int32)
    ln = np.ascontiguousarray(lens, np.int32)
    q = _f32(q)
    n_seq = ln.size
    out = np.zeros((n_seq, H, hd), np.float32)
    lib().orc_paged_attention(_p(data), _p(scales), _p(pt), pt.shape[1], _p(ln), n_seq, P, H, hd, _p(q),
                              _p(out), threads)
    return out


class _SynthSpec(C.Structure):  # chalot_synth_spec (include/chalot_b200.h)
    _fields_ = [("dim", C.c_uint32), ("hidden_dim", C.c_uint32), ("n_layers", C.c_uint32),
                ("n_heads", C.c_uint32), ("vocab_size", C.c_uint32), ("n_experts", C.c_uint32),
                ("top_k", C.c_uint32), ("int4_group_size", C.c_uint32),
                ("max_seq_len", C.c_uint32), ("rope_theta_x100", C.c_uint32),
                ("weight_std", C.c_float), ("seed", C.c_uint64), ("n_threads", C.c_int)]


def write_synthetic(path: str, *, dim, hidden_dim, n_layers, n_heads, vocab_size, n_experts=8, top_k=2,
                    int4_group_size=32, max_seq_len=512, rope_theta_x100=0, seed=0, weight_std=0.02,
                    n_threads=0) -> str:
    """The synthetic .myai writer, compiled into this library from the CUDA
    library's own writer sources (same bytes), for callers that must not load
    the CUDA library (the CPU reference arm of the benchmark)."""
    spec = _SynthSpec(dim, hidden_dim, n_layers, n_heads, vocab_size, n_experts, top_k, int4_group_size,
                      max_seq_len, rope_theta_x100, weight_std, seed, n_threads)
    L = lib()
    L.orc_write_synthetic.restype = C.c_int
    L.orc_write_synthetic.argtypes = [C.c_char_p, C.c_void_p]
    rc = L.orc_write_synthetic(path.encode(), C.byref(spec))
    if rc != 0:
        raise RuntimeError(f"orc_write_synthetic failed ({rc}): {path}")
    return path


def ensure_model(directory: str, name: str, shape: dict) -> str:
    """directory/name.myai, written once (through a temporary file)."""
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{name}.myai")
    if not os.path.exists(path):
        tmp = path + ".tmp"
        write_synthetic(tmp, **shape)
        os.replace(tmp, path)
    return path


def hw_threads() -> int:
    return int(lib().orc_hw_threads())


# ---- engine ----------------------------------------------------------------

class OracleEngine:
    """Engine::load/forward/generate restated on the CPU.

    threads=0 mirrors the reference's threading (one thread, one thread per
    selected expert); threads=N splits every matmul's rows over N threads.
    """

    def __init__(self, path: str, threads: int = 0):
        self._L = lib()
        h = self._L.orc_load(path.encode(), threads)
        if not h:
            raise RuntimeError(self._L.orc_error().decode())
        self._h = C.c_void_p(h)
        cfg = np.zeros(11, np.uint64)
        self._L.orc_config(self._h, _p(cfg))
        keys = ["dim", "hidden_dim", "n_layers", "n_heads", "head_dim", "vocab_size",
                "max_seq_len", "n_experts", "top_k", "int4_group_size", "total_bytes"]
        self.config = {k: int(v) for k, v in zip(keys, cfg)}

    def close(self):
        if getattr(self, "_h", None):
            self._L.orc_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def set_trace(self, on: bool = True):
        self._L.orc_set_trace(self._h, int(on))

    def trace(self, which: int) -> np.ndarray:
        c = self.config
        n = {0: c["n_layers"] * c["dim"], 1: c["n_layers"] * c["dim"],
             2: c["n_layers"] * c["n_experts"], 3: c["n_layers"] * c["top_k"],
             4: c["n_layers"] * c["top_k"]}[which]
        buf = np.zeros(n, np.float32)
        self._L.orc_get_trace(self._h, which, _p(buf), n)
        return buf

    def forward(self, token: int, pos: int) -> int:
        r = self._L.orc_forward(self._h, token, pos)
        if r < 0:
            raise RuntimeError(self._L.orc_error().decode())
        return int(r)

    def fill_kv_random(self, n: int, seed: int = 0):
        """Timing helper: makes positions [0, n) attendable without a prefill."""
        self._L.orc_fill_kv_random(self._h, n, seed)

    def logits(self) -> np.ndarray:
        out = np.empty(self.config["vocab_size"], np.float32)
        self._L.orc_get_logits(self._h, _p(out), out.size)
        return out

    def generate(self, prompt, max_new: int, repetition_penalty: float = 1.0,
                 repetition_window: int = 64, stop_tokens=()):
        p = np.ascontiguousarray(prompt, np.uint32)
        st = np.ascontiguousarray(list(stop_tokens) or [0], np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = C.c_size_t(0)
        r = self._L.orc_generate(self._h, _p(p), p.size, max_new, float(repetition_penalty),
                                 repetition_window, _p(st), len(stop_tokens), _p(out),
                                 C.byref(n))
        if r != 0:
            raise RuntimeError(self._L.orc_error().decode())
        return out[: n.value].tolist()
