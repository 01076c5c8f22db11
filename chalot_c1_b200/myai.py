"""The .myai weight-file format: synthetic writer and header inspection.

The writer and the parser are native (include/chalot_b200.h); this module is
their Python face plus the named model shapes used by the benchmarks.
"""
from __future__ import annotations

import ctypes as C
import os

from ._capi import ModelConfig, SynthSpec, check, lib

# Named shapes (dim, hidden, layers, heads, vocab, experts, top_k, group,
# max_seq, rope_theta*100, seed).
SHAPES = {
    # tiny synthetic MoE, CPU-runnable: d256 L4 H4 V4096 E8 top-2 g32
    "tiny": dict(dim=256, hidden_dim=1024, n_layers=4, n_heads=4, vocab_size=4096, n_experts=8,
                 top_k=2, int4_group_size=32, max_seq_len=512, rope_theta_x100=0, seed=0),
    # Qwen2.5-0.5B-shaped MoE: d896 L24 H14 V151936 E8 top-2 g32, theta 1e6
    "qwen": dict(dim=896, hidden_dim=4864, n_layers=24, n_heads=14, vocab_size=151936,
                 n_experts=8, top_k=2, int4_group_size=32, max_seq_len=2048,
                 rope_theta_x100=100000000, seed=1),
    # 1B-class MoE: d2048 L16 H16 V32000 E16 top-2 g32
    "1b": dict(dim=2048, hidden_dim=5632, n_layers=16, n_heads=16, vocab_size=32000,
               n_experts=16, top_k=2, int4_group_size=32, max_seq_len=512, rope_theta_x100=0,
               seed=2),
}


def write_synthetic(path: str, *, dim: int, hidden_dim: int, n_layers: int, n_heads: int,
                    vocab_size: int, n_experts: int = 8, top_k: int = 2,
                    int4_group_size: int = 32, max_seq_len: int = 512, rope_theta_x100: int = 0,
                    seed: int = 0, weight_std: float = 0.02, n_threads: int = 0) -> str:
    spec = SynthSpec(dim, hidden_dim, n_layers, n_heads, vocab_size, n_experts, top_k,
                     int4_group_size, max_seq_len, rope_theta_x100, weight_std, seed, n_threads)
    check(lib().chalot_myai_write_synthetic(path.encode(), C.byref(spec)))
    return path


def write_shape(path: str, name: str, **over) -> str:
    kw = dict(SHAPES[name])
    kw.update(over)
    return write_synthetic(path, **kw)


def ensure_shape(directory: str, name: str, **over) -> str:
    """Writes the named synthetic model once into `directory` and reuses it."""
    os.makedirs(directory, exist_ok=True)
    tag = "_".join(f"{k}{v}" for k, v in sorted(over.items()))
    path = os.path.join(directory, f"{name}{('_' + tag) if tag else ''}.myai")
    want = inspect_expected(name, **over)
    if not (os.path.exists(path) and os.path.getsize(path) == want):
        tmp = path + ".tmp"
        write_shape(tmp, name, **over)
        os.replace(tmp, path)
    return path


def inspect(path: str) -> dict:
    cfg = ModelConfig()
    check(lib().chalot_myai_inspect(path.encode(), C.byref(cfg)))
    return cfg.as_dict()


def validate(path: str) -> tuple:
    """chalot_myai_validate: (ok, report lines)."""
    buf = C.create_string_buffer(4096)
    rc = lib().chalot_myai_validate(path.encode(), buf, len(buf))
    if rc not in (0, -3):
        check(rc)
    return rc == 0, [line for line in buf.value.decode().splitlines() if line]


def inspect_expected(name: str, **over) -> int:
    """File size of a named shape, from the offset arithmetic alone."""
    kw = dict(SHAPES[name])
    kw.update(over)
    d, H, L, V, E, g = (kw["dim"], kw["hidden_dim"], kw["n_layers"], kw["vocab_size"],
                        kw["n_experts"], kw["int4_group_size"])
    expert = 2 * H * ((d + 1) // 2) + 2 * H * ((d + g - 1) // g) * 4 + d * ((H + 1) // 2) + \
        d * ((H + g - 1) // g) * 4
    layer = d * 4 + 3 * d * d + 3 * d * 4 + d * d + d * 4 + d * 4 + \
        ((E * d * 4 + E * 4) if E >= 2 else 0) + E * expert
    return 256 + V * d + V * 4 + L * layer + d * 4 + V * d + V * 4
