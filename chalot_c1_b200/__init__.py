"""chalot_c1_b200 — B200 (sm_100a) implementation of chalot_C1's sparse-MoE
decode hot path behind the reference's Engine / tensor API and .myai format.

The compute lives in ``_lib/libchalot_b200.so`` (CUDA kernels + C++ engine,
C ABI in include/chalot_b200.h); these modules are thin ctypes faces of it.
"""
from ._capi import ChalotError, LIB_PATH  # noqa: F401
from .engine import GREEDY, Engine, EpHub, SamplingConfig, Scheduler  # noqa: F401
from .myai import SHAPES, ensure_shape, inspect, write_shape, write_synthetic  # noqa: F401

__all__ = ["Engine", "EpHub", "SamplingConfig", "GREEDY", "ChalotError", "write_synthetic",
           "write_shape", "ensure_shape", "inspect", "SHAPES", "LIB_PATH"]
