"""The device's tanh (chalot_c1_b200/csrc/libm_f32.h, a restatement of the
method of the host libm's tanhf) must reproduce the system tanhf and expm1f
bit for bit: the attention soft-cap (src/tensor/activations.rs:133-135) feeds
every score through it. Compiled here for the host from the same header the
kernels include.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def both(tmp_path_factory):
    d = tmp_path_factory.mktemp("libm")
    src = d / "t.cpp"
    src.write_text('#include "libm_f32.h"\n'
                   'extern "C" float t_tanh(float x){return chalot::libm::tanh_f32(x);}\n'
                   'extern "C" float t_expm1(float x){return chalot::libm::expm1_f32(x);}\n')
    so = d / "t.so"
    subprocess.run(["g++", "-O2", "-ffp-contract=off", "-shared", "-fPIC",
                    "-I", os.path.join(ROOT, "chalot_c1_b200", "csrc"), str(src), "-o", str(so)],
                   check=True)
    mine = ctypes.CDLL(str(so))
    sysm = ctypes.CDLL("libm.so.6")
    for f in (mine.t_tanh, mine.t_expm1, sysm.tanhf, sysm.expm1f):
        f.restype = ctypes.c_float
        f.argtypes = [ctypes.c_float]
    return mine, sysm


@pytest.mark.parametrize("lo,hi,n", [(-1.5, 1.5, 200000), (-30, 30, 100000), (-1e-3, 1e-3, 50000)])
def test_tanh_matches_system_libm(both, lo, hi, n):
    mine, sysm = both
    xs = np.random.default_rng(n).uniform(lo, hi, n).astype(np.float32)
    a = np.array([sysm.tanhf(float(x)) for x in xs], np.float32).view(np.uint32)
    b = np.array([mine.t_tanh(float(x)) for x in xs], np.float32).view(np.uint32)
    assert (a == b).all(), xs[a != b][:5]


def test_expm1_matches_system_libm(both):
    mine, sysm = both
    xs = np.random.default_rng(3).uniform(-60, 60, 100000).astype(np.float32)
    a = np.array([sysm.expm1f(float(x)) for x in xs], np.float32).view(np.uint32)
    b = np.array([mine.t_expm1(float(x)) for x in xs], np.float32).view(np.uint32)
    assert (a == b).all(), xs[a != b][:5]


def test_system_expf_is_nearly_correctly_rounded():
    """The device evaluates libm's expf as exp in double rounded once; record
    how often the host's expf differs from that (1 ulp when it does)."""
    m = ctypes.CDLL("libm.so.6")
    m.expf.restype = ctypes.c_float
    m.expf.argtypes = [ctypes.c_float]
    xs = np.random.default_rng(1).uniform(-60, 0, 100000).astype(np.float32)
    a = np.array([m.expf(float(x)) for x in xs], np.float32).view(np.int32).astype(np.int64)
    b = np.exp(xs.astype(np.float64)).astype(np.float32).view(np.int32).astype(np.int64)
    d = np.abs(a - b)
    assert d.max() <= 1 and (d != 0).mean() < 2e-3
