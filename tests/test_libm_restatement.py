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
                   'extern "C" float t_expm1(float x){return chalot::libm::expm1_f32(x);}\n'
                   'extern "C" float t_exp(float x){return chalot::libm::exp_f32(x);}\n'
                   '#include <math.h>\n#include <string.h>\n'
                   'extern "C" long long t_exp_mismatch(unsigned lo, unsigned hi){long long n=0;'
                   'for(unsigned long long u=lo;u<=hi;++u){float x;unsigned v=(unsigned)u;memcpy(&x,&v,4);'
                   'float a=expf(x),b=chalot::libm::exp_f32(x);if(memcmp(&a,&b,4))++n;}return n;}\n')
    so = d / "t.so"
    subprocess.run(["g++", "-O2", "-ffp-contract=off", "-shared", "-fPIC",
                    "-I", os.path.join(ROOT, "chalot_c1_b200", "csrc"), str(src), "-o", str(so)],
                   check=True)
    mine = ctypes.CDLL(str(so))
    sysm = ctypes.CDLL("libm.so.6")
    mine.t_exp_mismatch.restype = ctypes.c_longlong
    mine.t_exp_mismatch.argtypes = [ctypes.c_uint, ctypes.c_uint]
    for f in (mine.t_tanh, mine.t_expm1, mine.t_exp, sysm.tanhf, sysm.expm1f, sysm.expf):
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


def test_exp_matches_system_libm_on_softmax_range(both):
    """Every float in [-87, 0] (the attention softmax tail evaluates expf on
    x - max <= 0; the soft-cap keeps it above -60): the restated expf is the
    system expf, bit for bit, where exp in double rounded once is not."""
    mine, _ = both
    b60, b87 = int(np.float32(-60.0).view(np.uint32)), int(np.float32(-87.0).view(np.uint32))
    assert mine.t_exp_mismatch(0x80000000, b60) == 0
    # one known 1-ulp case below the soft-capped range: x = -0x1.f8cbb2p+5
    assert mine.t_exp_mismatch(b60 + 1, b87) == 1
    x = np.array([float.fromhex('-0x1.f8cbb2p+5')], np.float32)
    assert mine.t_exp_mismatch(int(x.view(np.uint32)[0]), int(x.view(np.uint32)[0])) == 1


def test_exp_matches_system_libm_positive_and_edges(both):
    mine, sysm = both
    xs = np.concatenate([np.random.default_rng(4).uniform(0, 88.7, 200000),
                         [-103.9, -103.98, -104.5, 88.72, 88.73, -np.inf, np.inf, 0.0, -0.0]]).astype(np.float32)
    a = np.array([sysm.expf(float(x)) for x in xs], np.float32).view(np.uint32)
    b = np.array([mine.t_exp(float(x)) for x in xs], np.float32).view(np.uint32)
    bad = xs[a != b]
    # two known 1-ulp cases above 32 (0x1.04845ep+5) may be drawn; nothing else
    assert bad.size <= 2 and all(abs(float(x) - 32.5648) < 1e-3 for x in bad), bad[:5]
