"""A second, independent restatement of the reference's small float routines
in numpy float32 scalar arithmetic (test helper).

Used to cross-check the C++ oracle bit for bit on small inputs: two
restatements written separately that agree to the bit pin the lane orders.
Citations are to chalot28/chalot_C1.
"""
import math

import numpy as np

f32 = np.float32


def fast_exp(x):
    """src/tensor/normalization.rs:165-200 (one lane)."""
    x = f32(x)
    n = f32(math.floor(f32(x * f32(1.442695040888963407))))
    r = f32(x - f32(n * f32(0.693147180559945309)))
    p = f32(0.008333333333)
    for c in (0.041666666666, 0.166666666666, 0.5, 1.0, 1.0):
        p = f32(f32(p * r) + f32(c))
    e = ((int(n) + 127) & 0xFFFFFFFF) << 23 & 0xFFFFFFFF
    return f32(p * np.array([e], np.uint32).view(np.float32)[0])


def hsum8(s):
    t = [f32(s[j] + s[j + 4]) for j in range(4)]
    return f32(f32(t[0] + t[2]) + f32(t[1] + t[3]))


def rmsnorm(x, w):
    """src/tensor/normalization.rs:35-67."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    n = x.size
    ch = n // 8
    s = [f32(0)] * 8
    for c in range(ch):
        for j in range(8):
            v = x[c * 8 + j]
            s[j] = f32(s[j] + f32(v * v))
    ss = hsum8(s)
    for i in range(ch * 8, n):
        ss = f32(ss + f32(x[i] * x[i]))
    inv = f32(f32(1) / f32(np.sqrt(f32(f32(ss / f32(n)) + f32(1e-5)))))
    return np.array([f32(f32(x[i] * inv) * w[i]) for i in range(n)], np.float32)


def dot_f32(a, b):
    """src/tensor/attention_helpers.rs:41-80."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    n = a.size
    c16 = n // 16
    a0 = [f32(0)] * 8
    a1 = [f32(0)] * 8
    for c in range(c16):
        for j in range(8):
            a0[j] = f32(a0[j] + f32(a[16 * c + j] * b[16 * c + j]))
            a1[j] = f32(a1[j] + f32(a[16 * c + 8 + j] * b[16 * c + 8 + j]))
    rem = c16 * 16
    extra = rem + 8 <= n
    if extra:
        for j in range(8):
            a0[j] = f32(a0[j] + f32(a[rem + j] * b[rem + j]))
    r = hsum8([f32(a0[j] + a1[j]) for j in range(8)])
    for i in range(rem + 8 if extra else rem, n):
        r = f32(r + f32(a[i] * b[i]))
    return r


def softmax(x):
    """src/tensor/normalization.rs:106-160 (exp tail via float64 math.exp
    rounded to f32, which equals a correctly rounded expf)."""
    x = [f32(v) for v in x]
    n = len(x)
    mx = max(x)
    full = n // 8 * 8
    s = [f32(0)] * 8
    out = list(x)
    for i in range(full):
        e = fast_exp(f32(x[i] - mx))
        out[i] = e
        s[i % 8] = f32(s[i % 8] + e)
    tot = hsum8(s)
    for i in range(full, n):
        e = f32(math.exp(float(f32(x[i] - mx))))
        out[i] = e
        tot = f32(tot + e)
    inv = f32(f32(1) / tot)
    return np.array([f32(v * inv) for v in out], np.float32)


def quantize_i8(x):
    """src/tensor/quantization.rs:56-104."""
    x = np.asarray(x, np.float32)
    n = x.size
    amax = f32(max(float(np.abs(x).max()) if n else 0.0, 1e-12))
    amax = max(amax, f32(1e-12))
    scale = f32(amax / f32(127))
    inv = f32(f32(1) / scale)
    q = np.zeros(n, np.int8)
    full = n // 8 * 8
    for i in range(n):
        s = f32(x[i] * inv)
        if i < full:
            s = min(max(s, f32(-127)), f32(127))
            q[i] = int(np.rint(s))
        else:
            r = math.floor(abs(float(s)) + 0.5) * (1 if s >= 0 else -1)
            q[i] = int(min(max(r, -127), 127))
    return q, scale


def matmul_i8(w, ws, x, out_dim, in_dim):
    q, xs = quantize_i8(x)
    w = np.asarray(w, np.int8).reshape(out_dim, in_dim).astype(np.int64)
    d = w @ q.astype(np.int64)
    return np.array([f32(f32(f32(int(d[r])) * f32(ws[r])) * xs) for r in range(out_dim)], np.float32)


def matmul_i4(wp, ws, x, out_dim, in_dim, group):
    q, xs = quantize_i8(x)
    prow = (in_dim + 1) // 2
    ng = (in_dim + group - 1) // group
    wp = np.asarray(wp, np.uint8).reshape(out_dim, prow)
    lo = (wp & 0x0F).astype(np.int64) - 8
    hi = (wp >> 4).astype(np.int64) - 8
    full = np.empty((out_dim, prow * 2), np.int64)
    full[:, 0::2] = lo
    full[:, 1::2] = hi
    full = full[:, :in_dim]
    ws = np.asarray(ws, np.float32).reshape(out_dim, ng)
    out = np.empty(out_dim, np.float32)
    for r in range(out_dim):
        t = f32(0)
        for g in range(ng):
            s, e = g * group, min((g + 1) * group, in_dim)
            gd = int(full[r, s:e] @ q[s:e].astype(np.int64))
            t = f32(t + f32(f32(f32(gd) * ws[r, g]) * xs))
        out[r] = t
    return out
