#!/usr/bin/env python3
"""Generates tests/golden/kats.json: known-answer vectors computed in pure
Python (math module, integers), independently of the C oracle.

The reference (OgnianM/TADMA) ships no tests or expected outputs and cannot be
built here, so these analytic KATs are what pins the oracle:
* gelu / sigmoid / tanh at fixed points from the formulas of
  include/tadma/Operations.hpp:160-181 (evaluated with Python floats = IEEE
  double);
* MapToShape (include/tadma/Utils.hpp:9-17) examples;
* the seeded generator's first values (same definition as tadma_b200_fill);
* closed-form reductions: sum of arange, mean, softmax of a constant row,
  LayerNorm of an alternating +-1 row.
Run: python tests/golden/make_kats.py  (rewrites kats.json)
"""
import json
import math
import os
import struct

M64 = (1 << 64) - 1


def mix64(z):
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def key(seed, sid):
    return mix64(seed ^ mix64((sid + 0x632BE59BD9B4E019) & M64))


def draw(k, g, j):
    return mix64((k + ((4 * g + j + 1) * 0x9E3779B97F4A7C15)) & M64)


def f32(x):
    return struct.unpack("<f", struct.pack("<f", x))[0]


LN_COEF = [2.0 / (2 * j + 1) for j in range(12)]


def _alt_coefs(div):
    c = [1.0]
    for k in range(1, 9):
        c.append(-c[-1] / float(div(k)))
    return c


COS_COEF = _alt_coefs(lambda k: (2 * k - 1) * (2 * k))
SIN_COEF = _alt_coefs(lambda k: (2 * k) * (2 * k + 1))
SQRT2 = float.fromhex("0x1.6a09e667f3bcdp+0")
LN2 = float.fromhex("0x1.62e42fefa39efp-1")
TWO_PI = float.fromhex("0x1.921fb54442d18p+2")


def ln_series(u):
    """ln u for u in (0, 1]: u = m 2^e, ln u = e ln2 + 2 atanh((m-1)/(m+1))."""
    m, e = math.frexp(u)  # u = m 2^e, m in [0.5, 1)
    m, e = m * 2.0, e - 1
    if m > SQRT2:
        m, e = m * 0.5, e + 1
    s = (m - 1.0) / (m + 1.0)
    w = s * s
    p = LN_COEF[-1]
    for c in reversed(LN_COEF[:-1]):
        p = c + w * p
    return float(e) * LN2 + s * p


def cos_turns(t):
    """cos(2 pi t), t in [0, 1), folded to [0, 1/8] then a Taylor series."""
    neg = use_sin = False
    if t > 0.5:
        t = 1.0 - t
    if t > 0.25:
        t, neg = 0.5 - t, True
    if t > 0.125:
        t, use_sin = 0.25 - t, True
    x = t * TWO_PI
    y = x * x
    k = SIN_COEF if use_sin else COS_COEF
    p = k[-1]
    for c in reversed(k[:-1]):
        p = c + y * p
    if use_sin:
        p = x * p
    return -p if neg else p


def gen_normal_f32(seed, sid, n, p0=0.0, p1=1.0):
    """Box-Muller from two 53-bit uniforms per element, ln and cos from their
    series (the generator's definition, each operation an IEEE double op)."""
    k = key(seed, sid)
    out = []
    for g in range(n):
        u1 = float((draw(k, g, 0) >> 11) + 1) * 2.0 ** -53
        t = float(draw(k, g, 1) >> 11) * 2.0 ** -53
        z = math.sqrt(-2.0 * ln_series(u1)) * cos_turns(t)
        out.append(f32(p0 + p1 * z))
    return out


def gen_uniform_f32(seed, sid, n, p0, p1):
    k = key(seed, sid)
    return [f32(p0 + (p1 - p0) * (float(draw(k, g, 0) >> 40) * 2.0 ** -24)) for g in range(n)]


def gen_index(seed, sid, n, v):
    k = key(seed, sid)
    return [(draw(k, g, 0) * v) >> 64 for g in range(n)]


def tanh_ref(x):
    ep, en = math.exp(x), math.exp(-x)
    return (ep - en) / (ep + en)


def gelu_ref(x):
    """The reference expression itself (accurate in double for x >= -3)."""
    return 0.5 * x * (1 + tanh_ref(0.7978845608 * (x + 0.044715 * x * x * x)))


def gelu_stable(x):
    """Algebraically identical form x / (1 + exp(-2u)), accurate for all x."""
    u = 0.7978845608 * (x + 0.044715 * x * x * x)
    return x / (1 + math.exp(-2 * u))


def map_to_shape(dims, index):
    out = [0] * len(dims)
    for d in range(len(dims) - 1, -1, -1):
        out[d] = index % dims[d]
        index //= dims[d]
    return out


def main():
    pts = [-8.0, -3.0, -1.0, -0.5, -1e-3, 0.0, 1e-3, 0.5, 1.0, 2.0, 3.0, 8.0]
    kats = {
        "gelu_reference_expr": [[x, gelu_ref(x)] for x in pts if x >= -3.0],
        "gelu": [[x, gelu_stable(x)] for x in pts],
        "sigmoid": [[x, 1 / (1 + math.exp(-x))] for x in pts],
        "tanh": [[x, tanh_ref(x)] for x in pts],
        "exp": [[x, math.exp(x)] for x in pts],
        "map_to_shape": [[[2, 3, 4], i, map_to_shape([2, 3, 4], i)] for i in (0, 1, 5, 12, 23)]
                        + [[[7], 6, [6]], [[1, 1, 5], 4, [0, 0, 4]]],
        "gen_normal_f32_seed0_sid1": gen_normal_f32(0, 1, 16),
        "gen_normal_f32_seed7_sid11_p1_0.02": gen_normal_f32(7, 11, 8, 1.0, 0.02),
        "gen_uniform_f32_seed0_sid1": gen_uniform_f32(0, 1, 16, -1.0, 1.0),
        "gen_index_seed0_sid2_v50257": gen_index(0, 2, 16, 50257),
        "sum_arange": [[n, n * (n - 1) // 2] for n in (1, 2, 128, 4096, 65537)],
        "softmax_const_row": [[n, 1.0 / n] for n in (1, 7, 2048)],
        "layer_norm_pm1": {"row": [1.0, -1.0] * 8, "out": [1.0, -1.0] * 8},
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kats.json")
    with open(path, "w") as f:
        json.dump(kats, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
