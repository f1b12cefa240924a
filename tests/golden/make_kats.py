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


def gen_normal_f32(seed, sid, n, p0=0.0, p1=1.0):
    k = key(seed, sid)
    out = []
    for g in range(n):
        s = 0.0
        for j in range(4):
            s += float(draw(k, g, j) >> 40) * 2.0 ** -23 - 1.0
        z = s * 0.8660254037844386
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
