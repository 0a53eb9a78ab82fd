"""Generates the committed golden fixtures of tests/golden/ (run: python tests/golden/make_golden.py).

threefry_kat.json
    The published known-answer vectors of Threefry-2x32 with 20 rounds (Random123's kat_vectors; the same three
    vectors pin jax's threefry2x32).  Typed in, not computed: they pin the oracle's and the kernels' threefry.

exact_sum.npz
    The exact f32 sum's known answers.  The reference's kernel backend keeps an exact sum (TSpec.exact) and tests
    it bitwise against a numpy integer reference (tests/edge.py:2037-2064: _units, _f32_round, _exact_ref): every
    finite f32 is an integer in units of 2^-149; a bin's total is summed in Python integers and rounded once, to
    nearest with ties to even, to f32.  That reference is restated here (units / f32_round / exact_ref) and run on
    seeded value sets that reach every word of the 5-word accumulator: mixed signs, subnormals, values near the f32
    maximum, cancellations to exact zero, out-of-range bins (-3, 0, 7, 8 with 8 bins, tests/edge.py:162), and a total
beyond the f32 range, which the kernel contract reads out as NaN.
"""
import json
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

THREEFRY_KAT = [
    # key0, key1, ctr0, ctr1 -> out0, out1
    {"key": ["0x00000000", "0x00000000"], "ctr": ["0x00000000", "0x00000000"], "out": ["0x6b200159", "0x99ba4efe"]},
    {"key": ["0xffffffff", "0xffffffff"], "ctr": ["0xffffffff", "0xffffffff"], "out": ["0x1cb996fc", "0xbb002be7"]},
    {"key": ["0x13198a2e", "0x03707344"], "ctr": ["0x243f6a88", "0x85a308d3"], "out": ["0xc4923a9c", "0x483df7a0"]},
]


def units(v):
    """f32 values -> their exact values as Python ints in units of 2^-149 (tests/edge.py:2037-2042)."""
    b = np.asarray(v, np.float32).view(np.uint32).astype(np.int64)
    e, mant = (b >> 23) & 255, b & 0x7FFFFF
    m, p = np.where(e > 0, mant | 0x800000, mant), np.maximum(e - 1, 0)
    return [(-int(mi) if s else int(mi)) << int(pi) for s, mi, pi in zip(b >> 31, m, p)]


def f32_round(T):
    """the correctly rounded f32 (nearest, ties to even) of the integer T x 2^-149 (tests/edge.py:2045-2056)."""
    if T == 0:
        return np.float32(0.0)
    m = abs(T)
    sh = max(m.bit_length() - 24, 0)
    q, r = divmod(m, 1 << sh)
    if sh and (2 * r > (1 << sh) or (2 * r == (1 << sh) and q & 1)):
        q += 1
    with np.errstate(over="ignore"):
        v = np.float32(math.ldexp(float(q), sh - 149))
    return -v if T < 0 else v


def exact_ref(vals, bins, nbins):
    """per-bin exact totals, rounded once (tests/edge.py:2059-2064); out-of-range bins are dropped."""
    tot = [0] * nbins
    for u, i in zip(units(vals), np.asarray(bins)):
        if 0 <= int(i) < nbins:
            tot[int(i)] += u
    return np.array([f32_round(t) for t in tot], np.float32)


def value_sets():
    rng = np.random.default_rng(2037)
    sets = {}
    n = 1 << 14
    sets["uniform"] = (rng.uniform(-3, 3, n).astype(np.float32), rng.integers(0, 16, n).astype(np.int32), 16)
    # every exponent, both signs (reaches all five words), plus subnormals
    e = rng.integers(-149, 111, n)
    v = (rng.uniform(1, 2, n) * np.exp2(e.astype(np.float64))).astype(np.float32)
    v = np.where(rng.random(n) < 0.5, -v, v).astype(np.float32)
    v = v[np.isfinite(v)]
    sets["wide"] = (v, rng.integers(0, 8, len(v)).astype(np.int32), 8)
    sub = (rng.integers(1, 1 << 23, 4096).astype(np.uint32)).view(np.float32)
    sub = np.where(rng.random(4096) < 0.5, -sub, sub).astype(np.float32)
    sets["subnormal"] = (sub, rng.integers(0, 4, 4096).astype(np.int32), 4)
    big = np.float32(3.0e38) * np.ones(64, np.float32)
    sets["cancel"] = (np.concatenate([big, -big, np.float32([1e-45, -1e-45, 2.5, -2.5])]),
                      np.zeros(132, np.int32), 1)
    sets["oob"] = (np.float32([1.0, 2.0, 4.0, 8.0]), np.int32([-3, 0, 7, 8]), 8)
    # a total beyond the f32 range: the readout makes the bin NaN and counts it (backends/kernel/kernel.py:625-628)
    sets["overflow"] = (np.float32([3.0e38, 3.0e38, -1.0, 2.0]), np.int32([0, 0, 1, 1]), 2)
    return sets


def main():
    with open(os.path.join(HERE, "threefry_kat.json"), "w") as f:
        json.dump(THREEFRY_KAT, f, indent=1)
    arrays = {}
    for name, (v, b, nb) in value_sets().items():
        arrays[f"{name}_vals"] = v
        arrays[f"{name}_bins"] = b
        arrays[f"{name}_nb"] = np.int32(nb)
        ref = exact_ref(v, b, nb)
        arrays[f"{name}_expect"] = np.where(np.isfinite(ref), ref, np.float32(np.nan)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "exact_sum.npz"), **arrays)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
