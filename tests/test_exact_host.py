"""CPU: the exact f32 sum's arithmetic (tallymap_b200/csrc/tm_exact.h, included by every kernel that keeps an exact
tally) compiled for the host with g++, checked bitwise against

  * the golden known answers of tests/golden/exact_sum.npz (the restated integer reference of the reference's
    tests/edge.py:2037-2064), through the same add-with-carry and readout the device runs;
  * Python's exact integers on arbitrary 5-word states (any signs, words near +-2^63, totals beyond f32): the
    readout must be f32_round of sum_j w_j 2^(63 j), overflow exactly where that rounds beyond the f32 maximum;
  * the addend split: every f32 v equals (s0 + s1 2^63) 2^(63 j) units.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from tests.golden.make_golden import f32_round, units

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
SRC = os.path.join(HERE, "native", "exact_host.cpp")
SETS = ["uniform", "wide", "subnormal", "cancel", "oob", "overflow"]


@pytest.fixture(scope="module")
def xlib(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("exact") / "libexact_host.so")
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC", "-o", so, SRC], check=True)
    L = ctypes.CDLL(so)
    P = ctypes.c_void_p
    L.tmx_scatter.argtypes = [P, P, ctypes.c_longlong, ctypes.c_int, P, P]
    L.tmx_read.argtypes = [P, ctypes.c_int, P, P]
    L.tmx_addend.argtypes = [ctypes.c_float, P, P, P, P]
    return L


def ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def read(L, words):
    words = np.ascontiguousarray(words, np.int64).reshape(-1, 5)
    out = np.empty(len(words), np.float32)
    ovf = np.empty(len(words), np.int32)
    L.tmx_read(ptr(words), len(words), ptr(out), ptr(ovf))
    return out, ovf


@pytest.mark.parametrize("name", SETS)
def test_golden_known_answers(xlib, name):
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    vals, bins, nb, exp = d[name + "_vals"], d[name + "_bins"], int(d[name + "_nb"]), d[name + "_expect"]
    words = np.zeros((nb, 5), np.int64)
    flags = np.zeros(nb, np.uint32)
    xlib.tmx_scatter(ptr(vals), ptr(bins), len(vals), nb, ptr(words), ptr(flags))
    out, ovf = read(xlib, words)
    out = np.where((flags != 0) | (ovf != 0), np.float32(np.nan), out)
    assert np.array_equal(np.isnan(out), np.isnan(exp))
    ok = ~np.isnan(exp)
    assert np.array_equal(out[ok].view(np.uint32), exp[ok].view(np.uint32))


def test_readout_of_arbitrary_words(xlib):
    rng = np.random.default_rng(315)
    n = 20000
    w = rng.integers(-2**63, 2**63 - 1, (n, 5), dtype=np.int64, endpoint=True)
    # mostly small upper words (totals within f32), some at every magnitude, some words pinned near the edges
    scale = rng.integers(0, 5, (n, 5))
    w = np.where(scale[:, :1] == 0, w >> rng.integers(1, 63, (n, 5)), w)
    w[:, 2:] = np.where(rng.random((n, 3)) < 0.7, 0, w[:, 2:])
    w[:, 4] = np.where(rng.random(n) < 0.8, 0, w[:, 4] >> 60)
    w[::97, 0] = 2**63 - 1
    w[1::97, 0] = -2**63
    w[2::97, :] = 0
    w[3::97, 1:] = 0
    w[3::97, 0] = rng.integers(-2**24, 2**24, len(w[3::97]))
    w[4::97, 4] = rng.integers(-2**40, 2**40, len(w[4::97]))           # far beyond f32
    # totals at the f32 maximum's rounding boundary, (2^24 - 1/2) 2^253 units, and one unit either side, both signs
    edge = []
    for T in [(2**25 - 1) << 252, ((2**25 - 1) << 252) - 1, ((2**25 - 1) << 252) + 1, (2**24 - 1) << 253, 2**277]:
        for sgn in (1, -1):
            edge.append([sgn * ((T >> (63 * j)) & (2**63 - 1)) for j in range(5)])
    w = np.concatenate([w, np.array(edge, np.int64)])
    n = len(w)
    out, ovf = read(xlib, w)
    fmax = 3.4028234663852886e38
    for i in range(n):
        T = sum(int(w[i, j]) << (63 * j) for j in range(5))
        ref = f32_round(T)
        if not np.isfinite(ref) or abs(float(ref)) > fmax:
            assert ovf[i] == 1, (i, T)
            continue
        assert ovf[i] == 0, (i, T)
        assert out[i].view(np.uint32) == np.float32(ref).view(np.uint32), (i, T, out[i], ref)


def test_addend_split(xlib):
    rng = np.random.default_rng(63)
    bits = rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32)
    bits[:8] = [0, 0x80000000, 1, 0x7f7fffff, 0xff7fffff, 0x00800000, 0x7f800000, 0x7fc00000]
    v = bits.view(np.float32)
    j, s0, s1, nf = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int32()
    for x, u in zip(v[:20000], units(np.where(np.isfinite(v[:20000]), v[:20000], 0))):
        xlib.tmx_addend(ctypes.c_float(x), ctypes.byref(j), ctypes.byref(s0), ctypes.byref(s1), ctypes.byref(nf))
        if not np.isfinite(x):
            assert nf.value == 1
            continue
        assert nf.value == 0 and 0 <= j.value <= 4 and (s1.value == 0 or j.value <= 3)
        assert 0 <= abs(s0.value) < 2**63 and abs(s1.value) < 2**24
        assert (s0.value + (s1.value << 63)) << (63 * j.value) == u
