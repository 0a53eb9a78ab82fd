"""CPU tests of the oracle (the checker) against the golden fixtures, and of the host-side key arithmetic.

The oracle restates the reference's CPU kernel target; before it checks the GPU it is pinned here:
  * threefry2x32 against the published known-answer vectors (tests/golden/threefry_kat.json);
  * the exact f32 sum against the restated numpy integer reference of tests/edge.py:2037-2064
    (tests/golden/exact_sum.npz);
  * the reverse-mode replay against properties of the reference's checkpointed loop (_reverse.py:324-444):
    the checkpoint count C changes the work, never the result; and the gradient of a linear tally equals the
    forward tally divided by the parameter.
"""
import json
import os

import numpy as np
import pytest

from tallymap_b200 import prng

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def kat():
    with open(os.path.join(GOLD, "threefry_kat.json")) as f:
        return [(tuple(int(v, 16) for v in r["key"]), tuple(int(v, 16) for v in r["ctr"]),
                 tuple(int(v, 16) for v in r["out"])) for r in json.load(f)]


@pytest.mark.parametrize("case", range(3))
def test_threefry_kat_oracle(orc, case):
    k, c, o = kat()[case]
    assert orc.threefry2x32(k[0], k[1], c[0], c[1]) == o


@pytest.mark.parametrize("case", range(3))
def test_threefry_kat_host(case):
    k, c, o = kat()[case]
    a, b = prng.threefry2x32(k[0], k[1], c[0], c[1])
    assert (int(a), int(b)) == o


def test_host_keys_match_oracle(orc):
    key = prng.PRNGKey(7)
    assert np.array_equal(prng.split(key, 1000), orc.split(key, 1000))
    k2 = prng.split(prng.PRNGKey(1), 2)
    u = prng.uniform(k2[0], 5000)
    assert np.array_equal(u.view(np.uint32), orc.uniform(k2[0], 5000).view(np.uint32))
    assert u.min() >= 0.0 and u.max() < 1.0
    z = prng.uniform(k2[1], 5000, 0.1, 0.9)
    assert np.array_equal(z.view(np.uint32), orc.uniform(k2[1], 5000, 0.1, 0.9).view(np.uint32))
    assert z.min() >= np.float32(0.1) and z.max() < 0.9
    fk = prng.fold_in(key, np.arange(10, dtype=np.uint32))
    for i in range(10):
        assert tuple(int(v) for v in fk[i]) == orc.threefry2x32(key[0], key[1], 0, i)


@pytest.mark.parametrize("name", ["uniform", "wide", "subnormal", "cancel", "oob", "overflow"])
def test_exact_sum_golden(orc, name):
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    out, st = orc.exact_sum(d[name + "_vals"], d[name + "_bins"], int(d[name + "_nb"]))
    exp = d[name + "_expect"]
    assert np.array_equal(out, exp, equal_nan=True)
    nz = ~np.isnan(exp)
    assert np.array_equal(out[nz].view(np.uint32), exp[nz].view(np.uint32))   # signed zeros too
    assert st[3] == int(np.isnan(exp).sum())


def test_exact_sum_order_independent(orc):
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    v, b, nb = d["wide_vals"], d["wide_bins"], int(d["wide_nb"])
    p = np.random.default_rng(0).permutation(len(v))
    a, _ = orc.exact_sum(v, b, nb)
    c, _ = orc.exact_sum(v[p], b[p], nb)
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


def q1_inputs(n):
    return np.linspace(0.1, 0.99, n, dtype=np.float32), prng.split(prng.PRNGKey(0), n)


def rw_inputs(n, seed=1):
    kx, ks = prng.split(prng.PRNGKey(seed), 2)
    return prng.uniform(kx, n), prng.split(ks, n)


def test_q1_forward_basics(orc):
    x, k = q1_inputs(10000)
    r = orc.q1_fwd(x, k, 2.0)
    assert r["stats"].tolist() == [0, 0, 0, 0, 0]
    assert not r["trunc"].any()
    assert 2 <= r["k"].mean() <= 12
    # hist = theta * sum over steps of (1 - x): the gradient of hist.sum() is hist.sum() / theta
    g = orc.q1_grad(x, k, 2.0, np.ones(16, np.float32))
    assert abs(g["g"][0] - r["hist"].sum() / 2.0) <= 1e-5 * abs(g["g"][0])


@pytest.mark.parametrize("C", [1, 2, 4, 16, 64])
def test_replay_invariant_to_checkpoints(orc, C):
    """the checkpoint count changes the replay's work, not the order of the step VJPs: bitwise the same"""
    x, k = rw_inputs(2048)
    ct = np.random.default_rng(1).uniform(0.5, 1.5, 256).astype(np.float32)
    ref = orc.rw_grad(x, k, 1.0, ct, C=16)
    got = orc.rw_grad(x, k, 1.0, ct, C=C)
    assert got["g"].view(np.uint32)[0] == ref["g"].view(np.uint32)[0]
    assert np.array_equal(got["trunc"], ref["trunc"])


def test_rw_grad_is_linear_tally(orc):
    x, k = rw_inputs(4096)
    f = orc.rw_fwd(x, k, 1.0, nthreads=4)
    g = orc.rw_grad(x, k, 1.0, np.ones(256, np.float32), nthreads=4)
    assert abs(g["g"][0] - f["hist"].sum()) <= 1e-5 * abs(g["g"][0])
    assert f["side"].sum() == 4096


def test_rw_threads_deterministic_ints(orc):
    x, k = rw_inputs(4096)
    a = orc.rw_fwd(x, k, 1.0, nthreads=1)
    b = orc.rw_fwd(x, k, 1.0, nthreads=4)
    assert np.array_equal(a["k"], b["k"]) and np.array_equal(a["trunc"], b["trunc"])
    assert np.allclose(a["hist"], b["hist"], rtol=1e-5, atol=1e-6 * np.abs(a["hist"]).max())
    ga = orc.rw_grad(x, k, 1.0, np.ones(256, np.float32), nthreads=1)
    gb = orc.rw_grad(x, k, 1.0, np.ones(256, np.float32), nthreads=4)
    assert ga["g"].view(np.uint32)[0] == gb["g"].view(np.uint32)[0]      # exact tally: order-independent


def test_truncation_and_drops(orc):
    # x0 = 1.0 sits in bin 256 (dropped, counted); max_steps = 5 truncates most items
    x = np.float32([1.0, 0.5, -0.25, 1.5, np.nan, 0.0])
    k = prng.split(prng.PRNGKey(3), len(x))
    r = orc.rw_fwd(x, k, 1.0, max_steps=5)
    assert r["k"][2] == 0 and r["k"][3] == 0 and r["k"][4] == 0          # outside [0, 1] (NaN too): no step
    assert r["stats"][4] >= 1
    assert r["trunc"][1] and not r["trunc"][2]
    assert r["side"][1] >= 1                                              # x0 = 1.5 exits high at once


def test_empty(orc):
    x = np.zeros(0, np.float32)
    k = np.zeros((0, 2), np.uint32)
    r = orc.rw_fwd(x, k, 1.0)
    assert r["hist"].sum() == 0 and r["k"].size == 0
    g = orc.rw_grad(x, k, 1.0, np.ones(256, np.float32))
    assert g["g"][0] == 0.0


def test_oracle_sh_grad_energy(orc):
    """the oracle's tree adjoint: with ct_dep = 1 each root's E cotangent is the share of its energy that lands in
    range (1 up to rounding: children split E into z E and (1 - z) E), and X0 and depth get none (they only move
    integer bins)"""
    inp = orc.sh_inputs(200, seed=4)
    g = orc.sh_grad(*inp)
    assert np.median(np.abs(g["g_E"] - 1.0)) < 1e-5 and np.abs(g["g_E"] - 1.0).max() < 1e-2
    assert g["g_X0"][0] == 0.0 and not g["g_depth"].any()
    ct = np.random.default_rng(2).normal(size=512).astype(np.float32)
    g2 = orc.sh_grad(*inp, ct_dep=ct)
    # linearity in the cotangent
    g3 = orc.sh_grad(*inp, ct_dep=2 * ct)
    assert np.allclose(g3["g_E"], 2 * g2["g_E"], rtol=1e-6, atol=1e-6)


def test_onepass_order_within_tolerance(orc):
    """the oracle's one-pass summation order (C = -1, the checker of the one-pass kernels) against the reference's
    newest-first order: within the float tolerance, and bitwise when every contribution is exact"""
    from tallymap_b200 import prng
    kx, ks = prng.split(prng.PRNGKey(3), 2)
    x, k = prng.uniform(kx, 300), prng.split(ks, 300)
    ct = np.random.default_rng(1).normal(size=256).astype(np.float32)
    a, b = orc.rw_grad(x, k, 1.0, ct, C=-1)["g"], orc.rw_grad(x, k, 1.0, ct)["g"]
    assert abs(float(a[0]) - float(b[0])) <= 1e-5 * abs(float(b[0]))
    xq = np.linspace(0.1, 0.99, 200, dtype=np.float32)
    kq = prng.split(prng.PRNGKey(0), 200)
    a, b = orc.q1_grad(xq, kq, 2.0, np.ones(16, np.float32), C=-1)["g"], orc.q1_grad(xq, kq, 2.0, np.ones(16, np.float32))["g"]
    assert abs(float(a[0]) - float(b[0])) <= 1e-5 * abs(float(b[0]))
