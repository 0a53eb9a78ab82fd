"""GPU parity at the benchmark sizes: each benchmark configuration at its full N, the sm_100a kernels (through
libtm_b200.so's C ABI) against the CPU oracle run on ALL the same items.

Bar (the reference's tolerances, tests/invariants.py:86-91, 192-207): per-item trip counts, truncation flags, stats
and integer-valued tallies bitwise; f32 tallies within FT = 1e-5 of the largest bin (the oracle's checker mode: f64
partials, one rounding); gradients, summed in the exact cotangent tally, bitwise -- the one-pass programs against
the oracle summing in the one-pass order (C = -1), the replay programs against the oracle's checkpointed replay
(_reverse.py:324-444; its cotangents do not depend on C, so the oracle runs it with a C above the trip counts,
linear time) -- and the one-pass gradient within FT of the replay's.

These are the runs the benchmark times (bench.py): the heavy tail of the walk's trip counts, the items near its
20,000-step cap and the handful that truncate at 4M only appear at full size.  The oracle takes a minute or two of
host time on a 16-core host."""
import numpy as np
import pytest
import torch

from tallymap_b200 import backend as B
from tallymap_b200 import prng

pytestmark = pytest.mark.gpu
FT = 1e-5


def near(a, b, tol=FT):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() <= tol * max(np.abs(b).max(), 1e-30)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def run(prog, pi, bc, M, **kw):
    out = B.run(prog, pi, bc, consts=(M,), **kw)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    return [o.cpu().numpy() for o in out]


def test_rw_full_size_against_oracle(cuda, orc):
    """benchmark configuration 2, N = 4,194,304, max_steps 20,000: the forward, the one-pass value-and-grad (the
    benchmark's step) and the exact-order replay gradient"""
    n, M = 4194304, 20000
    kx, ks = prng.split(prng.PRNGKey(1), 2)
    x, k = prng.uniform(kx, n), prng.split(ks, n)
    ct = np.ones(256, np.float32)
    zs = np.zeros(2, np.float32)
    hist, side, stats, kk, tr = run(B.RW_FWD, [x, k], [np.float32(1.0)], M)
    v_hist, v_side, v_g, v_stats, v_k, v_tr = run(B.RW_VG1, [x, k], [np.float32(1.0), ct, zs], M)
    r_g, r_stats, r_tr = run(B.RW_GRAD, [x, k], [np.float32(1.0), ct, zs], M)

    ref = orc.rw_fwd(x, k, 1.0, max_steps=M, nthreads=0)
    assert np.array_equal(kk, ref["k"]) and np.array_equal(tr.astype(bool), ref["trunc"])
    assert np.array_equal(stats, ref["stats"])
    assert np.array_equal(side, ref["side"]) and near(hist, ref["hist"])
    assert ref["k"].max() > 15000                 # the heavy tail is in the comparison
    assert np.array_equal(v_k, ref["k"]) and np.array_equal(v_tr.astype(bool), ref["trunc"])
    assert np.array_equal(v_stats, ref["stats"]) and np.array_equal(v_side, ref["side"]) and near(v_hist, ref["hist"])

    one = orc.rw_grad(x, k, 1.0, ct, max_steps=M, C=-1, nthreads=0)
    assert np.array_equal(bits(v_g), bits(one["g"]))
    rep = orc.rw_grad(x, k, 1.0, ct, max_steps=M, C=M, nthreads=0)
    assert np.array_equal(bits(r_g), bits(rep["g"])) and np.array_equal(r_tr.astype(bool), rep["trunc"])
    assert abs(float(v_g[0]) - float(r_g[0])) <= FT * abs(float(r_g[0]))


def test_ph_full_size_against_oracle(cuda, orc):
    """benchmark configuration 3, N = 4,194,304 photons: the forward, the one-pass (forward-mode) value-and-grad and the
    replay gradient w.r.t. (mu_a, mu_s); trip counts depend on log/sin/cos/sqrt, the shared math on both sides"""
    n, M = 4194304, 100000
    keys = prng.split(prng.PRNGKey(2), n)
    bc = [np.float32(0.1), np.float32(10.0)]
    ct = np.random.default_rng(33).uniform(0.5, 1.5, (64, 64, 64)).astype(np.float32)
    dep, stats, kk, tr = run(B.PH_FWD, [keys], bc, M)
    v_dep, v_g, v_stats, v_k, v_tr = run(B.PH_VG1, [keys], bc + [ct], M)
    r_g, r_stats, r_tr = run(B.PH_GRAD, [keys], bc + [ct], M)

    ref = orc.ph_fwd(keys, max_steps=M)
    assert np.array_equal(kk, ref["k"]) and np.array_equal(tr.astype(bool), ref["trunc"])
    assert np.array_equal(stats, ref["stats"]) and near(dep, ref["dep"])
    assert np.array_equal(v_k, ref["k"]) and np.array_equal(v_stats, ref["stats"]) and near(v_dep, ref["dep"])
    one = orc.ph_grad(keys, ct=ct, max_steps=M, C=-1)
    assert np.array_equal(bits(v_g), bits(one["g"]))
    rep = orc.ph_grad(keys, ct=ct, max_steps=M, C=4096)
    assert np.array_equal(bits(r_g), bits(rep["g"])) and np.array_equal(r_tr.astype(bool), rep["trunc"])
    assert near(v_g, r_g)


def test_od_full_size_against_oracle(cuda, orc):
    """benchmark configuration 4, N = 1,048,576 Lorenz systems: every item's final state (each bin of Sum((N, 3)) is
    written once, so exact), the accepted + rejected step counts, the replay gradient w.r.t. beta and the one-pass
    forward-mode gradient"""
    n, M = 1048576, 50000
    inp = orc.od_inputs(n)
    beta = np.float32(8.0 / 3.0)
    ctf = np.random.default_rng(44).normal(size=(n, 3)).astype(np.float32)
    fin, mean, stats, kk, tr = run(B.OD_FWD, list(inp), [beta], M)
    g, g_stats, g_tr = run(B.OD_GRAD, list(inp), [beta, ctf, np.float32(0.5)], M)

    ref = orc.od_fwd(*inp, beta=beta, max_steps=M)
    assert np.array_equal(kk, ref["k"]) and np.array_equal(tr.astype(bool), ref["trunc"])
    assert np.array_equal(stats, ref["stats"])
    assert np.array_equal(bits(fin.reshape(n, 3)), bits(ref["final"]))
    assert abs(float(mean.reshape(-1)[0]) - float(ref["mean"][0])) <= FT * abs(float(ref["mean"][0]))
    rep = orc.od_grad(*inp, beta=beta, ct_final=ctf, ct_mean=0.5, max_steps=M, C=4096)
    assert np.array_equal(bits(g), bits(rep["g"])) and np.array_equal(g_tr.astype(bool), rep["trunc"])
    # the one-pass forward-mode launch (the bench's step): bitwise the oracle's forward mode at full size
    fin1, mean1, g1, st1, k1, tr1 = run(B.OD_VG1, list(inp), [beta, ctf, np.float32(0.5)], M)
    ref1 = orc.od_vg1(*inp, beta=beta, ct_final=ctf, ct_mean=0.5, max_steps=M)
    assert np.array_equal(bits(g1), bits(ref1["g"])) and np.array_equal(k1, ref["k"])
    assert np.array_equal(bits(fin1.reshape(n, 3)), bits(ref["final"])) and np.array_equal(st1, ref["stats"])
    assert abs(float(g1[0]) - float(g[0])) <= 1e-4 * abs(float(g[0]))


def test_sh_full_size_against_oracle(cuda, orc):
    """benchmark configuration 5, N = 1,048,576 primaries (about 10^9 particles through the spawn ring): particle
    count, spawned children, per-root trip counts and flags, stats; the deposit; the one-pass per-root gradient"""
    n, M = 1048576, 100000
    inp = orc.sh_inputs(n)
    dep, count, stats, kk, tr = run(B.SH_FWD, list(inp), [np.float32(1.0)], M)
    ctd = np.random.default_rng(55).uniform(-1, 1, 512).astype(np.float32)
    r = B.sh_value_and_grad(list(inp), np.float32(1.0), ctd, max_steps=M)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    v = {key: t.cpu().numpy() for key, t in r.items()}

    ref = orc.sh_fwd(*inp, max_steps=M)
    assert np.array_equal(count, ref["count"]) and np.array_equal(stats, ref["stats"]) and stats[1] == 0
    assert np.array_equal(kk, ref["k"]) and np.array_equal(tr.astype(bool), ref["trunc"])
    assert near(dep, ref["dep"])
    assert np.array_equal(v["count"], ref["count"]) and np.array_equal(v["k"], ref["k"]) and near(v["dep"], ref["dep"])
    one = orc.sh_vg1(*inp, ct_dep=ctd, max_steps=M)
    assert np.array_equal(bits(v["g_E"]), bits(one["g_E"]))
