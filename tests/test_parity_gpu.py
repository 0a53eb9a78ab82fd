"""GPU parity: the sm_100a kernels (through libtm_b200.so's C ABI) against the CPU oracle on the same inputs.

Bar (the reference's own tolerances, tests/invariants.py:86-91, 192-207): trip counts, truncation flags, stats and
every other integer output bitwise; f32 tallies within 1e-5 relative to the largest bin (atomic summation order
differs); gradients, which go through the exact cotangent tally, bitwise.
"""
import numpy as np
import pytest
import torch

from tallymap_b200 import backend as B
from tallymap_b200 import prng

pytestmark = pytest.mark.gpu
FT = 1e-5     # float tally tolerance, relative to the largest |bin| (tests/invariants.py:86-91)


def near(a, b, tol=FT):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    return np.abs(a - b).max() <= tol * scale


def q1_inputs(n):
    return np.linspace(0.1, 0.99, n, dtype=np.float32), prng.split(prng.PRNGKey(0), n)


def rw_inputs(n, seed=1):
    kx, ks = prng.split(prng.PRNGKey(seed), 2)
    return prng.uniform(kx, n), prng.split(ks, n)


def gpu_q1(x, k, theta, M=100):
    out = B.run(B.Q1_FWD, [x, k], [np.float32(theta)], consts=(M,))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    hist, stats, kk, tr = [o.cpu().numpy() for o in out]
    return dict(hist=hist, stats=stats, k=kk, trunc=tr.astype(bool))


def gpu_q1_grad(x, k, theta, ct, M=100):
    out = B.run(B.Q1_GRAD, [x, k], [np.float32(theta), ct], consts=(M,))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    g, stats, tr = [o.cpu().numpy() for o in out]
    return dict(g=g, stats=stats, trunc=tr.astype(bool))


def gpu_rw(x, k, drift, M=20000):
    out = B.run(B.RW_FWD, [x, k], [np.float32(drift)], consts=(M,))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    hist, side, stats, kk, tr = [o.cpu().numpy() for o in out]
    return dict(hist=hist, side=side, stats=stats, k=kk, trunc=tr.astype(bool))


def gpu_rw_grad(x, k, drift, ct_hist, ct_side=None, M=20000, C=None, order=None):
    ct_side = np.zeros(2, np.float32) if ct_side is None else ct_side
    out = B.run(B.RW_GRAD, [x, k], [np.float32(drift), ct_hist, ct_side], consts=(M,), rev_checkpoints=C,
                order=order)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    g, stats, tr = [o.cpu().numpy() for o in out]
    return dict(g=g, stats=stats, trunc=tr.astype(bool))


def same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


# ------------------------------------------------------------------------------------------------ Q1
@pytest.mark.parametrize("n", [1, 31, 10000])
def test_q1_forward(cuda, orc, n):
    x, k = q1_inputs(n)
    ref = orc.q1_fwd(x, k, 2.0)
    got = gpu_q1(x, k, 2.0)
    assert np.array_equal(got["k"], ref["k"])
    assert np.array_equal(got["trunc"], ref["trunc"])
    assert np.array_equal(got["stats"], ref["stats"])
    assert near(got["hist"], ref["hist"])


@pytest.mark.parametrize("ct", ["ones", "random"])
def test_q1_grad_bitwise(cuda, orc, ct):
    x, k = q1_inputs(10000)
    c = np.ones(16, np.float32) if ct == "ones" else np.random.default_rng(5).normal(size=16).astype(np.float32)
    ref = orc.q1_grad(x, k, 2.0, c)
    got = gpu_q1_grad(x, k, 2.0, c)
    assert same_bits(got["g"], ref["g"])
    assert np.array_equal(got["trunc"], ref["trunc"])
    assert np.array_equal(got["stats"], ref["stats"])


def test_q1_edge_inputs(cuda, orc):
    # NaN / negative / out-of-range starts, an exactly-on-threshold start, bins >= 16 (dropped and counted)
    x = np.float32([np.nan, -1.0, 0.05, 0.0500001, 1.5, 100.0, 0.99, 3e38, -0.0, 1e-30])
    k = prng.split(prng.PRNGKey(11), len(x))
    ref = orc.q1_fwd(x, k, 2.0)
    got = gpu_q1(x, k, 2.0)
    assert np.array_equal(got["k"], ref["k"])
    assert np.array_equal(got["stats"], ref["stats"]) and ref["stats"][4] > 0
    assert near(got["hist"], ref["hist"])


def test_q1_truncation(cuda, orc):
    x, k = q1_inputs(5000)
    ref = orc.q1_fwd(x, k, 2.0, max_steps=3)
    got = gpu_q1(x, k, 2.0, M=3)
    assert ref["trunc"].sum() > 0
    assert np.array_equal(got["trunc"], ref["trunc"]) and np.array_equal(got["k"], ref["k"])
    g_ref = orc.q1_grad(x, k, 2.0, np.ones(16, np.float32), max_steps=3)
    g_got = gpu_q1_grad(x, k, 2.0, np.ones(16, np.float32), M=3)
    assert np.array_equal(g_got["trunc"], g_ref["trunc"]) and same_bits(g_got["g"], g_ref["g"])


def test_empty_launch(cuda):
    x = np.zeros(0, np.float32)
    k = np.zeros((0, 2), np.uint32)
    got = gpu_rw(x, k, 1.0)
    assert got["hist"].sum() == 0 and got["k"].size == 0 and got["stats"].sum() == 0
    g = gpu_rw_grad(x, k, 1.0, np.ones(256, np.float32))
    assert g["g"][0] == 0.0


# ------------------------------------------------------------------------------------------------ RW
@pytest.mark.parametrize("n", [1000, 65536 + 7])
def test_rw_forward(cuda, orc, n):
    x, k = rw_inputs(n)
    ref = orc.rw_fwd(x, k, 1.0, nthreads=0)
    got = gpu_rw(x, k, 1.0)
    assert np.array_equal(got["k"], ref["k"])
    assert np.array_equal(got["trunc"], ref["trunc"])
    assert np.array_equal(got["stats"], ref["stats"])
    assert np.array_equal(got["side"], ref["side"])           # integer-valued: exact
    assert near(got["hist"], ref["hist"])


def test_rw_grad_bitwise(cuda, orc):
    x, k = rw_inputs(65536)
    ct = np.random.default_rng(7).uniform(0.5, 1.5, 256).astype(np.float32)
    ref = orc.rw_grad(x, k, 1.0, ct, nthreads=0)
    got = gpu_rw_grad(x, k, 1.0, ct)
    assert same_bits(got["g"], ref["g"])
    assert np.array_equal(got["trunc"], ref["trunc"])


@pytest.mark.parametrize("C", [1, 3, 16, 64, 1024])
def test_rw_grad_checkpoint_invariance(cuda, orc, C):
    """the replay's checkpoint count changes its work and memory, never the cotangent (the step VJPs run in the same
    order on the same states): every C is bitwise the oracle's C = 16 replay"""
    x, k = rw_inputs(8192, seed=4)
    ct = np.random.default_rng(8).uniform(0.5, 1.5, 256).astype(np.float32)
    ref = orc.rw_grad(x, k, 1.0, ct, nthreads=0)
    got = gpu_rw_grad(x, k, 1.0, ct, C=C)
    assert same_bits(got["g"], ref["g"]) and np.array_equal(got["trunc"], ref["trunc"])


@pytest.mark.parametrize("how", ["longest_first", "reversed", "random"])
def test_claim_order_changes_nothing(cuda, orc, how):
    """an item claim order moves work between threads, never a result: per-item flags at their own index, the
    exact gradient bitwise"""
    from tallymap_b200.api import longest_first
    x, k = rw_inputs(20000, seed=6)
    f = gpu_rw(x, k, 1.0)
    order = {"longest_first": longest_first(torch.from_numpy(f["k"])).numpy(),
             "reversed": np.arange(len(x), dtype=np.int32)[::-1].copy(),
             "random": np.random.default_rng(0).permutation(len(x)).astype(np.int32)}[how]
    ref = orc.rw_grad(x, k, 1.0, np.ones(256, np.float32), nthreads=0)
    got = gpu_rw_grad(x, k, 1.0, np.ones(256, np.float32), order=order)
    assert same_bits(got["g"], ref["g"]) and np.array_equal(got["trunc"], ref["trunc"])
    out = B.run(B.RW_FWD, [x, k], [np.float32(1.0)], consts=(20000,), order=order)
    kk = out[3].cpu().numpy()
    assert np.array_equal(kk, f["k"])


def test_rw_edge_inputs(cuda, orc):
    x = np.float32([1.0, 0.0, -1e-7, 1.0000001, np.nan, 0.5, 0.999, 1e-3])
    k = prng.split(prng.PRNGKey(9), len(x))
    for M in (1, 7, 20000):
        ref = orc.rw_fwd(x, k, 1.0, max_steps=M)
        got = gpu_rw(x, k, 1.0, M=M)
        assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
        assert np.array_equal(got["stats"], ref["stats"]) and np.array_equal(got["side"], ref["side"])
        assert near(got["hist"], ref["hist"])
        gr = orc.rw_grad(x, k, 1.0, np.ones(256, np.float32), max_steps=M)
        gg = gpu_rw_grad(x, k, 1.0, np.ones(256, np.float32), M=M)
        assert same_bits(gg["g"], gr["g"]) and np.array_equal(gg["trunc"], gr["trunc"])


# ------------------------------------------------------------------------------------------------ full size
def test_rw_full_size_properties(cuda):
    """benchmark configuration 2 at N = 4,194,304: size-independent checks (the oracle would take minutes here).
    The gradient of the linear tally drift * x is sum(hist) / drift; the run is bitwise repeatable in every integer
    output and in the exact gradient; every item exits or truncates."""
    n = 4194304
    x, k = rw_inputs(n)
    a = gpu_rw(x, k, 1.0)
    b = gpu_rw(x, k, 1.0)
    assert np.array_equal(a["k"], b["k"]) and np.array_equal(a["trunc"], b["trunc"])
    assert a["side"].sum() == n
    assert near(a["hist"], b["hist"])
    assert 1000 < a["k"].mean() < 1600 and a["k"].max() <= 20000
    ga = gpu_rw_grad(x, k, 1.0, np.ones(256, np.float32))
    gb = gpu_rw_grad(x, k, 1.0, np.ones(256, np.float32))
    assert same_bits(ga["g"], gb["g"])
    assert np.array_equal(ga["trunc"], a["trunc"])
    assert abs(float(ga["g"][0]) - float(a["hist"].sum(dtype=np.float64))) <= 1e-5 * abs(float(ga["g"][0]))


def test_api_contract(cuda):
    """Result: outputs poisoned with NaN when an item truncates; grad is one replay launch, NaN when truncated."""
    import tallymap_b200 as tm
    f = tm.vmap("walk1d", outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None),
                max_steps=20000)
    x, k = rw_inputs(4096)
    r = f(x, k, np.float32(1.0))
    assert int(r.stats["n_truncated"]) == 0 and not torch.isnan(r.outputs["hist"]).any()
    g = f.grad(x, k, np.float32(1.0), wrt=2, cotangents={"hist": torch.ones(256)})
    assert abs(float(g) - float(r.outputs["hist"].double().sum())) <= 1e-5 * abs(float(g))
    f3 = tm.vmap("walk1d", outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=3)
    r3 = f3(x, k, np.float32(1.0))
    assert int(r3.stats["n_truncated"]) > 0
    assert torch.isnan(r3.outputs["hist"]).all() and torch.isnan(r3.outputs["side"]).all()
    assert torch.isnan(f3.grad(x, k, np.float32(1.0), wrt=2, cotangents={"hist": torch.ones(256)}))
