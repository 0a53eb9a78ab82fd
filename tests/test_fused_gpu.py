"""GPU parity of the fused value-and-grad programs (one launch: the replay's count pass is the forward pass and
emits its tallies): forward outputs and gradient against the oracle and against the separate forward + replay
launches.  Integer outputs, stats and gradients bitwise; f32 tallies within the float-tally tolerance (atomic order)."""
import numpy as np
import pytest
import torch

import tallymap_b200 as tm
from tallymap_b200 import backend as B
from tallymap_b200 import prng

pytestmark = pytest.mark.gpu
FT = 1e-5


def near(a, b, tol=FT):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() <= tol * max(np.abs(b).max(), 1e-30)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def rw_inputs(n, seed=1):
    kx, ks = prng.split(prng.PRNGKey(seed), 2)
    return prng.uniform(kx, n), prng.split(ks, n)


def vg(prog, pi, bc, M, C=None):
    out = B.run(prog, pi, bc, consts=(M,), rev_checkpoints=C)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    return [o.cpu().numpy() for o in out]


@pytest.mark.parametrize("n,C", [(1, None), (777, None), (20000, None), (20000, 3), (20000, 64)])
def test_rw_vg(cuda, orc, n, C):
    x, k = rw_inputs(n, seed=4)
    ct_h = np.random.default_rng(n).normal(size=256).astype(np.float32)
    ct_s = np.float32([0.5, -2.0])
    hist, side, g, stats, kk, tr = vg(B.RW_VG, [x, k], [np.float32(1.0), ct_h, ct_s], 20000, C)
    # the pipelined kernel when every item fits the head (C >= max_steps), else the fused checkpointed replay
    assert B.run.last["kernel"] == ("rw_vg" if C is None else "rw_vg_replay")
    rf = orc.rw_fwd(x, k, 1.0)
    rg = orc.rw_grad(x, k, 1.0, ct_h)
    assert np.array_equal(kk, rf["k"]) and np.array_equal(tr.astype(bool), rf["trunc"])
    assert near(hist, rf["hist"]) and near(side, rf["side"])
    assert np.array_equal(bits(g), bits(rg["g"]))
    # stats: the forward's (dropped emits) plus the adjoint's (fixed-point overflow)
    assert np.array_equal(stats, rf["stats"] + rg["stats"])


@pytest.mark.parametrize("ct", ["ones", "random"])
def test_q1_vg(cuda, orc, ct):
    x = np.linspace(0.1, 0.99, 10000, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), 10000)
    c = np.ones(16, np.float32) if ct == "ones" else np.random.default_rng(5).normal(size=16).astype(np.float32)
    hist, g, stats, kk, tr = vg(B.Q1_VG, [x, k], [np.float32(2.0), c], 100)
    rf = orc.q1_fwd(x, k, 2.0)
    rg = orc.q1_grad(x, k, 2.0, c)
    assert np.array_equal(kk, rf["k"]) and np.array_equal(tr.astype(bool), rf["trunc"])
    assert near(hist, rf["hist"])
    assert np.array_equal(bits(g), bits(rg["g"]))


def test_q1_vg_truncation(cuda, orc):
    x = np.linspace(0.1, 0.99, 3000, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), 3000)
    hist, g, stats, kk, tr = vg(B.Q1_VG, [x, k], [np.float32(2.0), np.ones(16, np.float32)], 3)
    rf = orc.q1_fwd(x, k, 2.0, max_steps=3)
    assert rf["trunc"].sum() > 0 and np.array_equal(tr.astype(bool), rf["trunc"])
    assert np.array_equal(kk, rf["k"])


def test_api_value_and_grad_fused_matches_two_launches(cuda):
    n = 50000
    x, k = rw_inputs(n, seed=9)
    f = tm.vmap("walk1d", outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None))
    cts = {"hist": torch.ones(256), "side": torch.zeros(2)}
    r1, g1 = f.value_and_grad(x, k, np.float32(1.0), wrt=2, cotangents=cts, exact_order=True)
    assert B.run.last["kernel"] == "rw_vg"
    r2, g2 = f.value_and_grad(x, k, np.float32(1.0), wrt=2, cotangents=cts, fused=False)
    r3, g3 = f.value_and_grad(x, k, np.float32(1.0), wrt=2, cotangents=cts)      # the one-pass default
    assert B.run.last["kernel"] == "rw_vg_onepass"
    torch.cuda.synchronize()
    assert np.array_equal(bits(g1.cpu().numpy()), bits(g2.cpu().numpy()))
    assert near(g3.cpu().numpy(), g2.cpu().numpy())
    assert np.array_equal(r3.per_item.cpu().numpy(), r2.per_item.cpu().numpy())
    assert np.array_equal(r1.per_item.cpu().numpy(), r2.per_item.cpu().numpy())
    assert np.array_equal(r1.truncated.cpu().numpy(), r2.truncated.cpu().numpy())
    assert near(r1.outputs["hist"].cpu().numpy(), r2.outputs["hist"].cpu().numpy())
    assert int(r1.stats["n_truncated"]) == int(r2.stats["n_truncated"])


def test_rw_vg_full_size(cuda, orc):
    """N = 4,194,304: fused gradient bitwise the separate replay's; forward trip counts bitwise the forward's"""
    x, k = rw_inputs(4194304)
    ct_h = np.ones(256, np.float32)
    hist, side, g, stats, kk, tr = vg(B.RW_VG, [x, k], [np.float32(1.0), ct_h, np.zeros(2, np.float32)], 20000)
    out = B.run(B.RW_FWD, [x, k], [np.float32(1.0)], consts=(20000,))
    gout = B.run(B.RW_GRAD, [x, k], [np.float32(1.0), ct_h, np.zeros(2, np.float32)], consts=(20000,))
    torch.cuda.synchronize()
    assert np.array_equal(kk, out[3].cpu().numpy()) and np.array_equal(tr, out[4].cpu().numpy())
    assert np.array_equal(bits(g), bits(gout[0].cpu().numpy()))
    assert near(hist, out[0].cpu().numpy()) and near(side, out[1].cpu().numpy())


# ---------------------------------------------------------------------------------------------- one pass
# The walkers have no active carry: the one-pass programs sum each step's VJP as the forward runs (OnePassVG).  The
# per-item cotangent is summed oldest step first: bitwise the oracle run in that order (C = -1), within the float
# tolerance of the reference's newest-first order.
@pytest.mark.parametrize("n", [1, 777, 20000])
def test_rw_vg_onepass(cuda, orc, n):
    x, k = rw_inputs(n, seed=4)
    ct_h = np.random.default_rng(n).normal(size=256).astype(np.float32)
    ct_s = np.float32([0.5, -2.0])
    hist, side, g, stats, kk, tr = vg(B.RW_VG1, [x, k], [np.float32(1.0), ct_h, ct_s], 20000)
    rf = orc.rw_fwd(x, k, 1.0)
    assert np.array_equal(kk, rf["k"]) and np.array_equal(tr.astype(bool), rf["trunc"])
    assert near(hist, rf["hist"]) and near(side, rf["side"])
    r1 = orc.rw_grad(x, k, 1.0, ct_h, C=-1)
    assert np.array_equal(bits(g), bits(r1["g"]))
    rg = orc.rw_grad(x, k, 1.0, ct_h)
    assert near(g, rg["g"])
    assert np.array_equal(stats, rf["stats"] + rg["stats"])


@pytest.mark.parametrize("ct", ["ones", "random"])
def test_q1_vg_onepass(cuda, orc, ct):
    x = np.linspace(0.1, 0.99, 10000, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), 10000)
    c = np.ones(16, np.float32) if ct == "ones" else np.random.default_rng(5).normal(size=16).astype(np.float32)
    hist, g, stats, kk, tr = vg(B.Q1_VG1, [x, k], [np.float32(2.0), c], 100)
    rf = orc.q1_fwd(x, k, 2.0)
    assert np.array_equal(kk, rf["k"]) and np.array_equal(tr.astype(bool), rf["trunc"])
    assert near(hist, rf["hist"])
    assert np.array_equal(bits(g), bits(orc.q1_grad(x, k, 2.0, c, C=-1)["g"]))
    assert near(g, orc.q1_grad(x, k, 2.0, c)["g"])


def test_q1_vg_onepass_truncation_poisons(cuda):
    x = np.linspace(0.1, 0.99, 3000, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), 3000)
    f = tm.vmap("quickstart", outputs={"hist": tm.Sum((16,))}, in_axes=(0, 0, None), max_steps=3)
    r, g = f.value_and_grad(x, k, np.float32(2.0), wrt=2, cotangents={"hist": torch.ones(16)})
    assert B.run.last["kernel"] == "q1_vg_onepass"
    assert int(r.stats["n_truncated"]) > 0 and torch.isnan(g).all() and torch.isnan(r.outputs["hist"]).all()


def test_rw_vg_onepass_full_size(cuda, orc):
    """N = 4,194,304: the one-pass gradient within the float tolerance of the replay's; trip counts bitwise"""
    x, k = rw_inputs(4194304)
    ct_h = np.ones(256, np.float32)
    hist, side, g, stats, kk, tr = vg(B.RW_VG1, [x, k], [np.float32(1.0), ct_h, np.zeros(2, np.float32)], 20000)
    gout = B.run(B.RW_GRAD, [x, k], [np.float32(1.0), ct_h, np.zeros(2, np.float32)], consts=(20000,))
    out = B.run(B.RW_FWD, [x, k], [np.float32(1.0)], consts=(20000,))
    torch.cuda.synchronize()
    assert np.array_equal(kk, out[3].cpu().numpy()) and np.array_equal(tr, out[4].cpu().numpy())
    assert near(g, gout[0].cpu().numpy()) and near(hist, out[0].cpu().numpy())
