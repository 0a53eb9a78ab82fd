"""GPU parity of the branching shower (benchmark configuration 5): the warp-aggregated spawn ring against the oracle's
depth-first traversal.  With a ring large enough to drop nothing: particle count, spawned children, per-root trip
counts and truncation flags, and every stat bitwise; the depth deposit within the float-tally tolerance.  With a
tiny ring: children are dropped and counted, every popped child still runs exactly once, and no wait times out."""
import numpy as np
import pytest
import torch

from tallymap_b200 import backend as B

pytestmark = pytest.mark.gpu
FT = 1e-5


def gpu_sh(inp, X0=1.0, M=100000, Q=None):
    out = B.run(B.SH_FWD, list(inp), [np.float32(X0)], consts=(M,), queue=Q)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    dep, count, stats, k, tr = [o.cpu().numpy() for o in out]
    return dict(dep=dep, count=count, stats=stats, k=k, trunc=tr.astype(bool))


@pytest.mark.parametrize("n", [1, 777, 20000])
def test_sh_forward(cuda, orc, n):
    inp = orc.sh_inputs(n)
    ref = orc.sh_fwd(*inp)
    got = gpu_sh(inp)
    assert np.array_equal(got["count"], ref["count"])
    assert np.array_equal(got["stats"], ref["stats"]) and got["stats"][1] == 0
    assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
    assert np.abs(got["dep"].astype(np.float64) - ref["dep"]).max() <= FT * np.abs(ref["dep"]).max()


def test_sh_truncation(cuda, orc):
    inp = orc.sh_inputs(3000)
    ref = orc.sh_fwd(*inp, max_steps=1)
    got = gpu_sh(inp, M=1)
    assert ref["stats"][2] > 0 and ref["trunc"].any()
    assert np.array_equal(got["stats"], ref["stats"]) and np.array_equal(got["count"], ref["count"])
    assert np.array_equal(got["trunc"], ref["trunc"])


@pytest.mark.parametrize("Q", [64, 4096])
def test_sh_small_ring_drops(cuda, orc, Q):
    inp = orc.sh_inputs(5000)
    got = gpu_sh(inp, Q=Q)
    spawned, dropped = int(got["stats"][0]), int(got["stats"][1])
    assert dropped > 0
    assert int(got["count"][0]) == 5000 + spawned          # every root and every pushed child ran once


def test_sh_full_size(cuda, orc):
    """N = 1,048,576 primaries (~10^9 particles): counts repeatable; energy conserved into the deposit (up to the
    deposits dropped beyond depth 64, counted in stats[4])"""
    inp = orc.sh_inputs(1048576)
    a = gpu_sh(inp)
    b = gpu_sh(inp)
    assert np.array_equal(a["count"], b["count"]) and np.array_equal(a["stats"], b["stats"])
    assert np.array_equal(a["k"], b["k"])
    assert int(a["count"][0]) == 1048576 + int(a["stats"][0]) and a["stats"][1] == 0
    e0 = float(inp[0].astype(np.float64).sum())
    assert abs(float(a["dep"].astype(np.float64).sum()) - e0) <= 1e-3 * e0


# ---------------------------------------------------------------------------------------------- the tree adjoint
def gpu_sh_grad(inp, X0=1.0, ct=None, M=100000, Q=None, R=None):
    ct = np.ones(512, np.float32) if ct is None else ct
    r = B.tree_grad(list(inp), np.float32(X0), ct, max_steps=M, queue=Q, record=R)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    B.check_status(B.tree_grad.last["ctl"])
    out = {k: r[k].cpu().numpy() for k in ("ct_X0", "ct_E", "ct_depth")}
    out["info"] = r["info"]
    out["poisoned"] = bool(r["info"]["poisoned"].item())
    out["mismatch"] = int(r["info"]["mismatch"].item())
    out["fwd"] = [o.cpu().numpy() for o in r["forward"]]
    return out


@pytest.mark.parametrize("n", [1, 300, 3000])
def test_sh_tree_grad(cuda, orc, n):
    """the per-generation adjoint launches against the oracle's post-order traversal: every root's E and depth
    cotangent bitwise, the X0 cotangent (an exact tally) bitwise; the recording forward's outputs as the forward's"""
    inp = orc.sh_inputs(n, seed=7)
    ct = np.random.default_rng(n).normal(size=512).astype(np.float32)
    ref = orc.sh_grad(*inp, ct_dep=ct)
    got = gpu_sh_grad(inp, ct=ct)
    assert not got["poisoned"] and got["mismatch"] == 0
    assert np.array_equal(got["ct_E"].view(np.uint32), ref["g_E"].view(np.uint32))
    assert np.array_equal(got["ct_depth"].view(np.uint32), ref["g_depth"].view(np.uint32))
    assert np.array_equal(got["ct_X0"].view(np.uint32), ref["g_X0"].view(np.uint32))
    fr = orc.sh_fwd(*inp)
    dep, count, stats, k, tr = got["fwd"]
    assert np.array_equal(count, fr["count"]) and np.array_equal(stats, fr["stats"])
    assert np.array_equal(k, fr["k"]) and np.array_equal(tr.astype(bool), fr["trunc"])
    assert got["info"]["children"] == int(fr["stats"][0])
    assert sum(got["info"]["generation_sizes"]) == int(fr["stats"][0])
    assert got["info"]["launches"] == 2 + sum(1 for c in got["info"]["generation_sizes"][1:] if c) + 1


def test_sh_tree_grad_energy(cuda, orc):
    """with ct_dep = 1 a root's E cotangent is the fraction of its energy deposited in range: 1 up to rounding for
    every root whose tree stays within depth 64"""
    inp = orc.sh_inputs(5000, seed=9)
    got = gpu_sh_grad(inp)
    assert not got["poisoned"]
    assert np.abs(got["ct_E"] - 1.0).max() < 1e-2 and np.median(np.abs(got["ct_E"] - 1.0)) < 1e-5
    assert float(got["ct_X0"][0]) == 0.0 and not got["ct_depth"].any()


@pytest.mark.parametrize("how", ["record", "ring", "steps"])
def test_sh_tree_grad_poison(cuda, orc, how):
    """an incomplete record (capacity below the children, or children dropped by a small ring) or a truncated
    particle poisons every cotangent (tallymap/_reverse_spawn.py:30-38); the forward outputs stay as they are"""
    inp = orc.sh_inputs(2000, seed=3)
    kw = dict(record=dict(R=1000), ring=dict(Q=64), steps=dict(M=1))[how]
    got = gpu_sh_grad(inp, **kw)
    assert got["poisoned"]
    assert np.isnan(got["ct_E"]).all() and np.isnan(got["ct_X0"]).all() and np.isnan(got["ct_depth"]).all()
    if how == "record":
        ref = orc.sh_fwd(*inp)
        assert np.array_equal(got["fwd"][1], ref["count"]) and got["info"]["children"] == int(ref["stats"][0])


def test_sh_tree_grad_full_size(cuda, orc):
    """N = 1,048,576 roots (~10^9 recorded children): the tree adjoint against the oracle's post-order traversal of
    every root -- each root's E and depth cotangents and the X0 cotangent (an exact tally over all roots) bitwise --,
    repeatable bitwise, energy-conserving E cotangents"""
    inp = orc.sh_inputs(1048576)
    ct = np.random.default_rng(1048576).uniform(0.5, 1.5, 512).astype(np.float32)
    a = gpu_sh_grad(inp, ct=ct)
    b = gpu_sh_grad(inp, ct=ct)
    assert not a["poisoned"] and a["mismatch"] == 0
    assert np.array_equal(a["ct_E"].view(np.uint32), b["ct_E"].view(np.uint32))
    assert np.array_equal(a["ct_X0"].view(np.uint32), b["ct_X0"].view(np.uint32))
    ref = orc.sh_grad(*inp, ct_dep=ct)
    assert np.array_equal(a["ct_E"].view(np.uint32), ref["g_E"].view(np.uint32))
    assert np.array_equal(a["ct_depth"].view(np.uint32), ref["g_depth"].view(np.uint32))
    assert np.array_equal(a["ct_X0"].view(np.uint32), ref["g_X0"].view(np.uint32))
    e = gpu_sh_grad(inp)
    assert np.median(np.abs(e["ct_E"] - 1.0)) < 1e-5


# ---------------------------------------------------------------------------------------------- one pass
def near_roots(a, b):
    """per root: within 1e-5 relative, or 1e-6 absolute for near-zero roots (the float tolerance)"""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= np.maximum(1e-5 * np.abs(b), 1e-6)))


@pytest.mark.parametrize("n", [1, 777, 20000])
def test_sh_vg_onepass(cuda, orc, n):
    """forward mode through spawn in one launch: the forward's outputs as the forward's; g_E bitwise the oracle's
    forward mode (exact per-root sums) and within the float tolerance of the tree adjoint's"""
    inp = orc.sh_inputs(n)
    ct = np.random.default_rng(n).normal(size=512).astype(np.float32)
    r = B.sh_value_and_grad(list(inp), np.float32(1.0), ct)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    ref = orc.sh_fwd(*inp)
    assert np.array_equal(r["count"].cpu().numpy(), ref["count"])
    assert int(r["steps"][0]) >= int(r["count"][0]) + int(ref["k"].sum()) - n      # every particle steps once
    assert np.array_equal(r["k"].cpu().numpy(), ref["k"])
    assert np.array_equal(r["stats"].cpu().numpy(), ref["stats"])
    assert np.abs(r["dep"].cpu().numpy().astype(np.float64) - ref["dep"]).max() <= FT * np.abs(ref["dep"]).max()
    gE = r["g_E"].cpu().numpy()
    assert np.array_equal(gE.view(np.uint32), orc.sh_vg1(*inp, ct_dep=ct)["g_E"].view(np.uint32))
    tg = orc.sh_grad(*inp, ct_dep=ct)
    assert near_roots(gE, tg["g_E"])
    assert not r["g_depth"].any() and not tg["g_depth"].any() and float(tg["g_X0"][0]) == 0.0


def test_sh_api_value_and_grad_onepass(cuda):
    """value_and_grad of the shower runs the one spawn launch; against the recording forward + tree adjoint"""
    import tallymap_b200 as tm
    from oracle import oracle as orc
    inp = orc.sh_inputs(50000)
    f = tm.vmap("shower", outputs={"dep": tm.Sum((512,)), "count": tm.Sum((1,), torch.int32)},
                in_axes=(0, 0, 0, None))
    cts = {"dep": torch.from_numpy(np.random.default_rng(3).normal(size=512).astype(np.float32))}
    r1, (gE1, gX1) = f.value_and_grad(*inp, np.float32(1.0), wrt=(0, 3), cotangents=cts)
    assert B.run.last["kernel"] == "sh_vg_onepass"
    r2, (gE2, gX2) = f.value_and_grad(*inp, np.float32(1.0), wrt=(0, 3), cotangents=cts, exact_order=True)
    torch.cuda.synchronize()
    assert near_roots(gE1.cpu().numpy(), gE2.cpu().numpy())
    assert float(gX1) == 0.0 and float(gX2) == 0.0
    assert np.array_equal(r1.per_item.cpu().numpy(), r2.per_item.cpu().numpy())
    assert int(r1.outputs["count"][0]) == int(r2.outputs["count"][0])


def test_sh_energy_order_changes_no_result(cuda, orc):
    """roots claimed largest energy first (what the public API gives the shower's launches) against index order: the
    counts, trip counts, truncation flags and stats bitwise, the per-root g_E bitwise (exact sums), the deposit
    within the float tolerance (f32 atomics in another order)"""
    inp = orc.sh_inputs(20000)
    order = B.energy_order(torch.from_numpy(inp[0]).cuda())
    a = B.run(B.SH_FWD, list(inp), [np.float32(1.0)], consts=(100000,))
    b = B.run(B.SH_FWD, list(inp), [np.float32(1.0)], consts=(100000,), order=order)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    for x, y in zip(a[1:], b[1:]):
        assert torch.equal(x, y)
    assert float((a[0].double() - b[0].double()).abs().max()) <= FT * float(a[0].abs().max())
    ct = np.random.default_rng(9).normal(size=512).astype(np.float32)
    r1 = B.sh_value_and_grad(list(inp), np.float32(1.0), ct)
    r2 = B.sh_value_and_grad(list(inp), np.float32(1.0), ct, order=order)
    torch.cuda.synchronize()
    for k in ("count", "stats", "k", "trunc"):
        assert torch.equal(r1[k], r2[k]), k
    assert torch.equal(r1["g_E"].view(torch.int32), r2["g_E"].view(torch.int32))
    assert torch.equal(r1["g_E"].view(torch.int32),
                       torch.from_numpy(orc.sh_vg1(*inp, ct_dep=ct)["g_E"].view(np.int32)).cuda())


def test_sh_vg_onepass_small_queue_poisons(cuda, orc):
    """a queue too small: dropped children poison the gradient (NaN), never a silently partial one"""
    import tallymap_b200 as tm
    inp = orc.sh_inputs(5000)
    f = tm.vmap("shower", outputs={"dep": tm.Sum((512,)), "count": tm.Sum((1,), torch.int32)},
                in_axes=(0, 0, 0, None), spawn=tm.Queue(64))
    r, gE = f.value_and_grad(*inp, np.float32(1.0), wrt=0, cotangents={"dep": torch.ones(512)})
    assert int(r.stats["children_dropped"]) > 0 and torch.isnan(gE).all()
