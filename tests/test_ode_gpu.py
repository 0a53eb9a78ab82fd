"""GPU parity of the Lorenz RK45 ensemble (benchmark configuration 4): trip counts (accepted + rejected steps), truncation
flags, stats, the per-item final states (each bin of Sum((N, 3)) is written by one item, so it is exact) and the
exact beta gradient bitwise against the oracle; the mean-z scalar within the float-tally tolerance."""
import numpy as np
import pytest
import torch

from tallymap_b200 import backend as B

pytestmark = pytest.mark.gpu
BETA = np.float32(8.0 / 3.0)


def gpu_od(inp, beta=BETA, M=50000):
    out = B.run(B.OD_FWD, list(inp), [beta], consts=(M,))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    fin, mean, stats, k, tr = [o.cpu().numpy() for o in out]
    mean = mean.reshape(1)
    return dict(final=fin, mean=mean, stats=stats, k=k, trunc=tr.astype(bool))


def gpu_od_grad(inp, beta=BETA, ctf=None, ctm=1.0, M=50000, C=None):
    n = len(inp[0])
    ctf = np.ones((n, 3), np.float32) if ctf is None else ctf
    out = B.run(B.OD_GRAD, list(inp), [beta, ctf, np.float32(ctm)], consts=(M,), rev_checkpoints=C)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    g, stats, tr = [o.cpu().numpy() for o in out]
    return dict(g=g, stats=stats, trunc=tr.astype(bool))


@pytest.mark.parametrize("n", [1, 3000, 65536 + 5])
def test_od_forward(cuda, orc, n):
    inp = orc.od_inputs(n)
    ref = orc.od_fwd(*inp)
    got = gpu_od(inp)
    assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
    assert np.array_equal(got["stats"], ref["stats"])
    assert np.array_equal(got["final"].view(np.uint32), ref["final"].view(np.uint32))
    assert abs(float(got["mean"][0]) - float(ref["mean"][0])) <= 1e-5 * abs(float(ref["mean"][0]))


@pytest.mark.parametrize("C", [None, 2, 32])
def test_od_grad_bitwise(cuda, orc, C):
    inp = orc.od_inputs(4000, seed=11)
    ctf = np.random.default_rng(2).normal(size=(4000, 3)).astype(np.float32)
    ref = orc.od_grad(*inp, ct_final=ctf, ct_mean=0.5)
    got = gpu_od_grad(inp, ctf=ctf, ctm=0.5, C=C)
    assert np.array_equal(got["g"].view(np.uint32), ref["g"].view(np.uint32))
    assert np.array_equal(got["trunc"], ref["trunc"])


def test_od_truncation_and_ids(cuda, orc):
    sigma, rho, y0, ids = orc.od_inputs(2000, seed=5)
    ids = ids.copy()
    ids[::7] = -1                       # out-of-range ids: their emits are dropped and counted
    ids[3] = 2000
    inp = (sigma, rho, y0, ids)
    for M in (50, 50000):
        ref = orc.od_fwd(*inp, max_steps=M)
        got = gpu_od(inp, M=M)
        assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
        assert np.array_equal(got["stats"], ref["stats"]) and ref["stats"][4] > 0
        assert np.array_equal(got["final"].view(np.uint32), ref["final"].view(np.uint32))
        gr = orc.od_grad(*inp, max_steps=M)
        gg = gpu_od_grad(inp, M=M)
        assert np.array_equal(gg["g"].view(np.uint32), gr["g"].view(np.uint32))
        assert np.array_equal(gg["trunc"], gr["trunc"])


def test_od_full_size(cuda, orc):
    """N = 1,048,576: repeatable; the replay gradient agrees with a central difference of the forward pass"""
    inp = orc.od_inputs(1048576)
    a = gpu_od(inp)
    b = gpu_od(inp)
    assert np.array_equal(a["k"], b["k"]) and np.array_equal(a["final"], b["final"])
    g = gpu_od_grad(inp)
    h = np.float32(1e-3)
    fp = gpu_od(inp, beta=BETA + h)
    fm = gpu_od(inp, beta=BETA - h)
    lp = fp["final"].astype(np.float64).sum() + float(fp["mean"][0])
    lm = fm["final"].astype(np.float64).sum() + float(fm["mean"][0])
    fd = (lp - lm) / (float(BETA + h) - float(BETA - h))
    assert np.isfinite(g["g"]).all() and abs(float(g["g"][0]) - fd) <= 0.05 * abs(fd)
    # the one-pass forward mode (the bench's step) at full size: the replay's gradient within 1e-4, the forward's
    # trip counts and final states bitwise
    v = gpu_od_vg(inp)
    assert abs(float(v["g"][0]) - float(g["g"][0])) <= 1e-4 * abs(float(g["g"][0]))
    assert np.array_equal(v["k"], a["k"]) and np.array_equal(v["final"].view(np.uint32), a["final"].view(np.uint32))


# ---------------------------------------------------------------------------------------------- one pass
def gpu_od_vg(inp, beta=BETA, ctf=None, ctm=1.0, M=50000):
    n = len(inp[0])
    ctf = np.ones((n, 3), np.float32) if ctf is None else ctf
    out = B.run(B.OD_VG1, list(inp), [beta, ctf, np.float32(ctm)], consts=(M,))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    fin, mean, g, stats, k, tr = [o.cpu().numpy() for o in out]
    return dict(final=fin, mean=mean.reshape(1), g=g, stats=stats, k=k, trunc=tr.astype(bool))


@pytest.mark.parametrize("n", [1, 4000, 65536 + 5])
def test_od_vg_onepass(cuda, orc, n):
    """forward mode w.r.t. beta in one launch: the gradient bitwise the oracle's forward mode (the same order), within
    the float tolerance of the replay adjoint; trip counts, flags, stats and the final states bitwise the forward's"""
    inp = orc.od_inputs(n, seed=11)
    ctf = np.random.default_rng(2).normal(size=(n, 3)).astype(np.float32)
    got = gpu_od_vg(inp, ctf=ctf, ctm=0.5)
    ref = orc.od_vg1(*inp, ct_final=ctf, ct_mean=0.5)
    assert np.array_equal(got["g"].view(np.uint32), ref["g"].view(np.uint32))
    fw = orc.od_fwd(*inp)
    assert np.array_equal(got["k"], fw["k"]) and np.array_equal(got["trunc"], fw["trunc"])
    assert np.array_equal(got["stats"], fw["stats"])
    assert np.array_equal(got["final"].view(np.uint32), fw["final"].view(np.uint32))
    assert abs(float(got["mean"][0]) - float(fw["mean"][0])) <= 1e-5 * abs(float(fw["mean"][0]))
    rp = orc.od_grad(*inp, ct_final=ctf, ct_mean=0.5)
    assert abs(float(got["g"][0]) - float(rp["g"][0])) <= 1e-4 * max(abs(float(rp["g"][0])), 1e-6)


def test_od_vg_onepass_truncation_and_ids(cuda, orc):
    """dropped final bins contribute nothing (and are counted); max_steps = 50 truncates items: the flags and the
    gradient of what ran, bitwise the oracle's"""
    sigma, rho, y0, ids = orc.od_inputs(2000, seed=5)
    ids = ids.copy()
    ids[::7] = -1
    ids[3] = 2000
    inp = (sigma, rho, y0, ids)
    for M in (50, 50000):
        got = gpu_od_vg(inp, M=M)
        ref = orc.od_vg1(*inp, max_steps=M)
        assert np.array_equal(got["g"].view(np.uint32), ref["g"].view(np.uint32))
        assert np.array_equal(got["trunc"], ref["trunc"]) and np.array_equal(got["k"], ref["k"])
        assert got["stats"][4] > 0


def test_od_api_value_and_grad_onepass(cuda, orc):
    """value_and_grad of the Lorenz ensemble runs the one-pass launch (exact_order=True: the forward and the replay);
    a truncated item poisons both gradients"""
    import tallymap_b200 as tm
    inp = orc.od_inputs(3000, seed=7)
    f = tm.vmap("lorenz", outputs={"final": tm.Sum((3000, 3)), "mean_z": tm.Sum(())}, in_axes=(0, 0, 0, 0, None))
    cts = {"final": torch.ones(3000, 3), "mean_z": torch.tensor(0.25)}
    r1, g1 = f.value_and_grad(*inp, BETA, wrt=4, cotangents=cts)
    assert B.run.last["kernel"] == "od_vg_onepass"
    r2, g2 = f.value_and_grad(*inp, BETA, wrt=4, cotangents=cts, exact_order=True)
    torch.cuda.synchronize()
    assert abs(float(g1) - float(g2)) <= 1e-4 * abs(float(g2))
    assert torch.equal(r1.outputs["final"], r2.outputs["final"]) and torch.equal(r1.per_item, r2.per_item)
    ft = tm.vmap("lorenz", outputs={"final": tm.Sum((3000, 3)), "mean_z": tm.Sum(())}, in_axes=(0, 0, 0, 0, None),
                 max_steps=50)
    _, gt = ft.value_and_grad(*inp, BETA, wrt=4, cotangents=cts)
    torch.cuda.synchronize()
    assert torch.isnan(gt)


def test_od_vg_onepass_empty(cuda):
    """no items: no kernel runs; zero outputs and a zero gradient"""
    inp = (np.zeros(0, np.float32), np.zeros(0, np.float32), np.zeros((0, 3), np.float32), np.zeros(0, np.int32))
    got = gpu_od_vg(inp, ctf=np.zeros((0, 3), np.float32))
    assert got["final"].size == 0 and got["k"].size == 0 and float(got["g"][0]) == 0.0 and got["stats"].sum() == 0
