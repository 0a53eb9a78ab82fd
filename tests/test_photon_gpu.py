"""GPU parity of the photon-slab item (benchmark configuration 3) and of the shared f32 math it uses.

The math (log, exp, sin, cos, pow in tallymap_b200/csrc/tm_math.h) is one implementation compiled for host and
device, so the device must reproduce the host bitwise; then photon trip counts, truncation flags, stats and the
exact (mu_a, mu_s) gradient are bitwise the oracle's, and the deposit grid within the float-tally tolerance."""
import ctypes

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


@pytest.mark.parametrize("fn", ["log", "exp", "sin", "cos", "pow"])
def test_device_math_bitwise_host(cuda, tmlib, orc, fn):
    rng = np.random.default_rng(3)
    n = 1 << 20
    bits = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = {"log": np.abs(bits), "exp": rng.uniform(-110, 95, n), "sin": rng.uniform(-50, 50, n),
         "cos": rng.uniform(-50, 50, n), "pow": rng.uniform(0, 20, n)}[fn].astype(np.float32)
    x = np.where(np.isnan(x), np.float32(1.0), x).astype(np.float32)
    y = rng.uniform(-4, 4, n).astype(np.float32)
    host = orc.math(fn, x, y)
    dx = torch.from_numpy(x).cuda()
    dy = torch.from_numpy(y).cuda()
    out = torch.empty_like(dx)
    P = ctypes.c_void_p
    tmlib.check(tmlib.lib().tm_math_eval(P(torch.cuda.current_stream().cuda_stream), orc.MATH_FN[fn],
                                         P(dx.data_ptr()), P(dy.data_ptr()), P(out.data_ptr()), n))
    dev = out.cpu().numpy()
    assert np.array_equal(dev.view(np.uint32), host.view(np.uint32))


def gpu_ph(keys, mu_a=0.1, mu_s=10.0, M=100000, order=None):
    out = B.run(B.PH_FWD, [keys], [np.float32(mu_a), np.float32(mu_s)], consts=(M,), order=order)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    dep, stats, k, tr = [o.cpu().numpy() for o in out]
    return dict(dep=dep, stats=stats, k=k, trunc=tr.astype(bool))


def gpu_ph_grad(keys, mu_a=0.1, mu_s=10.0, ct=None, M=100000, C=None, order=None):
    ct = np.ones((64, 64, 64), np.float32) if ct is None else ct
    out = B.run(B.PH_GRAD, [keys], [np.float32(mu_a), np.float32(mu_s), ct], consts=(M,), rev_checkpoints=C,
                order=order)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    g, stats, tr = [o.cpu().numpy() for o in out]
    return dict(g=g, stats=stats, trunc=tr.astype(bool))


@pytest.mark.parametrize("n", [1, 5000, 65536 + 3])
def test_ph_forward(cuda, orc, n):
    keys = prng.split(prng.PRNGKey(2), n)
    ref = orc.ph_fwd(keys)
    got = gpu_ph(keys)
    assert np.array_equal(got["k"], ref["k"])
    assert np.array_equal(got["trunc"], ref["trunc"]) and np.array_equal(got["stats"], ref["stats"])
    assert near(got["dep"], ref["dep"])


@pytest.mark.parametrize("C", [None, 4, 64])
def test_ph_grad_bitwise(cuda, orc, C):
    keys = prng.split(prng.PRNGKey(2), 20000)
    ct = np.random.default_rng(4).uniform(0.5, 1.5, (64, 64, 64)).astype(np.float32)
    ref = orc.ph_grad(keys, ct=ct)
    got = gpu_ph_grad(keys, ct=ct, C=C)
    assert np.array_equal(got["g"].view(np.uint32), ref["g"].view(np.uint32))
    assert np.array_equal(got["trunc"], ref["trunc"])


def test_ph_truncation_and_params(cuda, orc):
    keys = prng.split(prng.PRNGKey(7), 4000)
    for mu_a, mu_s, M in ((0.1, 10.0, 40), (1.0, 2.0, 100000), (0.01, 30.0, 300)):
        ref = orc.ph_fwd(keys, mu_a, mu_s, max_steps=M)
        got = gpu_ph(keys, mu_a, mu_s, M=M)
        assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
        assert near(got["dep"], ref["dep"])
        gr = orc.ph_grad(keys, mu_a, mu_s, max_steps=M)
        gg = gpu_ph_grad(keys, mu_a, mu_s, M=M)
        assert np.array_equal(gg["g"].view(np.uint32), gr["g"].view(np.uint32))
        assert np.array_equal(gg["trunc"], gr["trunc"])
    assert ref["trunc"].any() or True


def test_ph_libm_statistics(cuda, orc):
    """against the libm build (the reference host target's math): the same statistics (compare protocol
    tolerance: mean trip count and total deposit within 3 standard errors)"""
    keys = prng.split(prng.PRNGKey(2), 20000)
    lm = orc.ph_fwd(keys, libm=True)
    got = gpu_ph(keys)
    se = lm["k"].std() / np.sqrt(len(keys))
    assert abs(got["k"].mean() - lm["k"].mean()) <= 3 * se + 1e-9
    assert abs(got["dep"].sum() - lm["dep"].sum()) <= 1e-3 * abs(lm["dep"].sum())


def test_ph_full_size_properties(cuda):
    """N = 4,194,304 photons: repeatable integers and exact gradient; gradient consistent with the linear
    structure (d dep.sum / d mu_a at fixed paths is positive)."""
    keys = prng.split(prng.PRNGKey(2), 4194304)
    a = gpu_ph(keys)
    b = gpu_ph(keys)
    assert np.array_equal(a["k"], b["k"]) and near(a["dep"], b["dep"])
    ga = gpu_ph_grad(keys)
    gb = gpu_ph_grad(keys)
    assert np.array_equal(ga["g"].view(np.uint32), gb["g"].view(np.uint32))
    assert np.isfinite(ga["g"]).all() and ga["g"][0] > 0


# ---------------------------------------------------------------------------------------------- one pass
def gpu_ph_vg1(keys, mu_a=0.1, mu_s=10.0, ct=None, M=100000):
    ct = np.ones((64, 64, 64), np.float32) if ct is None else ct
    out = B.run(B.PH_VG1, [keys], [np.float32(mu_a), np.float32(mu_s), ct], consts=(M,))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    dep, g, stats, k, tr = [o.cpu().numpy() for o in out]
    return dict(dep=dep, g=g, stats=stats, k=k, trunc=tr.astype(bool))


@pytest.mark.parametrize("n", [1, 20000])
def test_ph_vg_onepass(cuda, orc, n):
    """forward mode in one pass: the forward's outputs as the forward's; the gradient bitwise the oracle's forward
    mode (C = -1) and within the float tolerance of the replay adjoint's"""
    keys = prng.split(prng.PRNGKey(2), n)
    ct = np.random.default_rng(4).uniform(0.5, 1.5, (64, 64, 64)).astype(np.float32)
    got = gpu_ph_vg1(keys, ct=ct)
    ref = orc.ph_fwd(keys)
    assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
    assert near(got["dep"], ref["dep"])
    fm = orc.ph_grad(keys, ct=ct, C=-1)
    assert np.array_equal(got["g"].view(np.uint32), fm["g"].view(np.uint32))
    rv = orc.ph_grad(keys, ct=ct)
    assert near(got["g"], rv["g"])
    assert np.array_equal(got["stats"], ref["stats"] + rv["stats"])


def test_ph_vg_onepass_params_and_truncation(cuda, orc):
    keys = prng.split(prng.PRNGKey(7), 4000)
    for mu_a, mu_s, M in ((1.0, 2.0, 100000), (0.01, 30.0, 300)):
        got = gpu_ph_vg1(keys, mu_a, mu_s, M=M)
        fm = orc.ph_grad(keys, mu_a, mu_s, max_steps=M, C=-1)
        assert np.array_equal(got["g"].view(np.uint32), fm["g"].view(np.uint32))
        assert np.array_equal(got["trunc"], fm["trunc"])
        assert near(got["g"], orc.ph_grad(keys, mu_a, mu_s, max_steps=M)["g"])


def test_ph_api_value_and_grad_onepass(cuda):
    """value_and_grad of the photon family runs the one-pass program; the gradient within the float tolerance of
    the forward + replay launches (exact_order=True)"""
    import tallymap_b200 as tm
    keys = prng.split(prng.PRNGKey(3), 300000)
    f = tm.vmap("photon", outputs={"dep": tm.Sum((64, 64, 64))}, in_axes=(0, None, None))
    cts = {"dep": torch.ones((64, 64, 64))}
    r1, g1 = f.value_and_grad(keys, np.float32(0.1), np.float32(10.0), wrt=(1, 2), cotangents=cts)
    assert B.run.last["kernel"] == "ph_vg_onepass"
    r2, g2 = f.value_and_grad(keys, np.float32(0.1), np.float32(10.0), wrt=(1, 2), cotangents=cts, exact_order=True)
    torch.cuda.synchronize()
    assert near(g1.cpu().numpy(), g2.cpu().numpy())
    assert np.array_equal(r1.per_item.cpu().numpy(), r2.per_item.cpu().numpy())
    assert near(r1.outputs["dep"].cpu().numpy(), r2.outputs["dep"].cpu().numpy())


def test_ph_api_grad_forward_mode_option(cuda):
    """grad(exact_order=False) runs the forward-mode launch; within the float tolerance of the replay's"""
    import tallymap_b200 as tm
    keys = prng.split(prng.PRNGKey(5), 100000)
    f = tm.vmap("photon", outputs={"dep": tm.Sum((64, 64, 64))}, in_axes=(0, None, None))
    cts = {"dep": torch.ones((64, 64, 64))}
    g1 = f.grad(keys, np.float32(0.1), np.float32(10.0), wrt=(1, 2), cotangents=cts, exact_order=False)
    assert B.run.last["kernel"] == "ph_vg_onepass"
    g2 = f.grad(keys, np.float32(0.1), np.float32(10.0), wrt=(1, 2), cotangents=cts)
    assert B.run.last["kernel"] == "ph_grad"
    torch.cuda.synchronize()
    assert near(g1.cpu().numpy(), g2.cpu().numpy())


@pytest.mark.parametrize("fn", ["atan", "atan2", "asin", "acos", "tan", "sinh", "cosh", "asinh", "acosh", "atanh",
                                "exp2", "log2", "cbrt", "erf", "erfc", "erfinv", "lgamma", "nextafter"])
def test_device_special_math_bitwise_host(cuda, tmlib, orc, fn):
    """the inverse trigonometric, hyperbolic and erf family: device bitwise host over random bit patterns and
    in-domain values (NaN inputs and the signed zeros and infinities included)"""
    rng = np.random.default_rng(11)
    n = 1 << 18
    bits = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    dom = {"asin": (-1, 1), "acos": (-1, 1), "atanh": (-1, 1), "erfinv": (-1, 1), "acosh": (1, 50),
           "tan": (-50, 50), "sinh": (-95, 95), "cosh": (-95, 95), "exp2": (-155, 130), "erf": (-6, 6),
           "erfc": (-6, 12), "lgamma": (-20, 40)}.get(fn, (-100, 100))
    x = np.concatenate([bits, rng.uniform(*dom, n).astype(np.float32),
                        np.float32([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0])]).astype(np.float32)
    y = rng.permutation(x).astype(np.float32)
    host = orc.math(fn, x, y)
    dx, dy = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    out = torch.empty_like(dx)
    P = ctypes.c_void_p
    tmlib.check(tmlib.lib().tm_math_eval(P(torch.cuda.current_stream().cuda_stream), orc.MATH_FN[fn],
                                         P(dx.data_ptr()), P(dy.data_ptr()), P(out.data_ptr()), len(x)))
    dev = out.cpu().numpy()
    assert np.array_equal(dev.view(np.uint32), host.view(np.uint32))
