"""GPU parity of run-time lowered items (tallymap_b200.trace -> lower -> NVRTC): the traced quickstart walker and
1-D walk against the oracle and against the hand-lowered kernels -- trip counts, flags, stats and gradients bitwise,
float tallies within the float-tally tolerance -- and an item using the other lowered primitives, whose generated
gradient is checked against a central difference of its generated forward."""
import numpy as np
import pytest
import torch

import tallymap_b200 as tm
from tallymap_b200 import backend as B
from tallymap_b200 import prng

from items_lang import mixer, quickstart, walk

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


def np_out(r):
    return {k: v.cpu().numpy() for k, v in r.outputs.items()}


@pytest.mark.parametrize("n", [1, 3000, 65536])
def test_lowered_walk_forward(cuda, orc, n):
    x, k = rw_inputs(n, seed=2)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    r = f(x, k, np.float32(1.0))
    torch.cuda.synchronize()
    ref = orc.rw_fwd(x, k, 1.0)
    assert np.array_equal(r.per_item.cpu().numpy(), ref["k"])
    assert np.array_equal(r.truncated.cpu().numpy(), ref["trunc"])
    st = np.array([int(r.stats[s]) for s in B.STATS])
    assert np.array_equal(st, ref["stats"])
    o = np_out(r)
    if not ref["trunc"].any():
        assert near(o["hist"], ref["hist"]) and near(o["side"], ref["side"])
    hand = B.run(B.RW_FWD, [x, k], [np.float32(1.0)], consts=(20000,))
    assert np.array_equal(hand[3].cpu().numpy(), ref["k"])


@pytest.mark.parametrize("C", [None, 3])
def test_lowered_walk_grad_bitwise(cuda, orc, C):
    x, k = rw_inputs(20000, seed=3)
    ct = np.random.default_rng(4).normal(size=256).astype(np.float32)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    prog = f.lowered((x, k, np.float32(1.0))).grad_program((0,))
    out = B.run(prog, [x, k], [np.float32(1.0), ct, np.zeros(2, np.float32)], consts=(20000,), rev_checkpoints=C)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    g = out[0].cpu().numpy()
    ref = orc.rw_grad(x, k, 1.0, ct)
    hand = B.run(B.RW_GRAD, [x, k], [np.float32(1.0), ct, np.zeros(2, np.float32)], consts=(20000,))
    assert np.array_equal(bits(g), bits(ref["g"]))
    assert np.array_equal(bits(g), bits(hand[0].cpu().numpy()))
    # and through the API
    gg = f.grad(x, k, np.float32(1.0), wrt=2, cotangents={"hist": ct})
    assert np.array_equal(bits(gg.cpu().numpy().reshape(1)), bits(ref["g"]))


def test_lowered_quickstart(cuda, orc):
    x = np.linspace(0.1, 0.99, 10000, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), 10000)
    f = tm.vmap(quickstart, outputs={"hist": tm.Sum((16,))}, in_axes=(0, 0, None), max_steps=100)
    r, g = f.value_and_grad(x, k, np.float32(2.0), wrt=2, cotangents={"hist": np.ones(16, np.float32)})
    torch.cuda.synchronize()
    rf = orc.q1_fwd(x, k, 2.0)
    rg = orc.q1_grad(x, k, 2.0, np.ones(16, np.float32))
    assert np.array_equal(r.per_item.cpu().numpy(), rf["k"])
    assert near(np_out(r)["hist"], rf["hist"])
    assert np.array_equal(bits(g.cpu().numpy().reshape(1)), bits(rg["g"]))


def _mixer_args(n, a, b):
    keys = prng.split(prng.PRNGKey(8), n)
    rng = np.random.default_rng(1)
    pos = (0.3 * rng.standard_normal((n, 3))).astype(np.float32)
    steps = rng.integers(1, 7, n).astype(np.int32)
    return pos, keys, steps, np.float32(a), np.float32(b)


def test_lowered_mixer_forward_and_gradient(cuda):
    n = 4000
    outs = {"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), torch.int32), "end": tm.Sum(())}
    f = tm.vmap(mixer, outputs=outs, in_axes=(0, 0, 0, None, None), max_steps=64)
    args = _mixer_args(n, 0.3, 1.7)
    r1, r2 = f(*args), f(*args)
    torch.cuda.synchronize()
    # the int tally is exact: item i adds 1 to bin s % 4 for s < steps[i]
    steps = args[2]
    want = np.zeros(4, np.int64)
    for s in range(int(steps.max())):
        want[s % 4] += int((steps > s).sum())
    assert np.array_equal(r1.outputs["hits"].cpu().numpy(), want)
    assert np.array_equal(r1.per_item.cpu().numpy(), steps)
    assert near(r1.outputs["dep"].cpu().numpy(), r2.outputs["dep"].cpu().numpy(), 1e-6)
    # gradient of <1, dep> + 0.5 end w.r.t. (a, b) against a central difference of the forward (f64 sums)
    cts = {"dep": np.ones((8, 8, 8), np.float32), "end": np.float32(0.5)}
    g = f.grad(*args, wrt=(3, 4), cotangents=cts).cpu().numpy()

    def loss(a, b):
        r = f(*_mixer_args(n, a, b))
        return float(r.outputs["dep"].double().sum()) + 0.5 * float(r.outputs["end"].double().sum())
    for j, (a, b) in enumerate([(1e-3, 0.0), (0.0, 1e-3)]):
        fd = (loss(0.3 + a, 1.7 + b) - loss(0.3 - a, 1.7 - b)) / 2e-3
        assert abs(g[j] - fd) <= 2e-2 * abs(fd) + 1e-2, (j, g[j], fd)


def test_fixed_point_sums_are_order_independent(cuda, orc):
    """Sum(fixed_point=True): bitwise the same under any claim order, within one ulp of the oracle's f64 sums
    (the correctly rounded exact sum), while the plain f32 side tally is only within tolerance"""
    n = 200000
    x, k = rw_inputs(n, seed=6)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,), fixed_point=True), "side": tm.Sum((2,), fixed_point=True)},
                in_axes=(0, 0, None), max_steps=20000)
    L = f.lowered((x, k, np.float32(1.0)))
    outs = []
    for order in (None, np.arange(n, dtype=np.int32)[::-1].copy(),
                  np.random.default_rng(1).permutation(n).astype(np.int32)):
        o = B.run(L.fwd, [x, k], [np.float32(1.0)], consts=(20000,), order=order)
        torch.cuda.synchronize()
        B.check_status(B.run.last["ctl"])
        outs.append([t.cpu().numpy() for t in o])
    for o in outs[1:]:
        assert np.array_equal(bits(o[0]), bits(outs[0][0])) and np.array_equal(bits(o[1]), bits(outs[0][1]))
        assert np.array_equal(o[3], outs[0][3])
    ref = orc.rw_fwd(x, k, 1.0)          # f64 partial sums, rounded once
    h = outs[0][0]
    ulps = np.abs(h.view(np.int32).astype(np.int64) - ref["hist"].view(np.int32).astype(np.int64))
    assert ulps.max() <= 1 and (ulps == 0).mean() > 0.99
    assert np.array_equal(outs[0][1], ref["side"])


def test_jvp_walk_matches_primal_and_vjp(cuda):
    """forward mode of the walk w.r.t. drift: the hist tangent is sum(x) per bin, i.e. the hist itself at drift = 1
    (the same emits), and <ct, tangent> is the reverse-mode gradient"""
    x, k = rw_inputs(50000, seed=12)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    r, d = f.jvp(x, k, np.float32(1.0), wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    assert d["hist"].shape == (256,) and d["side"].shape == (2,)
    h, dh = r.outputs["hist"].cpu().numpy(), d["hist"].cpu().numpy()
    assert near(dh, h) and not d["side"].cpu().numpy().any()
    ct = np.random.default_rng(3).normal(size=256).astype(np.float32)
    g = float(f.grad(x, k, np.float32(1.0), wrt=2, cotangents={"hist": ct}))
    assert abs(float(np.dot(ct.astype(np.float64), dh)) - g) <= 1e-4 * abs(g)


def test_jacfwd_mixer_matches_vjp(cuda):
    n = 4000
    outs = {"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), torch.int32), "end": tm.Sum(())}
    f = tm.vmap(mixer, outputs=outs, in_axes=(0, 0, 0, None, None), max_steps=64)
    args = _mixer_args(n, 0.3, 1.7)
    J = f.jacfwd(*args, wrt=(3, 4))
    torch.cuda.synchronize()
    assert J["dep"].shape == (2, 8, 8, 8) and J["end"].shape == (2,)
    cts = {"dep": np.ones((8, 8, 8), np.float32), "end": np.float32(0.5)}
    g = f.grad(*args, wrt=(3, 4), cotangents=cts).cpu().numpy().astype(np.float64)
    jd = J["dep"].double().sum(dim=(1, 2, 3)).cpu().numpy() + 0.5 * J["end"].double().cpu().numpy()
    assert np.all(np.abs(jd - g) <= 1e-4 * np.abs(g) + 1e-3), (jd, g)
    # two lanes of arbitrary tangents: linear in the tangent
    _, d2 = f.jvp(*args, wrt=(3, 4), tangents=[[1.0, 0.0], [2.0, -1.0]])
    comb = 2.0 * J["dep"][0].double() - J["dep"][1].double()
    assert torch.allclose(d2["dep"][1].double(), comb, rtol=1e-4, atol=1e-3)


def _walk_host(x0, keys, M=20000):
    """the walk on the host (numpy f32, jax.random's threefry): per item its hits (step, x) in bin 128 and its exit"""
    from tallymap_b200.prng import threefry2x32
    x = x0.astype(np.float32).copy()
    n = len(x)
    alive = (x >= 0) & (x <= 1)
    k = np.zeros(n, np.int32)
    hits = [[] for _ in range(n)]
    step = 0
    with np.errstate(over="ignore"):
        while alive.any() and step < M:
            i = np.nonzero(alive)[0]
            o0, o1 = threefry2x32(keys[i, 0], keys[i, 1], np.uint32(0), np.uint32(step))
            a0, a1 = threefry2x32(o0, o1, np.uint32(0), np.uint32(0))
            u = (((a0 ^ a1) >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)
            b = (x[i] * np.float32(256)).astype(np.int32)
            for j in np.nonzero(b == 128)[0]:
                hits[i[j]].append((step, x[i[j]]))
            x[i] = x[i] + np.float32(0.02) * (np.float32(2.0) * u - np.float32(1.0))
            k[i] += 1
            step += 1
            alive = (x >= 0) & (x <= 1) & (k < M)
    return hits, k, (x > 1).astype(np.int32)


def test_records_canonical_layout(cuda):
    from items_lang import walk_records
    n = 300
    x, k = rw_inputs(n, seed=13)
    outs = {"hist": tm.Sum((256,)), "hits": tm.Records({"k": torch.int32, "x": torch.float32}, capacity=1 << 16),
            "exit": tm.Records({"k": torch.int32, "side": torch.int32}, capacity=n)}
    f = tm.vmap(walk_records, outputs=outs, in_axes=(0, 0, None), max_steps=20000)
    r1 = f(x, k, np.float32(1.0))
    r2 = f(x, k, np.float32(1.0))
    torch.cuda.synchronize()
    hits, K, side = _walk_host(x, k)
    want_k = np.array([s for h in hits for s, _ in h], np.int32)
    want_x = np.array([v for h in hits for _, v in h], np.float32)
    m = len(want_k)
    assert 0 < m < 1 << 16 and int(r1.stats["appended"]["hits"]) == m and int(r1.stats["appended"]["exit"]) == n
    for r in (r1, r2):            # deterministic layout, whatever order the records were claimed in
        h = {kk: v.cpu().numpy() for kk, v in r.outputs["hits"].items()}
        assert np.array_equal(h["k"][:m], want_k) and np.array_equal(bits(h["x"][:m]), bits(want_x))
        assert not h["k"][m:].any() and not h["x"][m:].any()
        e = {kk: v.cpu().numpy() for kk, v in r.outputs["exit"].items()}
        assert np.array_equal(e["k"], K) and np.array_equal(e["side"], side)
    assert np.array_equal(r1.per_item.cpu().numpy(), K)


def test_records_overflow_poisons(cuda):
    from items_lang import walk_records
    n = 300
    x, k = rw_inputs(n, seed=13)
    outs = {"hist": tm.Sum((256,)), "hits": tm.Records({"k": torch.int32, "x": torch.float32}, capacity=8),
            "exit": tm.Records({"k": torch.int32, "side": torch.int32}, capacity=n)}
    f = tm.vmap(walk_records, outputs=outs, in_axes=(0, 0, None), max_steps=20000)
    r = f(x, k, np.float32(1.0))
    torch.cuda.synchronize()
    assert int(r.stats["records_dropped"]["hits"]) == int(r.stats["appended"]["hits"]) - 8 > 0
    assert (r.outputs["hits"]["k"].cpu().numpy() == -1).all() and torch.isnan(r.outputs["hits"]["x"]).all()
    assert torch.isnan(r.outputs["hist"]).all()


def _eval(fn, in_specs, npi, specs, records, args, M, exact=()):
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as Tr
    tr = Tr.trace_item(fn, in_specs, npi, specs, records)
    return Evaluator(tr, M, exact).run(list(args[:npi]), list(args[npi:]))


def test_lowered_against_ir_evaluator_edges(cuda):
    """every primitive on awkward values, bitwise (through Records), against the IR evaluator"""
    from items_lang import edges
    vals = np.float32([np.nan, np.inf, -np.inf, -0.0, 0.0, 1e38, -1e38, 3e-39, -7.5, 7.5, 0.6, 123456.0, -2.0, 0.25])
    n = len(vals)
    keys = prng.split(prng.PRNGKey(21), n)
    steps = np.full(n, 3, np.int32)
    args = (vals, keys, steps, np.float32(0.7))
    fields = {"i": torch.int32, "q": torch.int32, "r": torch.int32, "b": torch.int32, "y": torch.float32,
              "z": torch.float32, "u": torch.int32}
    outs = {"h": tm.Sum((8,), torch.int32), "rec": tm.Records(fields, capacity=256)}
    f = tm.vmap(edges, outputs=outs, in_axes=(0, 0, 0, None), max_steps=10)
    r = f(*args)
    torch.cuda.synchronize()
    recspec = {"rec": (256, tuple((k, "f32" if v == torch.float32 else "i32") for k, v in sorted(fields.items())))}
    ref = _eval(edges, ["f32", "key", "i32", "f32"], 3, {"h": ((8,), "i32")}, recspec, args, 10)
    m = len(ref["records"]["rec"])
    assert m == 3 * n and int(r.stats["appended"]["rec"]) == m
    got = {k: v.cpu().numpy() for k, v in r.outputs["rec"].items()}
    for j, (fname, _) in enumerate(recspec["rec"][1]):
        want = np.array([rec[j] for rec in ref["records"]["rec"]])
        g = got[fname][:m]
        if g.dtype == np.float32:
            w = want.astype(np.float32)
            # bitwise, NaN payloads aside (the device's canonical NaN and the host's differ in sign and payload)
            same = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
            assert same.all() and np.isnan(w).sum() > 0, fname
        else:
            assert np.array_equal(g.astype(np.int64), want.astype(np.int64)), fname
    assert np.array_equal(r.outputs["h"].cpu().numpy(), ref["sums"]["h"])


def test_lowered_against_ir_evaluator_fixed_point_and_records(cuda):
    from items_lang import walk_records
    n = 400
    x, k = rw_inputs(n, seed=17)
    outs = {"hist": tm.Sum((256,), fixed_point=True),
            "hits": tm.Records({"k": torch.int32, "x": torch.float32}, capacity=1 << 16),
            "exit": tm.Records({"k": torch.int32, "side": torch.int32}, capacity=n)}
    f = tm.vmap(walk_records, outputs=outs, in_axes=(0, 0, None), max_steps=20000)
    r = f(x, k, np.float32(1.0))
    torch.cuda.synchronize()
    recs = {"hits": (1 << 16, (("k", "i32"), ("x", "f32"))), "exit": (n, (("k", "i32"), ("side", "i32")))}
    ref = _eval(walk_records, ["f32", "key", "f32"], 2, {"hist": ((256,), "f32")}, recs, (x, k, np.float32(1.0)),
                20000, exact=("hist",))
    assert np.array_equal(bits(r.outputs["hist"].cpu().numpy()), bits(ref["sums"]["hist"]))
    m = len(ref["records"]["hits"])
    hk = np.array([h[0] for h in ref["records"]["hits"]], np.int32)
    hx = np.array([h[1] for h in ref["records"]["hits"]], np.float32)
    assert np.array_equal(r.outputs["hits"]["k"].cpu().numpy()[:m], hk)
    assert np.array_equal(bits(r.outputs["hits"]["x"].cpu().numpy()[:m]), bits(hx))
    assert np.array_equal(r.per_item.cpu().numpy(), ref["results"][0])


def test_quickstart_grad_and_jvp_agree(cuda):
    """the reference's quickstart check (examples/quickstart.py:43-53): for loss = sum(hist ** 2), reverse mode
    (a replay with the cotangent 2 hist, taken from the forward) and forward mode (2 <hist, d hist / d theta>) agree
    to 1e-4"""
    n = 10000
    x = np.linspace(0.1, 0.99, n, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), n)
    f = tm.vmap(quickstart, outputs={"hist": tm.Sum((16,))}, in_axes=(0, 0, None), max_steps=100)
    r = f(x, k, np.float32(2.0))
    hist = r.outputs["hist"]
    g = float(f.grad(x, k, np.float32(2.0), wrt=2, cotangents={"hist": 2.0 * hist}))
    _, d = f.jvp(x, k, np.float32(2.0), wrt=2, tangents=[1.0])
    t = float(2.0 * (hist.double() * d["hist"].double()).sum())
    assert int(r.stats["n_truncated"]) == 0
    assert abs(g - t) <= 1e-4 * abs(t)


# ---------------------------------------------------------------------------------------------- spawn
def _shower_fn(Q=1 << 22, M=100000):
    from items_lang import shower
    return tm.vmap(shower, outputs={"dep": tm.Sum((512,)), "count": tm.Sum((1,), torch.int32)},
                   in_axes=(0, 0, 0, None), max_steps=M, spawn=tm.Queue(Q))


@pytest.mark.parametrize("n", [1, 777, 20000])
def test_lowered_shower_matches_oracle(cuda, orc, n):
    """the traced shower on the spawn runtime: particle count, spawned children, per-root trip counts, flags and
    stats bitwise against the oracle; the deposit within the float-tally tolerance"""
    E0, d0, keys = orc.sh_inputs(n)
    r = _shower_fn()(E0, d0, keys, np.float32(1.0))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    ref = orc.sh_fwd(E0, d0, keys, 1.0)
    o = np_out(r)
    assert np.array_equal(o["count"], ref["count"])
    st = np.array([int(r.stats[s]) for s in B.STATS])
    assert np.array_equal(st, ref["stats"]) and st[1] == 0
    assert np.array_equal(r.per_item.cpu().numpy(), ref["k"])
    assert np.array_equal(r.truncated.cpu().numpy(), ref["trunc"])
    assert near(o["dep"], ref["dep"])


def test_lowered_shower_matches_hand_lowered(cuda, orc):
    """the traced shower against the hand-lowered SH_FWD kernel on 2^18 roots (~2.5e8 particles)"""
    E0, d0, keys = orc.sh_inputs(1 << 18)
    r = _shower_fn()(E0, d0, keys, np.float32(1.0))
    torch.cuda.synchronize()
    hand = B.run(B.SH_FWD, [E0, d0, keys], [np.float32(1.0)], consts=(100000,))
    torch.cuda.synchronize()
    o = np_out(r)
    assert np.array_equal(o["count"], hand[1].cpu().numpy())
    assert np.array_equal(r.per_item.cpu().numpy(), hand[3].cpu().numpy())
    assert int(r.stats["spawned"]) == int(hand[2][0]) and int(r.stats["children_dropped"]) == 0
    assert near(o["dep"], hand[0].cpu().numpy())


def test_lowered_shower_small_queue_poisons(cuda, orc):
    """a Queue too small for the children idle threads wait for: dropped children are counted and every float
    output is NaN (_api.py:898-915); the integer count stays the particles that ran"""
    E0, d0, keys = orc.sh_inputs(5000)
    r = _shower_fn(Q=64)(E0, d0, keys, np.float32(1.0))
    torch.cuda.synchronize()
    dropped, spawned = int(r.stats["children_dropped"]), int(r.stats["spawned"])
    assert dropped > 0
    assert np.isnan(r.outputs["dep"].cpu().numpy()).all()
    assert int(r.outputs["count"][0]) == 5000 + spawned


@pytest.mark.parametrize("M", [100, 4])
def test_lowered_post_loop_spawn_matches_evaluator(cuda, M):
    """spawn after the loop (three generations of children); with max_steps = 4 the later generations truncate:
    counted in stats['children_truncated'] and poisoning the float output, not the roots' flags"""
    from items_lang import spawn_walk
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    n = 3000
    rng = np.random.default_rng(9)
    g = np.zeros(n, np.int32)
    x = rng.uniform(0.5, 1.5, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(11), n)
    f = tm.vmap(spawn_walk, outputs={"Q": tm.Sum((16,)), "C": tm.Sum((16,), torch.int32)}, in_axes=(0, 0, 0),
                max_steps=M, spawn=tm.Queue(4096))
    r = f(g, x, keys)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    tr = T.trace_item(spawn_walk, ["i32", "f32", "key"], 3, {"Q": ((16,), "f32"), "C": ((16,), "i32")}, spawn=True)
    ref = Evaluator(tr, M).run([g, x, keys], [])
    st = np.array([int(r.stats[s]) for s in B.STATS])
    assert np.array_equal(st, ref["stats"]) and st[0] == 3 * n
    assert np.array_equal(r.per_item.cpu().numpy(), ref["results"][0])
    assert np.array_equal(r.outputs["C"].cpu().numpy(), ref["sums"]["C"])
    if M == 4:
        assert st[2] > 0 and not r.truncated.any() and np.isnan(r.outputs["Q"].cpu().numpy()).all()
    else:
        assert near(r.outputs["Q"].cpu().numpy(), ref["sums"]["Q"])


# ---------------------------------------------------------------------------------------------- one-pass
def test_lowered_walk_value_and_grad_onepass(cuda, orc):
    """the traced walk has no active carry: value_and_grad is ONE generated one-pass launch; its gradient is bitwise
    the oracle summing each item's cotangent oldest step first, within the float tolerance of the replay's order"""
    x, k = rw_inputs(30000, seed=6)
    ct = np.random.default_rng(7).normal(size=256).astype(np.float32)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    r, g = f.value_and_grad(x, k, np.float32(1.0), wrt=2, cotangents={"hist": ct})
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    assert B.run.last["kernel"] == f.last_lowered.vg_program((0,)).kernel
    rf = orc.rw_fwd(x, k, 1.0)
    assert np.array_equal(r.per_item.cpu().numpy(), rf["k"]) and near(np_out(r)["hist"], rf["hist"])
    assert np.array_equal(bits(g.cpu().numpy()), bits(orc.rw_grad(x, k, 1.0, ct, C=-1)["g"][0]))
    g2 = f.value_and_grad(x, k, np.float32(1.0), wrt=2, cotangents={"hist": ct}, exact_order=True)[1]
    assert np.array_equal(bits(g2.cpu().numpy()), bits(orc.rw_grad(x, k, 1.0, ct)["g"][0]))
    assert near(g.cpu().numpy(), g2.cpu().numpy())


def test_lowered_quickstart_onepass_fixed_point(cuda, orc):
    """a fixed-point output in the one-pass program: bitwise the forward's exact tally; the gradient bitwise the
    oracle in the one-pass order"""
    x = np.linspace(0.1, 0.99, 10000, dtype=np.float32)
    k = prng.split(prng.PRNGKey(0), 10000)
    f = tm.vmap(quickstart, outputs={"hist": tm.Sum((16,), fixed_point=True)}, in_axes=(0, 0, None), max_steps=100)
    r, g = f.value_and_grad(x, k, np.float32(2.0), wrt=2, cotangents={"hist": torch.ones(16)})
    r0 = f(x, k, np.float32(2.0))
    torch.cuda.synchronize()
    assert np.array_equal(bits(np_out(r)["hist"]), bits(np_out(r0)["hist"]))
    assert np.array_equal(bits(g.cpu().numpy()), bits(orc.q1_grad(x, k, 2.0, np.ones(16, np.float32), C=-1)["g"][0]))


@pytest.mark.parametrize("ct", ["end", "dep"])
def test_lowered_mixer_value_and_grad_forward_mode(cuda, ct):
    """the mixer's carries depend on a and b: value_and_grad is ONE forward-mode launch (two tangent lanes
    contracted with the cotangents at each emit); its gradient within the float tolerance of the replay's
    (exact_order=True), its outputs the forward's"""
    kx = prng.split(prng.PRNGKey(3), 4096)
    rng = np.random.default_rng(2)
    pos = rng.uniform(-1, 1, (4096, 3)).astype(np.float32)
    n = rng.integers(1, 40, 4096).astype(np.int32)
    f = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), torch.int32), "end": tm.Sum(())},
                in_axes=(0, 0, 0, None, None), max_steps=64)
    cts = {"end": torch.ones(())} if ct == "end" else \
        {"dep": torch.from_numpy(rng.normal(size=(8, 8, 8)).astype(np.float32)), "end": torch.full((), 0.5)}
    args = (pos, kx, n, np.float32(0.3), np.float32(1.7))
    r, g = f.value_and_grad(*args, wrt=(3, 4), cotangents=cts)
    assert B.run.last["kernel"] == f.last_lowered.vg_program((0, 1)).kernel
    r2, g2 = f.value_and_grad(*args, wrt=(3, 4), cotangents=cts, exact_order=True)
    assert B.run.last["kernel"] == f.last_lowered.grad_program((0, 1)).kernel
    torch.cuda.synchronize()
    assert near(g.cpu().numpy(), g2.cpu().numpy())
    assert np.array_equal(r.per_item.cpu().numpy(), r2.per_item.cpu().numpy())
    assert np.array_equal(np_out(r)["hits"], np_out(r2)["hits"]) and near(np_out(r)["dep"], np_out(r2)["dep"])


# ---------------------------------------------------------------------------------------------- forward mode through spawn
def _decay_args(n=3000):
    rng = np.random.default_rng(12)
    return (np.zeros(n, np.int32), rng.uniform(0.5, 1.5, n).astype(np.float32), prng.split(prng.PRNGKey(13), n))


def _decay_eval(args, a):
    from items_lang import spawn_decay
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    tr = T.trace_item(spawn_decay, ["i32", "f32", "key", "f32"], 3, {"Q": ((8,), "f32")}, spawn=True)
    return Evaluator(tr, 10).run(list(args), [np.float32(a)])


def test_forward_mode_through_spawn(cuda):
    """value_and_grad and jvp of a spawning item w.r.t. a broadcast operand: children carry their weight's tangent;
    against a central difference of the IR evaluator (the outputs are polynomials of degree <= 3 in a)"""
    from items_lang import spawn_decay
    args = _decay_args()
    a, h = 1.1, 1.1e-2
    f = tm.vmap(spawn_decay, outputs={"Q": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=10,
                spawn=tm.Queue(1 << 16))
    ct = np.linspace(-1.0, 2.0, 8).astype(np.float32)
    r, g = f.value_and_grad(*args, np.float32(a), wrt=3, cotangents={"Q": torch.from_numpy(ct)})
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    assert int(r.stats["spawned"]) == 2 * len(args[0])
    qp, qm = _decay_eval(args, a + h)["sums"]["Q"], _decay_eval(args, a - h)["sums"]["Q"]
    dq = (qp - qm) / (2 * h)
    want = float(np.dot(ct.astype(np.float64), dq))
    assert abs(float(g) - want) <= 1e-3 * np.abs(ct.astype(np.float64) * dq).sum()
    q0 = _decay_eval(args, a)["sums"]["Q"]
    assert near(np_out(r)["Q"], q0)
    # forward mode with a tangent tally: the same derivative per bin
    _, dts = f.jvp(*args, np.float32(a), wrt=3, tangents=[1.0])
    torch.cuda.synchronize()
    assert np.abs(dts["Q"].cpu().numpy() - dq).max() <= 1e-3 * np.abs(dq).max()


def test_forward_mode_through_spawn_lanes_and_limits(cuda):
    """two tangent lanes through spawn: lane 1 seeded twice lane 0 gives twice the tangent; a max_steps that
    truncates children poisons value_and_grad's gradient and the float outputs (never a silently partial one)"""
    from items_lang import spawn_decay
    args = _decay_args(2000)
    f = tm.vmap(spawn_decay, outputs={"Q": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=10,
                spawn=tm.Queue(1 << 16))
    _, dts = f.jvp(*args, np.float32(1.1), wrt=3, tangents=np.array([[1.0], [2.0]], np.float32))
    torch.cuda.synchronize()
    d = dts["Q"].cpu().numpy()
    assert d.shape == (2, 8) and near(d[1], 2.0 * d[0], 1e-6)
    ft = tm.vmap(spawn_decay, outputs={"Q": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=2,
                 spawn=tm.Queue(1 << 16))
    r, g = ft.value_and_grad(*args, np.float32(1.1), wrt=3, cotangents={"Q": torch.ones(8)})
    torch.cuda.synchronize()
    assert int(r.stats["children_truncated"]) > 0 and int(r.stats["n_truncated"]) > 0
    assert torch.isnan(g).all() and torch.isnan(r.outputs["Q"]).all()


def test_traced_shower_value_and_grad(cuda, orc):
    """the traced shower's value_and_grad w.r.t. X0 runs forward mode through spawn in one launch: X0 moves only the
    deposit's bin, so the gradient is exactly 0 (as the tree adjoint's); the outputs are the forward's"""
    E0, d0, keys = orc.sh_inputs(3000)
    f = _shower_fn()
    r, g = f.value_and_grad(E0, d0, keys, np.float32(1.0), wrt=3, cotangents={"dep": torch.ones(512)})
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    assert B.run.last["kernel"] == f.last_lowered.vg_program((0,)).kernel
    assert float(g) == 0.0
    ref = orc.sh_fwd(E0, d0, keys, 1.0)
    assert np.array_equal(np_out(r)["count"], ref["count"]) and np.array_equal(r.per_item.cpu().numpy(), ref["k"])
    assert near(np_out(r)["dep"], ref["dep"])


def test_loop_free_item(cuda):
    """an item with no loop (a zero-step loop): outputs and per-item results against the IR evaluator, the one-pass
    gradient against the replay's and a central difference of the evaluator"""
    from items_lang import scatter
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    x, k = rw_inputs(20000, seed=21)
    a = 0.7
    f = tm.vmap(scatter, outputs={"h": tm.Sum((8,)), "s": tm.Sum(())}, in_axes=(0, 0, None))
    r = f(x, k, np.float32(a))
    torch.cuda.synchronize()
    tr = T.trace_item(scatter, ["f32", "key", "f32"], 2, {"h": ((8,), "f32"), "s": ((), "f32")})
    ev = lambda av: Evaluator(tr, 2 ** 31 - 1).run([x, k], [np.float32(av)])
    ref = ev(a)
    assert np.array_equal(bits(r.per_item.cpu().numpy()), bits(ref["results"][0]))
    assert near(np_out(r)["h"], ref["sums"]["h"]) and near(np_out(r)["s"], ref["sums"]["s"])
    cts = {"h": torch.linspace(-1, 1, 8), "s": torch.full((), 2.0)}
    r1, g1 = f.value_and_grad(x, k, np.float32(a), wrt=2, cotangents=cts)
    r2, g2 = f.value_and_grad(x, k, np.float32(a), wrt=2, cotangents=cts, exact_order=True)
    torch.cuda.synchronize()
    assert near(g1.cpu().numpy(), g2.cpu().numpy())
    h = 1e-3
    ct = np.linspace(-1, 1, 8)
    fd = lambda av: float(np.dot(ct, ev(av)["sums"]["h"]) + 2.0 * ev(av)["sums"]["s"][0])
    want = (fd(a + h) - fd(a - h)) / (2 * h)
    assert abs(float(g2) - want) <= 2e-3 * abs(want)


def test_lowered_compositions_against_ir_evaluator(cuda):
    """clip, sign, square and bernoulli on awkward values (NaN, +-inf, +-0, huge), bitwise through Records"""
    from items_lang import extras
    vals = np.float32([np.nan, np.inf, -np.inf, -0.0, 0.0, 1e38, -1e38, 3e-39, -7.5, 7.5, 0.6, 123456.0, -2.0, 0.25])
    n = len(vals)
    keys = prng.split(prng.PRNGKey(23), n)
    args = (vals, keys, np.full(n, 4, np.int32), np.float32(0.7))
    fields = {"y": torch.float32, "z": torch.float32, "h": torch.int32, "g": torch.int32}
    f = tm.vmap(extras, outputs={"rec": tm.Records(fields, capacity=128)}, in_axes=(0, 0, 0, None), max_steps=10)
    r = f(*args)
    torch.cuda.synchronize()
    recspec = {"rec": (128, tuple((k, "f32" if v == torch.float32 else "i32") for k, v in sorted(fields.items())))}
    ref = _eval(extras, ["f32", "key", "i32", "f32"], 3, {}, recspec, args, 10)
    m = len(ref["records"]["rec"])
    assert m == 4 * n and int(r.stats["appended"]["rec"]) == m
    got = {k: v.cpu().numpy() for k, v in r.outputs["rec"].items()}
    for j, (fname, _) in enumerate(recspec["rec"][1]):
        want = np.array([rec[j] for rec in ref["records"]["rec"]])
        g = got[fname][:m]
        if g.dtype == np.float32:
            w = want.astype(np.float32)
            same = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
            assert same.all(), fname
        else:
            assert np.array_equal(g.astype(np.int64), want.astype(np.int64)), fname


def test_per_item_operand_gradient(cuda):
    """grad w.r.t. a per-item operand (each item's own cotangent) and the broadcast one in one replay launch,
    against the closed form of an affine recursion (d x_k / d x_0 = a^k) in float64"""
    from items_lang import affine
    n, a = 20000, np.float32(0.9)
    x, k = rw_inputs(n, seed=31)
    ct = np.linspace(-1.0, 1.0, 8).astype(np.float32)
    f = tm.vmap(affine, outputs={"h": tm.Sum((8,))}, in_axes=(0, 0, None), max_steps=10)
    gx, ga = f.grad(x, k, a, wrt=(0, 2), cotangents={"h": torch.from_numpy(ct)})
    gx1 = f.grad(x, k, a, wrt=0, cotangents={"h": torch.from_numpy(ct)})
    torch.cuda.synchronize()
    assert gx.shape == (n,) and np.array_equal(bits(gx.cpu().numpy()), bits(gx1.cpu().numpy()))
    # the closed form in float64 (the draws exactly as the item's)
    xs = x.astype(np.float64)
    dxdx0 = np.ones(n)
    dxda = np.zeros(n)
    want_x = np.zeros(n)
    want_a = 0.0
    for s in range(6):
        kk = prng.fold_in(k, s)
        o0, o1 = prng.threefry2x32(kk[:, 0], kk[:, 1], np.uint32(0), np.uint32(0))
        u = (((o0 ^ o1) >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)
        dxda = xs + float(a) * dxda
        dxdx0 = float(a) * dxdx0
        xs = xs * float(a) + u.astype(np.float64)
        want_x += float(ct[s % 8]) * 2.0 * xs * dxdx0
        want_a += float((float(ct[s % 8]) * 2.0 * xs * dxda).sum())
    g = gx.cpu().numpy().astype(np.float64)
    assert np.abs(g - want_x).max() <= 1e-4 * np.abs(want_x).max()
    assert abs(float(ga) - want_a) <= 1e-4 * abs(want_a)


def test_forward_mode_of_fixed_point_outputs(cuda):
    """a fixed-point output in forward mode: its tangent tally is exact (bitwise the same under any claim order) and
    equals the plain tally's tangent within the float tolerance; the forward-mode value_and_grad agrees with the
    replay (exact_order=True)"""
    args = _mixer_args(4000, 0.3, 1.7)
    fx = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8), fixed_point=True), "hits": tm.Sum((4,), torch.int32),
                                 "end": tm.Sum(())}, in_axes=(0, 0, 0, None, None), max_steps=64)
    fp = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), torch.int32), "end": tm.Sum(())},
                 in_axes=(0, 0, 0, None, None), max_steps=64)
    tan = np.array([[1.0, 0.0], [0.0, 1.0]], np.float32)
    rx, dx = fx.jvp(*args, wrt=(3, 4), tangents=tan)
    rp, dp = fp.jvp(*args, wrt=(3, 4), tangents=tan)
    torch.cuda.synchronize()
    assert near(dx["dep"].cpu().numpy(), dp["dep"].cpu().numpy())
    assert np.array_equal(bits(rx.outputs["dep"].cpu().numpy()), bits(fx(*args).outputs["dep"].cpu().numpy()))
    prog = fx.last_lowered.jvp_program((0, 1), 2)
    outs = []
    for order in (None, np.arange(4000, dtype=np.int32)[::-1].copy()):
        o = B.run(prog, list(args[:3]), [args[3], args[4], tan], consts=(64,), order=order)
        torch.cuda.synchronize()
        outs.append(o[3].cpu().numpy())
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    cts = {"dep": torch.ones((8, 8, 8)), "end": torch.full((), 0.5)}
    r1, g1 = fx.value_and_grad(*args, wrt=(3, 4), cotangents=cts)
    r2, g2 = fx.value_and_grad(*args, wrt=(3, 4), cotangents=cts, exact_order=True)
    torch.cuda.synchronize()
    assert near(g1.cpu().numpy(), g2.cpu().numpy())
    assert np.array_equal(bits(r1.outputs["dep"].cpu().numpy()), bits(r2.outputs["dep"].cpu().numpy()))


def test_lowered_round_rem_reductions_against_ir_evaluator(cuda):
    """round, rem, mod, sum / max / min / all / any on awkward values, bitwise through Records"""
    from items_lang import rounding
    vals = np.float32([np.nan, np.inf, -np.inf, -0.0, 0.0, 1e38, -1e38, 3e-39, -7.5, 7.5, 0.6, 123456.0, -2.0, 2.5])
    n = len(vals)
    keys = prng.split(prng.PRNGKey(29), n)
    args = (vals, keys, np.full(n, 4, np.int32), np.float32(0.7))
    fields = {"r": torch.float32, "m": torch.float32, "o": torch.float32, "s": torch.float32, "x": torch.float32,
              "n": torch.float32, "a": torch.int32}
    f = tm.vmap(rounding, outputs={"rec": tm.Records(fields, capacity=128)}, in_axes=(0, 0, 0, None), max_steps=10)
    r = f(*args)
    torch.cuda.synchronize()
    recspec = {"rec": (128, tuple((k, "f32" if v == torch.float32 else "i32") for k, v in sorted(fields.items())))}
    ref = _eval(rounding, ["f32", "key", "i32", "f32"], 3, {}, recspec, args, 10)
    m = len(ref["records"]["rec"])
    assert m == 4 * n
    got = {k: v.cpu().numpy() for k, v in r.outputs["rec"].items()}
    for j, (fname, _) in enumerate(recspec["rec"][1]):
        want = np.array([rec[j] for rec in ref["records"]["rec"]])
        g = got[fname][:m]
        if g.dtype == np.float32:
            w = want.astype(np.float32)
            same = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
            assert same.all(), fname
        else:
            assert np.array_equal(g.astype(np.int64), want.astype(np.int64)), fname


def test_stop_gradient_and_rem_derivatives(cuda):
    """d/da of sum(rem(x a, 0.7) + stop_gradient(a) x) = sum(x): the replay, the one-pass program and forward mode"""
    from items_lang import stopped
    x, k = rw_inputs(100000, seed=41)
    f = tm.vmap(stopped, outputs={"h": tm.Sum(())}, in_axes=(0, 0, None))
    want = float(x.astype(np.float64).sum())
    g1 = f.grad(x, k, np.float32(1.3), wrt=2, cotangents={"h": torch.ones(())})
    g2 = f.value_and_grad(x, k, np.float32(1.3), wrt=2, cotangents={"h": torch.ones(())})[1]
    _, d = f.jvp(x, k, np.float32(1.3), wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    for g in (float(g1), float(g2), float(d["h"])):
        assert abs(g - want) <= 1e-5 * abs(want)


def test_log1p_expm1_tanh(cuda):
    """the compositions bitwise against the IR evaluator, and within 8 ulp of float64 references where finite"""
    from items_lang import transcend
    rng = np.random.default_rng(3)
    vals = np.concatenate([np.float32([np.nan, np.inf, -np.inf, -0.0, 0.0, -1.0, -0.999999, 1e-30, -1e-30, 3e-39, 88.0,
                                       -88.0, 20.0, -20.0]),
                           rng.uniform(-0.99, 10.0, 2000).astype(np.float32),
                           (10.0 ** rng.uniform(-20, 0, 2000)).astype(np.float32)])
    n = len(vals)
    keys = prng.split(prng.PRNGKey(2), n)
    fields = {"l": torch.float32, "e": torch.float32, "h": torch.float32}
    f = tm.vmap(transcend, outputs={"rec": tm.Records(fields, capacity=n)}, in_axes=(0, 0, None))
    r = f(vals, keys, np.float32(1.0))
    torch.cuda.synchronize()
    recspec = {"rec": (n, tuple((k, "f32") for k in sorted(fields)))}
    ref = _eval(transcend, ["f32", "key", "f32"], 2, {}, recspec, (vals, keys, np.float32(1.0)), 1)
    got = {k: v.cpu().numpy() for k, v in r.outputs["rec"].items()}
    x64 = vals.astype(np.float64)
    with np.errstate(all="ignore"):
        exact = {"l": np.log1p(x64), "e": np.expm1(x64), "h": np.tanh(x64)}
    for j, fname in enumerate(sorted(fields)):
        want = np.array([rec[j] for rec in ref["records"]["rec"]], np.float32)
        g = got[fname][:n]
        assert ((g.view(np.uint32) == want.view(np.uint32)) | (np.isnan(g) & np.isnan(want))).all(), fname
        e = exact[fname]
        ok = np.isfinite(e) & (np.abs(e) < 3e38)
        ulp = np.abs(g[ok].astype(np.float64) - e[ok]) / np.spacing(np.abs(e[ok]).astype(np.float32)).astype(np.float64)
        assert ulp.max() <= 8, (fname, ulp.max())


def test_gillespie_birth_death(cuda):
    """an exact SSA item (a float-time loop, a propensity vector, cumsum / searchsorted selection, int clips):
    per-item final counts and event counts and the integer histogram bitwise against the IR evaluator"""
    from items_lang import birth_death
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    n = 500
    x0 = np.random.default_rng(4).integers(0, 200, n).astype(np.int32)
    keys = prng.split(prng.PRNGKey(17), n)
    c = (np.float32(1.0), np.float32(0.4))
    f = tm.vmap(birth_death, outputs={"hist": tm.Sum((32,), torch.int32), "tau": tm.Sum(())},
                in_axes=(0, 0, None, None), max_steps=1 << 16)
    r = f(x0, keys, *c)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    tr = T.trace_item(birth_death, ["i32", "key", "f32", "f32"], 2, {"hist": ((32,), "i32"), "tau": ((), "f32")})
    ref = Evaluator(tr, 1 << 16).run([x0, keys], list(c))
    xs, ks = r.per_item
    assert np.array_equal(xs.cpu().numpy(), ref["results"][0]) and np.array_equal(ks.cpu().numpy(), ref["results"][1])
    assert np.array_equal(r.outputs["hist"].cpu().numpy(), ref["sums"]["hist"])
    assert near(np_out(r)["tau"], ref["sums"]["tau"])


def test_call_options(cuda):
    """the call options (_api.py:414-425): cuda_math='approx' (div.full / sqrt.approx) changes the tallied values
    within a few ulp and no control flow; 'fast' (also FMA contraction) agrees statistically; min_blocks_per_sm
    changes no bit of a fixed-point output; rev_checkpoints changes the replay's buffers, not the gradient"""
    from items_lang import divided
    n = 300
    x, k = rw_inputs(n, seed=23)
    a = np.float32(0.7)
    ref = _eval(divided, ["f32", "key", "f32"], 2, {"h": ((16,), "f32")}, {}, (x, k, a), 20000, exact=("h",))
    run = lambda **o: tm.vmap(divided, outputs={"h": tm.Sum((16,), fixed_point=True)}, in_axes=(0, 0, None),
                              max_steps=20000, **o)
    r0 = run()(x, k, a)
    torch.cuda.synchronize()
    assert np.array_equal(bits(r0.outputs["h"].cpu().numpy()), bits(ref["sums"]["h"]))
    assert np.array_equal(r0.per_item.cpu().numpy(), ref["results"][0])
    r1 = run(cuda_math="approx")(x, k, a)
    assert np.array_equal(r1.per_item.cpu().numpy(), ref["results"][0])
    assert near(r1.outputs["h"].cpu().numpy(), ref["sums"]["h"], 2e-6)
    r2 = run(cuda_math="fast")(x, k, a)
    same = (r2.per_item.cpu().numpy() == ref["results"][0]).mean()
    assert same > 0.95 and near(r2.outputs["h"].cpu().numpy(), ref["sums"]["h"], 0.05)
    r3 = run(min_blocks_per_sm=8)(x, k, a)
    assert np.array_equal(bits(r3.outputs["h"].cpu().numpy()), bits(r0.outputs["h"].cpu().numpy()))
    ct = {"h": torch.linspace(-1, 1, 16)}
    g0 = run().grad(x, k, a, wrt=2, cotangents=ct)
    g1 = run(rev_checkpoints=4).grad(x, k, a, wrt=2, cotangents=ct)
    assert near(g1.cpu().numpy(), g0.cpu().numpy())


def test_broadcast_vector_operand(cuda):
    """a broadcast float32[3] parameter vector: the forward, the replay gradient (f32[3]), the one-pass
    value_and_grad and jacfwd equal those of the same item with three broadcast scalars"""
    from items_lang import walk_theta, walk_theta_scalars
    n = 4000
    x, k = rw_inputs(n, seed=29)
    th = np.float32([0.5, 0.03, 0.1])
    outs = {"hist": tm.Sum((64,), fixed_point=True)}
    f = tm.vmap(walk_theta, outputs=outs, in_axes=(0, 0, None), max_steps=20000)
    g = tm.vmap(walk_theta_scalars, outputs=outs, in_axes=(0, 0, None, None, None), max_steps=20000)
    ct = {"hist": torch.linspace(-1, 1, 64)}
    rf, rg = f(x, k, th), g(x, k, *th)
    assert np.array_equal(bits(rf.outputs["hist"].cpu().numpy()), bits(rg.outputs["hist"].cpu().numpy()))
    assert np.array_equal(rf.per_item.cpu().numpy(), rg.per_item.cpu().numpy())
    gf = f.grad(x, k, th, wrt=2, cotangents=ct)
    gg = g.grad(x, k, *th, wrt=(2, 3, 4), cotangents=ct)
    assert gf.shape == (3,) and np.array_equal(bits(gf.cpu().numpy()), bits(gg.cpu().numpy()))
    _, vf = f.value_and_grad(x, k, th, wrt=2, cotangents=ct)
    assert vf.shape == (3,) and near(vf.cpu().numpy(), gf.cpu().numpy())
    J = f.jacfwd(x, k, th, wrt=2)["hist"].cpu().numpy()
    assert J.shape == (3, 64)
    assert near(J @ ct["hist"].numpy(), gf.cpu().numpy(), 1e-4)


def test_broadcast_tables(cuda):
    """items reading broadcast tables by traced indices (1-D and 2-D, float32 and int32, indices clamped and
    counted from the end): a lookup walk and a cell-list neighbour item bitwise against the IR evaluator (per-item
    results and fixed-point tallies); the neighbour energy's gradient w.r.t. its parameter vector (replay and one
    launch) against jacfwd"""
    from items_lang import lookup, neighbours
    from oracle.ir_eval import Evaluator
    rng = np.random.default_rng(5)
    n = 150
    x, k = rw_inputs(n, seed=31)
    xs = rng.uniform(0.5, 1.5, 100).astype(np.float32)
    pairs = rng.uniform(-1, 1, (100, 2)).astype(np.float32)
    f = tm.vmap(lookup, outputs={"h": tm.Sum((16,), fixed_point=True)}, in_axes=(0, 0, None, None, None),
                max_steps=20000)
    r = f(x, k, xs, pairs, np.float32(0.7))
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    ref = Evaluator(f.last_lowered.tr, 20000, ("h",)).run([x, k], [xs, pairs, np.float32(0.7)])
    assert np.array_equal(bits(r.outputs["h"].cpu().numpy()), bits(ref["sums"]["h"]))
    assert np.array_equal(r.per_item[0].cpu().numpy(), ref["results"][0])
    assert np.array_equal(bits(r.per_item[1].cpu().numpy()), bits(ref["results"][1]))
    N = 256
    pos = rng.uniform(0, 8, (N, 2)).astype(np.float32)
    cell = np.clip((pos[:, 1] / 2).astype(int), 0, 3) * 4 + np.clip((pos[:, 0] / 2).astype(int), 0, 3)
    order = np.argsort(cell, kind="stable").astype(np.int32)
    start = np.searchsorted(cell[order], np.arange(17)).astype(np.int32)
    th = np.float32([1.0, 0.5])
    ii = np.arange(N, dtype=np.int32)
    g = tm.vmap(neighbours, outputs={"u": tm.Sum((4,), fixed_point=True)}, in_axes=(0, None, None, None, None),
                max_steps=1 << 14)
    r2 = g(ii, order, start, pos, th)
    ref2 = Evaluator(g.last_lowered.tr, 1 << 14, ("u",)).run([ii], [order, start, pos, *th])
    assert np.array_equal(r2.per_item[0].cpu().numpy(), ref2["results"][0])
    assert np.array_equal(bits(r2.per_item[1].cpu().numpy()), bits(ref2["results"][1]))
    assert np.array_equal(bits(r2.outputs["u"].cpu().numpy()), bits(ref2["sums"]["u"]))
    ct = {"u": torch.tensor([1.0, -0.5, 0.25, 2.0])}
    gr = g.grad(ii, order, start, pos, th, wrt=4, cotangents=ct)
    _, gv = g.value_and_grad(ii, order, start, pos, th, wrt=4, cotangents=ct)
    J = g.jacfwd(ii, order, start, pos, th, wrt=4)["u"].cpu().numpy()
    assert gr.shape == (2,) and near(gr.cpu().numpy(), J @ ct["u"].numpy(), 1e-4)
    assert near(gv.cpu().numpy(), gr.cpu().numpy(), 1e-4)


def test_special_math_item(cuda):
    """an item using every math primitive beyond log / exp / sin / cos with the normal and exponential samplers:
    bitwise against the IR evaluator (per-item sums, a fixed-point tally); its gradient by replay and by forward
    mode agree"""
    from items_lang import special
    from oracle.ir_eval import Evaluator
    n = 1000
    x = np.random.default_rng(12).uniform(-1, 1, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(13), n)
    a = np.float32(0.8)
    f = tm.vmap(special, outputs={"h": tm.Sum((8,), fixed_point=True)}, in_axes=(0, 0, None), max_steps=100)
    r = f(x, keys, a)
    ref = Evaluator(f.last_lowered.tr, 100, ("h",)).run([x, keys], [a])
    assert np.array_equal(bits(r.per_item[0].cpu().numpy()), bits(ref["results"][0]))
    assert np.array_equal(r.per_item[1].cpu().numpy(), ref["results"][1])
    assert np.array_equal(bits(r.outputs["h"].cpu().numpy()), bits(ref["sums"]["h"]))
    ct = {"h": torch.linspace(-1, 1, 8)}
    g = f.grad(x, keys, a, wrt=2, cotangents=ct)
    J = f.jacfwd(x, keys, a, wrt=2)["h"].cpu().numpy()
    assert np.isfinite(float(g)) and near(float(g), float(J[0] @ ct["h"].numpy()), 1e-4)


def test_cond_switch_item(cuda):
    """lax.cond / switch / fori_loop inside the loop body: bitwise against the IR evaluator; the gradient by
    replay against jacfwd"""
    from items_lang import branchy
    from oracle.ir_eval import Evaluator
    n = 200
    x, k = rw_inputs(n, seed=37)
    a = np.float32(1.5)
    f = tm.vmap(branchy, outputs={"h": tm.Sum((8,), fixed_point=True)}, in_axes=(0, 0, None), max_steps=20000)
    r = f(x, k, a)
    ref = Evaluator(f.last_lowered.tr, 20000, ("h",)).run([x, k], [a])
    assert np.array_equal(r.per_item.cpu().numpy(), ref["results"][0])
    assert np.array_equal(bits(r.outputs["h"].cpu().numpy()), bits(ref["sums"]["h"]))
    ct = {"h": torch.linspace(-1, 1, 8)}
    g = f.grad(x, k, a, wrt=2, cotangents=ct)
    J = f.jacfwd(x, k, a, wrt=2)["h"].cpu().numpy()
    assert near(float(g), float(J[0] @ ct["h"].numpy()), 1e-4)


def test_vector_item_spheres(cuda):
    """a walk-on-spheres item written with jax.numpy-style vectors (per-item (2,) starts, a (4,) parameter vector):
    per-item hop counts bitwise and the tally within the float-tally tolerance of the IR evaluator; its gradient
    w.r.t. the parameter vector by replay against jacfwd"""
    from items_lang import spheres
    from oracle.ir_eval import Evaluator
    n = 400
    rng = np.random.default_rng(41)
    x0 = rng.uniform(0.1, 0.9, (n, 2)).astype(np.float32)
    point = (np.arange(n) % 8).astype(np.int32)
    keys = prng.split(prng.PRNGKey(43), n)
    th = np.float32([1.0, 3.0, 0.2, 0.1])
    f = tm.vmap(spheres, outputs={"u": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=4096)
    r = f(x0, point, keys, th)
    ref = Evaluator(f.last_lowered.tr, 4096).run([x0, point, keys], list(th))
    assert np.array_equal(r.per_item.cpu().numpy(), ref["results"][0])
    assert near(r.outputs["u"].cpu().numpy(), ref["sums"]["u"])
    ct = {"u": torch.linspace(-1, 1, 8)}
    g = f.grad(x0, point, keys, th, wrt=3, cotangents=ct)
    J = f.jacfwd(x0, point, keys, th, wrt=3)["u"].cpu().numpy()
    assert g.shape == (4,) and near(g.cpu().numpy(), J @ ct["u"].numpy(), 1e-4)


def test_n_active(cuda):
    """n_active (_api.py:466-469): only items i < n_active run -- the outputs and the gradient equal those of the
    prefix bitwise (fixed-point sums), the other items' per-item results are zero and never truncated"""
    n, m = 3000, 1234
    x, k = rw_inputs(n, seed=47)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,), fixed_point=True), "side": tm.Sum((2,), fixed_point=True)},
                in_axes=(0, 0, None), max_steps=20000)
    d = np.float32(1.0)
    r = f(x, k, d, n_active=m)
    rp = f(x[:m], k[:m], d)
    for nm in ("hist", "side"):
        assert np.array_equal(bits(r.outputs[nm].cpu().numpy()), bits(rp.outputs[nm].cpu().numpy()))
    kk = r.per_item.cpu().numpy()
    assert np.array_equal(kk[:m], rp.per_item.cpu().numpy()) and not kk[m:].any()
    assert not r.truncated[m:].cpu().numpy().any()
    ct = {"hist": torch.linspace(0, 1, 256), "side": torch.ones(2)}
    g = f.grad(x, k, d, wrt=2, cotangents=ct, n_active=m)
    gp = f.grad(x[:m], k[:m], d, wrt=2, cotangents=ct)
    assert np.array_equal(bits(g.cpu().numpy()), bits(gp.cpu().numpy()))


def test_vector_results(cuda):
    """an item returning a vector: Result.per_item holds an (N, 2) array bitwise the evaluator's"""
    from items_lang import drift2d
    from oracle.ir_eval import Evaluator
    n = 500
    x0 = np.random.default_rng(3).uniform(0.3, 0.7, (n, 2)).astype(np.float32)
    keys = prng.split(prng.PRNGKey(5), n)
    f = tm.vmap(drift2d, outputs={"exits": tm.Sum((4,))}, in_axes=(0, 0, None), max_steps=10000)
    r = f(x0, keys, np.float32(0.1))
    xy, k = r.per_item
    ref = Evaluator(f.last_lowered.tr, 10000).run([x0, keys], [np.float32(0.1)])
    assert tuple(xy.shape) == (n, 2)
    assert np.array_equal(bits(xy[:, 0].cpu().numpy()), bits(ref["results"][0]))
    assert np.array_equal(bits(xy[:, 1].cpu().numpy()), bits(ref["results"][1]))
    assert np.array_equal(k.cpu().numpy(), ref["results"][2])


def test_cond_branches_write_the_tally(cuda):
    """t.add / t.append inside lax.cond / lax.switch branches (tallymap/_rewrite.py:573-598): the traced branch_writes
    item against the IR evaluator (fixed-point sums, records and trip counts bitwise) and against the
    same item written with selects (branch_writes_where) -- outputs, records, the reverse-mode gradient w.r.t. the
    broadcast a and the per-item x, the one-pass value-and-grad and forward mode"""
    from items_lang import branch_writes, branch_writes_where
    n = 20000
    x = np.random.default_rng(3).uniform(0, 1, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(5), n)
    a = np.float32(1.3)
    # (a fixed-point Sum: bin 1 sums a * a some 2e5 times, beyond what an f32 accumulation holds to 1e-5)
    outs = {"h": tm.Sum((5,), fixed_point=True), "low": tm.Records({"k": torch.int32, "x": torch.float32})}
    fb = tm.vmap(branch_writes, outputs=outs, in_axes=(0, 0, None), max_steps=100)
    fw = tm.vmap(branch_writes_where, outputs=outs, in_axes=(0, 0, None), max_steps=100)
    rb, rw = fb(x, keys, a), fw(x, keys, a)
    torch.cuda.synchronize()
    recs = {"low": (1 << 20, (("k", "i32"), ("x", "f32")))}
    ref = _eval(branch_writes, ["f32", "key", "f32"], 2, {"h": ((5,), "f32")}, recs, (x, keys, a), 100,
                exact=("h",))
    hb, hw = rb.outputs["h"].cpu().numpy(), rw.outputs["h"].cpu().numpy()
    assert np.array_equal(bits(hb), bits(ref["sums"]["h"])) and np.array_equal(bits(hb), bits(hw))
    assert np.array_equal(rb.per_item.cpu().numpy(), ref["results"][0])
    m = len(ref["records"]["low"])
    assert m > 0 and int(rb.stats["appended"]["low"]) == m
    for j, fname in enumerate(("k", "x")):
        got = rb.outputs["low"][fname].cpu().numpy()[:m]
        assert np.array_equal(got, rw.outputs["low"][fname].cpu().numpy()[:m])
        assert np.array_equal(got, np.array([r[j] for r in ref["records"]["low"]], got.dtype))
    ct = {"h": torch.tensor([0.5, -1.0, 2.0, 1.5, -0.25])}
    gb = fb.grad(x, keys, a, wrt=(0, 2), cotangents=ct)
    gw = fw.grad(x, keys, a, wrt=(0, 2), cotangents=ct)
    torch.cuda.synchronize()
    assert near(gb[0].cpu().numpy(), gw[0].cpu().numpy(), 1e-6) and near(float(gb[1]), float(gw[1]), 1e-6)
    assert float(gb[1]) != 0.0
    _, vb = fb.value_and_grad(x, keys, a, wrt=2, cotangents=ct)
    _, db = fb.jvp(x, keys, a, wrt=2, tangents=[1.0])
    _, dw = fw.jvp(x, keys, a, wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    assert near(float(vb), float(gw[1]), 1e-5)
    assert near(db["h"].cpu().numpy(), dw["h"].cpu().numpy(), 1e-6)


def test_spawn_inside_a_cond_branch(cuda):
    """a child spawned from inside a lax.cond branch: the same tree, outputs and tree-adjoint gradient as the
    spawn's `when` gives (spawn_decay)"""
    from items_lang import spawn_decay, spawn_decay_cond
    args = _decay_args(3000)
    ct = {"Q": torch.from_numpy(np.linspace(-1.0, 2.0, 8).astype(np.float32))}
    res = []
    for fn in (spawn_decay_cond, spawn_decay):
        f = tm.vmap(fn, outputs={"Q": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=10, spawn=tm.Queue(1 << 16))
        r, (gw, ga) = f.value_and_grad(*args, np.float32(1.1), wrt=(1, 3), cotangents=ct)
        torch.cuda.synchronize()
        assert f.last_tree["children"] == 2 * 3000 and int(f.last_tree["mismatch"]) == 0
        res.append((np_out(r)["Q"], gw.cpu().numpy(), float(ga)))
    assert near(res[0][0], res[1][0]) and near(res[0][1], res[1][1], 1e-6) and near(res[0][2], res[1][2], 1e-6)


def test_inner_while_loops(cuda):
    """inner while loops (rejection sampling inside the step reading the step's key, three iterations in a cond
    branch, a halving loop and a traced-bound fori_loop after the stepping loop): trip counts, inner-loop counts and
    the int tally bitwise the IR evaluator's (run first, so every inner loop is known to end), the float tally within
    the float tolerance; the replay gradient, the one-pass value-and-grad and forward mode w.r.t. a (the tally is
    linear in a: its derivative is h / a) within 1e-5"""
    from items_lang import rejection
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as Tr
    n = 300
    x0 = np.random.default_rng(6).uniform(0.2, 0.8, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(17), n)
    a = np.float32(1.25)
    specs = {"h": ((9,), "f32"), "tries": ((2,), "i32")}
    ref = Evaluator(Tr.trace_item(rejection, ["f32", "key", "f32"], 2, specs), 1000).run([x0, keys], [a])
    f = tm.vmap(rejection, outputs={"h": tm.Sum((9,)), "tries": tm.Sum((2,), torch.int32)}, in_axes=(0, 0, None),
                max_steps=1000)
    r = f(x0, keys, a)
    torch.cuda.synchronize()
    per = r.per_item if isinstance(r.per_item, (tuple, list)) else (r.per_item,)
    for j in range(3):
        assert np.array_equal(per[j].cpu().numpy(), ref["results"][j]), j
    assert np.array_equal(r.outputs["tries"].cpu().numpy(), ref["sums"]["tries"])
    assert near(r.outputs["h"].cpu().numpy(), ref["sums"]["h"])
    ct = torch.linspace(-1.0, 1.0, 9)
    want = float(np.dot(ct.numpy().astype(np.float64), ref["sums"]["h"] / float(a)))
    g = f.grad(x0, keys, a, wrt=2, cotangents={"h": ct})
    _, gv = f.value_and_grad(x0, keys, a, wrt=2, cotangents={"h": ct})
    _, d = f.jvp(x0, keys, a, wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    assert abs(float(g) - want) <= 1e-5 * abs(want) and abs(float(gv) - want) <= 1e-5 * abs(want)
    assert near(d["h"].cpu().numpy(), ref["sums"]["h"] / float(a))


@pytest.mark.parametrize("name", ["newton", "rejection_active"])
def test_inner_while_loops_differentiated(cuda, name):
    """inner loops that read the differentiated a (newton: fixed-point iterations of y = x + a sin y, whose iterates
    write the tally, under an active stepping carry; rejection_active: a loop whose trip count and carry depend on a):
    the replay gradient (the inner loop transposed from recomputed states) and the forward-mode value-and-grad agree
    within 1e-5, the jvp's float32 tangent tally within 1e-4; newton's with a central difference of the IR evaluator within 1e-3, rejection_active's with the
    host count of its trip counts (its derivative, the trip counts being locally constant) within 1e-5"""
    import items_lang
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as Tr
    item = getattr(items_lang, name)
    n = 2000
    x0 = np.random.default_rng(9).uniform(0.1, 0.6, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(3), n)
    a, h = 0.35, 1e-3
    ct = torch.tensor([0.7, -1.3])
    f = tm.vmap(item, outputs={"h": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=10)
    g = float(f.grad(x0, keys, np.float32(a), wrt=2, cotangents={"h": ct}))
    _, gv = f.value_and_grad(x0, keys, np.float32(a), wrt=2, cotangents={"h": ct})
    _, d = f.jvp(x0, keys, np.float32(a), wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    gj = float(np.dot(ct.numpy().astype(np.float64), d["h"].cpu().numpy()))
    # (g and gv sum exact per-item cotangents; the jvp's tangent tally is a float32 atomic sum of some 10^5 emits,
    # whose rounding depends on the order the atomics ran in)
    assert abs(g - float(gv)) <= 1e-5 * abs(g) and abs(g - gj) <= 1e-4 * abs(g)
    if name == "newton":
        tr = Tr.trace_item(item, ["f32", "key", "f32"], 2, {"h": ((2,), "f32")})
        q = lambda aa: Evaluator(tr, 10).run([x0, keys], [np.float32(aa)])["sums"]["h"]
        want = float(np.dot(ct.numpy().astype(np.float64), (q(a + h) - q(a - h)) / (2 * h)))
        assert abs(g - want) <= 1e-3 * abs(want), (g, want)
        return
    # rejection_active: y = x + m a after m iterations (a trip count that steps with a): d h[0] / d a = the sum of
    # the trip counts, counted on the host in float32
    f32, m_all = np.float32, 0
    for x in x0:
        x = f32(x)
        for _ in range(5):
            y, m = x, 0
            while m < 4 and y < 1.0:
                y, m = f32(y + f32(a)), m + 1
            m_all += m
            x = f32(x + f32(0.1))
    want = float(ct[0]) * m_all
    assert abs(g - want) <= 1e-5 * abs(want), (g, want)


def test_wider_accumulators(cuda):
    """float64 and int64 Sums and scaled fixed-point Sums (tallymap/_api.py:55-84): the int64 and every scaled sum
    bitwise the IR evaluator's exact integers (wbig's words carry past 2^63 many times: the 128-bit readout), the
    float64 sum within 1e-12; the gradient w.r.t. a of the float outputs (linear in a) within 1e-5 of total / a"""
    from items_lang import accumulators
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as Tr
    from test_lower_cpu import _acc_outputs
    n = 1500
    x0 = np.random.default_rng(1).uniform(0.3, 0.7, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(2), n)
    a = np.float32(1.5)
    outs = _acc_outputs()
    wide = {"w64": ("f64", 2.0 ** 20), "wi32": ("i32", 1.0), "wbig": ("f64", 2.0 ** 50)}
    specs = {k: ((4,), "f32" if k in ("f64", "w64", "wbig") else "i32") for k in outs}
    ref = Evaluator(Tr.trace_item(accumulators, ["f32", "key", "f32"], 2, specs), 200, wide=wide).run([x0, keys], [a])
    f = tm.vmap(accumulators, outputs=outs, in_axes=(0, 0, None), max_steps=200)
    r = f(x0, keys, a)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in r.outputs.items()}
    assert got["i64"].dtype == np.int64 and np.array_equal(got["i64"], ref["sums"]["i64"])
    assert got["wi32"].dtype == np.int32 and np.array_equal(got["wi32"], ref["sums"]["wi32"])
    for k in ("w64", "wbig"):
        assert got[k].dtype == np.float64 and np.array_equal(got[k].view(np.uint64), ref["sums"][k].view(np.uint64)), k
    assert np.abs(got["f64"] - ref["sums"]["f64"]).max() <= 1e-12 * np.abs(ref["sums"]["f64"]).max()
    assert int(r.stats["fixed_point_overflow"]) == 0 and np.array_equal(r.per_item.cpu().numpy(), ref["results"][0])
    ct = {"f64": torch.tensor([0.5, -1.0, 2.0, 0.25], dtype=torch.float64), "wbig": torch.tensor([1.0, 0.0, 0.0, -1.0])}
    g = float(f.grad(x0, keys, a, wrt=2, cotangents=ct))
    _, gv = f.value_and_grad(x0, keys, a, wrt=2, cotangents=ct)
    want = (float(np.dot(ct["f64"].numpy(), ref["sums"]["f64"])) +
            float(np.dot(ct["wbig"].double().numpy(), ref["sums"]["wbig"]))) / float(a)
    assert abs(g - want) <= 1e-5 * abs(want) and float(gv) == g


def test_diagnostics_reports_kernel_resources(cuda):
    """tallymap_b200.diagnostics on a GPU: each recorded kernel's registers, local and shared memory and resident
    blocks per SM (tm_kernel_info), and the device"""
    x, k = rw_inputs(1000, seed=3)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    f(x, k, np.float32(1.0))
    torch.cuda.synchronize()
    d = tm.diagnostics()
    rec = [r for r in d["kernels"] if r["tag"] == "walk_fwd"][-1]
    res = rec["resources"]
    assert res["registers"] > 0 and res["blocks_per_sm"] >= 1 and res["sms"] == d["platform"]["sms"] >= 100
    assert d["platform"]["compute_capability"] == "10.0"


def test_bit_counts_on_device(cuda):
    """lax.population_count / lax.clz lowered through __popc / __clz: per item bitwise Python's bit counts"""
    from tallymap_b200 import lang as tl
    xs = np.int32([0, 1, -1, 2 ** 31 - 1, -(2 ** 31), 12345, -7, 256])
    f = tm.vmap(lambda t, x: (t, tl.population_count(x), tl.clz(x)), outputs={}, in_axes=(0,))
    r = f(xs)
    torch.cuda.synchronize()
    pc, cz = (v.cpu().numpy() for v in r.per_item)
    assert list(pc) == [bin(int(v) & 0xFFFFFFFF).count("1") for v in xs]
    assert list(cz) == [32 - (int(v) & 0xFFFFFFFF).bit_length() for v in xs]
