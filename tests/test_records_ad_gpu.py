"""Records outputs under forward and reverse mode (the reference's fill twin, tallymap/_records.py:1-19): the jvp
writes each record's float-field tangents beside it and the canonical layout moves them with it; the replay adjoint
reads a record's field cotangents at its canonical slot (the forward's per-item counts and offsets).  Checked
against central differences of the IR evaluator's canonical records, against each other (<ct, J t> both ways),
and for the poisoning of an overflowed output."""
import numpy as np
import pytest
import torch

import tallymap_b200 as tm
from tallymap_b200 import backend as B
from tallymap_b200 import prng

pytestmark = pytest.mark.gpu
CAP = 1 << 14


def _setup(n=2000, cap=CAP):
    from items_lang import decay_records
    rng = np.random.default_rng(21)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(23), n)
    outs = {"tot": tm.Sum(()), "hits": tm.Records({"k": torch.int32, "w": torch.float32}, capacity=cap),
            "last": tm.Records({"k": torch.int32, "w": torch.float32}, capacity=n)}
    f = tm.vmap(decay_records, outputs=outs, in_axes=(0, 0, None), max_steps=64)
    return f, w, keys


def _records(w, keys, a, n):
    """the IR evaluator's canonical records (item order, append order) of decay_records: hits w, last w"""
    from items_lang import decay_records
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    tr = T.trace_item(decay_records, ["f32", "key", "f32"], 2, {"tot": ((), "f32")},
                      {"hits": (CAP, (("k", "i32"), ("w", "f32"))), "last": (n, (("k", "i32"), ("w", "f32")))})
    r = Evaluator(tr, 64).run([w, keys], [np.float32(a)])
    hw = np.array([rec[1] for rec in r["records"]["hits"]], np.float64)
    lw = np.array([rec[1] for rec in r["records"]["last"]], np.float64)
    return hw, lw, float(r["sums"]["tot"][0])


def test_records_jvp_against_central_difference(cuda):
    f, w, keys = _setup()
    a, h = 1.05, 1e-3
    r, d = f.jvp(w, keys, np.float32(a), wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    m = int(r.stats["appended"]["hits"])
    assert 0 < m < CAP and int(r.stats["appended"]["last"]) == len(w)
    hp, lp, tp = _records(w, keys, a + h, len(w))
    hm, lm, tm_ = _records(w, keys, a - h, len(w))
    h0, l0, _ = _records(w, keys, a, len(w))
    assert len(hp) == len(hm) == len(h0) == m
    dh, dl = d["hits"]["w"].cpu().numpy().astype(np.float64), d["last"]["w"].cpu().numpy().astype(np.float64)
    assert np.allclose(dh[:m], (hp - hm) / (2 * h), rtol=1e-3, atol=1e-4) and not dh[m:].any()
    assert np.allclose(dl, (lp - lm) / (2 * h), rtol=1e-3, atol=1e-4)
    # the primal records in the canonical layout, bitwise the forward's
    r0 = f(w, keys, np.float32(a))
    torch.cuda.synchronize()
    for nm in ("hits", "last"):
        for fld in ("k", "w"):
            assert torch.equal(r.outputs[nm][fld], r0.outputs[nm][fld])
    assert abs(float(d["tot"]) - (tp - tm_) / (2 * h)) <= 1e-3 * abs((tp - tm_) / (2 * h))


def test_records_grad_matches_jvp(cuda):
    """the adjoint with cotangents on both Records outputs and the Sum against the jvp's contraction (and a central
    difference); a second call bitwise the same"""
    f, w, keys = _setup()
    a = np.float32(1.05)
    rng = np.random.default_rng(5)
    ct = {"tot": torch.tensor(0.3),
          "hits": {"w": torch.from_numpy(rng.normal(size=CAP).astype(np.float32))},
          "last": {"w": torch.from_numpy(rng.normal(size=len(w)).astype(np.float32))}}
    g = f.grad(w, keys, a, wrt=2, cotangents=ct)
    g2 = f.grad(w, keys, a, wrt=2, cotangents=ct)
    _, d = f.jvp(w, keys, a, wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    want = (0.3 * float(d["tot"]) + float((ct["hits"]["w"].double() * d["hits"]["w"].cpu().double()).sum())
            + float((ct["last"]["w"].double() * d["last"]["w"].cpu().double()).sum()))
    assert abs(float(g) - want) <= 1e-5 * max(abs(want), 1.0)
    assert torch.equal(g.view(torch.int32), g2.view(torch.int32))
    r, gv = f.value_and_grad(w, keys, a, wrt=2, cotangents=ct)
    torch.cuda.synchronize()
    assert torch.equal(gv.view(torch.int32), g.view(torch.int32)) and int(r.stats["appended"]["last"]) == len(w)


def test_records_grad_and_jvp_poison_on_overflow(cuda):
    f, w, keys = _setup(cap=64)
    g = f.grad(w, keys, np.float32(1.05), wrt=2, cotangents={"tot": torch.tensor(1.0)})
    r, d = f.jvp(w, keys, np.float32(1.05), wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    assert torch.isnan(g) and torch.isnan(d["hits"]["w"]).all() and torch.isnan(d["tot"])
    assert int(r.stats["records_dropped"]["hits"]) > 0


def test_records_replay_count_mismatch_flags(cuda):
    """the negative control of the replay's append count (_records.py twin: a final k != cnt poisons): the adjoint
    given one item's count off by one flags that item, and only it"""
    f, w, keys = _setup(n=500)
    a = np.float32(1.05)
    L = f.lowered((w, keys, a))
    fo = B.run(L.fwd, [w, keys], [a], consts=(64,))
    ys = fo[len(L.fwd.tallies) + 1:]
    prog = L.grad_program((0,))
    pi = [w, keys]
    for r, (nm, cap, _) in enumerate(L.fwd.records):
        cnt = ys[L.n_results + r].clone()
        if nm == "hits":
            cnt[7] += 1
        off = torch.cumsum(cnt.to(torch.int64), 0) - cnt.to(torch.int64)
        pi += [cnt, off]
    cts = [torch.zeros(())] + [torch.zeros(cap) for nm, cap, _ in L.fwd.records]
    out = B.run(prog, pi, [a] + cts, consts=(64,))
    torch.cuda.synchronize()
    tr = out[-1].cpu().numpy()
    assert tr[7] == 1 and tr.sum() == 1


def test_records_appended_before_the_loop(cuda):
    """appends before the loop, in it and after it into one output: the canonical layout bitwise the IR evaluator's;
    the tangents against a central difference; the adjoint against the jvp's contraction"""
    from items_lang import pre_records
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    n, cap = 1000, 8192
    rng = np.random.default_rng(3)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(9), n)
    f = tm.vmap(pre_records, outputs={"log": tm.Records({"k": torch.int32, "w": torch.float32}, capacity=cap)},
                in_axes=(0, 0, None), max_steps=16)
    tr = T.trace_item(pre_records, ["f32", "key", "f32"], 2, {}, {"log": (cap, (("k", "i32"), ("w", "f32")))})

    def ev(a):
        r = Evaluator(tr, 16).run([w, keys], [np.float32(a)])
        return np.array([x[0] for x in r["records"]["log"]]), np.array([x[1] for x in r["records"]["log"]], np.float32)
    a, h = 1.1, 1e-3
    r, d = f.jvp(w, keys, np.float32(a), wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    k0, w0 = ev(a)
    m = len(k0)
    assert int(r.stats["appended"]["log"]) == m and (k0 == -1).sum() == n and (k0 == 99).sum() == n
    assert np.array_equal(r.outputs["log"]["k"].cpu().numpy()[:m], k0)
    assert np.array_equal(r.outputs["log"]["w"].cpu().numpy()[:m].view(np.uint32), w0.view(np.uint32))
    fd = (ev(a + h)[1].astype(np.float64) - ev(a - h)[1]) / (2 * h)
    assert np.allclose(d["log"]["w"].cpu().numpy()[:m], fd, rtol=1e-3, atol=1e-4)
    ct = torch.from_numpy(rng.normal(size=cap).astype(np.float32))
    g = f.grad(w, keys, np.float32(a), wrt=2, cotangents={"log": {"w": ct}})
    torch.cuda.synchronize()
    want = float((ct.double() * d["log"]["w"].cpu().double()).sum())
    assert abs(float(g) - want) <= 1e-5 * max(abs(want), 1.0)


# ---------------------------------------------------------------------------------------------- count-then-fill
def _pair(n=2000):
    """the same item with a capacity-less Records output (count-then-fill) and with a large capacity (one pass)"""
    from items_lang import decay_records
    rng = np.random.default_rng(21)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(23), n)
    mk = lambda cap: tm.vmap(decay_records, outputs={
        "tot": tm.Sum(()), "hits": tm.Records({"k": torch.int32, "w": torch.float32}, capacity=cap),
        "last": tm.Records({"k": torch.int32, "w": torch.float32}, capacity=n)}, in_axes=(0, 0, None), max_steps=64)
    return mk(None), mk(CAP), w, keys


def test_count_then_fill_forward(cuda):
    """a Records output without a capacity: exactly the total records, each where the one-pass layout puts it; the
    other outputs (a Sum, a Records output with a capacity) as the one-pass call's"""
    ff, fo, w, keys = _pair()
    a = np.float32(1.05)
    r1, r2 = ff(w, keys, a), fo(w, keys, a)
    torch.cuda.synchronize()
    m = int(r2.stats["appended"]["hits"])
    assert int(r1.stats["appended"]["hits"]) == m and r1.outputs["hits"]["w"].shape == (m,)
    assert int(r1.stats["records_mismatch"]["hits"]) == 0 and int(r1.stats["records_dropped"]["hits"]) == 0
    for fld in ("k", "w"):
        assert torch.equal(r1.outputs["hits"][fld], r2.outputs["hits"][fld][:m])
        assert torch.equal(r1.outputs["last"][fld], r2.outputs["last"][fld])
    assert abs(float(r1.outputs["tot"]) - float(r2.outputs["tot"])) <= 1e-5 * abs(float(r2.outputs["tot"]))
    assert torch.equal(r1.per_item, r2.per_item)


def test_count_then_fill_jvp_and_grad(cuda):
    """forward mode and the adjoint of a count-then-fill output against the one-pass ones: the tangents bitwise,
    the gradient bitwise (the same cotangents at the same slots)"""
    ff, fo, w, keys = _pair()
    a = np.float32(1.05)
    r1, d1 = ff.jvp(w, keys, a, wrt=2, tangents=[1.0])
    r2, d2 = fo.jvp(w, keys, a, wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    m = int(r1.stats["appended"]["hits"])
    assert d1["hits"]["w"].shape == (m,) and torch.equal(d1["hits"]["w"], d2["hits"]["w"][:m])
    assert torch.equal(d1["last"]["w"], d2["last"]["w"])
    rng = np.random.default_rng(8)
    cth = rng.normal(size=CAP).astype(np.float32)
    ctl = torch.from_numpy(rng.normal(size=len(w)).astype(np.float32))
    g1 = ff.grad(w, keys, a, wrt=2, cotangents={"hits": {"w": torch.from_numpy(cth[:m])}, "last": {"w": ctl}})
    g2 = fo.grad(w, keys, a, wrt=2, cotangents={"hits": {"w": torch.from_numpy(cth)}, "last": {"w": ctl}})
    torch.cuda.synchronize()
    assert torch.equal(g1.view(torch.int32), g2.view(torch.int32))


def test_count_then_fill_with_an_overflowing_capacity_output(cuda):
    """count-then-fill beside an output whose capacity is too small: that output's records are cut at its capacity
    and poisoned (floats NaN, integers -1), every float output NaN, the capacity-less output's records intact"""
    from items_lang import decay_records
    rng = np.random.default_rng(21)
    n = 500
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(23), n)
    f = tm.vmap(decay_records, outputs={"tot": tm.Sum(()), "hits": tm.Records({"k": torch.int32, "w": torch.float32}),
                                         "last": tm.Records({"k": torch.int32, "w": torch.float32}, capacity=n // 2)},
                in_axes=(0, 0, None), max_steps=64)
    r = f(w, keys, np.float32(1.05))
    torch.cuda.synchronize()
    assert int(r.stats["records_dropped"]["last"]) == n - n // 2 and r.outputs["last"]["w"].shape == (n // 2,)
    assert torch.isnan(r.outputs["last"]["w"]).all() and (r.outputs["last"]["k"] == -1).all()
    assert torch.isnan(r.outputs["tot"])
    assert int(r.stats["records_mismatch"]["hits"]) == 0


@pytest.mark.parametrize("cap", [1 << 15, None])
def test_records_inside_inner_loops(cuda, cap):
    """Records appended inside inner loops (items_lang.loop_records): the canonical records bitwise the IR
    evaluator's; the adjoint -- the loop that reads a transposed iteration by iteration, the other re-run to count its
    appends -- against the jvp's contraction within 5e-5; one pass (a capacity) and count-then-fill alike"""
    from items_lang import loop_records
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    n = 1000
    x = np.random.default_rng(4).uniform(0.2, 0.9, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(6), n)
    a = np.float32(0.8)
    outs = {"h": tm.Sum((1,)), "r": tm.Records({"v": torch.float32}, capacity=cap)}
    f = tm.vmap(loop_records, outputs=outs, in_axes=(0, 0, None), max_steps=8)
    tr = T.trace_item(loop_records, ["f32", "key", "f32"], 2, {"h": ((1,), "f32")}, {"r": (1 << 15, (("v", "f32"),))})
    ref = Evaluator(tr, 8).run([x, keys], [a])
    want_v = np.array([rec[0] for rec in ref["records"]["r"]], np.float32)
    m = len(want_v)
    r = f(x, keys, a)
    torch.cuda.synchronize()
    assert m == 15 * n and int(r.stats["appended"]["r"]) == m
    assert np.array_equal(r.outputs["r"]["v"].cpu().numpy()[:m].view(np.uint32), want_v.view(np.uint32))
    ctv = torch.from_numpy(np.random.default_rng(7).normal(size=cap or m).astype(np.float32))
    ct = {"h": torch.tensor([0.4]), "r": {"v": ctv}}
    g = f.grad(x, keys, a, wrt=2, cotangents=ct)
    _, d = f.jvp(x, keys, a, wrt=2, tangents=[1.0])
    torch.cuda.synchronize()
    want = 0.4 * float(d["h"][0]) + float((ctv.double() * d["r"]["v"].cpu().double()).sum())
    # (the Sum's tangent is a float32 atomic sum of 4000 emits: its rounding depends on the atomics' order)
    assert abs(float(g) - want) <= 5e-5 * abs(want)
