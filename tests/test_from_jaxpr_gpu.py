"""GPU: the jaxpr front end end to end.  The reference's quickstart ItemProgram (duck-typed, tests/jaxpr_fixtures.py,
after retrace(cap=100)) through tallymap_b200.from_jaxpr.run -- the reference backend entry's signature -- against
the oracle: the histogram within the float tolerance, stats, trip counts and the program's own truncation flags
bitwise, in the reference's output order [sum tallies] + [stats] + [per-item results]; and the same jaxpr's item
function under tallymap_b200.vmap: its replay gradient w.r.t. theta bitwise the oracle's."""
import numpy as np
import pytest
import torch

import jaxpr_fixtures as J
import tallymap_b200 as tm
from tallymap_b200 import from_jaxpr as FJ
from tallymap_b200 import prng

pytestmark = pytest.mark.gpu


def _inputs(n):
    return np.linspace(0.1, 0.99, n, dtype=np.float32), prng.split(prng.PRNGKey(0), n)


@pytest.mark.parametrize("cap", [100, 3])
def test_reference_item_program_runs(cuda, orc, cap):
    x, k = _inputs(10000)
    out = FJ.run(J.quickstart_program(cap=cap), [x, k], [np.float32(2.0)], target="cuda", cuda_math="ieee")
    torch.cuda.synchronize()
    hist, stats, kk, tr = [o.cpu().numpy() for o in out]
    ref = orc.q1_fwd(x, k, 2.0, max_steps=cap)
    assert out[3].dtype == torch.bool
    assert np.array_equal(kk, ref["k"]) and np.array_equal(tr, ref["trunc"]) and np.array_equal(stats, ref["stats"])
    assert np.abs(hist.astype(np.float64) - ref["hist"]).max() <= 1e-5 * np.abs(ref["hist"]).max()
    if cap == 3:
        assert tr.any()


def test_jaxpr_item_gradient_bitwise(cuda, orc):
    fn, _ = FJ.item_function(J.quickstart(), ["hist"], 2)
    f = tm.vmap(fn, outputs={"hist": tm.Sum((16,))}, in_axes=(0, 0, None), max_steps=100)
    x, k = _inputs(10000)
    ct = np.random.default_rng(5).normal(size=16).astype(np.float32)
    g = f.grad(x, k, np.float32(2.0), wrt=2, cotangents={"hist": torch.from_numpy(ct)})
    ref = orc.q1_grad(x, k, 2.0, ct)
    assert np.array_equal(np.float32(g.cpu().numpy()).reshape(1).view(np.uint32), ref["g"].view(np.uint32))


def test_jaxpr_emit_inside_a_cond_branch(cuda):
    """the quickstart jaxpr with its emit inside a lax.cond branch (taken above x = 0.3): the histogram within the
    float tolerance of the IR evaluator's, nothing in the bins below the gate, trip counts exact; the replay
    gradient w.r.t. theta equal to that of the IR's own evaluation at theta +- h (the histogram is linear in theta)"""
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    fn, specs = FJ.item_function(J.quickstart(gate=0.3), ["hist"], 2)
    f = tm.vmap(fn, outputs={"hist": tm.Sum((16,))}, in_axes=(0, 0, None), max_steps=100)
    x, k = _inputs(10000)
    r = f(x, k, np.float32(2.0))
    torch.cuda.synchronize()
    tr = T.trace_item(fn, specs, 2, {"hist": ((16,), "f32")})
    ev = lambda th: Evaluator(tr, 100).run([x, k], [np.float32(th)])
    ref = ev(2.0)
    h = r.outputs["hist"].cpu().numpy().astype(np.float64)
    assert np.abs(h - ref["sums"]["hist"]).max() <= 1e-5 * np.abs(ref["sums"]["hist"]).max()
    assert h[:4].max() == 0.0 and np.array_equal(r.per_item.cpu().numpy(), ref["results"][0])
    ct = np.random.default_rng(5).normal(size=16).astype(np.float32)
    g = float(f.grad(x, k, np.float32(2.0), wrt=2, cotangents={"hist": torch.from_numpy(ct)}))
    want = float(np.dot(ct.astype(np.float64), (ev(2.5)["sums"]["hist"] - ev(1.5)["sums"]["hist"]) / 1.0))
    assert abs(g - want) <= 1e-4 * abs(want)


@pytest.mark.parametrize("C", [1 << 15, 64])
def test_reference_records_program_runs(cuda, C):
    """the reference's one-pass Records program (tallymap_claim + the cond that writes the claimed slot) through
    run(): every raw slot below min(total, C) holds one record, whose (node id, ordinal) key places it at the
    canonical slot (tallymap/_records.py:35-62 canon) with the field the IR evaluator gives that record, bitwise;
    the counts (per-item results) and trip counts exact; a capacity below the total keeps C of the records and
    drops no other write"""
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    from items_lang import quickstart_hits
    n = 10000
    x, k = _inputs(n)
    cid = np.arange(n, dtype=np.int32)
    out = FJ.run(J.records_program(C), [x, k, cid], [np.float32(2.0)], target="cuda", cuda_math="ieee")
    torch.cuda.synchronize()
    hist, hx, hi, hk, stats, kk, cnt = [o.cpu().numpy() for o in out]
    tq = T.trace_item(quickstart_hits, ["f32", "key", "f32"], 2, {"hist": ((16,), "f32")},
                      {"hits": (1 << 20, (("x", "f32"),))})
    ref = Evaluator(tq, 100).run([x, k], [np.float32(2.0)])
    want_cnt = ref["counts"]["hits"]
    total = int(want_cnt.sum())
    assert np.array_equal(cnt, want_cnt) and np.array_equal(kk, ref["results"][0]) and not stats.any()
    assert np.abs(hist - ref["sums"]["hist"]).max() <= 1e-5 * np.abs(ref["sums"]["hist"]).max()
    want_x = np.array([v[0] for v in ref["records"]["hits"]], np.float32)
    off = np.concatenate([[0], np.cumsum(want_cnt)[:-1]])
    m = min(total, C)
    assert total > 0 and (C > total or total > 2 * C)
    pos = off[hi[:m]] + hk[:m]
    assert (hk[:m] < want_cnt[hi[:m]]).all() and len(np.unique(pos)) == m
    assert np.array_equal(hx[:m].view(np.uint32), want_x[pos].view(np.uint32))
    assert not hx[m:].any() and not hi[m:].any() and not hk[m:].any()
