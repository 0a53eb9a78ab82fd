"""CPU: the jaxpr front end (tallymap_b200.from_jaxpr) on duck-typed jaxprs of the reference's quickstart item
(tests/jaxpr_fixtures.py, spelled as jax.make_jaxpr writes it): the item function it makes traces to IR that the IR
evaluator runs bitwise like the hand-written oracle (trip counts, truncation flags, stats; the histogram within the
float tolerance) and like the same item written with tallymap_b200.lang; its retrace(cap) form gives the same
trip counts and its own truncation flag; the lowering compiles it for sm_100a (NVRTC needs no GPU); primitives
outside the table raise UnsupportedError."""
import numpy as np
import pytest

import jaxpr_fixtures as J
from tallymap_b200 import from_jaxpr as FJ
from tallymap_b200 import prng
from tallymap_b200 import trace as T

SPECS = {"hist": ((16,), "f32")}


def _inputs(n):
    return np.linspace(0.1, 0.99, n, dtype=np.float32), prng.split(prng.PRNGKey(0), n)


def test_quickstart_jaxpr_against_oracle(orc):
    from oracle.ir_eval import Evaluator
    fn, specs = FJ.item_function(J.quickstart(), ["hist"], 2)
    assert specs == ["f32", "key", "f32"]
    tr = T.trace_item(fn, specs, 2, SPECS)
    assert sum(e.prim == "emit" for e in tr.body) == 1 and sum(e.prim == "bits" for e in tr.body) == 1
    x, k = _inputs(3000)
    r = Evaluator(tr, 100).run([x, k], [2.0])
    ref = orc.q1_fwd(x, k, 2.0)
    assert np.array_equal(r["results"][0], ref["k"]) and np.array_equal(r["trunc"], ref["trunc"])
    assert np.array_equal(r["stats"], ref["stats"])
    assert np.abs(r["sums"]["hist"] - ref["hist"]).max() <= 1e-6 * np.abs(ref["hist"]).max()
    # the same item written with tallymap_b200.lang: the same results bitwise
    from items_lang import quickstart
    tq = T.trace_item(quickstart, ["f32", "key", "f32"], 2, SPECS)
    rq = Evaluator(tq, 100).run([x, k], [2.0])
    assert np.array_equal(rq["results"][0], r["results"][0])
    assert np.array_equal(rq["sums"]["hist"].view(np.uint32), r["sums"]["hist"].view(np.uint32))


def test_emit_inside_a_cond_branch():
    """the reference's `t = lax.cond(pred, lambda t: t.add(...), lambda t: t, t)` (the tally threaded through a
    cond, tallymap/_rewrite.py:173-185, 573-598): the emit is made only where its branch is taken -- the IR equal
    to the same item written with tallymap_b200.lang and a select of the value, its histogram bitwise"""
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import lang as tl
    fn, specs = FJ.item_function(J.quickstart(gate=0.3), ["hist"], 2)
    tr = T.trace_item(fn, specs, 2, SPECS)
    (em,) = [e for e in tr.body if e.prim == "emit"]
    assert len(em.ins) == 3 and em.ins[2].dtype == T.BOOL

    def gated(t, x, key, theta):
        def body(c):
            k, x, t = c
            u = tl.random.uniform(tl.random.fold_in(key, k))
            t = t.add("hist", (x * 16).astype(tl.int32), tl.where(x > 0.3, theta * (1 - x), 0.0))
            return k + 1, x * (0.5 + 0.5 * u), t
        k, x, t = tl.while_loop(lambda c: c[1] > 0.05, body, (0, x, t))
        return t, k
    x, k = _inputs(3000)
    r = Evaluator(tr, 100).run([x, k], [2.0])
    rq = Evaluator(T.trace_item(gated, ["f32", "key", "f32"], 2, SPECS), 100).run([x, k], [2.0])
    assert np.array_equal(rq["results"][0], r["results"][0])
    assert np.array_equal(rq["sums"]["hist"].view(np.uint32), r["sums"]["hist"].view(np.uint32))
    assert r["sums"]["hist"][:4].max() == 0.0 and r["sums"]["hist"][5:].min() > 0.0


def test_scan_and_static_fori_loop():
    """jax's scan equation (lax.scan, and fori_loop of static bounds, which jax writes as a scan carrying the
    counter) unrolls like tallymap_b200.lang's scan / fori_loop: the IR evaluator's outputs bitwise equal to the
    same item written with lang"""
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import lang as tl
    fn, specs = FJ.item_function(J.scans(), ["hist"], 2)
    tr = T.trace_item(fn, specs, 2, SPECS)

    def item(t, x, key, theta):
        c = tl.fori_loop(0, 3, lambda i, c: c * 0.5 + float(i), x)
        cs, ys = tl.scan(lambda c, z: (c + z * theta, c * z), 0.0, tl.array([1.0, 2.0, 3.0]))
        t = t.add("hist", 0, c).add("hist", 1, cs).add("hist", 2, ys[2])
        return t, c
    x, k = _inputs(64)
    r = Evaluator(tr, 10).run([x, k], [np.float32(1.5)])
    rq = Evaluator(T.trace_item(item, ["f32", "key", "f32"], 2, SPECS), 10).run([x, k], [np.float32(1.5)])
    assert np.array_equal(r["results"][0].view(np.uint32), rq["results"][0].view(np.uint32))
    assert np.array_equal(r["sums"]["hist"].view(np.uint32), rq["sums"]["hist"].view(np.uint32))
    c = x
    for i in range(3):
        c = (c * np.float32(0.5) + np.float32(i)).astype(np.float32)
    assert np.array_equal(r["results"][0], c)
    assert r["sums"]["hist"][1] == 64 * 9.0 and r["sums"]["hist"][2] == 64 * 13.5


def test_records_one_pass_claims():
    """the reference's one-pass Records append in a jaxpr (tallymap_claim, then the field, the node id and the
    ordinal emitted at the claimed slot inside a cond; tallymap/_tally.py:335-351): with the items run in order (the
    IR evaluator) the raw slots are the canonical layout, the records of the same item written with lang's
    t.append; the forward program compiles with one slot counter per tally, and a derived program refuses the claim
    (the reference runs its fill twin there)"""
    from oracle.ir_eval import Evaluator
    import tallymap_b200 as tm
    import torch
    from items_lang import quickstart_hits
    C = 4096
    names = ["hist", "hits\x1fx", "hits\x1fi", "hits\x1fk"]
    fn, specs = FJ.item_function(J.quickstart_records(C), names, 3)
    assert specs == ["f32", "key", "i32", "f32"]
    sp = {"hist": ((16,), "f32"), names[1]: ((C,), "f32"), names[2]: ((C,), "i32"), names[3]: ((C,), "i32")}
    tr = T.trace_item(fn, specs, 3, sp)
    assert sum(e.prim == "claim" for e in tr.body) == 1
    assert sum(e.prim == "emit" and len(e.ins) == 3 for e in tr.body) == 3
    n = 3000
    x, k = _inputs(n)
    cid = np.arange(n, dtype=np.int32)
    r = Evaluator(tr, 100).run([x, k, cid], [2.0])
    tq = T.trace_item(quickstart_hits, ["f32", "key", "f32"], 2, SPECS, {"hits": (C, (("x", "f32"),))})
    rq = Evaluator(tq, 100).run([x, k], [2.0])
    cnt = rq["counts"]["hits"]
    m = len(rq["records"]["hits"])
    assert 0 < m < C and np.array_equal(r["results"][1], cnt)
    assert np.array_equal(r["results"][0], rq["results"][0]) and np.array_equal(r["sums"]["hist"], rq["sums"]["hist"])
    want = np.array([v[0] for v in rq["records"]["hits"]], np.float32)
    assert np.array_equal(r["sums"][names[1]][:m].astype(np.float32).view(np.uint32), want.view(np.uint32))
    assert np.array_equal(r["sums"][names[2]][:m], np.repeat(np.arange(n), cnt))
    assert np.array_equal(r["sums"][names[3]][:m], np.concatenate([np.arange(c) for c in cnt]))
    assert not r["sums"][names[1]][m:].any()
    outs = {"hist": tm.Sum((16,)), names[1]: tm.Sum((C,)), names[2]: tm.Sum((C,), torch.int32),
            names[3]: tm.Sum((C,), torch.int32)}
    f = tm.vmap(fn, outputs=outs, in_axes=(0, 0, 0, None), max_steps=100)
    L = f.lowered((x[:8], k[:8], cid[:8], np.float32(2.0)))
    assert L.fwd.kernel > 0 and L.fwd.claims == 4 and "atomicAdd(&c.claims[3], 1ull)" in L.fwd_source
    with pytest.raises(T.UnsupportedError, match="fill twin"):
        L.grad_program((0,))


def test_retraced_program_carries_its_own_cap(orc):
    """the reference backend receives retrace(cap)'s program: its loop counter stops the loop and its own
    `truncated` is the second per-item result, equal to the oracle's flags at max_steps = 3"""
    from oracle.ir_eval import Evaluator
    p = J.quickstart_program(cap=3)
    fn, specs = FJ.item_function(p.cj, ["hist"], p.nP)
    tr = T.trace_item(fn, specs, 2, SPECS)
    x, k = _inputs(2000)
    r = Evaluator(tr, 10 ** 6).run([x, k], [2.0])
    ref = orc.q1_fwd(x, k, 2.0, max_steps=3)
    assert ref["trunc"].any()
    assert np.array_equal(r["results"][0], ref["k"])
    assert np.array_equal(np.asarray(r["results"][1]).astype(bool), ref["trunc"])
    assert not np.asarray(r["trunc"]).any()                # (the runtime's own ceiling is far above the cap)


def test_lowers_and_compiles(tmlib):
    import tallymap_b200 as tm
    fn, specs = FJ.item_function(J.quickstart(), ["hist"], 2)
    f = tm.vmap(fn, outputs={"hist": tm.Sum((16,))}, in_axes=(0, 0, None), max_steps=100)
    x, k = _inputs(8)
    L = f.lowered((x, k, np.float32(2.0)))
    assert isinstance(L.fwd.kernel, int) and "random_bits32" in L.fwd_source
    g = L.grad_program((0,))          # the replay adjoint w.r.t. theta lowers from the same IR
    assert g.tallies[0].exact


def test_constant_folding_and_lax_integer_semantics():
    """all-constant equations fold in numpy with the aval's dtype; lax.div / lax.rem of integers truncate toward
    zero (not Python's floor), on traced values and on constants alike"""
    from oracle.ir_eval import Evaluator
    a, b, q, r, qc, rc, s = J.Var(J.I), J.Var(J.I), J.Var(J.I), J.Var(J.I), J.Var(J.I), J.Var(J.I), J.Var(J.F)
    eqns = [J.Eqn("div", [a, b], [q]), J.Eqn("rem", [a, b], [r]),
            J.Eqn("div", [J.Literal(-7, J.I), J.Literal(2, J.I)], [qc]),
            J.Eqn("rem", [J.Literal(-7, J.I), J.Literal(2, J.I)], [rc]),
            J.Eqn("sub", [J.Literal(1.0, J.F), J.Literal(0.25, J.F)], [s])]
    cj = J.ClosedJaxpr(J.Jaxpr([a, b], [q, r, qc, rc, s], eqns))
    fn, specs = FJ.item_function(cj, [], 2)
    tr = T.trace_item(fn, specs, 2, {})
    A = np.int32([7, -7, 7, -7, 0, 5])
    Bv = np.int32([2, 2, -2, -2, 3, 5])
    res = Evaluator(tr, 1).run([A, Bv], [])["results"]
    assert list(res[0]) == [3, -3, -3, 3, 0, 1] and list(res[1]) == [1, -1, 1, -1, 0, 0]
    assert list(res[2]) == [-3] * 6 and list(res[3]) == [-1] * 6 and np.all(np.asarray(res[4]) == 0.75)


def test_vector_structure_primitives():
    """cumsum / cummax (reverse), rev, pad (interior, negative edge), dot_general (matrix-vector with a constant
    matrix, and a vector dot), dynamic_update_slice at a traced start, jit (jax >= 0.7's name of pjit),
    random_clone, iota_2x32_shape and platform_index: the IR evaluator's values bitwise those of numpy float32 in the
    reference's order (sequential running values; dot sums from zero, acc + x * y, no fused multiply-add)"""
    from oracle.ir_eval import Evaluator
    V, E, L = J.Var, J.Eqn, J.Literal
    x, th, k = V(J.F), V(J.F), V(J.I)
    x2, xb, x2b, thb, v = V(J.F), V(J.F, (1,)), V(J.F, (1,)), V(J.F, (1,)), V(J.F, (3,))
    c, r, pd, mv, d, u, cm = V(J.F, (3,)), V(J.F, (3,)), V(J.F, (5,)), V(J.F, (2,)), V(J.F), V(J.F, (5,)), V(J.F, (3,))
    jin, jout, jv = V(J.F, (3,)), V(J.F, (3,)), V(J.F, (3,))
    inner = J.ClosedJaxpr(J.Jaxpr([jin], [jout], [J.Eqn("rev", [jin], [jout], dimensions=(0,))]))
    hi, lo = V(J.U, (4,)), V(J.U, (4,))
    M = L(np.array([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], np.float32), J.F)
    M.aval = J.Aval((2, 3), J.F)
    eqns = [E("mul", [x, L(2.0, J.F)], [x2]),
            E("broadcast_in_dim", [x], [xb], shape=(1,), broadcast_dimensions=()),
            E("broadcast_in_dim", [x2], [x2b], shape=(1,), broadcast_dimensions=()),
            E("broadcast_in_dim", [th], [thb], shape=(1,), broadcast_dimensions=()),
            E("concatenate", [xb, x2b, thb], [v], dimension=0),
            E("cumsum", [v], [c], axis=0, reverse=False),
            E("jit", [c], [r], jaxpr=inner, name="flip"),
            E("pad", [r, L(0.5, J.F)], [pd], padding_config=((1, -1, 1),)),
            E("dot_general", [M, v], [mv], dimension_numbers=(((1,), (0,)), ((), ())), precision=None,
              preferred_element_type=np.float32),
            E("dot_general", [v, v], [d], dimension_numbers=(((0,), (0,)), ((), ())), precision=None,
              preferred_element_type=np.float32),
            E("dynamic_update_slice", [pd, mv, k], [u]),
            E("cummax", [v], [cm], axis=0, reverse=True),
            E("random_clone", [v], [jv]),
            E("iota_2x32_shape", [], [hi, lo], shape=(4,))]
    cj = J.ClosedJaxpr(J.Jaxpr([x, k, th], [c, pd, mv, d, u, cm, lo], eqns))
    fn, specs = FJ.item_function(cj, [], 2)
    tr = T.trace_item(fn, specs, 2, {})
    n = 40
    xs = np.random.default_rng(4).normal(size=n).astype(np.float32)
    ks = (np.arange(n) % 7 - 1).astype(np.int32)
    t = np.float32(0.7)
    res = [np.asarray(v) for v in Evaluator(tr, 1).run([xs, ks], [t])["results"]]
    f = np.float32
    for i in range(n):
        vv = [xs[i], f(xs[i] * f(2)), t]
        cc = [vv[0], f(vv[0] + vv[1]), f(f(vv[0] + vv[1]) + vv[2])]
        rr = cc[::-1]
        pp = [f(0.5), rr[0], f(0.5), rr[1], f(0.5)]
        mm = [f(f(f(f(0) + f(1 * vv[0])) + f(2 * vv[1])) + f(3 * vv[2])),
              f(f(f(f(0) + f(4 * vv[0])) + f(5 * vv[1])) + f(6 * vv[2]))]
        dd = f(f(f(f(0) + f(vv[0] * vv[0])) + f(vv[1] * vv[1])) + f(vv[2] * vv[2]))
        s0 = int(np.clip(ks[i], 0, 3))
        uu = pp[:s0] + mm + pp[s0 + 2:]
        c2 = vv[2]
        c1 = max(vv[1], c2)
        c0 = max(vv[0], c1)
        want = cc + pp + mm + [dd] + uu + [c0, c1, c2] + [0, 1, 2, 3]
        got = [res[j][i] for j in range(len(want))]
        assert np.array_equal(np.float32(got[:-4]).view(np.uint32), np.float32(want[:-4]).view(np.uint32)), i
        assert got[-4:] == [0, 1, 2, 3]
    assert FJ._platform_index([("cpu",), ("cuda", "rocm"), None]) == 1 and FJ._platform_index([("cpu",), None]) == 1


def test_sort_primitive():
    """lax.sort of (keys, iota) (jnp.argsort's form) and of keys alone: stable and ascending in lax.sort's total order
    (NaNs last, -0 equal to +0, each value keeping its bits), bitwise against numpy's stable argsort"""
    from oracle.ir_eval import Evaluator
    V, E, L = J.Var, J.Eqn, J.Literal
    x, y, z = V(J.F), V(J.F), V(J.F)
    xb, yb, zb, nb = V(J.F, (1,)), V(J.F, (1,)), V(J.F, (1,)), V(J.F, (1,))
    v, io, sv, perm, sv2 = V(J.F, (5,)), V(J.I, (5,)), V(J.F, (5,)), V(J.I, (5,)), V(J.F, (5,))
    b = lambda s_, d_: E("broadcast_in_dim", [s_], [d_], shape=(1,), broadcast_dimensions=())
    eqns = [b(x, xb), b(y, yb), b(z, zb), b(L(-0.0, J.F), nb),
            E("concatenate", [xb, nb, yb, zb, xb], [v], dimension=0),
            E("iota", [], [io], dtype=np.int32, shape=(5,), dimension=0, sharding=None),
            E("sort", [v, io], [sv, perm], dimension=0, is_stable=True, num_keys=1),
            E("sort", [v], [sv2], dimension=0, is_stable=True, num_keys=1)]
    cj = J.ClosedJaxpr(J.Jaxpr([x, y, z], [sv, perm, sv2], eqns))
    fn, specs = FJ.item_function(cj, [], 3)
    tr = T.trace_item(fn, specs, 3, {})
    vals = np.float32([0.0, -0.0, 1.5, -2.0, np.nan, -np.nan, np.inf, -np.inf, 1.5])
    g = np.array(np.meshgrid(vals, vals, vals)).reshape(3, -1)
    xs, ys, zs = (g[i].astype(np.float32) for i in range(3))
    res = [np.asarray(r) for r in Evaluator(tr, 1).run([xs, ys, zs], [])["results"]]
    for i in range(len(xs)):
        key = np.float32([xs[i], -0.0, ys[i], zs[i], xs[i]])
        order = np.argsort(np.where(key == 0, np.float32(0), key), kind="stable")
        got_v = np.float32([res[j][i] for j in range(5)])
        got_p = [int(res[5 + j][i]) for j in range(5)]
        got_v2 = np.float32([res[10 + j][i] for j in range(5)])
        assert got_p == list(order), (key, got_p, order)
        assert np.array_equal(got_v.view(np.uint32), key[order].view(np.uint32))
        assert np.array_equal(got_v2.view(np.uint32), key[order].view(np.uint32))


def test_gather_and_table_slices():
    """lax.gather as jnp indexing writes it -- a scalar index into a broadcast table (clip and fill modes), a vector
    of indices into a per-item vector, an element and a row of a 2-D table -- and dynamic_slice of a 2-D table's
    row: broadcast arrays become tables (as tallymap_b200.vmap passes them); the IR evaluator's values equal numpy's
    clamped reads, NaN where a fill-mode start is out of range"""
    from types import SimpleNamespace as NS
    from oracle.ir_eval import Evaluator
    V, E, L = J.Var, J.Eqn, J.Literal
    dn = lambda off, col, smap: NS(offset_dims=off, collapsed_slice_dims=col, start_index_map=smap,
                                   operand_batching_dims=(), start_indices_batching_dims=())
    PROM, FILL = "GatherScatterMode.PROMISE_IN_BOUNDS", "GatherScatterMode.FILL_OR_DROP"
    i, j, vec, tab, tab2 = V(J.I), V(J.I), V(J.F, (4,)), V(J.F, (100,)), V(J.F, (8, 3))
    ib, ij, i3, g1, g2, g3, g4, g5, ds, row = (V(J.I, (1,)), V(J.I, (2,)), V(J.I, (3, 1)), V(J.F), V(J.F),
                                              V(J.F, (3,)), V(J.F), V(J.F, (3,)), V(J.F, (1, 3)), V(J.F, (3,)))
    jb, iv = V(J.I, (1,)), V(J.I, (3,))
    b = lambda s_, d_, shape=(1,): E("broadcast_in_dim", [s_], [d_], shape=shape, broadcast_dimensions=())
    eqns = [b(i, ib), b(j, jb),
            E("concatenate", [ib, jb], [ij], dimension=0),
            E("concatenate", [ib, jb, ib], [iv], dimension=0),
            E("reshape", [iv], [i3], new_sizes=(3, 1), dimensions=None),
            E("gather", [tab, ib], [g1], dimension_numbers=dn((), (0,), (0,)), slice_sizes=(1,), mode=PROM,
              fill_value=None, indices_are_sorted=False, unique_indices=False),
            E("gather", [tab, ib], [g2], dimension_numbers=dn((), (0,), (0,)), slice_sizes=(1,), mode=FILL,
              fill_value=None, indices_are_sorted=False, unique_indices=False),
            E("gather", [vec, i3], [g3], dimension_numbers=dn((), (0,), (0,)), slice_sizes=(1,), mode=PROM,
              fill_value=None, indices_are_sorted=False, unique_indices=False),
            E("gather", [tab2, ij], [g4], dimension_numbers=dn((), (0, 1), (0, 1)), slice_sizes=(1, 1), mode=PROM,
              fill_value=None, indices_are_sorted=False, unique_indices=False),
            E("gather", [tab2, ib], [g5], dimension_numbers=dn((0,), (0,), (0,)), slice_sizes=(1, 3), mode=PROM,
              fill_value=None, indices_are_sorted=False, unique_indices=False),
            E("dynamic_slice", [tab2, j, L(0, J.I)], [ds], slice_sizes=(1, 3)),
            E("reshape", [ds], [row], new_sizes=(3,), dimensions=None)]
    cj = J.ClosedJaxpr(J.Jaxpr([i, j, vec, tab, tab2], [g1, g2, g3, g4, g5, row], eqns))
    fn, specs = FJ.item_function(cj, [], 3)
    assert specs[3:] == [("table", "f32", (100,)), ("table", "f32", (8, 3))]
    tr = T.trace_item(fn, specs, 3, {})
    rng = np.random.default_rng(8)
    n = 60
    ii = rng.integers(-5, 110, n).astype(np.int32)
    jj = rng.integers(-2, 10, n).astype(np.int32)
    vv = rng.normal(size=(n, 4)).astype(np.float32)
    t1 = rng.normal(size=100).astype(np.float32)
    t2 = rng.normal(size=(8, 3)).astype(np.float32)
    res = [np.asarray(r) for r in Evaluator(tr, 1).run([ii, jj, vv], [t1, t2])["results"]]
    for q in range(n):
        c1 = int(np.clip(ii[q], 0, 99))
        want = [t1[c1], t1[ii[q]] if 0 <= ii[q] < 100 else np.nan]
        want += [vv[q, int(np.clip(z, 0, 3))] for z in (ii[q], jj[q], ii[q])]
        want += [t2[int(np.clip(ii[q], 0, 7)), int(np.clip(jj[q], 0, 2))]]
        want += list(t2[int(np.clip(ii[q], 0, 7))]) + list(t2[int(np.clip(jj[q], 0, 7))])
        got = [res[z][q] for z in range(len(want))]
        assert np.array_equal(np.float32(got), np.float32(want), equal_nan=True), q


def test_inner_while_in_a_jaxpr():
    """a while equation inside the item's loop body (jax writes an inner lax.while_loop as a nested while): an inner
    loop of the trace, as the same item written with lang, bitwise"""
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import lang as tl
    V, E, L = J.Var, J.Eqn, J.Literal
    x = V(J.F)
    # the stepping loop: (k, x) while k < 5; its body runs an inner loop (j, y) = while j < k: (j + 1, y * 0.5 + x)
    bk, bx, ij, cq, ij2, iy2, t0, jo, yo, bk2, bx2 = (V(J.I), V(J.F), V(J.I), V(J.B), V(J.I), V(J.F), V(J.F), V(J.I),
                                                      V(J.F), V(J.I), V(J.F))
    ck, cx, cc, ik = V(J.I), V(J.F), V(J.B), V(J.I)
    icond = J.ClosedJaxpr(J.Jaxpr([ik, ij, V(J.F)], [cq], [E("lt", [ij, ik], [cq])]))
    ibx = V(J.F)
    ibody = J.ClosedJaxpr(J.Jaxpr([ibx, ij2, iy2], [jo, yo], [E("add", [ij2, L(1, J.I)], [jo]),
                                                             E("mul", [iy2, L(0.5, J.F)], [t0]),
                                                             E("add", [t0, ibx], [yo])]))
    jf, yf = V(J.I), V(J.F)
    body = J.ClosedJaxpr(J.Jaxpr([bk, bx], [bk2, bx2], [
        E("while", [bk, bx, L(0, J.I), bx], [jf, yf], cond_jaxpr=icond, body_jaxpr=ibody, cond_nconsts=1,
          body_nconsts=1),
        E("add", [bk, L(1, J.I)], [bk2]),
        E("mul", [yf, L(0.75, J.F)], [bx2])]))
    cond = J.ClosedJaxpr(J.Jaxpr([ck, cx], [cc], [E("lt", [ck, L(5, J.I)], [cc])]))
    ko, xo = V(J.I), V(J.F)
    cj = J.ClosedJaxpr(J.Jaxpr([x], [ko, xo], [E("while", [L(0, J.I), x], [ko, xo], cond_jaxpr=cond, body_jaxpr=body,
                                                    cond_nconsts=0, body_nconsts=0)]))
    fn, specs = FJ.item_function(cj, [], 1)
    tr = T.trace_item(fn, specs, 1, {})
    assert [e.prim for e in tr.body].count("while") == 1

    def item(t, x):
        def body(c):
            k, x = c
            _, y = tl.while_loop(lambda d: d[0] < k, lambda d: (d[0] + 1, d[1] * 0.5 + x), (0, x))
            return k + 1, y * 0.75
        k, x = tl.while_loop(lambda c: c[0] < 5, body, (0, x))
        return t, k, x
    xs = np.random.default_rng(2).normal(size=32).astype(np.float32)
    r = Evaluator(tr, 10).run([xs], [])
    rq = Evaluator(T.trace_item(item, ["f32"], 1, {}), 10).run([xs], [])
    assert np.array_equal(np.asarray(r["results"][1]).view(np.uint32), np.asarray(rq["results"][1]).view(np.uint32))


def test_scatter_primitives():
    """x.at[i].set / add / multiply / max into a vector (lax.scatter and its combining forms): static and traced
    indices, an out-of-range index dropped (fill_or_drop, jax's default) or clamped (clip); the IR evaluator's values
    equal numpy's in update order"""
    from types import SimpleNamespace as NS
    from oracle.ir_eval import Evaluator
    V, E, L = J.Var, J.Eqn, J.Literal
    dn = NS(update_window_dims=(), inserted_window_dims=(0,), scatter_dims_to_operand_dims=(0,),
            operand_batching_dims=(), scatter_indices_batching_dims=())
    DROP, CLIP = "GatherScatterMode.FILL_OR_DROP", "GatherScatterMode.CLIP"
    x, y, i = V(J.F, (4,)), V(J.F), V(J.I)
    ib, s1, s2, s3, s4, s5 = V(J.I, (1,)), V(J.F, (4,)), V(J.F, (4,)), V(J.F, (4,)), V(J.F, (4,)), V(J.F, (4,))
    sc = lambda p_, ins, out, mode: E(p_, ins, [out], dimension_numbers=dn, indices_are_sorted=True,
                                      unique_indices=True, mode=mode, update_jaxpr=None, update_consts=())
    eqns = [E("broadcast_in_dim", [i], [ib], shape=(1,), broadcast_dimensions=()),
            sc("scatter", [x, ib, y], s1, DROP),
            sc("scatter-add", [x, ib, y], s2, CLIP),
            sc("scatter-mul", [x, L(np.array([2], np.int32), J.I), y], s3, DROP),
            sc("scatter-max", [x, ib, y], s4, DROP),
            sc("scatter-add", [x, L(np.array([7], np.int32), J.I), y], s5, DROP)]
    cj = J.ClosedJaxpr(J.Jaxpr([x, y, i], [s1, s2, s3, s4, s5], eqns))
    fn, specs = FJ.item_function(cj, [], 3)
    tr = T.trace_item(fn, specs, 3, {})
    n = 30
    rng = np.random.default_rng(3)
    xs = rng.normal(size=(n, 4)).astype(np.float32)
    ys = rng.normal(size=n).astype(np.float32)
    ii = rng.integers(-2, 6, n).astype(np.int32)
    res = [np.asarray(r) for r in Evaluator(tr, 1).run([xs, ys, ii], [])["results"]]
    for q in range(n):
        x0, v, k = xs[q], ys[q], int(ii[q])
        want = []
        a = x0.copy()
        if 0 <= k < 4:
            a[k] = v
        want.append(a)
        a = x0.copy()
        a[int(np.clip(k, 0, 3))] += v
        want.append(a)
        a = x0.copy()
        a[2] *= v
        want.append(a)
        a = x0.copy()
        if 0 <= k < 4:
            a[k] = np.maximum(a[k], v)
        want.append(a)
        want.append(x0.copy())
        got = np.float32([res[j][q] for j in range(20)]).reshape(5, 4)
        assert np.array_equal(got, np.float32(want)), q


def test_split_and_reduce_prod():
    """lax.split of a vector into pieces and reduce_prod: the pieces' sums and products as numpy float32 gives them
    (products left to right)"""
    from oracle.ir_eval import Evaluator
    V, E = J.Var, J.Eqn
    v, p1, p2, s1, r2 = V(J.F, (5,)), V(J.F, (2,)), V(J.F, (3,)), V(J.F), V(J.F)
    eqns = [E("split", [v], [p1, p2], sizes=(2, 3), axis=0),
            E("reduce_sum", [p1], [s1], axes=(0,)),
            E("reduce_prod", [p2], [r2], axes=(0,))]
    cj = J.ClosedJaxpr(J.Jaxpr([v], [s1, r2], eqns))
    fn, specs = FJ.item_function(cj, [], 1)
    tr = T.trace_item(fn, specs, 1, {})
    vs = np.random.default_rng(2).normal(size=(20, 5)).astype(np.float32)
    r = Evaluator(tr, 1).run([vs], [])["results"]
    f = np.float32
    assert np.array_equal(np.float32(r[0]), (vs[:, 0] + vs[:, 1]).astype(np.float32))
    assert np.array_equal(np.float32(r[1]), ((vs[:, 2] * vs[:, 3]).astype(f) * vs[:, 4]).astype(f))


def test_unlowered_primitive_raises():
    x, y = J.Var(J.F), J.Var(J.F)
    cj = J.ClosedJaxpr(J.Jaxpr([x], [y], [J.Eqn("fft", [x], [y])]))
    fn, specs = FJ.item_function(cj, [], 1)
    with pytest.raises(T.UnsupportedError, match="'fft' is not lowered"):
        T.trace_item(fn, specs, 1, {})
    # a value of two dimensions (or an axis operation on a (k, 1) array) would be read in the wrong order: refused
    a, b, c = J.Var(J.F, (3, 1)), J.Var(J.F, (3, 1)), J.Var(J.F, (3, 2))
    for eq in (J.Eqn("concatenate", [a, b], [c], dimension=1), J.Eqn("cumsum", [a], [b], axis=1, reverse=False)):
        with pytest.raises(T.UnsupportedError, match="shape"):
            FJ._Interp(None).apply(eq, [T.Vec([1.0, 2.0, 3.0]), T.Vec([1.0, 2.0, 3.0])][:len(eq.invars)])
    # a key of another PRNG implementation would give other bits: refused, as a typed input and at random_wrap
    with pytest.raises(T.UnsupportedError, match="threefry2x32 only"):
        FJ.item_function(J.ClosedJaxpr(J.Jaxpr([J.Var("key<rbg>")], [], [])), [], 1)
    q, k = J.Var(J.U, (2,)), J.Var("key<rbg>")
    cj = J.ClosedJaxpr(J.Jaxpr([q], [], [J.Eqn("random_wrap", [q], [k], impl="rbg")]))
    fn, specs = FJ.item_function(cj, [], 1)
    with pytest.raises(T.UnsupportedError, match="threefry2x32 only"):
        T.trace_item(fn, specs, 1, {})
