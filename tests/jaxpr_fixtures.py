"""Duck-typed jaxprs for the jaxpr front end's tests (JAX is not installed here): objects with the attributes
tallymap_b200.from_jaxpr reads -- eqn.primitive.name / .params / .invars / .outvars, var.aval.shape / .dtype,
literal.val, jaxpr.invars / .outvars / .eqns / .constvars, closed.jaxpr / .consts -- spelled the way jax.make_jaxpr
writes the reference's quickstart item (examples/quickstart.py:19-30) under jax 0.6-0.8:

    def walker(t, x, key, theta):
        def body(c):
            k, x, t = c
            u = jax.random.uniform(jax.random.fold_in(key, k))
            t = t.add("hist", (x * NB).astype(jnp.int32), theta * (1.0 - x))
            return k + 1, x * (0.5 + 0.5 * u), t
        k, x, t = lax.while_loop(lambda c: c[1] > 0.05, body, (0, x, t))
        return t, k

with jax.random.split(PRNGKey(0), N)'s raw uint32[2] keys (fold_in and uniform wrap them with random_wrap and unwrap
the result; uniform is a pjit of random_bits and the mantissa fill), the item's tally leaf first (ItemProgram.cj's
invars: [tallies] + [per-item] + [broadcast]), and its retrace(cap=max_steps) form (the loop counter in the carry,
`truncated` as a second per-item result: tallymap/_rewrite.py:251, 502-528)."""
import itertools

import numpy as np

_ids = itertools.count()


class Aval:
    def __init__(self, shape, dtype):
        self.shape, self.dtype = tuple(shape), dtype

    def __repr__(self):
        return f"{self.dtype}{list(self.shape)}"


class Var:
    def __init__(self, dtype, shape=()):
        self.aval = Aval(shape, dtype)
        self.n = next(_ids)


class Literal:
    def __init__(self, val, dtype):
        self.val = val
        self.aval = Aval((), dtype)


class Primitive:
    def __init__(self, name):
        self.name = name


class Eqn:
    def __init__(self, prim, invars, outvars, **params):
        self.primitive, self.invars, self.outvars, self.params = Primitive(prim), invars, outvars, params


class Jaxpr:
    def __init__(self, invars, outvars, eqns, constvars=()):
        self.invars, self.outvars, self.eqns, self.constvars = invars, outvars, eqns, list(constvars)


class ClosedJaxpr:
    def __init__(self, jaxpr, consts=()):
        self.jaxpr, self.consts = jaxpr, list(consts)


F, I, U, B, KEY = "float32", "int32", "uint32", "bool", "key<fry>"


def uniform_pjit():
    """jax.random.uniform(key, (), f32, 0, 1) as the pjit jax.random.uniform binds: random_wrap, random_bits, the
    mantissa fill, then max(lo, f * (hi - lo) + lo)"""
    q, r, s = Var(U, (2,)), Var(F), Var(F)
    t, u, v, w, x, y, z, ba, bb, bc, bd = (Var(KEY), Var(U), Var(U), Var(U), Var(F), Var(F), Var(F), Var(F), Var(F),
                                           Var(F), Var(F))
    eqns = [Eqn("random_wrap", [q], [t], impl="fry"),
            Eqn("random_bits", [t], [u], bit_width=32, shape=()),
            Eqn("shift_right_logical", [u, Literal(9, U)], [v]),
            Eqn("or", [v, Literal(1065353216, U)], [w]),
            Eqn("bitcast_convert_type", [w], [x], new_dtype="float32"),
            Eqn("sub", [x, Literal(1.0, F)], [y]),
            Eqn("sub", [s, r], [z]),
            Eqn("mul", [y, z], [ba]),
            Eqn("add", [ba, r], [bb]),
            Eqn("reshape", [bb], [bc], new_sizes=(), dimensions=None),
            Eqn("max", [r, bc], [bd])]
    return ClosedJaxpr(Jaxpr([q, r, s], [bd], eqns))


def _gated_emit(bx, gate, bh, bf, bh2, bi):
    """`t = lax.cond(x > gate, lambda t: t.add("hist", bin, v), lambda t: t, t)` as jax writes it: the predicate
    converted to an int32 branch index, the branches (false first) taking the closed-over bin and value and the
    tally, the false branch returning its tally operand"""
    cp, ci = Var(B), Var(I)
    fi, fv, fh = Var(I), Var(F), Var(F, (16,))
    ti, tv, th, to = Var(I), Var(F), Var(F, (16,)), Var(F, (16,))
    false_b = ClosedJaxpr(Jaxpr([fi, fv, fh], [fh], []))
    true_b = ClosedJaxpr(Jaxpr([ti, tv, th], [to], [Eqn("tallymap_emit", [th, ti, tv], [to])]))
    return [Eqn("gt", [bx, Literal(gate, F)], [cp]),
            Eqn("convert_element_type", [cp], [ci], new_dtype="int32", weak_type=False),
            Eqn("cond", [ci, bf, bh2, bh], [bi], branches=(false_b, true_b))]


def quickstart(cap=None, gate=None):
    """the quickstart item's closed jaxpr; cap: retrace(cap=max_steps)'s form (loop counter + truncated result);
    gate: the emit inside a lax.cond branch, made only on steps that start above x = gate"""
    hist, x0, key, theta = Var(F, (16,)), Var(F), Var(U, (2,)), Var(F)
    # body: consts (key, theta), carry ([cnt,] k, x, hist)
    bkey, btheta = Var(U, (2,)), Var(F)
    bcnt, bk, bx, bh = Var(I), Var(I), Var(F), Var(F, (16,))
    m, ku, n, o, p = Var(KEY), Var(U), Var(KEY), Var(U, (2,)), Var(F)
    be, bf, bg, bh2, bi, bj, bk2, bl, bm, bcnt2 = (Var(F), Var(I), Var(F), Var(F), Var(F, (16,)), Var(I), Var(F),
                                                   Var(F), Var(F), Var(I))
    body_eqns = [Eqn("random_wrap", [bkey], [m], impl="fry"),
                 Eqn("convert_element_type", [bk], [ku], new_dtype="uint32", weak_type=False),
                 Eqn("random_fold_in", [m, ku], [n]),
                 Eqn("random_unwrap", [n], [o]),
                 Eqn("pjit", [o, Literal(0.0, F), Literal(1.0, F)], [p], jaxpr=uniform_pjit(), name="_uniform"),
                 Eqn("mul", [bx, Literal(16.0, F)], [be]),
                 Eqn("convert_element_type", [be], [bf], new_dtype="int32", weak_type=False),
                 Eqn("sub", [Literal(1.0, F), bx], [bg]),
                 Eqn("mul", [btheta, bg], [bh2]),
                 *([Eqn("tallymap_emit", [bh, bf, bh2], [bi])] if gate is None else
                   _gated_emit(bx, gate, bh, bf, bh2, bi)),
                 Eqn("add", [bk, Literal(1, I)], [bj]),
                 Eqn("mul", [Literal(0.5, F), p], [bk2]),
                 Eqn("add", [Literal(0.5, F), bk2], [bl]),
                 Eqn("mul", [bx, bl], [bm])]
    carry_in = [bk, bx, bh]
    carry_out = [bj, bm, bi]
    if cap is not None:
        body_eqns.append(Eqn("add", [bcnt, Literal(1, I)], [bcnt2]))
        carry_in, carry_out = [bcnt] + carry_in, [bcnt2] + carry_out
    body = ClosedJaxpr(Jaxpr([bkey, btheta] + carry_in, carry_out, body_eqns))
    ccnt, ck, cx, ch, cq = Var(I), Var(I), Var(F), Var(F, (16,)), Var(B)
    if cap is None:
        cond = ClosedJaxpr(Jaxpr([ck, cx, ch], [cq], [Eqn("gt", [cx, Literal(0.05, F)], [cq])]))
    else:
        c1, c2 = Var(B), Var(B)
        cond = ClosedJaxpr(Jaxpr([ccnt, ck, cx, ch], [cq], [Eqn("lt", [ccnt, Literal(cap, I)], [c1]),
                                                             Eqn("gt", [cx, Literal(0.05, F)], [c2]),
                                                             Eqn("and", [c1, c2], [cq])]))
    ok, ox, oh, ocnt = Var(I), Var(F), Var(F, (16,)), Var(I)
    outs = ([ocnt] if cap is not None else []) + [ok, ox, oh]
    init = ([Literal(0, I)] if cap is not None else []) + [Literal(0, I), x0, hist]
    eqns = [Eqn("while", [key, theta] + init, outs, cond_jaxpr=cond, body_jaxpr=body, cond_nconsts=0,
                body_nconsts=2)]
    results = [ok]
    if cap is not None:                       # truncated = the loop ran out of steps with its predicate still true
        t1, t2, tr = Var(B), Var(B), Var(B)
        eqns += [Eqn("ge", [ocnt, Literal(cap, I)], [t1]), Eqn("gt", [ox, Literal(0.05, F)], [t2]),
                 Eqn("and", [t1, t2], [tr])]
        results.append(tr)
    return ClosedJaxpr(Jaxpr([hist, x0, key, theta], [oh] + results, eqns))


def scans():
    """a loop-free item with jax's two spellings of a static loop:

        def item(t, x, key, theta):
            c = lax.fori_loop(0, 3, lambda i, c: c * 0.5 + i, x)          # a scan carrying (i, c)
            cs, ys = lax.scan(lambda c, z: (c + z * theta, c * z), 0.0, jnp.array([1.0, 2.0, 3.0]))
            t = t.add("hist", 0, c).add("hist", 1, cs).add("hist", 2, ys[2])
            return t, c
    """
    hist, x0, key, theta = Var(F, (16,)), Var(F), Var(U, (2,)), Var(F)
    bi, bc, bi1, m, bf, bc1 = Var(I), Var(F), Var(I), Var(F), Var(F), Var(F)
    b1 = ClosedJaxpr(Jaxpr([bi, bc], [bi1, bc1], [
        Eqn("add", [bi, Literal(1, I)], [bi1]),
        Eqn("mul", [bc, Literal(0.5, F)], [m]),
        Eqn("convert_element_type", [bi], [bf], new_dtype="float32", weak_type=False),
        Eqn("add", [m, bf], [bc1])]))
    th, c, z, zt, c1, y = Var(F), Var(F), Var(F), Var(F), Var(F), Var(F)
    b2 = ClosedJaxpr(Jaxpr([th, c, z], [c1, y], [
        Eqn("mul", [z, th], [zt]),
        Eqn("add", [c, zt], [c1]),
        Eqn("mul", [c, z], [y])]))
    i3, c3, cs, ys, y2s, y2, h1, h2, h3 = (Var(I), Var(F), Var(F), Var(F, (3,)), Var(F, (1,)), Var(F),
                                           Var(F, (16,)), Var(F, (16,)), Var(F, (16,)))
    zs = Literal(np.array([1.0, 2.0, 3.0], np.float32), F)
    zs.aval = Aval((3,), F)
    eqns = [Eqn("scan", [Literal(0, I), x0], [i3, c3], jaxpr=b1, length=3, reverse=False, num_consts=0,
                num_carry=2, linear=(False, False), unroll=1),
            Eqn("scan", [theta, Literal(0.0, F), zs], [cs, ys], jaxpr=b2, length=3, reverse=False, num_consts=1,
                num_carry=1, linear=(False, False, False), unroll=1),
            Eqn("slice", [ys], [y2s], start_indices=(2,), limit_indices=(3,), strides=None),
            Eqn("squeeze", [y2s], [y2], dimensions=(0,)),
            Eqn("tallymap_emit", [hist, Literal(0, I), c3], [h1]),
            Eqn("tallymap_emit", [h1, Literal(1, I), cs], [h2]),
            Eqn("tallymap_emit", [h2, Literal(2, I), y2], [h3])]
    return ClosedJaxpr(Jaxpr([hist, x0, key, theta], [h3, c3], eqns))


RSEP = "\x1f"


def quickstart_records(C=4096):
    """the quickstart walker with a Records output in the reference's ONE-PASS form (tallymap/_tally.py:302-351,
    _api.py:727-733): each step that starts in bin 3 appends {"x": x}.  The item's tallies are hist, then the record
    field tally 'hits\x1fx' and the key tallies 'hits\x1fi' (the item's node id) and 'hits\x1fk' (its ordinal),
    each of the capacity C; the per-item operands end with the hidden node id (arange(N)); the append ordinal rides
    in the carry and is the second per-item result (the item's count).  Per append:

        tok, slot = tallymap_claim(t['hits\x1fk'], w, k, r=0)
        ok = w & (slot >= 0) & (slot < C)
        (hx, hi, hk) = lax.cond(ok, put1, lambda ts: ts, (t['hits\x1fx'], t['hits\x1fi'], tok))
        k = k + w
    """
    hist, hx, hki, hkk = Var(F, (16,)), Var(F, (C,)), Var(I, (C,)), Var(I, (C,))
    x0, key, cid, theta = Var(F), Var(U, (2,)), Var(I), Var(F)
    bkey, btheta, bcid = Var(U, (2,)), Var(F), Var(I)
    bk, bx, bh, bhx, bhi, bhk, bkr = Var(I), Var(F), Var(F, (16,)), Var(F, (C,)), Var(I, (C,)), Var(I, (C,)), Var(I)
    m, ku, n, o, p = Var(KEY), Var(U), Var(KEY), Var(U, (2,)), Var(F)
    be, bf, bg, bh2, bi, bj, bk2, bl, bm = Var(F), Var(I), Var(F), Var(F), Var(F, (16,)), Var(I), Var(F), Var(F), Var(F)
    w, tk, slot, s0, s1, ok0, ok, oi = Var(B), Var(I, (C,)), Var(I), Var(B), Var(B), Var(B), Var(B), Var(I)
    hx2, hi2, hk2, wi, kr2 = Var(F, (C,)), Var(I, (C,)), Var(I, (C,)), Var(I), Var(I)
    # the branches: (slot, x, cid, k, field tally, key tallies) -> the three tallies
    ids = [Var(I), Var(F), Var(I), Var(I), Var(F, (C,)), Var(I, (C,)), Var(I, (C,))]
    put = [Var(I), Var(F), Var(I), Var(I), Var(F, (C,)), Var(I, (C,)), Var(I, (C,))]
    pa, pb, pc = Var(F, (C,)), Var(I, (C,)), Var(I, (C,))
    identity = ClosedJaxpr(Jaxpr(ids, ids[4:], []))
    put1 = ClosedJaxpr(Jaxpr(put, [pa, pb, pc], [Eqn("tallymap_emit", [put[4], put[0], put[1]], [pa]),
                                                 Eqn("tallymap_emit", [put[5], put[0], put[2]], [pb]),
                                                 Eqn("tallymap_emit", [put[6], put[0], put[3]], [pc])]))
    body_eqns = [Eqn("random_wrap", [bkey], [m], impl="fry"),
                 Eqn("convert_element_type", [bk], [ku], new_dtype="uint32", weak_type=False),
                 Eqn("random_fold_in", [m, ku], [n]),
                 Eqn("random_unwrap", [n], [o]),
                 Eqn("pjit", [o, Literal(0.0, F), Literal(1.0, F)], [p], jaxpr=uniform_pjit(), name="_uniform"),
                 Eqn("mul", [bx, Literal(16.0, F)], [be]),
                 Eqn("convert_element_type", [be], [bf], new_dtype="int32", weak_type=False),
                 Eqn("sub", [Literal(1.0, F), bx], [bg]),
                 Eqn("mul", [btheta, bg], [bh2]),
                 Eqn("tallymap_emit", [bh, bf, bh2], [bi]),
                 Eqn("eq", [bf, Literal(3, I)], [w]),
                 Eqn("tallymap_claim", [bhk, w, bkr], [tk, slot], r=0),
                 Eqn("ge", [slot, Literal(0, I)], [s0]),
                 Eqn("lt", [slot, Literal(C, I)], [s1]),
                 Eqn("and", [w, s0], [ok0]),
                 Eqn("and", [ok0, s1], [ok]),
                 Eqn("convert_element_type", [ok], [oi], new_dtype="int32", weak_type=False),
                 Eqn("cond", [oi, slot, bx, bcid, bkr, bhx, bhi, tk], [hx2, hi2, hk2], branches=(identity, put1)),
                 Eqn("convert_element_type", [w], [wi], new_dtype="int32", weak_type=False),
                 Eqn("add", [bkr, wi], [kr2]),
                 Eqn("add", [bk, Literal(1, I)], [bj]),
                 Eqn("mul", [Literal(0.5, F), p], [bk2]),
                 Eqn("add", [Literal(0.5, F), bk2], [bl]),
                 Eqn("mul", [bx, bl], [bm])]
    body = ClosedJaxpr(Jaxpr([bkey, btheta, bcid, bk, bx, bh, bhx, bhi, bhk, bkr],
                             [bj, bm, bi, hx2, hi2, hk2, kr2], body_eqns))
    ck, cx, ch, chx, chi, chk, ckr, cq = (Var(I), Var(F), Var(F, (16,)), Var(F, (C,)), Var(I, (C,)), Var(I, (C,)),
                                          Var(I), Var(B))
    cond = ClosedJaxpr(Jaxpr([ck, cx, ch, chx, chi, chk, ckr], [cq], [Eqn("gt", [cx, Literal(0.05, F)], [cq])]))
    ok_, ox, oh, ohx, ohi, ohk, okr = Var(I), Var(F), Var(F, (16,)), Var(F, (C,)), Var(I, (C,)), Var(I, (C,)), Var(I)
    eqns = [Eqn("while", [key, theta, cid, Literal(0, I), x0, hist, hx, hki, hkk, Literal(0, I)],
                [ok_, ox, oh, ohx, ohi, ohk, okr], cond_jaxpr=cond, body_jaxpr=body, cond_nconsts=0, body_nconsts=3)]
    return ClosedJaxpr(Jaxpr([hist, hx, hki, hkk, x0, key, cid, theta], [oh, ohx, ohi, ohk, ok_, okr], eqns))


class TSpec:
    """the reference's TSpec, as ItemProgram.tallies holds them (tallymap/_api.py:204-220)"""

    def __init__(self, name, size, dtype="float32", kind="sum"):
        self.name, self.size, self.dtype, self.kind = name, size, np.dtype(dtype), kind
        self.shape = (size,)


class ItemProgram:
    """the fields of the reference's ItemProgram (tallymap/_api.py:231-281) the backend entry reads"""

    def __init__(self, cj, tallies, nP, nB, trunc=None, spawn=None):
        self.cj, self.tallies, self.nP, self.nB, self.trunc, self.spawn = cj, tuple(tallies), nP, nB, trunc, spawn
        self.tag = "primal"


def records_program(C=4096):
    """the one-pass Records quickstart as the reference's backend entry receives it (no retrace cap: the loop ends on
    its own)"""
    return ItemProgram(quickstart_records(C), [TSpec("hist", 16), TSpec("hits" + RSEP + "x", C),
                                               TSpec("hits" + RSEP + "i", C, "int32"),
                                               TSpec("hits" + RSEP + "k", C, "int32")], nP=3, nB=1)


def quickstart_program(cap=100):
    return ItemProgram(quickstart(cap), [TSpec("hist", 16)], nP=2, nB=1, trunc=1)
