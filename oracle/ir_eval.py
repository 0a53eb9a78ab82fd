"""TEST INFRASTRUCTURE (not product code): a CPU evaluator of traced items -- the scalar IR of tallymap_b200.trace --
used as the oracle of the run-time lowering (tallymap_b200/lower.py).  Only tests/ may use it.

It runs each item's equations one at a time with the IR's semantics, which the lowering must reproduce on the
device:
  * f32 arithmetic in numpy float32 (one IEEE rounding per operation, no FMA); int32 wrapping, uint32 modulo 2^32;
  * log / exp / sin / cos / pow: the backend's shared f32 math through the oracle library (oracle.math);
  * f32 -> int32 conversion toward zero, saturating, NaN -> 0 (the reference's _rz conversions,
    backends/kernel/host.py:133-146); lax.max / lax.min (NaN wins, max(-0, +0) = +0);
  * jax.random: threefry2x32 (tallymap_b200.prng), fold_in = threefry(key, (0, m)), bits[i] = o0 ^ o1 of
    threefry(key, (0, i)), uniform = the mantissa fill;
  * the loop: while kc < max_steps and pred (retrace(cap), tallymap/_rewrite.py:517-528), truncated iff the cap
    stopped it;
  * emits: an index outside the output is dropped and counted in stats[4]; an emit with a third operand (a write in
    a lax.cond branch) only where that predicate holds; f32 Sums accumulate in f64 (the checker mode: compare within
    the float-tally tolerance), int32 Sums exactly, fixed_point f32 Sums through the oracle's exact accumulator
    (oracle.exact_sum, pinned to the golden known answers: compare bitwise), scaled fixed-point Sums (wide=) as exact
    Python integers;
  * an inner while loop (a "while" equation): its condition and body until the condition fails;
  * a Records slot claim of a reference jaxpr ("claim"): the next slot of a per-launch counter in item order, -1 when
    not `when` or past the capacity;
  * Records: each item's records in append order, items in item order (the canonical layout);
  * spawn (tallymap/_tally.py:284-302): a spawned child runs the same item from its leaves with the same broadcast
    operands, after the roots, first in first out (no queue limit); its per-item results are discarded, its
    truncation counts in stats[2], every spawn in stats[0].
"""
import math

import numpy as np

from tallymap_b200 import prng
from tallymap_b200 import trace as T

from . import oracle as orc

F32 = np.float32
_MATH = {p: p for p in ("log", "exp", "sin", "cos", "atan", "asin", "acos", "tan", "sinh", "cosh", "asinh", "acosh",
                         "atanh", "exp2", "log2", "cbrt", "erf", "erfc", "erfinv", "lgamma")}


def _wrap32(v):
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


def _f2i(x):
    x = float(x)
    if x != x:
        return 0
    if x >= 2147483648.0:
        return 2147483647
    if x <= -2147483648.0:
        return -2147483648
    return int(math.trunc(x))


def _f2u(x):
    x = float(x)
    if x != x or x <= 0.0:
        return 0
    if x >= 4294967296.0:
        return 4294967295
    return int(math.trunc(x))


def _jmax(a, b):
    if a > b or a != a:
        return a
    if b > a or b != b:
        return b
    return F32(a + b) if a == 0 else a


def _jmin(a, b):
    if a < b or a != a:
        return a
    if b < a or b != b:
        return b
    return F32(-(F32(-a) + F32(-b))) if a == 0 else a


def _unit(bits):
    return F32(np.array([(bits >> 9) | 0x3F800000], np.uint32).view(np.float32)[0] - F32(1.0))


def _tf(k0, k1, c0, c1):
    o0, o1 = prng.threefry2x32(np.uint32(k0), np.uint32(k1), np.uint32(c0), np.uint32(c1))
    return int(o0), int(o1)


def _floordiv(a, b, dt):
    if b == 0:
        return 0
    if dt == T.U32:
        return a // b
    if b == -1:
        return _wrap32(-a)
    q = abs(a) // abs(b)
    q = q if (a < 0) == (b < 0) else -q
    return q - 1 if q * b != a and ((a < 0) != (b < 0)) else q


def _floormod(a, b, dt):
    if b == 0 or (dt != T.U32 and b == -1):
        return 0
    if dt == T.U32:
        return a % b
    r = int(math.fmod(a, b))
    return r + b if r != 0 and ((r < 0) != (b < 0)) else r


def _convert(v, src, dst):
    if src == T.F32:
        return {T.I32: _f2i(v), T.U32: _f2u(v), T.BOOL: bool(v != 0)}[dst]
    if src == T.I32:
        return {T.F32: F32(v), T.U32: v & 0xFFFFFFFF, T.BOOL: v != 0}[dst]
    if src == T.U32:
        return {T.F32: F32(v), T.I32: _wrap32(v), T.BOOL: v != 0}[dst]
    return {T.F32: F32(1.0) if v else F32(0.0), T.I32: int(v), T.U32: int(v)}[dst]


def _eval(e, a):
    """-> the output value(s) of equation e for input values a"""
    p, d = e.prim, e.ins[0].dtype if e.ins else None
    if p in ("add", "sub", "mul"):
        if d == T.F32:
            with np.errstate(all="ignore"):
                return {"add": a[0] + a[1], "sub": a[0] - a[1], "mul": a[0] * a[1]}[p]
        r = {"add": a[0] + a[1], "sub": a[0] - a[1], "mul": a[0] * a[1]}[p]
        return _wrap32(r) if d == T.I32 else r & 0xFFFFFFFF
    if p == "div":
        with np.errstate(all="ignore"):
            return F32(a[0] / a[1])
    if p in ("lt", "le", "gt", "ge", "eq", "ne"):
        return {"lt": a[0] < a[1], "le": a[0] <= a[1], "gt": a[0] > a[1], "ge": a[0] >= a[1], "eq": a[0] == a[1],
                "ne": a[0] != a[1]}[p]
    if p == "idiv":
        return _floordiv(a[0], a[1], d)
    if p == "irem":
        return _floormod(a[0], a[1], d)
    if p == "neg":
        return F32(-a[0]) if d == T.F32 else (_wrap32(-a[0]) if d == T.I32 else (-a[0]) & 0xFFFFFFFF)
    if p in ("and", "or", "xor"):
        if d == T.BOOL:
            return {"and": a[0] and a[1], "or": a[0] or a[1], "xor": a[0] != a[1]}[p]
        r = {"and": a[0] & a[1], "or": a[0] | a[1], "xor": a[0] ^ a[1]}[p]
        return _wrap32(r) if d == T.I32 else r & 0xFFFFFFFF
    if p == "not":
        return (not a[0]) if d == T.BOOL else (_wrap32(~a[0]) if d == T.I32 else (~a[0]) & 0xFFFFFFFF)
    if p == "popc":
        return bin(int(a[0]) & 0xFFFFFFFF).count("1")
    if p == "clz":
        return 32 - (int(a[0]) & 0xFFFFFFFF).bit_length()
    if p == "shl":
        sh = a[1] & 0xFFFFFFFF
        return 0 if sh >= 32 else (_wrap32(a[0] << sh) if d == T.I32 else (a[0] << sh) & 0xFFFFFFFF)
    if p == "shr":
        sh = a[1] & 0xFFFFFFFF
        if d == T.U32:
            return 0 if sh >= 32 else a[0] >> sh
        return (-1 if a[0] < 0 else 0) if sh >= 32 else a[0] >> sh
    if p in _MATH:
        return F32(orc.math(_MATH[p], np.array([a[0]], np.float32))[0])
    if p in ("pow", "atan2", "nextafter"):
        return F32(orc.math(p, np.array([a[0]], np.float32), np.array([a[1]], np.float32))[0])
    if p == "sqrt":
        with np.errstate(all="ignore"):
            return F32(np.sqrt(F32(a[0])))
    if p == "floor":
        return F32(np.floor(a[0]))
    if p == "round":
        return F32(np.rint(F32(a[0])))
    if p == "rem":
        with np.errstate(all="ignore"):
            return F32(np.fmod(F32(a[0]), F32(a[1])))
    if p == "stop":
        return a[0]
    if p == "abs":
        return F32(abs(a[0])) if d == T.F32 else _wrap32(abs(a[0]))
    if p == "max":
        return _jmax(a[0], a[1]) if d == T.F32 else max(a[0], a[1])
    if p == "min":
        return _jmin(a[0], a[1]) if d == T.F32 else min(a[0], a[1])
    if p == "select":
        return a[1] if a[0] else a[2]
    if p == "inrange":
        return 0 <= a[0] < e.params["n"]
    if p == "gather":       # a broadcast table's element (the index is clamped into range by the tracer)
        v = a[0][a[1]]
        return F32(v) if e.outs[0].dtype == T.F32 else int(v)
    if p == "convert":
        return _convert(a[0], d, e.outs[0].dtype)
    if p == "bitcast":
        src, dst = d, e.outs[0].dtype
        if src == T.F32:
            u = int(np.float32(a[0]).view(np.uint32))
        else:
            u = int(a[0]) & 0xFFFFFFFF
        if dst == T.F32:
            return np.uint32(u).view(np.float32)
        return _wrap32(u) if dst == T.I32 else u
    if p == "threefry":
        return _tf(*a)
    if p == "bits":
        o0, o1 = _tf(a[0], a[1], 0, a[2])
        return o0 ^ o1
    if p == "uniform01":
        o0, o1 = _tf(a[0], a[1], 0, a[2])
        return _unit(o0 ^ o1)
    raise NotImplementedError(p)


def _lit(x):
    if x.dtype == T.F32:
        return F32(x.value)
    if x.dtype == T.BOOL:
        return bool(x.value)
    return int(x.value)


class Evaluator:
    """evaluate traced item `tr` over items: run(per_item operands, broadcast values) -> dict of outputs"""

    def __init__(self, tr, max_steps, exact=(), max_items=10 ** 7, wide=None):
        """wide: {output: (dtype "f64" | "i32" | "i64", scale)} -- the scaled fixed-point Sums (tallymap/_api.py:55-84),
        kept as exact Python integers sum(round(v * scale)) and read out as float(total) / scale, float(int) being
        the correctly rounded double of the exact total, then the output's type (toward zero for an integer)"""
        self.tr, self.M, self.exact, self.max_items = tr, int(max_steps), set(exact), max_items
        self.wide = dict(wide or {})

    def _val(self, x, env):
        return env[x.id] if isinstance(x, T.Var) else _lit(x)

    def _run_eqns(self, eqns, env, out):
        for e in eqns:
            a = [self._val(x, env) for x in e.ins]
            if e.prim == "while":                  # (an inner loop: its condition and body until the condition fails)
                prm = e.params
                vals = a
                while True:
                    for cv, v in zip(prm["carry"], vals):
                        env[cv.id] = v
                    self._run_eqns(prm["cond"], env, out)
                    if not bool(self._val(prm["cond_out"], env)):
                        break
                    self._run_eqns(prm["body"], env, out)
                    vals = [self._val(x, env) for x in prm["body_out"]]
                for o, v in zip(e.outs, vals):
                    env[o.id] = v
                continue
            if e.prim == "claim":                  # (a Records slot claim: the launch's counter, in item order)
                nm, c = e.params["tally"], self._claims.get(e.params["tally"], 0)
                if a[0]:
                    self._claims[nm] = c + 1
                env[e.outs[0].id] = np.int32(c if a[0] and c < e.params["capacity"] else -1)
                continue
            if e.prim == "emit":
                if len(a) < 3 or a[2]:              # (a third operand: the predicate of a write in a cond branch)
                    out["emits"].append((e.params["tally"], a[0], a[1]))
                continue
            if e.prim == "append":
                if a[0]:
                    out["appends"].append((e.params["records"], tuple(a[1:])))
                continue
            if e.prim == "spawn":
                if a[0]:
                    out["spawns"].append(tuple(a[1:]))
                continue
            r = _eval(e, a)
            if len(e.outs) == 1:
                env[e.outs[0].id] = r
            else:
                for o, v in zip(e.outs, r):
                    env[o.id] = v

    def run(self, per_item, bc):
        tr = self.tr
        self._claims = {}
        n = len(per_item[0]) if per_item else 0
        specs = tr.specs
        sums = {}
        exact_pairs = {nm: ([], []) for nm in self.exact}
        wide_tot = {nm: [0] * (int(np.prod(specs[nm][0])) if specs[nm][0] else 1) for nm in self.wide}
        wide_flag = {nm: [False] * len(wide_tot[nm]) for nm in self.wide}
        for nm, (shape, dt) in specs.items():
            S = int(np.prod(shape)) if shape else 1
            sums[nm] = np.zeros(S, np.float64 if dt == T.F32 else np.int64)
        records = {nm: [] for nm in tr.records}
        counts = {nm: np.zeros(n, np.int32) for nm in tr.records}
        stats = np.zeros(5, np.int64)
        results = [np.zeros(n, np.int64 if (isinstance(y, T.Var) and y.dtype != T.F32) or
                            (isinstance(y, T.Lit) and y.dtype != T.F32) else np.float32) for y in tr.results]
        trunc = np.zeros(n, bool)
        leaves_of = []                    # the per-item input variables, flattened as a child carries them
        for x in tr.inputs[:tr.n_per_item]:
            leaves_of += [x.a, x.b] if isinstance(x, T.Key) else (list(x) if isinstance(x, tuple) else [x])
        work = []
        for i in range(n):
            env = {}
            for x, col in zip(tr.inputs[:tr.n_per_item], per_item):
                v = col[i]
                if isinstance(x, T.Key):
                    env[x.a.id], env[x.b.id] = int(np.uint32(v[0])), int(np.uint32(v[1]))
                elif isinstance(x, tuple):
                    for xj, vj in zip(x, v):
                        env[xj.id] = F32(vj) if xj.dtype == T.F32 else int(vj)
                else:
                    env[x.id] = F32(v) if x.dtype == T.F32 else int(v)
            work.append((i, env))
        w = 0
        while w < len(work):
            i, env = work[w]
            work[w] = None
            w += 1
            for x, v in zip(tr.inputs[tr.n_per_item:], bc):
                if isinstance(x, T.Table):
                    env[x.var.id] = np.asarray(v, np.float32 if x.dtype == T.F32 else np.int64).reshape(-1)
                else:
                    env[x.id] = F32(v) if x.dtype == T.F32 else int(v)
            out = {"emits": [], "appends": [], "spawns": []}
            self._run_eqns(tr.pre, env, out)
            carry = [self._val(x, env) for x in tr.carry_in]
            kc = 0

            def pred(c):
                for v, x in zip(tr.carry, c):
                    env[v.id] = x
                self._run_eqns(tr.cond, env, out)
                return bool(self._val(tr.cond_out, env))
            while kc < self.M and pred(carry):
                for v, x in zip(tr.carry, carry):
                    env[v.id] = x
                self._run_eqns(tr.body, env, out)
                carry = [self._val(x, env) for x in tr.body_out]
                kc += 1
            tr_i = kc >= self.M and pred(carry)
            for v, x in zip(tr.post_carry, carry):
                env[v.id] = x
            self._run_eqns(tr.post, env, out)
            if i is None:
                stats[2] += int(tr_i)
            else:
                trunc[i] = tr_i
                for r, y in enumerate(tr.results):
                    results[r][i] = self._val(y, env)
            for ch in out["spawns"]:
                stats[0] += 1
                work.append((None, {x.id: v for x, v in zip(leaves_of, ch)}))
            if self.max_items and len(work) > self.max_items:
                raise RuntimeError("ir_eval: the spawn tree outgrew max_items")
            for nm, idx, v in out["emits"]:
                S = len(sums[nm])
                if not 0 <= idx < S:
                    stats[4] += 1
                elif nm in self.exact:
                    exact_pairs[nm][0].append(v)
                    exact_pairs[nm][1].append(idx)
                elif nm in self.wide:
                    x = float(v) * float(self.wide[nm][1])
                    if not abs(x) < 9.2e18:
                        stats[3] += 1
                        wide_flag[nm][idx] = True
                    else:
                        wide_tot[nm][idx] += round(x)
                else:
                    sums[nm][idx] += float(v) if specs[nm][1] == T.F32 else int(v)
            for nm, fields in out["appends"]:
                records[nm].append(tuple(F32(f + F32(0.0)) if isinstance(f, np.floating) else f for f in fields))
                counts[nm][i] += 1
        for nm, (vals, bins) in exact_pairs.items():
            sums[nm] = orc.exact_sum(np.array(vals, np.float32), np.array(bins, np.int32), len(sums[nm]))[0]
        for nm, (dt, scale) in self.wide.items():
            vals = []
            for tot, flag in zip(wide_tot[nm], wide_flag[nm]):
                v = float(tot) * (1.0 / float(scale))
                if dt == "f64":
                    big = not abs(v) <= 1.7976931348623157e308
                    stats[3] += int(big and not flag)
                    vals.append(math.nan if flag or big else v)
                else:
                    lim = 2 ** 63 if dt == "i64" else 2 ** 31
                    stats[3] += int(not -lim <= v < lim)
                    # (the device's conversion toward zero saturates)
                    vals.append(0 if v != v else lim - 1 if v >= lim else -lim if v < -lim else int(v))
            sums[nm] = np.array(vals, np.float64 if dt == "f64" else np.int64)
        return dict(sums=sums, records=records, counts=counts, stats=stats, results=results, trunc=trunc)
