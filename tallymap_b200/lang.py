"""The operations an item function may use, for tracing (tallymap_b200.trace): a scalar subset of jax.numpy,
jax.random and lax.while_loop with jax's semantics, the ones the reference's op table lowers for these items
(tallymap/backends/kernel/op_table.py: arithmetic, comparisons, select, conversions, transcendentals, threefry,
random_bits / fold_in / split, while, round, rem, stop_gradient), and compositions of them with jax's semantics
(clip, sign, square, mod, log1p, expm1, tanh, the reductions sum / max / min / all / any, cumsum and searchsorted
over a per-item vector, random.bernoulli); the inverse trigonometric, hyperbolic, exp2 / log2 / cbrt and erf / erfc /
erfinv primitives (random.normal over erfinv as jax.random forms it, random.exponential, gumbel, categorical,
randint), ceil, log10, logistic, isfinite and the other jax.numpy compositions below; small vectors with jax.numpy's
elementwise semantics (trace.Vec: array, stack, dot, reductions, a traced index read as jnp does); broadcast tables
read by traced indices (trace.Table); cond / switch (both branches traced, results selected, a branch's t.add /
t.append / t.spawn made only where it is taken, an inner loop in a branch iterating only where it is taken);
while_loop -- the item's first top-level one is its stepping loop, any other an inner loop --; fori_loop (static
bounds: unrolled; a traced bound: an inner loop) and scan of a static length.

    from tallymap_b200 import lang as tl

    def walk(t, x, key, drift):
        def body(c):
            k, x, t = c
            u = tl.random.uniform(tl.random.fold_in(key, k))
            t = t.add("hist", (x * 256).astype(tl.int32), drift * x)
            return k + 1, x + 0.02 * (2 * u - 1), t
        k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
        t = t.add("side", (x > 1).astype(tl.int32), 1.0)
        return t, k

Transcendentals are the backend's shared f32 math (identical on the host oracle and the device); f32 -> int32
conversion truncates toward zero, saturating, NaN -> 0 (the reference's _rz conversions).
"""
import builtins

from . import trace as T

float32, int32, uint32, bool_ = "float32", "int32", "uint32", "bool"
while_loop = T.while_loop


pi = 3.141592653589793         # jnp.pi: a Python float, rounded to float32 where it meets a traced value
e = 2.718281828459045


def _vmap1(f, x):
    return T.Vec(f(v) for v in x) if isinstance(x, T.Vec) else None


def _un(prim, x, out=None):
    if isinstance(x, T.Vec):
        return _vmap1(lambda v: _un(prim, v, out), x)
    x = T._lit(x)
    if isinstance(x, T.Lit):
        raise T.TraceError(f"tallymap_b200.lang.{prim} of a literal")
    return T._cur().emit(prim, [x], [out or x.dtype])[0]


def _f32(prim, x):
    if isinstance(x, T.Vec):
        return _vmap1(lambda v: _f32(prim, v), x)
    x = T._lit(x)
    if x.dtype != T.F32:
        raise T.TraceError(f"tallymap_b200.lang.{prim} takes float32")
    return _un(prim, x)


def log(x):
    return _f32("log", x)


def exp(x):
    return _f32("exp", x)


def sin(x):
    return _f32("sin", x)


def cos(x):
    return _f32("cos", x)


def sqrt(x):
    return _f32("sqrt", x)


def floor(x):
    return _f32("floor", x)


def ceil(x):
    """jnp.ceil: -floor(-x) (exact)"""
    return -floor(-x)


def arctan(x):
    return _f32("atan", x)


def arctan2(y, x):
    """jnp.arctan2(y, x) (lax.atan2): the angle of (x, y) in (-pi, pi], C's signed-zero and infinite cases"""
    if isinstance(x, T.Vec) or isinstance(y, T.Vec):
        return T._vec_map2(arctan2, y, x)
    y0 = y if isinstance(y, T.Var) else None
    x0 = x if isinstance(x, T.Var) else None
    y, x = T._lit(y, x0), T._lit(x, y0)
    if x.dtype != T.F32 or y.dtype != T.F32:
        raise T.TraceError("tallymap_b200.lang.arctan2 takes float32")
    return T._cur().emit("atan2", [y, x], [T.F32])[0]


def arcsin(x):
    return _f32("asin", x)


def arccos(x):
    return _f32("acos", x)


def tan(x):
    return _f32("tan", x)


def sinh(x):
    return _f32("sinh", x)


def cosh(x):
    return _f32("cosh", x)


def arcsinh(x):
    return _f32("asinh", x)


def arccosh(x):
    return _f32("acosh", x)


def arctanh(x):
    return _f32("atanh", x)


def exp2(x):
    return _f32("exp2", x)


def log2(x):
    return _f32("log2", x)


def log10(x):
    """jnp.log10: log(x) / log(10) in float32, as jax.numpy forms it"""
    return log(x) / 2.30258512


def cbrt(x):
    return _f32("cbrt", x)


def erf(x):
    """jax.scipy.special.erf / lax.erf"""
    return _f32("erf", x)


def erfc(x):
    """jax.scipy.special.erfc / lax.erfc"""
    return _f32("erfc", x)


def erfinv(x):
    """jax.scipy.special.erfinv / lax.erf_inv: the inverse of erf on (-1, 1), +-inf at +-1"""
    return _f32("erfinv", x)


def population_count(x):
    """lax.population_count of an int32 / uint32: the set bits of its 32-bit pattern"""
    if T._lit(x).dtype not in (T.I32, T.U32):
        raise T.TraceError("tallymap_b200.lang.population_count of an integer")
    return _un("popc", x)


def clz(x):
    """lax.clz of an int32 / uint32: the leading zero bits of its 32-bit pattern (32 for 0)"""
    if T._lit(x).dtype not in (T.I32, T.U32):
        raise T.TraceError("tallymap_b200.lang.clz of an integer")
    return _un("clz", x)


def lgamma(x):
    """jax.scipy.special.gammaln / lax.lgamma: ln|Gamma(x)| (+inf at 0 and the negative integers); it has no
    derivative rule here, as the reference's op table has no digamma"""
    return _f32("lgamma", x)


def nextafter(x, y):
    """jnp.nextafter / lax.nextafter: the float32 next to x in the direction of y (C's nextafterf); not
    differentiable"""
    if isinstance(x, T.Vec) or isinstance(y, T.Vec):
        return T._vec_map2(nextafter, x, y)
    x0 = x if isinstance(x, T.Var) else None
    y0 = y if isinstance(y, T.Var) else None
    x, y = T._lit(x, y0), T._lit(y, x0)
    if x.dtype != T.F32 or y.dtype != T.F32:
        raise T.TraceError("tallymap_b200.lang.nextafter takes float32")
    return T._binary("nextafter", x, y)


def logistic(x):
    """jax.nn.sigmoid / lax.logistic: 1 / (1 + exp(-x))"""
    return 1.0 / (1.0 + exp(-x))


def isfinite(x):
    """jnp.isfinite: neither infinite nor NaN (x - x is 0 exactly then)"""
    return (x - x) == 0.0


atan, atan2, asin, acos, asinh, acosh, atanh = arctan, arctan2, arcsin, arccos, arcsinh, arccosh, arctanh
sigmoid = logistic


def abs(x):   # noqa: A001 (jnp.abs)
    return _un("abs", x)


def power(x, y):
    if isinstance(x, T.Vec) or isinstance(y, T.Vec):
        return T._vec_map2(power, x, y)
    x0 = x if isinstance(x, T.Var) else None
    y0 = y if isinstance(y, T.Var) else None
    x, y = T._lit(x, y0), T._lit(y, x0)
    if x.dtype != T.F32 or y.dtype != T.F32:
        raise T.TraceError("tallymap_b200.lang.power takes float32")
    return T._cur().emit("pow", [x, y], [T.F32])[0]


def maximum(a, b):
    """jax.lax.max: NaN if either is NaN, max(-0, +0) = +0"""
    return T._binary("max", a, b)


def minimum(a, b):
    return T._binary("min", a, b)


def where(c, a, b):
    if isinstance(c, T.Vec) or isinstance(a, T.Vec) or isinstance(b, T.Vec):
        n = next(len(v) for v in (c, a, b) if isinstance(v, T.Vec))
        at = lambda v, i: tuple.__getitem__(v, i) if isinstance(v, T.Vec) else v
        if any(isinstance(v, T.Vec) and len(v) != n for v in (c, a, b)):
            raise T.TraceError("tallymap_b200.lang.where: vectors of different lengths")
        return T.Vec(where(at(c, i), at(a, i), at(b, i)) for i in range(n))
    c = T._lit(c)
    if c.dtype != T.BOOL:
        raise T.TraceError("tallymap_b200.lang.where: the condition must be bool")
    a0 = a if isinstance(a, T.Var) else None
    b0 = b if isinstance(b, T.Var) else None
    a, b = T._lit(a, b0), T._lit(b, a0)
    if a.dtype != b.dtype:
        raise T.TraceError(f"tallymap_b200.lang.where of {a.dtype} and {b.dtype}")
    return T._cur().emit("select", [c, a, b], [a.dtype])[0]


def _branch_select(picks, results):
    """the elementwise selection of branch results of one structure: picks[j] -> bool, branch j taken.  A leaf that
    is not a value (the tally handle, a tally of the jaxpr front end) passes through when every branch returns that
    same object, as a branch that writes the tally and returns it, or returns it untouched, does"""
    flat = [T._flatten(r) for r in results]
    leaves0, rebuild = flat[0]
    for lv, _ in flat[1:]:
        if len(lv) != len(leaves0):
            raise T.TraceError("tallymap_b200.lang.cond: the branches return different structures")
    out = []
    for k in range(len(leaves0)):
        xs = [f[0][k] for f in flat]
        if builtins.any(isinstance(x, T.TallyToken) for x in xs):
            if builtins.any(x is not xs[0] for x in xs[1:]):
                raise T.TallyError("tallymap_b200.lang.cond: the branches must use each tally the same way (write "
                                   "it and return it, or return it untouched) (tallymap/_rewrite.py:178-182)")
            out.append(xs[0])
            continue
        r = xs[0]
        for j in range(1, len(xs)):
            r = where(picks[j]() if isinstance(picks[j], _Pick) else picks[j], xs[j], r)
        out.append(r)
    return rebuild(out)


_EFFECTS = ("emit", "append", "spawn", "claim")     # (claim: a Records slot claim of the jaxpr front end)


class _Pick:
    """a branch predicate formed on first use: no equation for a branch whose result and effects need none"""

    def __init__(self, make):
        self.make, self.v = make, None

    def __call__(self):
        if self.v is None:
            self.v = self.make()
        return self.v


def _predicate(tr, n0, taken):
    """make the effects traced into tr.eqns[n0:] (one branch) happen only where `taken` (a bool): an emit carries
    the predicate as a third operand, an append's and a spawn's `when` is ANDed with it (a nested branch's own
    predicate included).  The branches of a lax.cond run as straight-line code, their results selected (as jax does
    under vmap); the reference's backends run only the taken branch's t.add / t.spawn / t.append
    (tallymap/_rewrite.py:573-598 threads the tally through lax.switch), and the predicate gives the same"""
    if isinstance(taken, _Pick):
        # (formed from values defined before the branch: its equations go in at the branch's start)
        m = len(tr.eqns)
        taken = taken()
        new = tr.eqns[m:]
        del tr.eqns[m:]
        tr.eqns[n0:n0] = new
    out = tr.eqns[:n0]
    for e in tr.eqns[n0:]:
        if e.prim == "while" and not (isinstance(taken, T.Lit) and taken.value):
            # (an inner loop in a branch iterates only where the branch is taken: its condition ANDed with the
            # predicate, so a loop that would not end on the other branch's values never starts, and the effects
            # in its body need no predicate of their own)
            p = dict(e.params)
            c = tr.new(T.BOOL)
            p["cond"] = list(p["cond"]) + [T.Eqn("and", [p["cond_out"], taken], [c], {})]
            p["cond_out"] = c
            out.append(T.Eqn("while", e.ins, e.outs, p))
            continue
        if e.prim not in _EFFECTS:
            out.append(e)
            continue
        k = 2 if e.prim == "emit" else 0
        old = e.ins[k] if len(e.ins) > k else T.Lit(True, T.BOOL)
        if isinstance(taken, T.Lit) and not taken.value or isinstance(old, T.Lit) and not old.value:
            continue                                   # (never taken: the effect is gone)
        if isinstance(taken, T.Lit):
            w = old
        elif isinstance(old, T.Lit):
            w = taken
        else:
            w = tr.new(T.BOOL)
            out.append(T.Eqn("and", [old, taken], [w], {}))
        ins = list(e.ins)
        if k < len(ins):
            ins[k] = w
        elif not isinstance(w, T.Lit):
            ins.append(w)
        out.append(T.Eqn(e.prim, ins, e.outs, e.params))
    tr.eqns[:] = out


def _branches(funs, operands, picks):
    """trace each branch on the same operands, its effects (t.add, t.append, t.spawn) predicated on picks[j]; a
    while loop in a branch is an inner loop (never the item's stepping loop), run only where its branch is taken"""
    tr = T._cur()
    st = getattr(tr, "loop_state", None)
    res = []
    for f, taken in zip(funs, picks):
        n0 = len(tr.eqns)
        if st is not None:
            st["branch"] = st.get("branch", 0) + 1
        try:
            res.append(f(*operands))
        finally:
            if st is not None:
                st["branch"] -= 1
        if builtins.any(e.prim in _EFFECTS or e.prim == "while" for e in tr.eqns[n0:]):
            _predicate(tr, n0, taken)
    return res


def cond(pred, true_fun, false_fun, *operands):
    """lax.cond: both branches traced, their results selected elementwise by pred, their tally writes made only by
    the taken one"""
    pred = T._lit(pred)
    if pred.dtype != T.BOOL:
        raise T.TraceError("tallymap_b200.lang.cond: the predicate must be bool")
    npred = _Pick(lambda: ~pred) if isinstance(pred, T.Var) else T.Lit(not pred.value, T.BOOL)
    f, t = _branches((false_fun, true_fun), operands, (npred, pred))
    return _branch_select((npred, pred), (f, t))


def switch(index, branches, *operands):
    """lax.switch: the index clamped into range, each branch traced, a chain of selects; the tally writes made only
    by the taken branch"""
    index = T._lit(index)
    if index.dtype != T.I32:
        raise T.TraceError("tallymap_b200.lang.switch: the index must be int32")
    n = len(branches)
    idx = clip(index, 0, n - 1) if isinstance(index, T.Var) else T.Lit(max(0, min(n - 1, int(index.value))), T.I32)
    picks = [_Pick(lambda j=j: idx == j) if isinstance(idx, T.Var) else T.Lit(idx.value == j, T.BOOL)
             for j in range(n)]
    res = _branches(branches, operands, picks)
    return _branch_select(picks, res)


def fori_loop(lower, upper, body_fun, init_val):
    """lax.fori_loop: with Python int bounds the body applied upper - lower times, unrolled (a static trip count);
    with a traced bound, jax's while form -- (i, val) carried while i < upper, an inner loop"""
    if not (isinstance(lower, int) and isinstance(upper, int)):
        lo = T._lit(lower)
        hi = T._lit(upper)
        if lo.dtype != T.I32 or hi.dtype != T.I32:
            raise T.TraceError("tallymap_b200.lang.fori_loop: int32 bounds")
        return while_loop(lambda c: c[0] < upper, lambda c: (c[0] + 1, body_fun(c[0], c[1])), (lower, init_val))[1]
    if upper - lower > 4096:
        raise T.UnsupportedError("tallymap_b200.lang.fori_loop: at most 4096 unrolled iterations")
    v = init_val
    for i in range(lower, upper):
        v = body_fun(i, v)
    return v


def array(xs, dtype=None):
    """jnp.array / jnp.stack of scalars (traced values or Python numbers) -> a vector with elementwise semantics"""
    xs = [x.item() if hasattr(x, "item") and not isinstance(x, (T.Var, T.Lit)) else x for x in xs]   # numpy numbers
    xs = [float(x) if dtype == float32 and isinstance(x, (int, float)) else x for x in xs]
    v = T.Vec(xs)
    return v.astype(dtype) if dtype in (float32, int32) and any(isinstance(x, T.Var) for x in xs) else v


stack = array


def zeros(n, dtype=float32):
    """jnp.zeros((n,)): a vector of literal zeros"""
    return T.Vec([0.0 if dtype == float32 else 0] * int(n if isinstance(n, int) else n[0]))


def ones(n, dtype=float32):
    return T.Vec([1.0 if dtype == float32 else 1] * int(n if isinstance(n, int) else n[0]))


def prod(xs):
    """jnp.prod of a vector: the products left to right"""
    xs = tuple(xs)
    out = xs[0]
    for x in xs[1:]:
        out = out * x
    return out


def mean(xs):
    """jnp.mean of a float32 vector: the left-to-right sum divided by the length"""
    return sum(xs) / float(len(xs))


def _arg(xs, better):
    """the first index of the extreme element (jnp.argmax / argmin; a NaN wins, as jax's)"""
    xs = tuple(xs)
    best, idx = xs[0], 0
    for j, x in enumerate(xs[1:], 1):
        take = better(x, best)
        if isinstance(x, T.Var) and x.dtype == T.F32:
            take = take | ((x != x) & (best == best))
        best, idx = where(take, x, best), where(take, j, idx)
    return idx


def argmax(xs):
    return _arg(xs, lambda x, b: x > b)


def argmin(xs):
    return _arg(xs, lambda x, b: x < b)


def _cum(xs, f):
    out, acc = [], None
    for x in tuple(xs):
        acc = x if acc is None else f(acc, x)
        out.append(acc)
    return T.Vec(out)


def cumprod(xs):
    """jnp.cumprod of a vector: the running products, left to right"""
    return _cum(xs, lambda a, b: a * b)


def cummax(xs):
    """lax.cummax of a vector: the running maxima"""
    return _cum(xs, maximum)


def cummin(xs):
    return _cum(xs, minimum)


def isnan(x):
    """jnp.isnan: x != x"""
    return x != x


def isinf(x):
    """jnp.isinf: |x| == inf"""
    return abs(x) == float("inf")


def nan_to_num(x, nan=0.0, posinf=3.4028234663852886e38, neginf=-3.4028234663852886e38):
    """jnp.nan_to_num of float32: NaN -> nan, +inf -> posinf (the largest float32 by default), -inf -> neginf"""
    return where(x != x, nan, where(x == float("inf"), posinf, where(x == -float("inf"), neginf, x)))


def logaddexp(a, b):
    """jnp.logaddexp as jax forms it: a + b where a - b is NaN (equal infinities, or a NaN), else
    max(a, b) + log1p(exp(-|a - b|))"""
    amax = maximum(a, b)
    delta = a - b
    return where(delta != delta, a + b, amax + log1p(exp(-abs(delta))))


def hypot(a, b):
    """jnp.hypot as jax forms it: x = max(|a|, |b|), y = min(...), x sqrt(1 + (y / x)^2) (x itself where it is 0),
    +inf where either is +-inf"""
    a, b = abs(a), abs(b)
    inf = (a == float("inf")) | (b == float("inf"))
    x, y = maximum(a, b), minimum(a, b)
    r = where(x == 0.0, x, x * sqrt(1.0 + square(y / where(x == 0.0, 1.0, x))))
    return where(inf, float("inf"), r)


def norm(xs):
    """jnp.linalg.norm of a vector (the 2-norm): sqrt of the left-to-right sum of squares"""
    return sqrt(sum(T.Vec(xs) * T.Vec(xs)))


def deg2rad(x):
    return x * (pi / 180.0)


def rad2deg(x):
    return x * (180.0 / pi)


def dot(a, b):
    """jnp.dot of two vectors: the products summed left to right"""
    return sum(T.Vec(a) * T.Vec(b))


def scan(f, init, xs=None, length=None):
    """lax.scan with a static length (len(xs), or `length`), unrolled: carry, y = f(carry, x) per step; -> (the
    final carry, the ys stacked: a vector of the per-step scalars, a tuple of vectors for tuple outputs, None for
    None).  xs: a vector, or a tuple of vectors scanned together"""
    if xs is None:
        if not isinstance(length, int):
            raise T.UnsupportedError("tallymap_b200.lang.scan: a static length (Python int) or xs")
        n, at = length, (lambda i: None)
    elif isinstance(xs, tuple) and not isinstance(xs, T.Vec) and xs and isinstance(xs[0], tuple):
        n = len(xs[0])
        at = lambda i: tuple(tuple.__getitem__(x, i) for x in xs)
    else:
        n = len(xs)
        at = lambda i: tuple.__getitem__(xs, i)
    if n > 4096:
        raise T.UnsupportedError("tallymap_b200.lang.scan: at most 4096 unrolled steps")
    carry, ys = init, []
    for i in range(n):
        carry, y = f(carry, at(i))
        ys.append(y)
    if not ys or ys[0] is None:
        return carry, None
    if isinstance(ys[0], tuple) and not isinstance(ys[0], T.Vec):
        return carry, tuple(T.Vec(y[j] for y in ys) for j in range(len(ys[0])))
    return carry, T.Vec(ys)


def round(x):   # noqa: A001 (jnp.round)
    """jnp.round: to the nearest integer, ties to even"""
    return _f32("round", x)


def stop_gradient(x):
    """lax.stop_gradient: the value itself, with no derivative (no cotangent, no tangent) through it"""
    if isinstance(x, T.Vec):
        return _vmap1(stop_gradient, x)
    x = T._lit(x)
    if isinstance(x, T.Lit):
        return x
    return T._cur().emit("stop", [x], [x.dtype])[0]


def rem(a, b):
    """lax.rem of float32: C's fmod (the sign of a)"""
    if isinstance(a, T.Vec) or isinstance(b, T.Vec):
        return T._vec_map2(rem, a, b)
    r = T._binary("rem", a, b)
    if r.dtype != T.F32:
        raise T.TraceError("tallymap_b200.lang.rem takes float32 (use % for integers)")
    return r


def mod(a, b):
    """jnp.mod / jnp.remainder of float32: the sign of b (rem, plus b when the signs differ)"""
    if isinstance(a, T.Vec) or isinstance(b, T.Vec):
        return T._vec_map2(mod, a, b)
    r = rem(a, b)
    return where((r != 0.0) & ((r < 0.0) != (b < 0.0)), r + b, r)


def sum(xs):   # noqa: A001 (jnp.sum of a per-item vector)
    """jnp.sum of a tuple of scalars (a per-item vector), added left to right"""
    xs = tuple(xs)
    out = xs[0]
    for x in xs[1:]:
        out = out + x
    return out


def max(xs):   # noqa: A001 (jnp.max of a per-item vector)
    """jnp.max of a tuple of scalars: lax.max left to right"""
    xs = tuple(xs)
    out = xs[0]
    for x in xs[1:]:
        out = maximum(out, x)
    return out


def min(xs):   # noqa: A001 (jnp.min of a per-item vector)
    xs = tuple(xs)
    out = xs[0]
    for x in xs[1:]:
        out = minimum(out, x)
    return out


def all(bs):   # noqa: A001 (jnp.all of a tuple of bools)
    bs = tuple(bs)
    out = bs[0]
    for b in bs[1:]:
        out = out & b
    return out


def any(bs):   # noqa: A001 (jnp.any of a tuple of bools)
    bs = tuple(bs)
    out = bs[0]
    for b in bs[1:]:
        out = out | b
    return out


def log1p(x):
    """jnp.log1p, by Goldberg's method (What Every Computer Scientist Should Know About Floating-Point Arithmetic,
    1991, Theorem 4): u = 1 + x; x itself where u rounds to 1, else log(u) * (x / (u - 1)), whose rounding error in
    u cancels; +inf for +inf"""
    u = 1.0 + x
    return where((u == 1.0) | (u == float("inf")), x, log(u) * (x / (u - 1.0)))


def expm1(x):
    """jnp.expm1, by Kahan's method: u = exp(x); x where u rounds to 1, -1 where u - 1 does, u itself where it
    overflows, else (u - 1) * (x / log(u))"""
    u = exp(x)
    um = u - 1.0
    return where(u == 1.0, x, where(um == -1.0, -1.0, where(u == float("inf"), u, um * (x / log(u)))))


def tanh(x):
    """jnp.tanh from expm1: with e = expm1(-2|x|), tanh(|x|) = -e / (e + 2), the sign of x restored (tanh(-0) = -0)"""
    ax = abs(x)
    e = expm1(-2.0 * ax)
    t = (-e) / (e + 2.0)
    return where(x < 0.0, -t, where(x > 0.0, t, x))


def cumsum(xs):
    """jnp.cumsum of a per-item vector (a tuple): the running sums, added left to right"""
    out = []
    acc = None
    for x in xs:
        acc = x if acc is None else acc + x
        out.append(acc)
    return tuple(out)


def searchsorted(a, v, side="left"):
    """jnp.searchsorted of v in the sorted per-item vector a: the count of elements < v (side "left") or <= v
    ("right"), as int32"""
    if side not in ("left", "right"):
        raise T.TraceError("tallymap_b200.lang.searchsorted: side 'left' or 'right'")
    if isinstance(a, T.Table):
        # a sorted 1-D table: binary search, bit_length(n) steps unrolled, each a gather and two selects
        if len(a.shape) != 1:
            raise T.TraceError("tallymap_b200.lang.searchsorted: a 1-D table")
        n = a.shape[0]
        lo, hi = 0, n
        for _ in range(n.bit_length()):
            act = T.Lit(True, T.BOOL) if isinstance(lo, int) and isinstance(hi, int) else (lo < hi)
            mid = (lo + hi) // 2
            c = (a[mid] < v) if side == "left" else (a[mid] <= v)
            lo, hi = where(act & c, mid + 1, lo), where(act & ~c, mid, hi)
        return lo
    cnt = None
    for x in a:
        c = (x < v) if side == "left" else (x <= v)
        c = c.astype(int32)
        cnt = c if cnt is None else cnt + c
    return cnt


def _sort_network(keys, payloads=()):
    """odd-even transposition sort of a vector of keys, each payload vector permuted with it: n passes of adjacent
    compare-exchanges, a swap when the right key is smaller or the left is NaN (NaNs last, as jnp.sort and lax.sort's
    total order; -0 and +0 compare equal); equal keys never swap, so the order is stable.  -> (sorted keys, [the
    payloads in that order])"""
    v = list(tuple(keys))
    ps = [list(tuple(q)) for q in payloads]
    n = len(v)
    for p in range(n):
        for j in range(p % 2, n - 1, 2):
            a, b = v[j], v[j + 1]
            flt = any((isinstance(z, T.Var) and z.dtype == T.F32) or isinstance(z, float) for z in (a, b))
            swap = (b < a) | ((a != a) & (b == b)) if flt else (b < a)
            v[j], v[j + 1] = where(swap, b, a), where(swap, a, b)
            for q in ps:
                q[j], q[j + 1] = where(swap, q[j + 1], q[j]), where(swap, q[j], q[j + 1])
    return T.Vec(v), [T.Vec(q) for q in ps]


def _sorted_pairs(xs):
    """the sorted vector and its stable ascending order's indices"""
    v, (idx,) = _sort_network(xs, [list(range(len(tuple(xs))))])
    return v, idx


def sort(xs):
    """jnp.sort of a vector: ascending, NaNs last, stable"""
    return _sorted_pairs(xs)[0]


def argsort(xs):
    """jnp.argsort of a vector: the stable ascending order's indices (int32)"""
    return _sorted_pairs(xs)[1]


def interp(x, xp, fp, left=None, right=None):
    """jnp.interp as jax forms it: i = clip(searchsorted(xp, x, 'right'), 1, n - 1), fp[i-1] + (x - xp[i-1]) /
    (xp[i] - xp[i-1]) (fp[i] - fp[i-1]) (fp[i-1] where the step is below 2^-46), fp[0] / fp[-1] (or left / right)
    outside [xp[0], xp[-1]]; xp and fp vectors or 1-D tables"""
    n = len(xp)
    i = clip(searchsorted(xp, x, side="right"), 1, n - 1)
    xi, xm, fi, fm = xp[i], xp[i - 1], fp[i], fp[i - 1]
    df, dx, delta = fi - fm, xi - xm, x - xm
    dx0 = abs(dx) <= 1.4210854715202004e-14
    f = where(dx0, fm, fm + (delta / where(dx0, 1.0, dx)) * df)
    f = where(x < xp[0], fp[0] if left is None else left, f)
    return where(x > xp[-1], fp[-1] if right is None else right, f)


def bitcast_convert_type(x, new_dtype):
    """lax.bitcast_convert_type between the 32-bit types (float32, int32, uint32): the same bits, another type"""
    if isinstance(x, T.Vec):
        return T.Vec(bitcast_convert_type(v, new_dtype) for v in x)
    dst = T._dt(new_dtype)
    x = T._lit(x)
    if dst == T.BOOL or x.dtype == T.BOOL:
        raise T.TraceError("tallymap_b200.lang.bitcast_convert_type: 32-bit types only")
    if x.dtype == dst:
        return x
    if isinstance(x, T.Lit):
        import numpy as np
        src = {T.F32: np.float32, T.I32: np.int32, T.U32: np.uint32}[x.dtype]
        out = {T.F32: np.float32, T.I32: np.int32, T.U32: np.uint32}[dst]
        v = np.array([x.value], src).view(out)[0]
        return T.Lit(float(v) if dst == T.F32 else int(v), dst)
    return T._cur().emit("bitcast", [x], [dst])[0]


def clip(x, a_min, a_max):
    """jnp.clip: maximum(a_min, x), then minimum(a_max, .) (lax.max / min semantics: NaN propagates)"""
    return minimum(a_max, maximum(a_min, x))


def sign(x):
    """jnp.sign (lax.sign): -1, +1, the zero itself for +-0 (its sign kept), NaN for NaN"""
    if isinstance(x, T.Vec):
        return _vmap1(sign, x)
    x = T._lit(x)
    if x.dtype == T.F32:
        return where(x > 0.0, 1.0, where(x < 0.0, -1.0, x))
    return where(x > 0, 1, where(x < 0, -1, 0))


def square(x):
    """jnp.square: x * x"""
    return x * x


class random:
    """jax.random on raw uint32[2] key data, partitionable threefry (bitwise jax.random's)"""

    @staticmethod
    def _u32(x):
        x = T._lit(x)
        if x.dtype == T.I32:
            x = x.astype(uint32) if isinstance(x, T.Var) else T.Lit(int(x.value) & 0xFFFFFFFF, T.U32)
        if x.dtype != T.U32:
            raise T.TraceError("tallymap_b200.lang.random: integer data expected")
        return x

    @staticmethod
    def fold_in(key, data):
        """jax.random.fold_in: threefry2x32(key, (0, data))"""
        o = T._cur().emit("threefry", [key.a, key.b, T.Lit(0, T.U32), random._u32(data)], [T.U32, T.U32])
        return T.Key(o[0], o[1])

    @staticmethod
    def split(key, num=2):
        """jax.random.split(key, num): key i = threefry2x32(key, (0, i))"""
        return tuple(random.fold_in(key, i) for i in range(int(num)))

    @staticmethod
    def bits(key, shape=()):
        """jax.random.bits(key, shape, uint32): element i = o0 ^ o1 of threefry2x32(key, (0, i))"""
        n = _count(shape)
        out = T.Vec(T._cur().emit("bits", [key.a, key.b, T.Lit(i, T.U32)], [T.U32])[0] for i in range(n))
        return out[0] if shape == () else out

    @staticmethod
    def bernoulli(key, p=0.5, shape=()):
        """jax.random.bernoulli: uniform(key, shape) < p"""
        u = random.uniform(key, shape)
        return u < p

    @staticmethod
    def normal(key, shape=(), dtype=float32):
        """jax.random.normal: sqrt(2) erf_inv(u) for u = uniform(key, shape, minval=nextafter(-1, 0), maxval=1)"""
        if dtype != float32:
            raise T.TraceError("tallymap_b200.lang.random.normal: float32 only")
        u = random.uniform(key, shape, minval=-0.99999994, maxval=1.0)
        return 1.41421354 * erfinv(u)

    @staticmethod
    def exponential(key, shape=(), dtype=float32):
        """jax.random.exponential: -log1p(-u) for u = uniform(key, shape)"""
        u = random.uniform(key, shape, dtype)
        return -log1p(-u)

    @staticmethod
    def truncated_normal(key, lower, upper, shape=(), dtype=float32):
        """jax.random.truncated_normal for Python-number bounds: u uniform on (erf(lower / sqrt2), erf(upper /
        sqrt2)), sqrt2 erfinv(u), clipped inside (lower, upper) by one float32 step (the bounds' erf in float32,
        correctly rounded as the shared math's)"""
        if not (isinstance(lower, (int, float)) and isinstance(upper, (int, float))):
            raise T.UnsupportedError("tallymap_b200.lang.random.truncated_normal: Python-number bounds only")
        import math
        import numpy as np
        s2 = np.float32(math.sqrt(2.0))
        lo, hi = np.float32(lower), np.float32(upper)
        ea = float(np.float32(math.erf(float(np.float32(lo / s2)))))
        eb = float(np.float32(math.erf(float(np.float32(hi / s2)))))
        u = random.uniform(key, shape, dtype, minval=ea, maxval=eb)
        out = float(s2) * erfinv(u)
        return clip(out, float(np.nextafter(lo, np.float32(np.inf))), float(np.nextafter(hi, np.float32(-np.inf))))

    @staticmethod
    def laplace(key, shape=(), dtype=float32):
        """jax.random.laplace: sign(u) log1p(-|u|) for u = uniform(key, shape, minval=-1 + 2^-24, maxval=1)"""
        u = random.uniform(key, shape, dtype, minval=-0.99999994, maxval=1.0)
        return sign(u) * log1p(-abs(u))

    @staticmethod
    def rademacher(key, shape=(), dtype=int32):
        """jax.random.rademacher: 2 bernoulli(key, 0.5, shape) - 1, as int32 (+-1)"""
        b = random.bernoulli(key, 0.5, shape).astype(int32)
        return 2 * b - 1

    @staticmethod
    def gumbel(key, shape=(), dtype=float32):
        """jax.random.gumbel: -log(-log(u)) for u = uniform(key, shape, minval=float32 tiny, maxval=1)"""
        u = random.uniform(key, shape, dtype, minval=1.1754943508222875e-38, maxval=1.0)
        return -log(-log(u))

    @staticmethod
    def categorical(key, logits):
        """jax.random.categorical over a vector of logits: argmax(gumbel(key, (n,)) + logits), an int32 index"""
        logits = T.Vec(logits)
        return argmax(random.gumbel(key, (len(logits),)) + logits)

    @staticmethod
    def choice(key, a, shape=(), replace=True, p=None):
        """jax.random.choice with replacement: an index drawn by randint(0, n) (p None) or by inverse-CDF sampling,
        searchsorted(cumsum(p), cumsum(p)[-1] * (1 - uniform)); the index itself for an int `a`, else a[index]"""
        if not replace:
            raise T.UnsupportedError("tallymap_b200.lang.random.choice: replace=False is not lowered")
        n = a if isinstance(a, int) else len(a)
        if p is None:
            ind = random.randint(key, shape, 0, n)
        else:
            pc = cumsum(T.Vec(p))
            u = random.uniform(key, shape)
            draw = lambda v: searchsorted(pc, pc[-1] * (1.0 - v))
            ind = T.Vec(draw(v) for v in u) if isinstance(u, T.Vec) else draw(u)
        if isinstance(a, int):
            return ind
        av = T.Vec(a)
        return T.Vec(av[i] for i in ind) if isinstance(ind, T.Vec) else av[ind]

    @staticmethod
    def randint(key, shape=(), minval=0, maxval=2):
        """jax.random.randint for int32 Python-int bounds: two 32-bit draws from split(key) combined modulo the
        span with jax's uint32 arithmetic (every product wraps modulo 2^32), minval where maxval <= minval"""
        if not (isinstance(minval, int) and isinstance(maxval, int)):
            raise T.UnsupportedError("tallymap_b200.lang.random.randint: Python int bounds only")
        import builtins
        lo = builtins.max(-2 ** 31, builtins.min(2 ** 31 - 1, minval))
        hi = builtins.max(-2 ** 31, builtins.min(2 ** 31 - 1, maxval))
        out_of_range = maxval > 2 ** 31 - 1
        span = (hi - lo) & 0xFFFFFFFF if hi > lo else 1
        if out_of_range and hi > lo:
            span = (span + 1) & 0xFFFFFFFF
        k1, k2 = random.split(key)
        hb, lb = random.bits(k1, shape), random.bits(k2, shape)
        # jax forms the multiplier 2^32 mod span in uint32: (2^16 mod span)^2 wraps modulo 2^32 before its remainder
        # (lax.mul on uint32), so for a span above 2^16 the square is 2^32 -> 0 and the multiplier is 0
        mult = (2 ** 16) % span if span else 0
        mult = ((mult * mult) & 0xFFFFFFFF) % span if span else 0

        def one(h, l):
            off = (h % span) * mult + (l % span)
            return (off % span).astype(int32) + lo
        if span == 0:          # (the full 2^32 range: the wrapped span is 0 and jax's remainders are by 0)
            raise T.UnsupportedError("tallymap_b200.lang.random.randint: a span of 2^32 is not lowered")
        return T.Vec(one(h, l) for h, l in zip(hb, lb)) if shape != () else one(hb, lb)

    @staticmethod
    def uniform(key, shape=(), dtype=float32, minval=0.0, maxval=1.0):
        """jax.random.uniform: the mantissa fill of random bits in [1, 2) minus 1, then max(lo, f * (hi - lo) + lo)"""
        if dtype != float32:
            raise T.TraceError("tallymap_b200.lang.random.uniform: float32 only")
        n = _count(shape)
        out = []
        for i in range(n):
            f = T._cur().emit("uniform01", [key.a, key.b, T.Lit(i, T.U32)], [T.F32])[0]
            if not (isinstance(minval, float) and isinstance(maxval, float) and minval == 0.0 and maxval == 1.0):
                # jax computes max(lo, f * (hi - lo) + lo); for lo = 0, hi = 1 that is f itself, bitwise
                lo, hi = minval, maxval
                if isinstance(hi, T.Var) or isinstance(lo, T.Var):
                    f = maximum(lo, f * (hi - lo) + lo)
                else:           # float32 bounds and their float32 difference, as jax forms them
                    import numpy as np
                    lo32, hi32 = np.float32(lo), np.float32(hi)
                    f = maximum(float(lo32), f * float(np.float32(hi32 - lo32)) + float(lo32))
            out.append(f)
        return out[0] if shape == () else T.Vec(out)


def _count(shape):
    if shape == ():
        return 1
    if isinstance(shape, int):
        shape = (shape,)
    if len(shape) != 1:
        raise T.TraceError("tallymap_b200.lang.random: shape () or (n,)")
    return int(shape[0])
