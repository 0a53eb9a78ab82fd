"""The jaxpr front end of the lowering: an item program as JAX traces it -- the closed jaxpr of ONE item that the
reference builds in tallymap.vmap (tallymap/_api.py:559-668, ItemProgram.cj: invars = [tallies] + [per-item
leaves] + [broadcast leaves], outvars = [tallies] + [per-item results]) -- turned into this package's scalar IR
(trace.py), which lower.py compiles for sm_100a.  The reference lowers the same jaxprs with its own emitter
(tallymap/backends/kernel/codegen.py:815, Emitter.run_jaxpr, over the op table of op_table.py).

How: `item_function` returns a Python item function fn(t, *leaves) that INTERPRETS the jaxpr equation by
equation with this package's traced values (lang / trace), so tracing it (trace.trace_item, or tallymap_b200.vmap
of it) records exactly the IR a hand-written item of the same program would.  Each equation is read through
`eqn.primitive.name`, `eqn.params`, `eqn.invars` / `eqn.outvars` and each variable's `aval` (shape, dtype); a
literal operand has `.val`; sub-jaxprs (`while`'s cond_jaxpr / body_jaxpr, `cond`'s branches, `scan`'s and `pjit`'s
jaxpr) are interpreted in place.  Nothing here imports JAX: any objects with those attributes work (the CPU tests use
duck-typed equation lists).

Values: a scalar of shape () is a traced scalar or a numpy constant (equations whose operands are all constants are
folded in numpy with the aval's dtype, as XLA would fold them); a small 1-D array is a trace.Vec; a PRNG key
(typed key<fry>, or uint32[2] key data under random_wrap) is a trace.Key; a tally array is a reference to its
output.  `tallymap_emit(t, idx, val)` becomes an emit at the flat index the reference's Tally.add has formed
(out-of-range indices dropped and counted, _tally.py:29-57); `tallymap_spawn(q, when, *leaves)` a spawn;
`tallymap_claim(tok, when, k)` (a Records output's one-pass append, _tally.py:141-160, 335-351) a slot claim on the
key tally `tok` (trace._claim), whose fields the jaxpr then emits at the slot.

The primitives read are those of jax.numpy / jax.random / lax on scalars and small vectors that the reference's
op table lowers (op_table.py:47 RULES): arithmetic, comparisons, bitwise and shifts, select_n, clamp, conversions
and bitcasts, the transcendentals, integer_pow, the random primitives (random_seed / wrap / unwrap / fold_in /
bits / split, threefry2x32), while (the item's one top-level loop), cond (its branches' tally writes made only by
the taken branch), scan of a static length (unrolled; jax's static fori_loop), pjit and the call wrappers, shape
operations on scalars and small vectors (reshape, broadcast_in_dim, squeeze, expand_dims, slice, dynamic_slice,
dynamic_update_slice, concatenate, pad, rev, iota, reductions, cumsum / cumprod / cummax / cummin, dot_general with
a result of at most one dimension, sort on one key, gather as jnp indexing writes it -- a broadcast array of two
dimensions or above 64 elements is a table read by index --, element scatters into a vector: x.at[i].set / add /
multiply / min / max), jit (jax >= 0.7's name for pjit), random_clone / random_key_data, iota_2x32_shape and
platform_index.  Anything else raises UnsupportedError, as the reference's emitter does for a primitive its table
lacks (backends/kernel/__init__.py:81-82): never a fallback.

`run(p, pi, bc, target, cuda_math, schedule, ndev, min_blocks_per_sm)` is the reference's backend entry
(tallymap/backends/kernel/__init__.py:135-185) over a reference ItemProgram: its jaxpr through this front end,
compiled and launched through the C ABI, the outputs in the reference's order [sum tallies] + [stats] + [per-item
results].
"""
import collections

import numpy as np

from . import lang as tl
from . import trace as T

_DT = {"float32": T.F32, "int32": T.I32, "uint32": T.U32, "bool": T.BOOL}
_NP = {T.F32: np.float32, T.I32: np.int32, T.U32: np.uint32, T.BOOL: np.bool_}


def _is_key(aval):
    return "key" in str(aval.dtype)


def aval_spec(aval, per_item=True):
    """the trace_item input spec of a jaxpr input: "f32" / "i32" / "u32" / "key" for a scalar, (dtype, n) for a
    small vector; a broadcast array of two dimensions, or of one above BC_VECTOR_MAX elements, is a table
    ("table", dtype, shape), read by index (as tallymap_b200.vmap passes it)"""
    shape = tuple(aval.shape)
    if _is_key(aval):
        _threefry_impl(str(aval.dtype))
    from .api import BC_VECTOR_MAX
    dt0 = _DT.get(str(aval.dtype))
    if not per_item and not _is_key(aval) and dt0 in (T.F32, T.I32) and (
            len(shape) == 2 or (len(shape) == 1 and (shape[0] > BC_VECTOR_MAX or dt0 == T.I32))):
        return ("table", dt0, shape)
    if _is_key(aval):
        if shape != ():
            raise T.UnsupportedError("tallymap_b200.from_jaxpr: a per-item key operand must be one key")
        return "key"
    dt = _DT.get(str(aval.dtype))
    if dt is None or dt == T.BOOL:
        raise T.UnsupportedError(f"tallymap_b200.from_jaxpr: operand dtype {aval.dtype} is not lowered")
    if shape == ():
        return dt
    if dt == T.U32 and shape == (2,):
        return "key"              # raw key data (jax.random.PRNGKey / split's uint32[2]): the two words of a key
    if len(shape) == 1:
        return (dt, int(shape[0]))
    raise T.UnsupportedError(f"tallymap_b200.from_jaxpr: operand shape {shape} is not lowered")


class _TallyRef(T.TallyToken):
    """a tally array of the jaxpr (one Sum output, or the spawn queue token): the item's tally handle, and which
    output it is; the loop carries it as the tracer carries the handle"""

    def __init__(self, tok, name):          # (the handle's state stays on `tok`)
        self.tok, self.name = tok, name


def _dtype(aval):
    return _DT.get(str(aval.dtype))


def _const(val, aval):
    """a literal operand -> a numpy scalar of its dtype, or a Vec of them"""
    dt = _dtype(aval)
    if dt is None:
        raise T.UnsupportedError(f"tallymap_b200.from_jaxpr: literal of dtype {aval.dtype}")
    a = np.asarray(val, dtype=_NP[dt])
    if a.shape == ():
        return _NP[dt](a)
    return T.Vec(_NP[dt](x) for x in a.reshape(-1))


def _isconst(x):
    return isinstance(x, np.generic) or (isinstance(x, T.Vec) and all(isinstance(v, np.generic) for v in x))


def _py(x):
    """numpy constants -> Python numbers (the tracer's literals take the traced operand's type)"""
    if isinstance(x, np.generic):
        return x.item()
    if isinstance(x, T.Vec):
        return T.Vec(_py(v) for v in x)
    return x


def _cast(x, dt):
    """a traced or constant value as dtype dt (numpy for constants, astype for traced values)"""
    if isinstance(x, T.Vec):
        return T.Vec(_cast(v, dt) for v in x)
    if isinstance(x, np.generic):
        if dt == T.I32 or dt == T.U32:
            if isinstance(x, np.floating):
                with np.errstate(all="ignore"):
                    f = np.float32(x)
                    if np.isnan(f):
                        return _NP[dt](0)
                    lo, hi = (-2 ** 31, 2 ** 31 - 1) if dt == T.I32 else (0, 2 ** 32 - 1)
                    return _NP[dt](int(np.clip(np.trunc(np.float64(f)), lo, hi)))
            return _NP[dt](int(x) & 0xFFFFFFFF if dt == T.U32 else ((int(x) + 2 ** 31) % 2 ** 32) - 2 ** 31)
        if dt == T.BOOL:
            return np.bool_(x != 0)
        return np.float32(x)
    x = T._lit(x)
    return x.astype(dt) if x.dtype != dt else x


# ------------------------------------------------------------------------------------------------ elementwise
def _fold(fn, args, dt):
    """fn over numpy constants in dtype dt (elementwise over Vecs)"""
    if any(isinstance(a, T.Vec) for a in args):
        n = max(len(a) for a in args if isinstance(a, T.Vec))
        at = lambda a, i: tuple.__getitem__(a, i) if isinstance(a, T.Vec) else a
        return T.Vec(_fold(fn, [at(a, i) for a in args], dt) for i in range(n))
    with np.errstate(all="ignore"):
        r = fn(*args)
    return _NP[dt](r) if dt is not None else r


def _np_trunc_div(a, b):
    if b == 0:
        return -1
    q = abs(int(a)) // abs(int(b))
    return q if (a < 0) == (b < 0) else -q


def _np_trunc_rem(a, b):
    if b == 0:
        return int(a)
    return int(a) - _np_trunc_div(a, b) * int(b)


_FOLD2 = {
    "add": lambda a, b: a + b, "sub": lambda a, b: a - b, "mul": lambda a, b: a * b,
    "max": lambda a, b: np.maximum(a, b) if not (np.isnan(a) or np.isnan(b)) else a + b,
    "min": lambda a, b: np.minimum(a, b) if not (np.isnan(a) or np.isnan(b)) else a + b,
    "eq": lambda a, b: a == b, "ne": lambda a, b: a != b, "lt": lambda a, b: a < b, "le": lambda a, b: a <= b,
    "gt": lambda a, b: a > b, "ge": lambda a, b: a >= b,
    "and": lambda a, b: a & b, "or": lambda a, b: a | b, "xor": lambda a, b: a ^ b,
}


def _tdiv(a, b, dt):
    """lax.div: float division, or integer division truncated toward zero (lax semantics)"""
    if dt == T.F32:
        return a / b
    if dt == T.U32:
        return a // b
    q = a // b                                        # floor division
    fix = ((a % b) != 0) & ((a < 0) != (b < 0))
    return q + fix.astype(tl.int32)


def _trem(a, b, dt):
    """lax.rem: C's remainder (the sign of the dividend)"""
    if dt == T.F32:
        return tl.rem(a, b)
    if dt == T.U32:
        return a % b
    r = a % b                                         # floor modulo
    return tl.where((r != 0) & ((a < 0) != (b < 0)), r - b, r)


def _shift_right_logical(a, b, dt):
    if dt == T.U32:
        return a >> b
    return tl.bitcast_convert_type(tl.bitcast_convert_type(a, tl.uint32) >> _cast(b, T.U32), tl.int32)


def _shift_right_arithmetic(a, b, dt):
    if dt == T.I32:
        return a >> b
    return tl.bitcast_convert_type(tl.bitcast_convert_type(a, tl.int32) >> _cast(b, T.I32), tl.uint32)


def _round(x, method):
    """lax.round: rounding_method 1 (ROUND_TO_NEAREST_EVEN, jnp.round) or 0 (AWAY_FROM_ZERO)"""
    if int(method) == 1:
        return tl.round(x)
    t = tl.sign(x) * tl.floor(tl.abs(x))              # toward zero
    return tl.where(tl.abs(x - t) >= 0.5, t + tl.sign(x), t)


_UNARY = {
    "exp": tl.exp, "log": tl.log, "sin": tl.sin, "cos": tl.cos, "tan": tl.tan, "tanh": tl.tanh, "sqrt": tl.sqrt,
    "log1p": tl.log1p, "expm1": tl.expm1, "atan": tl.arctan, "asin": tl.arcsin, "acos": tl.arccos,
    "sinh": tl.sinh, "cosh": tl.cosh, "asinh": tl.arcsinh, "acosh": tl.arccosh, "atanh": tl.arctanh,
    "erf": tl.erf, "erfc": tl.erfc, "erf_inv": tl.erfinv, "exp2": tl.exp2, "cbrt": tl.cbrt, "logistic": tl.logistic,
    "floor": tl.floor, "ceil": tl.ceil, "abs": tl.abs, "sign": tl.sign, "is_finite": tl.isfinite,
    "stop_gradient": tl.stop_gradient, "square": lambda x: x * x, "neg": lambda x: -x, "not": lambda x: ~x,
    "rsqrt": lambda x: 1.0 / tl.sqrt(x), "lgamma": tl.lgamma, "population_count": tl.population_count,
    "clz": tl.clz,
}
_NP_UNARY = {"population_count": lambda v: bin(int(v) & 0xFFFFFFFF).count("1"),
             "clz": lambda v: 32 - (int(v) & 0xFFFFFFFF).bit_length(),
             "neg": np.negative, "abs": np.abs, "not": np.invert, "floor": np.floor, "ceil": np.ceil,
             "sign": np.sign, "exp": np.exp, "log": np.log, "sqrt": np.sqrt, "square": np.square}


class UnsupportedPrimitive(T.UnsupportedError):
    pass


class _Interp:
    """evaluates jaxprs over traced values; `tok` is the item's tally handle, `names` the tally outputs in invar
    order (the spawn queue as '__spawn__')"""

    def __init__(self, tok):
        self.tok = tok
        self.depth = 0            # > 0 inside the top-level loop's cond / body

    # -------------------------------------------------------------------------------------------- plumbing
    def read(self, env, v):
        if hasattr(v, "val"):
            return _const(v.val, v.aval)
        return env[id(v)]

    def eval(self, jaxpr, consts, args):
        env = {}
        for v, c in zip(getattr(jaxpr, "constvars", ()), consts):
            env[id(v)] = _const(c, v.aval) if not isinstance(c, (T.Var, T.Vec, T.Key)) else c
        if len(args) != len(jaxpr.invars):
            raise T.TraceError(f"tallymap_b200.from_jaxpr: {len(args)} values for {len(jaxpr.invars)} inputs")
        for v, a in zip(jaxpr.invars, args):
            env[id(v)] = a
        for e in jaxpr.eqns:
            ins = [self.read(env, v) for v in e.invars]
            outs = self.apply(e, ins)
            for v, o in zip(e.outvars, outs):
                env[id(v)] = o
        return [self.read(env, v) for v in jaxpr.outvars]

    def call(self, closed, args):
        jaxpr = getattr(closed, "jaxpr", closed)
        consts = getattr(closed, "consts", ())
        return self.eval(jaxpr, list(consts), list(args))

    # -------------------------------------------------------------------------------------------- equations
    def apply(self, e, a):
        p = e.primitive.name
        prm = e.params
        out_aval = e.outvars[0].aval if e.outvars else None
        odt = _dtype(out_aval) if out_aval is not None else None
        idt = _dtype(e.invars[0].aval) if e.invars and not _is_key(e.invars[0].aval) else None
        # values are scalars and vectors (a shape with one dimension above 1 is its row-major vector): a result with
        # two, or an axis operation on an operand of more than one dimension, would be read in the wrong order
        for v in e.outvars:
            shp = tuple(getattr(getattr(v, "aval", None), "shape", ()) or ())
            if sum(int(d) != 1 for d in shp) > 1:
                raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} giving an array of shape {shp} (per-item "
                                           "values are scalars and vectors)")
        if p in _AXIS_OPS:
            for v, x in zip(e.invars, a):
                shp = tuple(getattr(getattr(v, "aval", None), "shape", ()) or ())
                if len(shp) > 1 and not isinstance(x, T.Table):
                    raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} of an array of shape {shp} (vectors "
                                               "only)")

        # calls: interpreted in place
        if p == "custom_lin":
            raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: custom_lin (a linearized custom_vjp) is not lowered "
                                       "inside an item, as the reference's kernel backend refuses it")
        if p in ("pjit", "jit", "closed_call", "core_call", "remat", "remat2", "checkpoint", "custom_jvp_call",
                 "custom_vjp_call", "custom_vjp_call_jaxpr"):
            sub = prm.get("jaxpr") or prm.get("call_jaxpr") or prm.get("fun_jaxpr")
            if sub is None:
                raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} without a jaxpr")
            n = len(getattr(sub, "jaxpr", sub).invars)
            return self.call(sub, a[:n])
        if p == "while":
            return self.while_(e, a)
        if p == "cond":
            return self.cond(e, a)
        if p == "scan":
            return self.scan(e, a)
        if p == "tallymap_emit":
            ref, idx, val = a
            if not isinstance(ref, _TallyRef):
                raise T.TraceError("tallymap_b200.from_jaxpr: an emit into something other than a tally")
            idxs = list(idx) if isinstance(idx, T.Vec) else [idx]
            vals = list(val) if isinstance(val, T.Vec) else [val] * len(idxs)
            for i, v in zip(idxs, vals):
                T._add_flat(self.tok, ref.name, _py(i), _py(v))
            return [ref]
        if p == "tallymap_claim":
            # (a Records output's one-pass append, tallymap/_tally.py:335-351: the slot, then its fields emitted
            # there inside a cond on `ok`; the ordinal operand k is read only by the reference's fill twin)
            ref, when = a[0], a[1]
            if not isinstance(ref, _TallyRef):
                raise T.TraceError("tallymap_b200.from_jaxpr: a claim on something other than a tally")
            return [ref, T._claim(self.tok, ref.name, _py(when))]
        if p == "tallymap_spawn":
            q, when, *leaves = a
            self.tok.spawn(tuple(_py(x) for x in leaves), when=_py(when))
            return [q]
        if p in _RANDOM:
            return _RANDOM[p](self, e, a)
        if p == "threefry2x32":
            k0, k1, x0, x1 = [_py(x) for x in a]
            o = T._cur().emit("threefry", [T._lit(_cast(k0, T.U32)), T._lit(_cast(k1, T.U32)),
                                           T._lit(_cast(x0, T.U32)), T._lit(_cast(x1, T.U32))], [T.U32, T.U32])
            return list(o)

        # shape operations on scalars and small vectors
        if p in ("reshape", "squeeze", "expand_dims", "copy", "copy_p", "optimization_barrier", "broadcast_in_dim",
                 "convert_element_type", "bitcast_convert_type", "reduce_precision"):
            return [self.shape_op(p, e, a, odt)]
        if p == "iota":
            n = int(prm["shape"][0]) if prm.get("shape") else 1
            return [T.Vec(_NP[odt](i) for i in range(n))]
        if p == "slice":
            (x,) = a
            s0, s1 = int(prm["start_indices"][0]), int(prm["limit_indices"][0])
            st = int(prm["strides"][0]) if prm.get("strides") else 1
            return [T.Vec(tuple.__getitem__(x, i) for i in range(s0, s1, st))]
        if p == "gather":
            return [_gather(e, a[0], a[1], prm)]
        if p in _SCATTER:
            return [_scatter(p, e, a[0], a[1], a[2], prm)]
        if p == "dynamic_slice" and isinstance(a[0], T.Table) and len(a[0].shape) == 2:
            return [_table_slice(a[0], [_py(v) for v in a[1:3]], [int(d) for d in prm["slice_sizes"]])]
        if p == "dynamic_slice":
            x, i = a[0], a[1]
            size = int(prm["slice_sizes"][0])
            n = len(x)
            if isinstance(i, np.generic):
                s = int(np.clip(int(i), 0, n - size))
                return [T.Vec(tuple.__getitem__(x, j) for j in range(s, s + size))]
            if size != 1:
                raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: dynamic_slice of more than one element at a "
                                           "traced index")
            return [T.Vec([_index_clamped(x, _py(i))])]
        if p == "concatenate":
            out = []
            for x in a:
                out += list(x) if isinstance(x, T.Vec) else [x]
            return [T.Vec(out)]
        if p in ("reduce_sum", "reduce_max", "reduce_min", "reduce_and", "reduce_or", "reduce_prod", "argmax",
                 "argmin"):
            (x,) = a
            if _isconst(x):
                f = {"reduce_sum": np.sum, "reduce_max": np.max, "reduce_min": np.min, "reduce_and": np.all,
                     "reduce_or": np.any, "reduce_prod": np.prod, "argmax": np.argmax, "argmin": np.argmin}[p]
                return [_NP[odt](f(np.array(list(x))))]
            f = {"reduce_sum": tl.sum, "reduce_max": tl.max, "reduce_min": tl.min, "reduce_and": tl.all,
                 "reduce_or": tl.any, "reduce_prod": tl.prod, "argmax": tl.argmax, "argmin": tl.argmin}[p]
            return [f(_py(x))]
        if p == "split":
            # (jnp.split / lax.split of a vector: consecutive pieces of the given sizes)
            (x,) = a
            xs, out, o = list(x) if isinstance(x, T.Vec) else [x], [], 0
            for n_ in prm["sizes"]:
                out.append(T.Vec(xs[o:o + int(n_)]))
                o += int(n_)
            return out

        if p == "sort":
            return _sort(a, int(prm.get("num_keys", 1)), tuple(e.invars[0].aval.shape))
        if p == "rev":
            (x,) = a
            return [T.Vec(reversed(list(x))) if isinstance(x, T.Vec) else x]
        if p == "transpose":
            if tuple(prm.get("permutation", ())) not in ((), (0,)):
                raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: transpose of more than one dimension")
            return [a[0]]
        if p == "pad":
            return [_pad(a[0], a[1], prm["padding_config"])]
        if p in _CUM:
            return [_cumulative(p, a[0], bool(prm.get("reverse", False)), odt)]
        if p == "dot_general":
            return [_dot_general(e, a[0], a[1], prm["dimension_numbers"], odt)]
        if p == "dynamic_update_slice":
            return [_dynamic_update_slice(a[0], a[1], a[2] if len(a) > 2 else np.int32(0))]
        if p == "iota_2x32_shape":
            shape = tuple(int(d) for d in prm["shape"])
            n = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if shape == ():
                return [np.uint32(0), np.uint32(0)]
            return [T.Vec([np.uint32(0)] * n), T.Vec(np.uint32(i) for i in range(n))]
        if p == "platform_index":
            return [np.int32(_platform_index(prm["platforms"]))]

        # elementwise (on scalars and vectors: a result with two dimensions above 1 would be a broadcast matrix)
        if out_aval is not None and sum(int(d) != 1 for d in out_aval.shape) > 1:
            raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} of arrays of shape {tuple(out_aval.shape)} "
                                       "is not lowered")
        if p == "select_n":
            which, *cases = a
            if _isconst(which) and not isinstance(which, T.Vec):
                return [cases[int(which)]]
            if len(cases) == 2:
                c = _py(which)
                if _dtype(e.invars[0].aval) != T.BOOL:
                    c = c != 0
                return [tl.where(c, _py(cases[1]), _py(cases[0]))]
            r = _py(cases[0])
            for j in range(1, len(cases)):
                r = tl.where(_py(which) == j, _py(cases[j]), r)
            return [r]
        if p == "clamp":
            lo, x, hi = a
            if all(_isconst(v) for v in a):
                return [_fold(lambda l, x_, h: np.minimum(np.maximum(x_, l), h), [lo, x, hi], odt)]
            return [tl.minimum(tl.maximum(_py(x), _py(lo)), _py(hi))]
        if p == "integer_pow":
            (x,) = a
            y = int(prm["y"])
            if _isconst(x):
                return [_fold(lambda v: v ** y if y >= 0 else 1 / v ** -y, [x], odt)]
            return [_vec(lambda v: T.int_pow(v, y), _py(x))]
        if p == "round":
            (x,) = a
            return [_vec(lambda v: _round(v, prm.get("rounding_method", 0)), _py(x))]
        if p in _UNARY:
            (x,) = a
            if _isconst(x) and p in _NP_UNARY:
                return [_fold(_NP_UNARY[p], [x], odt)]
            if _isconst(x):
                raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} of a constant is not folded")
            return [_UNARY[p](_py(x))]
        if p in ("div", "rem", "pow", "atan2", "nextafter", "shift_left", "shift_right_logical",
                 "shift_right_arithmetic") or p in _FOLD2:
            x, y = a
            if _isconst(x) and _isconst(y):
                return [self.fold2(p, x, y, idt, odt)]
            x, y = _py(x), _py(y)
            if p == "div":
                return [_tdiv(x, y, idt)]
            if p == "rem":
                return [_trem(x, y, idt)]
            if p == "pow":
                return [tl.power(x, y)]
            if p == "atan2":
                return [tl.arctan2(x, y)]
            if p == "nextafter":
                return [tl.nextafter(x, y)]
            if p == "shift_left":
                return [x << y]
            if p == "shift_right_logical":
                return [_shift_right_logical(x, y, idt)]
            if p == "shift_right_arithmetic":
                return [_shift_right_arithmetic(x, y, idt)]
            # (a constant operand on either side: Python's reflected operators reach the traced operand's method)
            ops = {"add": lambda: x + y, "sub": lambda: x - y, "mul": lambda: x * y,
                   "max": lambda: tl.maximum(x, y), "min": lambda: tl.minimum(x, y),
                   "eq": lambda: x == y, "ne": lambda: x != y, "lt": lambda: x < y, "le": lambda: x <= y,
                   "gt": lambda: x > y, "ge": lambda: x >= y, "and": lambda: x & y, "or": lambda: x | y,
                   "xor": lambda: x ^ y}
            return [ops[p]()]
        raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: primitive {p!r} is not lowered")

    def fold2(self, p, x, y, idt, odt):
        if p == "div":
            return _fold(lambda a, b: a / b if idt == T.F32 else _np_trunc_div(a, b), [x, y], odt)
        if p == "rem":
            return _fold(lambda a, b: np.fmod(a, b) if idt == T.F32 else _np_trunc_rem(a, b), [x, y], odt)
        if p == "pow":
            return _fold(lambda a, b: np.float32(np.float64(a) ** np.float64(b)), [x, y], odt)
        if p == "shift_left":
            return _fold(lambda a, b: 0 if int(b) >= 32 else (int(a) << int(b)) & 0xFFFFFFFF, [x, y], None) \
                if odt == T.U32 else _fold(lambda a, b: _cast(np.uint32(0 if int(b) >= 32 else
                                                                        (int(a) << int(b)) & 0xFFFFFFFF), T.I32),
                                           [x, y], odt)
        if p in ("shift_right_logical", "shift_right_arithmetic"):
            raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} of constants is not folded")
        if p in _FOLD2:
            return _fold(_FOLD2[p], [x, y], odt)
        raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} of constants is not folded")

    def shape_op(self, p, e, a, odt):
        x = a[0]
        shape = tuple(e.outvars[0].aval.shape)
        if p == "convert_element_type":
            return _cast(x, _DT[str(e.params["new_dtype"])] if str(e.params["new_dtype"]) in _DT else odt)
        if p == "bitcast_convert_type":
            if _isconst(x):
                return _fold(lambda v: np.array([v]).view(_NP[odt])[0], [x], odt)
            return tl.bitcast_convert_type(_py(x), {T.F32: tl.float32, T.I32: tl.int32, T.U32: tl.uint32}[odt])
        if p == "reduce_precision":
            return x
        n = int(np.prod(shape)) if shape else 1
        if shape == () or n == 1 and len(shape) <= 1 and not isinstance(x, T.Vec):
            if isinstance(x, T.Vec):
                if len(x) != 1:
                    raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} of {len(x)} elements to a scalar")
                x = tuple.__getitem__(x, 0)
            return T.Vec([x]) if shape == (1,) else x
        if sum(d != 1 for d in shape) > 1:
            raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: arrays of shape {shape} are not lowered")
        # (a shape with at most one dimension above 1, as (k, 1) gather indices: its row-major elements)
        if isinstance(x, T.Vec):
            if len(x) == n:
                return x
            if len(x) == 1:
                return T.Vec([tuple.__getitem__(x, 0)] * n)
            raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: {p} from {len(x)} to {n} elements")
        return T.Vec([x] * n)

    # -------------------------------------------------------------------------------------------- control flow
    def while_(self, e, a):
        prm = e.params
        cn, bn = int(prm["cond_nconsts"]), int(prm["body_nconsts"])
        cconst, bconst, init = a[:cn], a[cn:cn + bn], a[cn + bn:]
        self.depth += 1
        try:
            flat = [(_py(x) if not isinstance(x, T.Vec) else _py(x)) for x in init]

            def cond_fun(c):
                return _py(self.call(prm["cond_jaxpr"], list(cconst) + list(c))[0])

            def body_fun(c):
                return tuple(_py(x) for x in self.call(prm["body_jaxpr"], list(bconst) + list(c)))
            out = tl.while_loop(cond_fun, body_fun, tuple(flat))
        finally:
            self.depth -= 1
        return list(out)

    def cond(self, e, a):
        idx, *ops = a
        branches = e.params["branches"]
        fns = [(lambda br: (lambda *xs: tuple(_py(v) for v in self.call(br, list(xs)))))(br) for br in branches]
        if _isconst(idx):
            return list(fns[int(np.clip(int(idx), 0, len(fns) - 1))](*[_py(x) for x in ops]))
        i = _py(idx)
        if _dtype(e.invars[0].aval) == T.BOOL:
            i = i.astype(tl.int32)
        r = tl.switch(i, fns, *[_py(x) for x in ops])
        return list(r) if isinstance(r, tuple) else [r]


    def scan(self, e, a):
        """lax.scan of a static length (and jax's fori_loop of static bounds, which it writes as a scan): unrolled
        like tallymap_b200.lang.scan; the scanned inputs and stacked outputs are vectors of scalars (a tally may
        ride in the carry: t.add inside the body)"""
        prm = e.params
        nc, nk, n = int(prm["num_consts"]), int(prm["num_carry"]), int(prm["length"])
        if n > 4096:
            raise T.UnsupportedError("tallymap_b200.from_jaxpr: a scan of more than 4096 steps (unrolled)")
        consts, carry, xs = list(a[:nc]), list(a[nc:nc + nk]), list(a[nc + nk:])
        for x in xs:
            if not isinstance(x, T.Vec) or len(x) != n:
                raise T.UnsupportedError("tallymap_b200.from_jaxpr: a scanned input that is not a vector of the "
                                         "scan's length")
        ny = len(e.outvars) - nk
        ys = [[None] * n for _ in range(ny)]
        for i in (range(n - 1, -1, -1) if prm.get("reverse") else range(n)):
            out = self.call(prm["jaxpr"], consts + carry + [tuple.__getitem__(x, i) for x in xs])
            carry = list(out[:nk])
            for j, y in enumerate(out[nk:]):
                if isinstance(y, (T.Vec, T.TallyToken)):
                    raise T.UnsupportedError("tallymap_b200.from_jaxpr: a scan's stacked output is a vector of "
                                             "scalars (per-item arrays have one dimension)")
                ys[j][i] = y
        return carry + [T.Vec(y) for y in ys]


_CUM = {"cumsum": (np.add, lambda u, w: u + w), "cumprod": (np.multiply, lambda u, w: u * w),
        "cummax": (np.maximum, tl.maximum), "cummin": (np.minimum, tl.minimum)}


def _arith(f_np, f_tl, u, w, dt=None):
    """one binary step on constants (numpy, in the operands' dtype) or traced values"""
    if isinstance(u, np.generic) and isinstance(w, np.generic):
        with np.errstate(all="ignore"):
            r = f_np(u, w)
        return _NP[dt](r) if dt is not None else r
    return f_tl(_py(u), _py(w))


def _cumulative(p, x, reverse, dt):
    """lax.cumsum / cumprod / cummax / cummin of a vector: the running value element by element, from the last
    element when reverse (the reference's sequential loop, backends/kernel/op_table.py:930-961)"""
    xs = list(x) if isinstance(x, T.Vec) else [x]
    f_np, f_tl = _CUM[p]
    out, acc = [None] * len(xs), None
    for i in (range(len(xs) - 1, -1, -1) if reverse else range(len(xs))):
        acc = xs[i] if acc is None else _arith(f_np, f_tl, acc, xs[i], dt)
        out[i] = acc
    return T.Vec(out)


def _pad(x, v, config):
    """lax.pad of a vector by padding_config ((lo, hi, interior),): interior copies of v between elements, then lo /
    hi copies at the ends (a negative lo / hi crops)"""
    ((lo, hi, interior),) = [tuple(int(c) for c in cfg) for cfg in config]
    xs = list(x) if isinstance(x, T.Vec) else [x]
    out = []
    for i, y in enumerate(xs):
        if i:
            out += [v] * interior
        out.append(y)
    out = [v] * max(lo, 0) + out[max(-lo, 0):]
    out = out + [v] * max(hi, 0) if hi >= 0 else out[:len(out) + hi]
    return T.Vec(out)


def _dot_general(e, x, y, dimension_numbers, dt):
    """lax.dot_general over row-major flattened operands (their shapes from the avals): per output element, a sum
    from the literal zero in contraction order, acc = acc + x * y with no fused multiply-add (the reference's rule,
    backends/kernel/op_table.py:964-1003)"""
    (lc, rc), (lb, rb) = dimension_numbers
    ls, rs = tuple(e.invars[0].aval.shape), tuple(e.invars[1].aval.shape)
    xs = list(x) if isinstance(x, T.Vec) else [x]
    ys = list(y) if isinstance(y, T.Vec) else [y]
    lf = [d for d in range(len(ls)) if d not in lc and d not in lb]
    rf = [d for d in range(len(rs)) if d not in rc and d not in rb]
    bshape = tuple(ls[d] for d in lb)
    cshape = tuple(ls[d] for d in lc)
    oshape = bshape + tuple(ls[d] for d in lf) + tuple(rs[d] for d in rf)
    if len(oshape) > 1:
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a dot_general whose result has more than one dimension")
    out = []
    for oidx in np.ndindex(*oshape):
        bi, li_, ri_ = oidx[:len(lb)], oidx[len(lb):len(lb) + len(lf)], oidx[len(lb) + len(lf):]
        acc = _NP[dt](0)
        for cidx in np.ndindex(*cshape):
            li, ri = [0] * len(ls), [0] * len(rs)
            for j, d in enumerate(lb):
                li[d] = bi[j]
            for j, d in enumerate(rb):
                ri[d] = bi[j]
            for j, d in enumerate(lf):
                li[d] = li_[j]
            for j, d in enumerate(rf):
                ri[d] = ri_[j]
            for j, (dl, dr) in enumerate(zip(lc, rc)):
                li[dl] = cidx[j]
                ri[dr] = cidx[j]
            u = xs[int(np.ravel_multi_index(li, ls))] if ls else xs[0]
            w = ys[int(np.ravel_multi_index(ri, rs))] if rs else ys[0]
            acc = _arith(np.add, lambda s_, t_: s_ + t_, acc, _arith(np.multiply, lambda s_, t_: s_ * t_, u, w, dt), dt)
        out.append(acc)
    return out[0] if oshape == () else T.Vec(out)


def _dynamic_update_slice(x, upd, start):
    """lax.dynamic_update_slice of a vector: the update written from the start index clamped so that it fits; a
    traced start selects per element"""
    xs = list(x) if isinstance(x, T.Vec) else [x]
    us = list(upd) if isinstance(upd, T.Vec) else [upd]
    n, m = len(xs), len(us)
    if isinstance(start, T.Vec):
        start = tuple.__getitem__(start, 0)
    if isinstance(start, (np.generic, int)):
        s = int(np.clip(int(start), 0, n - m))
        return T.Vec(xs[:s] + us + xs[s + m:])
    s = tl.clip(_py(start), 0, n - m)
    out = []
    for j in range(n):
        r = _py(xs[j])
        for i in range(m):
            if 0 <= j - i <= n - m:
                r = tl.where(s == j - i, _py(us[i]), r)
        out.append(r)
    return T.Vec(out)


def _sort(ops, num_keys, shape):
    """lax.sort of vectors on the first operand (jnp.sort; jnp.argsort sorts (x, iota)): stable, ascending in
    lax.sort's total order -- NaNs last, -0 equal to +0 -- the other operands permuted with it (the reference's
    stable insertion sort gives the same order, backends/kernel/op_table.py:1006-1044)"""
    if num_keys != 1:
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a sort on more than one key")
    if len(shape) > 1:
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a sort of more than one dimension")
    if shape == () or len(ops[0]) <= 1:
        return list(ops)
    if all(_isconst(x) for x in ops):
        k = np.array(list(ops[0]))
        order = np.argsort(np.where(k == 0, np.zeros_like(k), k), kind="stable")
        return [T.Vec(list(x)[i] for i in order) for x in ops]
    v, rest = tl._sort_network(_py(ops[0]), [_py(x) for x in ops[1:]])
    return [v] + rest


def _mode(mode):
    """a gather's index mode (GatherScatterMode): 'fill' (out-of-range starts read the fill value), else 'clip'
    (clip and promise_in_bounds: the start clamped so the slice fits, XLA's gather)"""
    m = str(mode).upper()
    if "ONE_HOT" in m:
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a one-hot gather")
    return "fill" if ("FILL" in m or "DROP" in m) else "clip"


def _read(x, idx, shape):
    """operand x (a Vec, a table or a scalar) at the in-range multi-index idx (static ints or traced int32)"""
    if isinstance(x, T.Table):
        return x[tuple(idx)] if len(idx) > 1 else x[idx[0]]
    if not isinstance(x, T.Vec):
        return x
    flat = None
    for i, n in zip(idx, shape):
        flat = i if flat is None else flat * n + i
    if isinstance(flat, (int, np.integer)):
        return tuple.__getitem__(x, int(flat))
    return x[flat]


def _table_slice(tab, starts, sizes):
    """lax.dynamic_slice of a 2-D table: one element (sizes (1, 1)) or one whole row (sizes (1, m)), the starts
    clamped so the slice fits"""
    (n, m), (s0, s1) = tab.shape, sizes
    if s0 != 1 or s1 not in (1, m):
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a dynamic_slice of a table other than an element or "
                                   "a row")
    i = _clamp_start(starts[0], n - 1)
    if s1 == m:
        return T.Vec(tab[i]) if m > 1 else T.Vec([tab[i, 0]])
    return T.Vec([tab[i, _clamp_start(starts[1], m - 1)]])


def _clamp_start(i, hi):
    if isinstance(i, (int, np.integer)):
        return int(np.clip(int(i), 0, hi))
    return tl.clip(i, 0, hi)


_SCATTER = {"scatter": (None, lambda o, u: u), "scatter-add": (np.add, lambda o, u: o + u),
            "scatter_add": (np.add, lambda o, u: o + u), "scatter-mul": (np.multiply, lambda o, u: o * u),
            "scatter_mul": (np.multiply, lambda o, u: o * u), "scatter-min": (np.minimum, tl.minimum),
            "scatter_min": (np.minimum, tl.minimum), "scatter-max": (np.maximum, tl.maximum),
            "scatter_max": (np.maximum, tl.maximum)}


def _scatter(p, e, x, idx, upd, prm):
    """lax.scatter / scatter-add / -mul / -min / -max into a vector, as x.at[i].set / add / multiply / min / max
    write it: each update (the updates in order, one element per index vector of the indices' last axis) combined
    into the element its index names; an out-of-range index drops its update (mode fill_or_drop, jax's default for
    scatters) or is clamped (clip, promise_in_bounds); a traced index selects per element"""
    dn = prm["dimension_numbers"]
    oshape = tuple(e.invars[0].aval.shape)
    if len(oshape) != 1 or tuple(getattr(dn, "operand_batching_dims", ()) or ()):
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a scatter into anything but a vector")
    if tuple(dn.update_window_dims) or tuple(dn.inserted_window_dims) != (0,):
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a scatter of windows (element scatters only)")
    n = oshape[0]
    clip = _mode(prm.get("mode")) == "clip" and "FILL" not in str(prm.get("mode")).upper()
    f_np, f_tl = _SCATTER[p]
    xs = list(x) if isinstance(x, T.Vec) else [x]
    ivals = list(idx) if isinstance(idx, T.Vec) else [idx]
    uvals = list(upd) if isinstance(upd, T.Vec) else [upd] * len(ivals)
    for i, u in zip(ivals, uvals):
        i = _py(i)
        if isinstance(i, int):
            if not 0 <= i < n:
                if not clip:
                    continue
                i = int(np.clip(i, 0, n - 1))
            xs[i] = u if f_np is None else _arith(f_np, f_tl, xs[i], u)
            continue
        i = tl.clip(i, 0, n - 1) if clip else i
        for j in range(n):
            new_j = u if f_np is None else _arith(f_np, f_tl, xs[j], u)
            xs[j] = tl.where(i == j, _py(new_j), _py(xs[j]))
    return T.Vec(xs)


def _gather(e, x, idx, prm):
    """lax.gather in the forms jnp indexing writes for 1-D and 2-D operands: each index vector (the last axis of
    the indices) starts a slice of `slice_sizes`, the collapsed dimensions dropped, the rest kept; the result at
    most one-dimensional.  Out-of-range starts are clamped so the slice fits (mode clip / promise_in_bounds), or read
    the fill value (mode fill: NaN for floats, the type's minimum for int32 unless fill_value is given) -- the
    reference's gather rule, backends/kernel/op_table.py:1085-1180"""
    dn = prm["dimension_numbers"]
    oshape = tuple(e.invars[0].aval.shape)
    ishape = tuple(e.invars[1].aval.shape)
    sizes = [int(d) for d in prm["slice_sizes"]]
    if tuple(getattr(dn, "operand_batching_dims", ()) or ()):
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a batched gather")
    smap = [int(d) for d in dn.start_index_map]
    collapsed = set(int(d) for d in dn.collapsed_slice_dims)
    K = ishape[-1] if ishape else 1
    nb = int(np.prod(ishape[:-1], dtype=np.int64)) if len(ishape) > 1 else 1
    kept = [d for d in range(len(oshape)) if d not in collapsed]
    ksize = [sizes[d] for d in kept]
    if len(ishape) > 2 or (nb > 1 and any(k > 1 for k in ksize)) or sum(k > 1 for k in ksize) > 1:
        raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: a gather whose result has more than one dimension")
    mode = _mode(prm.get("mode"))
    iv = list(idx) if isinstance(idx, T.Vec) else [idx]
    odt = _dtype(e.outvars[0].aval)
    fill = prm.get("fill_value")
    if fill is None:
        fill = float("nan") if odt == T.F32 else -2 ** 31
    out = []
    for b in range(nb):
        starts, ok = [0] * len(oshape), None
        for q, d in enumerate(smap):
            s_ = _py(iv[b * K + q])
            hi = oshape[d] - sizes[d]
            if mode == "fill" and not isinstance(s_, int):
                inr = (s_ >= 0) & (s_ <= hi)
                ok = inr if ok is None else ok & inr
            elif mode == "fill" and not 0 <= s_ <= hi:
                ok = False
            starts[d] = _clamp_start(s_, hi)
        for off in np.ndindex(*[sizes[d] for d in range(len(oshape))]):
            pos = [starts[d] + off[d] if off[d] else starts[d] for d in range(len(oshape))]
            v = _read(x, pos, oshape)
            if ok is False:
                v = _NP[odt](fill) if odt in _NP else fill
            elif ok is not None:
                v = tl.where(ok, _py(v), fill if odt == T.F32 else int(fill))
            out.append(v)
    shape = tuple(e.outvars[0].aval.shape)
    return out[0] if shape == () or (len(out) == 1 and not shape) else T.Vec(out)


def _platform_index(platforms):
    """lax.platform_dependent's branch index for a CUDA device: the branch naming cuda / gpu, else the default
    (the reference's rule, backends/kernel/op_table.py:1650-1659)"""
    plats = list(platforms)
    for i, ps in enumerate(plats):
        if ps is not None and any(x in ("cuda", "gpu") for x in ps):
            return i
    for i, ps in enumerate(plats):
        if ps is None:
            return i
    raise UnsupportedPrimitive("tallymap_b200.from_jaxpr: lax.platform_dependent without a cuda / gpu branch or a "
                               "default")


_AXIS_OPS = frozenset(("cumsum", "cumprod", "cummax", "cummin", "reduce_sum", "reduce_max", "reduce_min",
                       "reduce_and", "reduce_or", "reduce_prod", "argmax", "argmin", "concatenate", "sort", "rev",
                       "pad", "split", "slice", "dynamic_update_slice"))

_STRUCTURAL = ("pjit", "jit", "closed_call", "core_call", "remat", "remat2", "checkpoint", "custom_jvp_call",
               "custom_vjp_call", "custom_vjp_call_jaxpr", "while", "cond", "scan", "tallymap_emit", "tallymap_claim",
               "tallymap_spawn", "threefry2x32", "reshape", "squeeze", "expand_dims", "copy", "copy_p",
               "optimization_barrier", "broadcast_in_dim", "convert_element_type", "bitcast_convert_type",
               "reduce_precision", "iota", "slice", "gather", "dynamic_slice", "dynamic_update_slice", "concatenate",
               "reduce_sum", "reduce_max", "reduce_min", "reduce_and", "reduce_or", "reduce_prod", "split", "argmax",
               "argmin", "sort", "rev", "transpose", "pad", "dot_general", "iota_2x32_shape", "platform_index",
               "select_n", "clamp", "scatter", "scatter-add", "scatter_add", "scatter-mul", "scatter_mul",
               "scatter-min", "scatter_min", "scatter-max", "scatter_max", "integer_pow", "round", "div", "rem", "pow",
               "atan2", "nextafter", "shift_left", "shift_right_logical", "shift_right_arithmetic")


def supported_primitives():
    """the names of the jaxpr primitives this front end lowers, sorted (tallymap.supported_primitives)"""
    return sorted(set(_STRUCTURAL) | set(_CUM) | set(_UNARY) | set(_FOLD2) | set(_RANDOM))


def _vec(f, x):
    return T.Vec(f(v) for v in x) if isinstance(x, T.Vec) else f(x)


def _index_clamped(x, i):
    n = len(x)
    i = tl.clip(i, 0, n - 1) if not isinstance(i, int) else int(np.clip(i, 0, n - 1))
    return tuple.__getitem__(x, i) if isinstance(i, int) else x[i]


# ------------------------------------------------------------------------------------------------ jax.random
def _key_of(x):
    if isinstance(x, T.Key):
        return x
    if isinstance(x, T.Vec) and len(x) == 2:
        return T.Key(T._lit(_cast(tuple.__getitem__(x, 0), T.U32)), T._lit(_cast(tuple.__getitem__(x, 1), T.U32)))
    raise T.TraceError("tallymap_b200.from_jaxpr: a PRNG key was expected")


def _r_seed(it, e, a):
    (s,) = a
    s = _py(s)
    seed = T.Lit(int(s) & 0xFFFFFFFF, T.U32) if isinstance(s, int) else _cast(s, T.U32)
    return [T.Key(T.Lit(0, T.U32) if not isinstance(s, int) or s >= 0 else T.Lit(0xFFFFFFFF, T.U32), seed)]


def _threefry_impl(name):
    """a key implementation this front end computes: threefry2x32 (jax's default, printed "fry"); another (rbg,
    unsafe_rbg) would give other bits, so it raises instead"""
    n = str(name).lower()
    if "fry" not in n:
        raise UnsupportedPrimitive(f"tallymap_b200.from_jaxpr: PRNG implementation {name!r} (threefry2x32 only)")


def _r_wrap(it, e, a):
    _threefry_impl(e.params.get("impl", "fry"))
    return [_key_of(a[0])]


def _r_unwrap(it, e, a):
    k = _key_of(a[0])
    return [T.Vec([k.a, k.b])]


def _r_fold_in(it, e, a):
    k, m = a
    return [tl.random.fold_in(_key_of(k), _py(m))]


def _r_bits(it, e, a):
    if int(e.params.get("bit_width", 32)) != 32:
        raise T.UnsupportedError("tallymap_b200.from_jaxpr: random_bits of a width other than 32")
    shape = tuple(e.params.get("shape", ()))
    if len(shape) > 1:
        raise T.UnsupportedError(f"tallymap_b200.from_jaxpr: random_bits of shape {shape}")
    return [tl.random.bits(_key_of(a[0]), shape if shape else ())]


def _r_split(it, e, a):
    shape = tuple(e.params.get("shape", (2,)))
    n = int(np.prod(shape))
    return [_KeyVec(tl.random.split(_key_of(a[0]), n))]


class _KeyVec(tuple):
    """the keys of random_split (indexed by the slicing that follows it)"""


_RANDOM = {"random_seed": _r_seed, "random_wrap": _r_wrap, "random_unwrap": _r_unwrap, "random_fold_in": _r_fold_in,
           "random_bits": _r_bits, "random_split": _r_split, "random_key_data": _r_unwrap,
           "random_clone": lambda it, e, a: [a[0]]}


# ------------------------------------------------------------------------------------------------ the item
def item_function(closed, tallies, n_per_item):
    """-> (fn, in_specs): fn(t, *leaves) interprets the item jaxpr `closed` (invars [tallies] + [per-item leaves] +
    [broadcast leaves], outvars [tallies] + [per-item results]); tallies: the names of its tally inputs in order
    (a spawn queue token named '__spawn__'); in_specs: trace_item's spec of each leaf."""
    jaxpr = getattr(closed, "jaxpr", closed)
    nT = len(tallies)
    specs = [aval_spec(v.aval, j < n_per_item) for j, v in enumerate(jaxpr.invars[nT:])]

    def fn(t, *leaves):
        it = _Interp(t)
        refs = [_TallyRef(t, name) for name in tallies]
        vals = []
        for x, v in zip(leaves, jaxpr.invars[nT:]):
            if isinstance(x, T.Key) and not _is_key(v.aval):
                x = T.Vec([x.a, x.b])            # raw uint32[2] key data, as the jaxpr reads it
            vals.append(x)
        outs = it.call(closed, refs + vals)
        for o, name in zip(outs[:nT], tallies):
            if not (isinstance(o, _TallyRef) and o.name == name):
                raise T.TallyError(f"tallymap_b200.from_jaxpr: tally output {name!r} is not the tally it received")
        res = []
        for o in outs[nT:]:
            if isinstance(o, (T.Key, _KeyVec)):
                raise T.UnsupportedError("tallymap_b200.from_jaxpr: a key as a per-item result")
            if isinstance(o, np.bool_):
                o = bool(o)
            res.append(_py(o) if not isinstance(o, T.Vec) else _py(o))
        return (t,) + tuple(res)
    return fn, specs


# ------------------------------------------------------------------------------------------------ backend entry
# lowered programs by (jaxpr object, options), the jaxpr kept alive beside its program so that its id cannot be reused
# by another jaxpr while the entry exists; the least recently used entries beyond PROGRAMS_MAX are dropped
_PROGRAMS = collections.OrderedDict()
PROGRAMS_MAX = 64


def run(p, pi, bc, target="cuda", cuda_math="approx", schedule="item", ndev=1, min_blocks_per_sm=None, **_):
    """The reference's backend entry (tallymap/backends/kernel/__init__.py:135-185) over a reference ItemProgram
    `p` (p.cj: the item's closed jaxpr after retrace(cap) -- its loop counter and `truncated` result included --;
    p.tallies: TSpec-like entries with .name, .kind ('sum' / 'spawn'), .dtype, .size or .shape; p.nP / p.nB: the
    per-item / broadcast leaf counts; p.spawn: a Queue-like with .capacity or None).  pi / bc: the per-item and
    broadcast leaves (keys as uint32[..., 2] key data, as KB.run passes them).  -> [sum tallies] + [stats int32[5]]
    + [per-item results], as torch tensors on the current CUDA device, in the reference's order.

    The jaxpr's own loop counter enforces max_steps (retrace(cap)); the backend's runtime ceiling is set above it.
    target must be 'cuda' (no CPU fallback); cuda_math / min_blocks_per_sm are the lowering's options (an unknown
    cuda_math raises); schedule is accepted for signature compatibility (the runtime refills at step granularity
    either way); ndev > 1 partitions are the caller's (each rank runs its own items, tallymap_b200.parallel)."""
    if target != "cuda":
        raise NotImplementedError("tallymap_b200 runs on CUDA devices only (no CPU fallback)")
    from . import api
    from . import backend as B
    import torch
    sums = [s for s in p.tallies if getattr(s, "kind", "sum") == "sum"]
    names = [s.name for s in p.tallies]
    key = (id(p.cj), cuda_math, min_blocks_per_sm)
    ent = _PROGRAMS.get(key)
    mf = ent[1] if ent is not None and ent[0] is p.cj else None
    if mf is not None:
        _PROGRAMS.move_to_end(key)
    if mf is None:
        fn, _ = item_function(p.cj, names, int(p.nP))
        outputs = {}
        for s in sums:
            shape = tuple(getattr(s, "shape", None) or (int(s.size),))
            outputs[s.name] = api.Sum(shape, torch.int32 if "int" in str(s.dtype) else torch.float32)
        spawn = getattr(p, "spawn", None)
        opts = {"cuda_math": "ieee" if cuda_math is None else cuda_math}
        if min_blocks_per_sm is not None:
            opts["min_blocks_per_sm"] = int(min_blocks_per_sm)
        # the jaxpr's own loop counter caps the loop (retrace(cap)); the runtime's ceiling sits above it
        mf = api.vmap(fn, outputs=outputs, in_axes=(0,) * int(p.nP) + (None,) * int(p.nB), max_steps=2 ** 31 - 1,
                      spawn=api.Queue(int(spawn.capacity)) if spawn is not None else None, **opts)
        _PROGRAMS[key] = (p.cj, mf)
        while len(_PROGRAMS) > PROGRAMS_MAX:
            _PROGRAMS.popitem(last=False)
    L = mf.lowered(tuple(pi) + tuple(bc))
    spawn = getattr(p, "spawn", None)
    out = B.run(L.fwd, list(pi), list(bc), consts=(mf.max_steps,),
                queue=int(spawn.capacity) if spawn is not None else None)
    nt = len(L.fwd.tallies)
    stats = out[nt]
    ys = out[nt + 1:][:L.n_results]
    yav = [v.aval for v in getattr(p.cj, "jaxpr", p.cj).outvars[len(p.tallies):]]
    per = [y.bool() if str(a.dtype) == "bool" else y for y, a in zip(ys, yav)]
    return list(out[:nt]) + [stats] + per
