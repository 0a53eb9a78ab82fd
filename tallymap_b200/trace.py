"""A scalar tracer for item functions: the stand-in for the jaxpr the reference's kernel backend lowers
(tallymap/backends/kernel/kernel.py:428-451 `function()`, codegen.py:494-980 `Emitter`).

An item is a Python function of (t, *per_item, *broadcast) written against `tallymap_b200.lang` (a jnp / jax.random /
lax.while_loop / Tally.add subset).  Tracing it with placeholder values records a flat list of scalar equations, a
jaxpr-like IR:

    Eqn(prim, ins, outs, params)   ins: Var or Lit; outs: Var

with dtypes f32, i32, u32 and bool.  The item's first top-level while loop is its stepping loop (the reference's
step schedule splits an item the same way: backends/kernel/kernel.py:225-295 into pre / cond / body / post), so a
traced item is four equation lists: `pre` (before the loop), `cond` and `body` (on the loop carry), `post` (after
it).  Any other while loop -- inside the stepping loop, inside a cond branch, after it -- is ONE equation "while"
holding its own condition and body lists (an inner loop; _nested_while).

Emits (`t.add(name, index, value)`) are equations of prim "emit"; a tuple index is flattened row-major with any
out-of-range coordinate giving -1 (tallymap/_tally.py:248-282), which the lowering drops and counts in stats[4].
"""
import dataclasses
import itertools

F32, I32, U32, BOOL = "f32", "i32", "u32", "bool"
TF32, TI32 = "tf32", "ti32"          # a broadcast table of float32 / int32 (read by gather)
TABLE_ELT = {TF32: F32, TI32: I32}
_CTX = []


class TraceError(TypeError):
    """an item function this tracer cannot trace (a type error in the item, or a construct outside the language)"""


class UnsupportedError(TraceError, NotImplementedError):
    """a valid item whose construct the kernel backend does not lower (tallymap/_api.py:198 UnsupportedError, a
    NotImplementedError there too); never a fallback: nothing else runs the item"""


class TallyError(TraceError):
    """the tally handle used in a way a write-through tally cannot honour: read as a value, dropped from the carry,
    or moved to another carry position (tallymap/_rewrite.py:31 TallyError)"""


@dataclasses.dataclass(frozen=True)
class Lit:
    value: object
    dtype: str


@dataclasses.dataclass
class Eqn:
    prim: str
    ins: list
    outs: list
    params: dict


class Trace:
    """one traced function body (a list of equations) and the variable counter it shares with nested bodies"""

    def __init__(self, ids=None):
        self.eqns = []
        self.ids = ids if ids is not None else itertools.count()

    def new(self, dtype):
        return Var(self, next(self.ids), dtype)

    def emit(self, prim, ins, out_dtypes, **params):
        outs = [self.new(d) for d in out_dtypes]
        self.eqns.append(Eqn(prim, list(ins), outs, params))
        return outs


def _cur():
    if not _CTX:
        raise TraceError("tallymap_b200.lang: operations on traced values outside a trace")
    return _CTX[-1]


def _lit(x, like=None):
    if isinstance(x, (Var, Lit)):
        return x
    if isinstance(x, bool):
        return Lit(bool(x), BOOL)
    if isinstance(x, int):
        # a Python int takes the other operand's type (a weak type, as jax's)
        if like is not None and like.dtype == F32:
            return Lit(float(x), F32)
        if like is not None and like.dtype == U32:
            return Lit(int(x) & 0xFFFFFFFF, U32)
        return Lit(int(x), I32)
    if isinstance(x, float):
        if like is not None and like.dtype in (I32, U32):
            raise TraceError("tallymap_b200.lang: a float literal combined with an integer value (use astype)")
        return Lit(float(x), F32)
    if isinstance(x, TallyToken):
        raise TallyError("tallymap_b200.lang: the tally handle is not a value (it is written with t.add, not read)")
    raise TraceError(f"tallymap_b200.lang: unsupported operand {x!r}")


def dtype_of(x):
    return x.dtype


def _binary(prim, a, b, out=None):
    if isinstance(a, Vec) or isinstance(b, Vec):
        return _vec_map2(lambda x, y: _binary(prim, x, y, out), a, b)
    a0 = a if isinstance(a, Var) else None
    b0 = b if isinstance(b, Var) else None
    a = _lit(a, b0)
    b = _lit(b, a0)
    if a.dtype != b.dtype:
        raise TraceError(f"tallymap_b200.lang: {prim} of {a.dtype} and {b.dtype} (convert with astype)")
    if isinstance(a, Lit) and isinstance(b, Lit):
        raise TraceError("tallymap_b200.lang: an operation on two literals")
    return _cur().emit(prim, [a, b], [out or a.dtype])[0]


class Var:
    """a traced scalar"""
    __slots__ = ("trace", "id", "dtype")

    def __init__(self, trace, id_, dtype):
        self.trace, self.id, self.dtype = trace, id_, dtype

    def __repr__(self):
        return f"v{self.id}:{self.dtype}"

    def __hash__(self):
        return hash(self.id)

    def __eq__(self, o):
        return _binary("eq", self, o, BOOL)

    def __ne__(self, o):
        return _binary("ne", self, o, BOOL)

    def __lt__(self, o):
        return _binary("lt", self, o, BOOL)

    def __le__(self, o):
        return _binary("le", self, o, BOOL)

    def __gt__(self, o):
        return _binary("gt", self, o, BOOL)

    def __ge__(self, o):
        return _binary("ge", self, o, BOOL)

    def __pow__(self, o):
        """x ** n: lax.integer_pow for a Python int n (binary powering), lax.pow otherwise"""
        if isinstance(o, int) and not isinstance(o, bool):
            return int_pow(self, o)
        from . import lang
        return lang.power(self, o)

    def __rpow__(self, o):
        from . import lang
        return lang.power(o, self)

    def __add__(self, o):
        return _binary("add", self, o)

    def __radd__(self, o):
        return _binary("add", o, self)

    def __sub__(self, o):
        return _binary("sub", self, o)

    def __rsub__(self, o):
        return _binary("sub", o, self)

    def __mul__(self, o):
        return _binary("mul", self, o)

    def __rmul__(self, o):
        return _binary("mul", o, self)

    def __truediv__(self, o):
        if self.dtype != F32 and not (isinstance(o, Var) and o.dtype == F32):
            raise TraceError("tallymap_b200.lang: '/' is float division (use // for integers)")
        return _binary("div", self, o)

    def __rtruediv__(self, o):
        return _binary("div", o, self)

    def __floordiv__(self, o):
        if self.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: // on integers only")
        return _binary("idiv", self, o)

    def __mod__(self, o):
        if self.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: % on integers only")
        return _binary("irem", self, o)

    def __rfloordiv__(self, o):
        if self.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: // on integers only")
        return _binary("idiv", o, self)

    def __rmod__(self, o):
        if self.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: % on integers only")
        return _binary("irem", o, self)

    def __neg__(self):
        return _cur().emit("neg", [self], [self.dtype])[0]

    def __and__(self, o):
        return _binary("and", self, o)

    def __rand__(self, o):
        return _binary("and", o, self)

    def __or__(self, o):
        return _binary("or", self, o)

    def __ror__(self, o):
        return _binary("or", o, self)

    def __xor__(self, o):
        return _binary("xor", self, o)

    def __lshift__(self, o):
        if self.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: << on integers only")
        return _binary("shl", self, o)

    def __rshift__(self, o):
        """logical for uint32, arithmetic for int32 (lax.shift_right_logical / _arithmetic)"""
        if self.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: >> on integers only")
        return _binary("shr", self, o)

    def __rlshift__(self, o):
        return _binary("shl", o, self)

    def __rrshift__(self, o):
        return _binary("shr", o, self)

    def __invert__(self):
        return _cur().emit("not", [self], [self.dtype])[0]

    def __bool__(self):
        raise TraceError("tallymap_b200.lang: a traced value has no Python truth value (use lang.where / while_loop)")

    def astype(self, dtype):
        dtype = _dt(dtype)
        if dtype == self.dtype:
            return self
        return _cur().emit("convert", [self], [dtype])[0]


def _dt(d):
    from . import lang
    m = {lang.float32: F32, lang.int32: I32, lang.uint32: U32, lang.bool_: BOOL, F32: F32, I32: I32, U32: U32,
         BOOL: BOOL}
    if d not in m:
        raise TraceError(f"tallymap_b200.lang: unsupported dtype {d!r}")
    return m[d]


class Key:
    """a traced PRNG key: its two uint32 words (jax.random key data)"""
    __slots__ = ("a", "b")

    def __init__(self, a, b):
        self.a, self.b = a, b


def _vec_map2(f, a, b):
    la = len(a) if isinstance(a, Vec) else None
    lb = len(b) if isinstance(b, Vec) else None
    if la is not None and lb is not None and la != lb:
        raise TraceError(f"tallymap_b200.lang: vectors of {la} and {lb} elements")
    n = la if la is not None else lb
    return Vec(f(tuple.__getitem__(a, i) if la is not None else a, tuple.__getitem__(b, i) if lb is not None else b)
               for i in range(n))


def int_pow(x, n):
    """x ** n for a Python int n (lax.integer_pow): binary powering, then the reciprocal for n < 0"""
    if n == 0:
        return x * 0.0 + 1.0
    m, acc, base = abs(n), None, x
    while m > 0:
        if m & 1:
            acc = base if acc is None else acc * base
        m >>= 1
        if m > 0:
            base = base * base
    return 1.0 / acc if n < 0 else acc


class Vec(tuple):
    """a small float32 / int32 / bool vector of traced scalars with jax.numpy's elementwise semantics (the item's
    per-item and broadcast vectors, tl.array / tl.stack): arithmetic, comparisons, logical ops and lang's math
    functions apply per element, a scalar operand broadcasts; t[i] with a traced int32 index reads an element as
    jax.numpy does (a negative index counts from the end, then the index is clamped into range) through a chain of
    selects, so the element read stays differentiable.  Unpacking and iteration are a tuple's."""
    __hash__ = tuple.__hash__

    @property
    def shape(self):
        return (len(self),)

    @property
    def at(self):
        """x.at[i].set(y) / add / multiply / min / max / get, jax.numpy's functional updates: a negative index counts
        from the end; an update at an index still out of range is dropped (mode 'drop', jnp's default for updates)
        or clamped (mode 'clip'); a traced index selects per element"""
        return _VecAt(self)

    def _op(prim, out=None):
        return lambda self, o: _binary(prim, self, o, out)

    def _rop(prim, out=None):
        return lambda self, o: _binary(prim, o, self, out)

    __add__, __radd__ = _op("add"), _rop("add")
    __sub__, __rsub__ = _op("sub"), _rop("sub")
    __mul__, __rmul__ = _op("mul"), _rop("mul")
    __truediv__, __rtruediv__ = _op("div"), _rop("div")
    __floordiv__, __mod__ = _op("idiv"), _op("irem")
    __and__, __rand__, __or__, __ror__, __xor__ = _op("and"), _rop("and"), _op("or"), _rop("or"), _op("xor")
    __lt__, __le__, __gt__, __ge__ = _op("lt", BOOL), _op("le", BOOL), _op("gt", BOOL), _op("ge", BOOL)
    __eq__, __ne__ = _op("eq", BOOL), _op("ne", BOOL)
    del _op, _rop

    def __neg__(self):
        return Vec(-x for x in tuple.__iter__(self))

    def __invert__(self):
        return Vec(~x for x in tuple.__iter__(self))

    def __pow__(self, n):
        return Vec(x ** n for x in tuple.__iter__(self))

    def astype(self, dtype):
        return Vec(x.astype(dtype) if isinstance(x, Var) else x for x in tuple.__iter__(self))

    def sum(self):
        from . import lang
        return lang.sum(self)

    def __getitem__(self, i):
        if isinstance(i, (int, slice)) and not isinstance(i, bool):
            r = tuple.__getitem__(self, i)
            return Vec(r) if isinstance(i, slice) else r
        i = _lit(i)
        if not isinstance(i, Var) or i.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: a vector index is an integer")
        from . import lang
        n = len(self)
        ii = lang.minimum(i, n - 1).astype(I32) if i.dtype == U32 else \
            lang.clip(lang.where(i < 0, i + n, i), 0, n - 1)
        r = tuple.__getitem__(self, 0)
        for j in range(1, n):
            r = lang.where(ii == j, tuple.__getitem__(self, j), r)
        return r


class _VecAt:
    __slots__ = ("v",)

    def __init__(self, v):
        self.v = v

    def __getitem__(self, i):
        return _VecRef(self.v, i)


class _VecRef:
    __slots__ = ("v", "i")

    def __init__(self, v, i):
        self.v, self.i = v, i

    def get(self, mode=None):
        if mode not in (None, "clip", "promise_in_bounds"):
            raise UnsupportedError(f"tallymap_b200.lang: x.at[i].get(mode={mode!r})")
        return self.v[self.i]

    def _update(self, y, f, mode):
        from . import lang
        if mode not in (None, "drop", "fill", "clip", "promise_in_bounds"):
            raise UnsupportedError(f"tallymap_b200.lang: x.at[i] update with mode={mode!r}")
        clip = mode in ("clip", "promise_in_bounds")
        xs, n, i = list(tuple.__iter__(self.v)), len(self.v), self.i
        if isinstance(i, bool):
            raise TraceError("tallymap_b200.lang: a vector index is an integer")
        if isinstance(i, int):
            i = i + n if i < 0 else i
            if not 0 <= i < n:
                if not clip:
                    return Vec(xs)
                i = min(max(i, 0), n - 1)
            xs[i] = f(xs[i], y)
            return Vec(xs)
        i = _lit(i)
        if not isinstance(i, Var) or i.dtype != I32:
            raise TraceError("tallymap_b200.lang: a vector index is an int32")
        ii = lang.where(i < 0, i + n, i)
        if clip:
            ii = lang.clip(ii, 0, n - 1)
        return Vec(lang.where(ii == j, f(x, y), x) for j, x in enumerate(xs))

    def set(self, y, mode=None):
        return self._update(y, lambda x, y_: y_, mode)

    def add(self, y, mode=None):
        return self._update(y, lambda x, y_: x + y_, mode)

    def multiply(self, y, mode=None):
        return self._update(y, lambda x, y_: x * y_, mode)

    def min(self, y, mode=None):
        from . import lang
        return self._update(y, lang.minimum, mode)

    def max(self, y, mode=None):
        from . import lang
        return self._update(y, lang.maximum, mode)


class Table:
    """a broadcast array of float32 or int32, shape (n,) or (n, m), read-only in the item: t[i] (a 1-D table's
    element; a 2-D table's row i as a tuple of m values) and t[i, j], with jax.numpy's indexing semantics for a
    traced index (a negative index counts from the end, then the index is clamped into range: XLA's gather start
    index clamp, backends/kernel/op_table.py:1085-1146); a Python int index out of range raises IndexError"""
    __slots__ = ("var", "shape")

    def __init__(self, var, shape):
        self.var, self.shape = var, tuple(int(d) for d in shape)

    def __len__(self):
        return self.shape[0]

    @property
    def dtype(self):
        return TABLE_ELT[self.var.dtype]

    def _index(self, i, n):
        """a Python int (static) or a traced int32 index in [0, n)"""
        if isinstance(i, bool):
            raise TraceError("tallymap_b200.lang: a table index is an integer")
        if isinstance(i, int):
            if not -n <= i < n:
                raise IndexError(f"tallymap_b200.lang: index {i} is out of bounds for a table axis of size {n}")
            return i % n
        i = _lit(i)
        if not isinstance(i, Var) or i.dtype not in (I32, U32):
            raise TraceError("tallymap_b200.lang: a table index is an integer")
        from . import lang
        if i.dtype == U32:
            return lang.minimum(i, n - 1).astype(I32)
        return lang.clip(lang.where(i < 0, i + n, i), 0, n - 1)

    def _gather(self, flat):
        size = self.shape[0] * (self.shape[1] if len(self.shape) > 1 else 1)
        return _cur().emit("gather", [self.var, _lit(flat)], [self.dtype], n=size)[0]

    def __getitem__(self, idx):
        idx = idx if isinstance(idx, tuple) else (idx,)
        if len(idx) > len(self.shape) or not idx:
            raise TraceError(f"tallymap_b200.lang: {len(idx)} indices for a table of shape {self.shape}")
        ii = [self._index(i, n) for i, n in zip(idx, self.shape)]
        if len(self.shape) == 1:
            return self._gather(ii[0])
        row = ii[0] * self.shape[1]
        if len(ii) == 2:
            return self._gather(row + ii[1])
        return tuple(self._gather(row + j) for j in range(self.shape[1]))


class TallyToken:
    """the tally handle `t` of an item: t.add(name, index, value) records an emit, t.append(name, {field: value},
    when=...) a record; both return the handle"""

    def __init__(self, specs, records=None, child=None):
        self.specs = specs           # name -> (shape, dtype)
        self.records = records or {}  # name -> (capacity, ((field, dtype), ...) sorted by field)
        self.child = child           # the per-item operands' specs: what a spawned child carries

    def spawn(self, child, when=True):
        """push a child item (tallymap/_tally.py:284-302, spawn): `child` holds its per-item operands with the
        structure of the mapped per-item arguments (a tuple of them, in their order; a key as a key, a vector as a
        tuple; one per-item argument may be given bare); it runs the same item function with the same broadcast
        operands, and its per-item results are discarded"""
        if self.child is None:
            raise TraceError("tallymap_b200.lang: spawn needs a Queue (tallymap_b200.vmap(..., spawn=Queue(n)))")
        if len(self.child) == 1 and not (isinstance(child, tuple) and len(child) == 1):
            child = (child,)
        if not isinstance(child, tuple) or len(child) != len(self.child):
            raise TraceError(f"tallymap_b200.lang: a spawned child has the structure of the mapped per-item "
                             f"arguments ({len(self.child)} of them)")
        w = _lit(when)
        if w.dtype != BOOL:
            raise TraceError("tallymap_b200.lang: spawn's `when` must be a scalar bool")
        leaves = []
        for x, s in zip(child, self.child):
            if s == "key":
                if not isinstance(x, Key):
                    raise TraceError("tallymap_b200.lang: a child's key operand must be a key")
                leaves += [x.a, x.b]
                continue
            if isinstance(s, tuple):
                if not isinstance(x, tuple) or len(x) != s[1]:
                    raise TraceError(f"tallymap_b200.lang: a child's vector operand has {s[1]} elements")
                xs, dt = x, s[0]
            else:
                xs, dt = (x,), s
            for v in xs:
                if isinstance(v, (Key, tuple)):
                    raise TraceError("tallymap_b200.lang: a spawned child has the structure of the mapped inputs")
                v = _lit(v)
                if isinstance(v, Lit):
                    v = Lit(float(v.value), F32) if dt == F32 else Lit(int(v.value), dt)
                if v.dtype != dt:
                    raise TraceError(f"tallymap_b200.lang: a child's operand is {dt}, got {v.dtype}")
                leaves.append(v)
        _cur().eqns.append(Eqn("spawn", [w] + leaves, [], {}))
        return self

    def append(self, name, fields, when=True):
        """a Records output's append (tallymap/_tally.py:302-364): the fields of one record, written when `when`"""
        if name not in self.records:
            raise TraceError(f"tallymap_b200.lang: no Records output named {name!r}")
        cap, spec = self.records[name]
        if sorted(fields) != [f for f, _ in spec]:
            raise TraceError(f"tallymap_b200.lang: Records {name!r} has fields {[f for f, _ in spec]}")
        w = _lit(when)
        if w.dtype != BOOL:
            raise TraceError("tallymap_b200.lang: append's `when` must be bool")
        vals = []
        for f, dt in spec:
            v = _lit(fields[f])
            if isinstance(v, Lit):
                v = Lit(float(v.value), F32) if dt == F32 else Lit(int(v.value), dt)
            if v.dtype != dt:
                raise TraceError(f"tallymap_b200.lang: Records {name!r} field {f!r} is {dt}, got {v.dtype}")
            vals.append(v)
        _cur().eqns.append(Eqn("append", [w] + vals, [], dict(records=name)))
        return self

    def add(self, name, index, value):
        """tally[name][index] += value (_tally.py:248-282): index an int32 (a flat index of a 1-D output) or a
        tuple of them, one per dimension; a vector index (or coordinate) with a scalar or vector value makes one
        emit per element, in element order, a scalar broadcast; an index outside the output is dropped and
        counted in stats['dropped_emits']"""
        if name not in self.specs:
            raise TraceError(f"tallymap_b200.lang: no output named {name!r} (outputs: {sorted(self.specs)})")
        coords = isinstance(index, tuple) and not isinstance(index, Vec)
        parts = list(index) if coords else [index]
        vecs = [p for p in parts + [value] if isinstance(p, Vec)]
        if vecs:
            n = len(vecs[0])
            if any(len(v) != n for v in vecs):
                raise TraceError(f"tallymap_b200.lang: t.add({name!r}, ...) of vectors of different lengths")
            at = lambda p, j: tuple.__getitem__(p, j) if isinstance(p, Vec) else p
            for j in range(n):
                self.add(name, tuple(at(p, j) for p in parts) if coords else at(index, j), at(value, j))
            return self
        shape, dt = self.specs[name]
        tr = _cur()
        idx = _flat_index(index, shape)
        v = _lit(value)
        if isinstance(v, Lit):
            v = Lit(float(v.value), F32) if dt == F32 else Lit(int(v.value), I32)
        if v.dtype != dt:
            raise TraceError(f"tallymap_b200.lang: output {name!r} sums {dt}, got {v.dtype}")
        tr.eqns.append(Eqn("emit", [idx, v], [], dict(tally=name)))
        return self


def _add_flat(tok, name, flat, value):
    """tally[name].flat[flat] += value for a flat int32 index into the output's row-major layout (the index the
    reference's Tally.add has already formed, with -1 for a coordinate out of range, _tally.py:260-271): the
    emit of the jaxpr front end (tallymap_b200.from_jaxpr); out-of-range indices are dropped and counted"""
    if name not in tok.specs:
        raise TraceError(f"tallymap_b200: no output named {name!r} (outputs: {sorted(tok.specs)})")
    _, dt = tok.specs[name]
    i = _lit(flat)
    if i.dtype == U32:
        i = i.astype(I32) if isinstance(i, Var) else Lit(int(i.value), I32)
    if i.dtype != I32:
        raise TraceError("tallymap_b200: tally indices are int32")
    v = _lit(value)
    if isinstance(v, Lit):
        v = Lit(float(v.value), F32) if dt == F32 else Lit(int(v.value), I32)
    if v.dtype != dt:
        raise TraceError(f"tallymap_b200: output {name!r} sums {dt}, got {v.dtype}")
    _cur().eqns.append(Eqn("emit", [i, v], [], dict(tally=name)))
    return tok


def _claim(tok, name, when):
    """a Records output's one-pass slot claim as the reference's jaxprs hold it (tallymap/_tally.py:141-160
    claim_p, its kernel rule backends/kernel/kernel.py:1052-1070): the next slot of the raw buffer behind the int32
    Sum `name` (its capacity = the tally's size) from a per-launch counter, or -1 when `when` is false or the buffer
    is full (the counter still counts: it holds the true total).  The jaxpr front end's `tallymap_claim`; the fields
    are then ordinary emits at the slot.  -> the slot, an int32"""
    if name not in tok.specs:
        raise TraceError(f"tallymap_b200: a claim on {name!r}, which is not a tally")
    shape, dt = tok.specs[name]
    w = _lit(when)
    if w.dtype != BOOL:
        raise TraceError("tallymap_b200: a claim's `when` must be a scalar bool")
    cap = 1
    for d in shape:
        cap *= int(d)
    return _cur().emit("claim", [w], [I32], tally=name, capacity=cap)[0]


def _flat_index(index, shape):
    """row-major flat index; any coordinate outside its dimension gives -1 (_tally.py:260-271)"""
    if not isinstance(index, tuple):
        index = (index,)
    if len(shape) == 0:
        if index not in ((), (0,)):
            raise TraceError("tallymap_b200.lang: a scalar output takes index 0 or ()")
        return Lit(0, I32)
    if len(index) != len(shape):
        raise TraceError(f"tallymap_b200.lang: index of {len(index)} coordinates for an output of shape {shape}")
    if len(index) == 1:
        i = _lit(index[0])
        if i.dtype != I32:
            raise TraceError("tallymap_b200.lang: tally indices are int32")
        return i
    flat, ok = None, None
    for i, n in zip(index, shape):
        i = _lit(i)
        if i.dtype != I32:
            raise TraceError("tallymap_b200.lang: tally indices are int32")
        inb = _cur().emit("inrange", [i], [BOOL], n=int(n))[0]
        ok = inb if ok is None else (ok & inb)
        flat = i if flat is None else flat * int(n) + i
    return _cur().emit("select", [ok, flat, Lit(-1, I32)], [I32])[0]


@dataclasses.dataclass
class Traced:
    """a traced item: pre / cond / body / post equation lists and the variables that connect them"""
    inputs: list             # per-item operands, then broadcast ones: Var, Key, or a tuple of Vars (a vector)
    n_per_item: int
    pre: list
    carry_in: list           # the loop's initial carry (Var | Lit), the tally token excluded
    carry: list              # the carry variables as the cond / body see them
    cond: list
    cond_out: Var
    body: list
    body_out: list           # the carry after one step (Var | Lit)
    post_carry: list         # the carry variables the post-loop code sees (the loop's final carry)
    post: list
    results: list            # per-item results (Var | Lit)
    specs: dict
    records: dict = dataclasses.field(default_factory=dict)
    result_groups: list = None   # per returned value: (first flat result, n for a vector or None for a scalar)


class _Loop:
    pass


def _walk(eqns):
    """every equation of `eqns`, those inside nested while loops included"""
    for e in eqns:
        yield e
        if e.prim == "while":
            yield from _walk(e.params["cond"])
            yield from _walk(e.params["body"])


def _nested_while(cond_fun, body_fun, init):
    """a while loop other than the item's stepping loop -- inside its body or condition, or after it -- as ONE
    equation "while" whose params hold its own condition and body (the reference's emitter writes it as a C while
    loop, op_table.py:1414-1450): ins = the initial carry (the tally handle passes through in its position), outs =
    the final carry; the condition and body may read any value defined before the loop.  A spawn inside it is not
    lowered (a step pushes at most two children)."""
    tr = _cur()
    flat_in, rebuild = _flatten(init)
    cond_tr, body_tr = Trace(tr.ids), Trace(tr.ids)
    carry = []
    for x in flat_in:
        carry.append(x if isinstance(x, TallyToken) else body_tr.new(_lit(x).dtype))
    _CTX.append(cond_tr)
    try:
        c = cond_fun(rebuild(carry))
    finally:
        _CTX.pop()
    if not isinstance(c, Var) or c.dtype != BOOL:
        raise TraceError("tallymap_b200.lang: a while loop's condition must be a traced bool")
    if any(e.prim in ("emit", "append", "spawn", "claim") for e in _walk(cond_tr.eqns)):
        raise TraceError("tallymap_b200.lang: a while loop's condition may not write the tally")
    _CTX.append(body_tr)
    try:
        out = body_fun(rebuild(carry))
    finally:
        _CTX.pop()
    if any(e.prim == "spawn" for e in _walk(body_tr.eqns)):
        raise UnsupportedError("tallymap_b200.lang: t.spawn inside an inner while loop is not lowered (spawn in "
                               "the item's loop body or after it)")
    flat_out, _ = _flatten(out)
    if len(flat_out) != len(flat_in):
        raise TraceError("tallymap_b200.lang: the loop body must return a carry of the same structure")
    cvars, body_out = [], []
    for a, b, cv in zip(flat_in, flat_out, carry):
        if isinstance(a, TallyToken) != isinstance(b, TallyToken):
            raise TallyError("tallymap_b200.lang: the tally handle must stay in its carry position")
        if isinstance(a, TallyToken):
            continue
        v = _lit(b, cv)
        if v.dtype != cv.dtype:
            raise TraceError(f"tallymap_b200.lang: a loop carry of {cv.dtype} became {v.dtype} in the body")
        cvars.append(cv)
        body_out.append(v)
    outs = [tr.new(v.dtype) for v in cvars]
    tr.eqns.append(Eqn("while", [_lit(x) for x in flat_in if not isinstance(x, TallyToken)], outs,
                       dict(carry=cvars, cond=cond_tr.eqns, cond_out=c, body=body_tr.eqns, body_out=body_out)))
    it = iter(outs)
    return rebuild([x if isinstance(x, TallyToken) else next(it) for x in carry])


def while_loop(cond_fun, body_fun, init):
    """lax.while_loop; the carry is a tuple of scalars, keys and the tally handle.  The item's first loop at its
    top level is its stepping loop (the runtime refills threads at its step granularity); any other loop -- inside
    it, or after it -- is an inner loop (_nested_while)"""
    tr = _cur()
    st = getattr(tr, "loop_state", None)
    if st is None or st.get("depth", 0) != 0 or st.get("done") or st.get("branch"):
        return _nested_while(cond_fun, body_fun, init)
    flat_in, rebuild = _flatten(init)
    carry = []
    body_tr = Trace(tr.ids)
    cond_tr = Trace(tr.ids)
    for x in flat_in:
        if isinstance(x, TallyToken):
            carry.append(x)
        else:
            v = _lit(x)
            carry.append(body_tr.new(v.dtype))
    # cond and body see the same carry variables
    cvars = [c for c in carry]
    st["depth"] = 1
    _CTX.append(cond_tr)
    try:
        c = cond_fun(rebuild(cvars))
    finally:
        _CTX.pop()
    if not isinstance(c, Var) or c.dtype != BOOL:
        raise TraceError("tallymap_b200.lang: the loop condition must be a traced bool")
    _CTX.append(body_tr)
    try:
        out = body_fun(rebuild(cvars))
    finally:
        _CTX.pop()
    st["depth"] = 0
    flat_out, _ = _flatten(out)
    if len(flat_out) != len(flat_in):
        raise TraceError("tallymap_b200.lang: the loop body must return a carry of the same structure")
    for a, b in zip(flat_in, flat_out):
        if isinstance(a, TallyToken) != isinstance(b, TallyToken):
            raise TallyError("tallymap_b200.lang: the tally handle must stay in its carry position")
    # the loop's results: fresh variables (the final carry)
    post = [x if isinstance(x, TallyToken) else tr.new(x.dtype) for x in carry]
    st.update(done=True, init=[x for x in flat_in], carry=cvars, cond=cond_tr.eqns, cond_out=c,
              body=body_tr.eqns, body_out=flat_out, post_carry=post, pre_len=len(tr.eqns))
    return rebuild(post)


def _flatten(tree):
    """flatten a carry (nested tuples of Var / Key / literals / TallyToken) into scalars; -> (leaves, rebuild)"""
    leaves, spec = [], []

    def go(x):
        if isinstance(x, tuple):
            spec.append(("vec" if isinstance(x, Vec) else "tuple", len(x)))
            for y in tuple.__iter__(x):
                go(y)
        elif isinstance(x, Key):
            spec.append(("key",))
            leaves.extend([x.a, x.b])
        else:
            spec.append(("leaf",))
            leaves.append(x)
    go(tree)

    def rebuild(vals):
        it = iter(vals)
        sp = iter(spec)

        def build():
            s = next(sp)
            if s[0] == "tuple":
                return tuple(build() for _ in range(s[1]))
            if s[0] == "vec":
                return Vec(build() for _ in range(s[1]))
            if s[0] == "key":
                return Key(next(it), next(it))
            return next(it)
        return build()
    return leaves, rebuild


def trace_item(fn, in_specs, n_per_item, specs, records=None, spawn=False):
    """trace item function `fn(t, *args)`; in_specs: per argument "f32" | "i32" | "u32" | "key" | ("f32", n)
    (a per-item vector); specs: Sum output name -> (shape, dtype); records: Records output name -> (capacity,
    ((field, dtype), ...)).  -> Traced"""
    tr = Trace()
    tr.loop_state = {"depth": 0}
    args = []
    for s in in_specs:
        if s == "key":
            args.append(Key(tr.new(U32), tr.new(U32)))
        elif isinstance(s, tuple) and s[0] == "table":
            args.append(Table(tr.new({F32: TF32, I32: TI32}[s[1]]), s[2]))
        elif isinstance(s, tuple):
            args.append(Vec(tr.new(s[0]) for _ in range(s[1])))
        else:
            args.append(tr.new(s))
    tok = TallyToken(specs, records, list(in_specs[:n_per_item]) if spawn else None)
    _CTX.append(tr)
    try:
        out = fn(tok, *args)
    finally:
        _CTX.pop()
    st = tr.loop_state
    if not st.get("done"):
        # no loop: a loop of zero steps (its predicate false), all the item's code after it
        st.update(done=True, init=[], carry=[], cond=[], cond_out=Lit(False, BOOL), body=[], body_out=[],
                  post_carry=[], pre_len=0)
    out = out if isinstance(out, tuple) else (out,)
    if not out or not isinstance(out[0], TallyToken):
        raise TallyError("tallymap_b200.lang: an item returns (t, *per_item_results)")
    results, groups = [], []
    for r in out[1:]:               # a returned vector: one per-item result per element, regrouped by the API
        if isinstance(r, tuple):
            if not r or any(isinstance(x, (tuple, Key, TallyToken)) for x in r):
                raise TraceError("tallymap_b200.lang: a per-item result is a scalar or a flat vector of scalars")
            groups.append((len(results), len(r)))
            results += [_lit(x) for x in r]
        else:
            groups.append((len(results), None))
            results.append(_lit(r))
    pre = tr.eqns[:st["pre_len"]]
    post = tr.eqns[st["pre_len"]:]
    keep = lambda xs: [x for x in xs if not isinstance(x, TallyToken)]
    if any(e.prim == "spawn" for e in pre):
        raise UnsupportedError("tallymap_b200.lang: spawn before the loop is not lowered "
                               "(spawn in the loop or after it)")
    if sum(e.prim == "spawn" for e in st["body"]) > 2 or sum(e.prim == "spawn" for e in post) > 2:
        raise UnsupportedError("tallymap_b200.lang: at most two spawns per loop step and two after the loop")
    return Traced(inputs=args, n_per_item=n_per_item, pre=pre, carry_in=[_lit(x) for x in keep(st["init"])],
                  carry=keep(st["carry"]), cond=st["cond"], cond_out=st["cond_out"], body=st["body"],
                  body_out=[_lit(x) for x in keep(st["body_out"])], post_carry=keep(st["post_carry"]), post=post,
                  results=results, specs=specs, records=records or {}, result_groups=groups)
