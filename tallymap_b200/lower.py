"""Lowering of a traced item (tallymap_b200.trace.Traced) to CUDA C for the persistent-thread runtime, and its
compilation at run time (NVRTC, sm_100a) into a registered kernel.

The reference lowers an item jaxpr to straight-line C inside its generated kernel (backends/kernel/kernel.py:428-451,
codegen.py:494-980) and compiles with NVRTC (backends/kernel/compile.py:160-173).  Here the item becomes an ITEM
struct of the hand-written runtime (csrc/tm_runtime.cuh): the pre-loop code is `start`, the loop predicate `cond`, the
loop body `step`, the post-loop code `finish` -- the step schedule of kernel.py:225-295, which needs exactly one
top-level loop.  Its reverse mode is the replay adjoint of _reverse.py:1079-1180 (vjp_prog): the same runtime's
replay_kernel with a generated step VJP (reverse mode over the body's equations, only for float values that depend on
a differentiated operand: _reverse.py:208 `_active`), the broadcast cotangents summed per item in f32 and emitted once
into an exact tally.

Launch layouts are the backend's (backend.ItemProgram): forward = [per-item][broadcast][consts i32[1]][order] |
[tallies][ctl][stats] | [per-item results][truncated]; reverse = [per-item][broadcast][output cotangents][consts
i32[3]][order] | [g f32[W]][exact words][ctl][stats] | [truncated][replay scratch].
"""
import ctypes
import dataclasses
import hashlib
import os
import time

import numpy as np
import torch

from . import _lib
from . import trace as T

CSRC = os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc")
PRIV_BYTES = 4096        # outputs up to this size are privatised per block in shared memory (kernel.py:300)
CTYPE = {T.F32: "float", T.I32: "i32", T.U32: "u32", T.BOOL: "bool", T.TF32: "const float*", T.TI32: "const i32*"}
SPAWN_STACK_SHARED = 8   # a lane's private stack entries in shared memory (csrc/tm_spawn.cuh kStackShared)
TDTYPE = {T.F32: torch.float32, T.I32: torch.int32, T.U32: torch.int32, T.BOOL: torch.uint8}


class LowerError(T.UnsupportedError):
    """a traced item (or a derived program of it) this lowering does not produce"""


# ------------------------------------------------------------------------------------------------ C expressions
def c_lit(lit):
    if lit.dtype == T.F32:
        v = float(np.float32(lit.value))
        if np.isnan(v):
            return "__int_as_float(0x7fc00000)"
        if np.isinf(v):
            return "__int_as_float(0x7f800000)" if v > 0 else "__int_as_float((int)0xff800000u)"
        return float(v).hex() + "f"
    if lit.dtype == T.I32:
        v = int(lit.value)
        return "(i32)(-2147483647 - 1)" if v == -2 ** 31 else f"(i32){v}"
    if lit.dtype == T.U32:
        return f"{int(lit.value) & 0xFFFFFFFF}u"
    return "true" if lit.value else "false"


_BIN = {"add": "+", "sub": "-", "mul": "*", "div": "/", "lt": "<", "le": "<=", "gt": ">", "ge": ">=", "eq": "==",
        "ne": "!="}
_MATH = {"log": "tmm::logf", "exp": "tmm::expf", "sin": "tmm::sinf", "cos": "tmm::cosf", "atan": "tmm::atanf",
         "asin": "tmm::asinf", "acos": "tmm::acosf", "tan": "tmm::tanf", "sinh": "tmm::sinhf", "cosh": "tmm::coshf",
         "asinh": "tmm::asinhf", "acosh": "tmm::acoshf", "atanh": "tmm::atanhf", "exp2": "tmm::exp2f",
         "log2": "tmm::log2f", "cbrt": "tmm::cbrtf", "erf": "tmm::erff", "erfc": "tmm::erfcf",
         "erfinv": "tmm::erfinvf", "lgamma": "tmm::lgammaf"}
# d out / d x of the unary math primitives above beyond log / exp / sin / cos, as C over the input's and the
# output's expressions (jax's jvp rules: lax.py atan, asin, acos, tan, sinh, cosh, asinh, acosh, atanh, exp2, log2,
# cbrt; special.py erf, erfc, erf_inv)
_DERIV = {
    "atan": lambda a, o: f"tm_fdiv(1.0f, (1.0f + {a} * {a}))",
    "asin": lambda a, o: f"tm_fdiv(1.0f, tm_fsqrt((1.0f - {a}) * (1.0f + {a})))",
    "acos": lambda a, o: f"(-tm_fdiv(1.0f, tm_fsqrt((1.0f - {a}) * (1.0f + {a}))))",
    "tan": lambda a, o: f"(1.0f + {o} * {o})",
    "sinh": lambda a, o: f"tmm::coshf({a})",
    "cosh": lambda a, o: f"tmm::sinhf({a})",
    "asinh": lambda a, o: f"tm_fdiv(1.0f, tm_fsqrt({a} * {a} + 1.0f))",
    "acosh": lambda a, o: f"tm_fdiv(1.0f, tm_fsqrt(({a} - 1.0f) * ({a} + 1.0f)))",
    "atanh": lambda a, o: f"tm_fdiv(1.0f, ((1.0f - {a}) * (1.0f + {a})))",
    "exp2": lambda a, o: f"({o} * 0.693147182f)",
    "log2": lambda a, o: f"tm_fdiv(1.0f, ({a} * 0.693147182f))",
    "cbrt": lambda a, o: f"tm_fdiv(1.0f, (3.0f * ({o} * {o})))",
    "erf": lambda a, o: f"(1.12837917f * tmm::expf(-({a} * {a})))",
    "erfc": lambda a, o: f"(-1.12837917f * tmm::expf(-({a} * {a})))",
    "erfinv": lambda a, o: f"(0.886226925f * tmm::expf({o} * {o}))",
}


def c_expr(e, a):
    """the C expression of equation e's single output; a: its inputs' C expressions"""
    p, d = e.prim, e.ins[0].dtype if e.ins else None
    if p in ("add", "sub", "mul") and d in (T.I32,):
        return f"(i32)((u32)({a[0]}) {_BIN[p]} (u32)({a[1]}))"         # wrapping int32 arithmetic
    if p == "div":      # f32 only ('/' of integers does not trace); the call's cuda_math decides the instruction
        return f"tm_fdiv({a[0]}, {a[1]})"
    if p in _BIN:
        return f"({a[0]} {_BIN[p]} {a[1]})"
    if p == "idiv":
        return f"tm_floordiv({a[0]}, {a[1]})"
    if p == "irem":
        return f"tm_floormod({a[0]}, {a[1]})"
    if p == "neg":
        return f"(-{a[0]})" if d == T.F32 else f"(i32)(0u - (u32)({a[0]}))"
    if p in ("and", "or", "xor"):
        op = {"and": "&", "or": "|", "xor": "^"}[p]
        return f"({a[0]} {op} {a[1]})" if d != T.BOOL else f"({a[0]} {op} {a[1]})"
    if p == "not":
        return f"(!{a[0]})" if d == T.BOOL else f"(~{a[0]})"
    if p == "popc":     # lax.population_count: set bits of the 32-bit pattern
        return f"({CTYPE[d]})__popc((unsigned)({a[0]}))"
    if p == "clz":      # lax.clz: leading zero bits of the 32-bit pattern (32 for 0)
        return f"({CTYPE[d]})__clz((int)({a[0]}))"
    if p == "shl":      # (a shift by 32 or more gives 0, as lax.shift_left; C would leave it undefined)
        return f"((u32)({a[1]}) >= 32u ? ({CTYPE[d]})0 : ({CTYPE[d]})((u32)({a[0]}) << (u32)({a[1]})))"
    if p == "shr":      # logical for u32, arithmetic for i32; 32 or more: 0, or the sign for i32
        if d == T.U32:
            return f"((u32)({a[1]}) >= 32u ? 0u : ({a[0]} >> (u32)({a[1]})))"
        return f"((u32)({a[1]}) >= 32u ? ({a[0]} < 0 ? (i32)-1 : (i32)0) : ({a[0]} >> (u32)({a[1]})))"
    if p in _MATH:
        return f"{_MATH[p]}({a[0]})"
    if p == "atan2":
        return f"tmm::atan2f({a[0]}, {a[1]})"
    if p == "nextafter":
        return f"tmm::nextafterf({a[0]}, {a[1]})"
    if p == "sqrt":
        return f"tm_fsqrt({a[0]})"
    if p == "floor":
        return f"floorf({a[0]})"
    if p == "round":    # jnp.round: to nearest, ties to even (an exact operation: host and device agree)
        return f"rintf({a[0]})"
    if p == "rem":      # lax.rem of f32: C's fmodf, exact
        return f"fmodf({a[0]}, {a[1]})"
    if p == "stop":     # lax.stop_gradient: the value itself
        return f"({a[0]})"
    if p == "abs":
        return f"fabsf({a[0]})" if d == T.F32 else f"tm_iabs({a[0]})"
    if p == "pow":
        return f"tmm::powf({a[0]}, {a[1]})"
    if p == "max":
        return f"tm_max({a[0]}, {a[1]})"
    if p == "min":
        return f"tm_min({a[0]}, {a[1]})"
    if p == "select":
        return f"({a[0]} ? {a[1]} : {a[2]})"
    if p == "inrange":
        return f"((u32)({a[0]}) < {int(e.params['n'])}u)"
    if p == "gather":   # a broadcast table's element; the index is in range by construction (trace.Table)
        return f"__ldg(&{a[0]}[{a[1]}])"
    if p == "convert":
        return _convert(d, e.outs[0].dtype, a[0])
    if p == "bitcast":  # lax.bitcast_convert_type between 32-bit types: the same bits
        return _bitcast(d, e.outs[0].dtype, a[0])
    if p == "bits":
        return f"random_bits32(Key{{{a[0]}, {a[1]}}}, {a[2]})"
    if p == "uniform01":
        return f"uniform01(Key{{{a[0]}, {a[1]}}}, {a[2]})"
    raise LowerError(f"tallymap_b200.lower: no lowering for {p}")


def _bitcast(src, dst, x):
    if src == dst:
        return f"({x})"
    if src == T.F32:
        return f"__float_as_uint({x})" if dst == T.U32 else f"__float_as_int({x})"
    if dst == T.F32:
        return f"__uint_as_float((u32)({x}))"
    return f"({CTYPE[dst]})({x})"


def _convert(src, dst, x):
    if src == T.F32:
        return {T.I32: f"f2i({x})", T.U32: f"__float2uint_rz({x})", T.BOOL: f"({x} != 0.0f)"}[dst]
    if src == T.I32:
        return {T.F32: f"__int2float_rn({x})", T.U32: f"(u32)({x})", T.BOOL: f"({x} != 0)"}[dst]
    if src == T.U32:
        return {T.F32: f"__uint2float_rn({x})", T.I32: f"(i32)({x})", T.BOOL: f"({x} != 0u)"}[dst]
    return {T.F32: f"({x} ? 1.0f : 0.0f)", T.I32: f"(i32)({x})", T.U32: f"(u32)({x})"}[dst]


PRELUDE = r"""
#include "tm_tally.cuh"
#include "tm_math.h"
namespace tmb {
__device__ __forceinline__ float tm_max(float a, float b) {   // lax.max: NaN wins, max(-0, +0) = +0
  return (a > b || a != a) ? a : ((b > a || b != b) ? b : (a == 0.0f ? a + b : a));
}
__device__ __forceinline__ float tm_min(float a, float b) {   // lax.min: NaN wins, min(-0, +0) = -0
  return (a < b || a != a) ? a : ((b < a || b != b) ? b : (a == 0.0f ? -((-a) + (-b)) : a));
}
__device__ __forceinline__ i32 tm_max(i32 a, i32 b) { return a > b ? a : b; }
__device__ __forceinline__ i32 tm_min(i32 a, i32 b) { return a < b ? a : b; }
__device__ __forceinline__ i32 tm_iabs(i32 a) { return a < 0 ? (i32)(0u - (u32)a) : a; }
__device__ __forceinline__ i32 tm_floordiv(i32 a, i32 b) {   // jnp.floor_divide; x // 0 = 0 here
  if (b == 0) return 0;
  if (b == -1) return (i32)(0u - (u32)a);
  const i32 q = a / b;
  return (q * b != a && ((a < 0) != (b < 0))) ? q - 1 : q;
}
__device__ __forceinline__ i32 tm_floormod(i32 a, i32 b) {
  if (b == 0 || b == -1) return 0;
  const i32 r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
__device__ __forceinline__ u32 tm_floordiv(u32 a, u32 b) { return b ? a / b : 0u; }
__device__ __forceinline__ u32 tm_floormod(u32 a, u32 b) { return b ? a % b : 0u; }
// f32 division and square root by the call's cuda_math: 'ieee' (no define) correctly rounded; 'approx' and 'fast'
// the f32 PTX XLA:GPU emits, div.full (at most 2 ulp) and sqrt.approx (backends/kernel/__init__.py:9-12, 141-146)
#if defined(TM_MATH_APPROX) || defined(TM_MATH_FAST)
__device__ __forceinline__ float tm_fdiv(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float tm_fsqrt(float a) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
#else
__device__ __forceinline__ float tm_fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float tm_fsqrt(float a) { return __fsqrt_rn(a); }
#endif
}  // namespace tmb
// the entry point's launch bounds: min_blocks_per_sm=N caps registers for N resident blocks per SM
#ifdef TM_MIN_BLOCKS
#define TM_MAIN_BOUNDS __launch_bounds__(TM_BLOCK, TM_MIN_BLOCKS)
#else
#define TM_MAIN_BOUNDS __launch_bounds__(TM_BLOCK)
#endif
"""


# ------------------------------------------------------------------------------------------------ program analysis
def _ids(xs):
    return {x.id for x in xs if isinstance(x, T.Var)}


def _uses(eqns):
    """the variables `eqns` read, an inner while loop's reads of values defined before it included"""
    u = set()
    for e in eqns:
        u |= _ids(e.ins)
        if e.prim == "while":
            p = e.params
            inner = _uses(p["cond"]) | _uses(p["body"]) | _ids(p["body_out"]) | _ids([p["cond_out"]])
            u |= inner - _defs_deep(p["cond"] + p["body"]) - _ids(p["carry"])
    return u


def _defs_deep(eqns):
    return {o.id for e in T._walk(eqns) for o in e.outs}


def _defs(eqns):
    d = set()
    for e in eqns:
        d |= _ids(e.outs)
    return d


class Item:
    """the layout facts of a traced item shared by its forward and reverse lowering"""

    def __init__(self, tr, in_specs, name, exact=(), acc=None):
        self.tr, self.name = tr, name
        self.exact = set(exact)                 # Sum(fixed_point=True) f32 outputs: exact bins
        # the wider accumulators: name -> ("f64",) | ("i64",) | ("wide", torch dtype, scale)
        self.acc = dict(acc or {})
        self.in_specs = list(in_specs)
        npi = tr.n_per_item
        self.pi = tr.inputs[:npi]
        self.bc = [b.var if isinstance(b, T.Table) else b for b in tr.inputs[npi:]]
        for b in self.bc:
            if not isinstance(b, T.Var):
                raise LowerError("tallymap_b200.lower: broadcast operands are scalars, vectors or tables")
        if any(e.prim == "emit" for e in tr.cond):
            raise LowerError("tallymap_b200.lower: the loop condition may not emit")
        self.specs = list(tr.specs.items())     # [(name, (shape, dtype))]
        # the per-item input variables, each with its loader
        self.loads = []                         # (var, C expression with `item`)
        for j, (x, s) in enumerate(zip(self.pi, self.in_specs[:npi])):
            if isinstance(x, T.Key):
                self.loads += [(x.a, f"__ldg(&c.in{j}[item]).x"), (x.b, f"__ldg(&c.in{j}[item]).y")]
            elif isinstance(x, tuple):
                self.loads += [(v, f"__ldg(&c.in{j}[item * {len(x)} + {i}])") for i, v in enumerate(x)]
            else:
                self.loads.append((x, f"__ldg(&c.in{j}[item])"))
        self.bc_ids = {b.id: k for k, b in enumerate(self.bc)}
        # spawning items (tallymap/_tally.py spawn): a child carries the per-item input leaves, in load order
        self.spawns = any(e.prim == "spawn" for e in tr.body + tr.post)
        self.post_spawns = any(e.prim == "spawn" for e in tr.post)
        if self.spawns and tr.records:
            raise NotImplementedError("tallymap_b200: Records outputs of a spawning item are not lowered")
        # Records slot claims of the jaxpr front end: one launch counter per claimed tally (by its output position)
        self.claims = any(e.prim == "claim" for e in T._walk(tr.pre + tr.body + tr.post))
        if self.claims and self.spawns:
            raise NotImplementedError("tallymap_b200: Records slot claims in a spawning item are not lowered")
        # step counters: carries that start at 0 and gain 1 per step equal the step index (not stored by the replay)
        self.counter = set()
        by_id = {o.id: e for e in tr.body for o in e.outs}
        for j, (ci, co) in enumerate(zip(tr.carry_in, tr.body_out)):
            if isinstance(ci, T.Lit) and ci.dtype == T.I32 and ci.value == 0 and isinstance(co, T.Var):
                e = by_id.get(co.id)
                if e is not None and e.prim == "add" and len(e.ins) == 2 and isinstance(e.ins[0], T.Var) and \
                        e.ins[0].id == tr.carry[j].id and isinstance(e.ins[1], T.Lit) and e.ins[1].value == 1:
                    self.counter.add(j)
        # pre-loop values (inputs included) that later code reads: kept in the per-thread context
        later = _uses(tr.cond) | _uses(tr.body) | _uses(tr.post) | _ids(tr.body_out) | _ids(tr.results) | \
            _ids([tr.cond_out])
        pre_defined = _defs(tr.pre) | {v.id for v, _ in self.loads}
        self.saved = sorted(later & pre_defined)
        self.vars = {}
        for v, _ in self.loads:
            self.vars[v.id] = v
        for e in tr.pre + tr.cond + tr.body + tr.post:
            for o in e.outs:
                self.vars[o.id] = o
        for b in self.bc:
            self.vars[b.id] = b
        for v in tr.carry + tr.post_carry:
            self.vars[v.id] = v


def _bc_setup(k, b):
    """setup's line for broadcast operand k: a scalar is read once into the context, a table keeps its pointer"""
    if b.dtype in T.TABLE_ELT:
        return f"    c.b{k} = static_cast<{CTYPE[b.dtype]}>(P.p[kBc{k}]);"
    return f"    c.b{k} = __ldg(static_cast<const {CTYPE[b.dtype]}*>(P.p[kBc{k}]));"


def _names_pre(it):
    """C names in start(): locals for everything"""
    return {i: f"v{i}" for i in it.vars} | {i: f"c.b{k}" for i, k in it.bc_ids.items()}


def _names_loop(it, carry, state="s"):
    n = {i: f"c.p{i}" for i in it.saved} | {i: f"c.b{k}" for i, k in it.bc_ids.items()}
    for j, v in enumerate(carry):
        n[v.id] = f"{state}.c{j}"
    return n


def _spawn_code(when_c, leaves_c):
    """one spawn: the next of the step's two child slots (the spawn runtime's step interface)"""
    st = [f"if ({when_c}) {{ Child& o_ = n_out == 0 ? o0 : o1;"]
    st += [f" o_.l{m} = {v};" for m, v in enumerate(leaves_c)]
    st.append(" ++n_out; }")
    return "".join(st)


def _bits(v, dt):
    """a 4-byte value's bits as an i32 (a record word)"""
    return f"__float_as_int({v})" if dt == T.F32 else f"(i32)({v})"


def _from_bits(w, dt):
    return f"__int_as_float({w})" if dt == T.F32 else (f"({w} != 0)" if dt == T.BOOL else f"({CTYPE[dt]})({w})")


def _spawn_record_code(it, gen, last):
    """-> spawner(when, leaves) of the recording forward (the reference's rec_primal, _reverse_spawn.py:85-109): the
    child goes to the step's child slot as in the forward, and gets a record slot (one atomic per converged group of
    spawning lanes) holding its leaves' bits, the spawning item's previous newest child (`prev`: the item's children
    form a chain, newest first) and, once the child has run, its own newest child (`last`); its generation goes to the
    compact generation array.  gen / last: C lvalues of the spawning item's generation and newest child."""
    L = len(it.loads)
    RS = L + 2

    def spawner(when_c, leaves_c):
        st = [f"if ({when_c}) {{ Child& o_ = n_out == 0 ? o0 : o1;"]
        st += [f" o_.l{m} = {v};" for m, v in enumerate(leaves_c)]
        st.append(" const unsigned m_ = __activemask(); const int ld_ = __ffs(m_) - 1; const int ln_ = threadIdx.x & 31;"
                  " unsigned long long b_ = 0ull; if (ln_ == ld_) b_ = atomicAdd(c.tree, (unsigned long long)__popc(m_));"
                  " b_ = __shfl_sync(m_, b_, ld_) + (unsigned long long)__popc(m_ & ((1u << ln_) - 1u));"
                  " const i32 r_ = b_ < c.R ? (i32)b_ : -1;"
                  f" if (r_ >= 0) {{ i32* w_ = c.rec + (i64)r_ * {RS};")
        st += [f" w_[{m}] = {_bits(f'o_.l{m}', v.dtype)};" for m, (v, _) in enumerate(it.loads)]
        st.append(f" w_[{L}] = {last}; w_[{L + 1}] = -1;"
                  f" c.rgen[r_] = (unsigned short)({gen} + 1 < 65535 ? {gen} + 1 : 65535); }}")
        st.append(f" o_.slot = r_; o_.gen = {gen} + 1; {last} = r_; ++n_out; }}")
        return "".join(st)
    return spawner


def _emit_code(eqns, names, emitter, indent="    ", skip_emits=False, appender=None, spawner=None, claimer=None):
    """straight-line C for eqns; names: id -> C expression (updated with the locals defined here)"""
    out = []
    for e in eqns:
        a = [names[x.id] if isinstance(x, T.Var) else c_lit(x) for x in e.ins]
        if e.prim == "spawn":
            if spawner is not None:
                out.append(indent + spawner(a[0], a[1:]))
            continue
        if e.prim == "append":
            if appender is not None:
                out.append(indent + appender(e.params["records"], a[0], a[1:]))
            continue
        if e.prim == "while":
            # an inner loop (the reference's while rule, backends/kernel/op_table.py:1414-1450): its carry in
            # mutable locals, the condition and body re-evaluated each iteration, the next carry through temporaries
            p = e.params
            for o, x in zip(e.outs, e.ins):
                out.append(f"{indent}{CTYPE[o.dtype]} v{o.id} = {_ref(x, names)};")
                names[o.id] = f"v{o.id}"
            for cv, o in zip(p["carry"], e.outs):
                names[cv.id] = f"v{o.id}"
            out.append(f"{indent}while (true) {{")
            sub = dict(skip_emits=skip_emits, appender=appender, spawner=spawner, claimer=claimer)
            out += _emit_code(p["cond"], names, emitter, indent + "  ", **sub)
            out.append(f"{indent}  if (!({_ref(p['cond_out'], names)})) break;")
            out += _emit_code(p["body"], names, emitter, indent + "  ", **sub)
            nxt = [f"const {CTYPE[o.dtype]} n{o.id} = {_ref(b, names)};" for o, b in zip(e.outs, p["body_out"])]
            out += [indent + "  " + x for x in nxt]
            out += [f"{indent}  v{o.id} = n{o.id};" for o in e.outs]
            out.append(f"{indent}}}")
            continue
        if e.prim == "claim":
            if claimer is None:
                raise LowerError("tallymap_b200.lower: a Records slot claim (tallymap_claim) lowers in the forward "
                                 "program only: the reference's derived programs run its fill twin")
            out.append(indent + claimer(e, a[0]))
            names[e.outs[0].id] = f"v{e.outs[0].id}"
            continue
        if e.prim == "emit":
            if not skip_emits:
                st = emitter(e.params["tally"], a[0], a[1])
                # (a third operand: the emit's predicate, a write inside a lax.cond branch)
                out.append(indent + (f"if ({a[2]}) {{ {st} }}" if len(a) > 2 else st))
            continue
        if e.prim == "threefry":
            o0, o1 = e.outs
            out.append(f"{indent}u32 v{o0.id}, v{o1.id};")
            out.append(f"{indent}threefry2x32({a[0]}, {a[1]}, {a[2]}, {a[3]}, v{o0.id}, v{o1.id});")
            names[o0.id], names[o1.id] = f"v{o0.id}", f"v{o1.id}"
            continue
        o = e.outs[0]
        out.append(f"{indent}const {CTYPE[o.dtype]} v{o.id} = {c_expr(e, a)};")
        names[o.id] = f"v{o.id}"
    return out


def _ref(x, names):
    return names[x.id] if isinstance(x, T.Var) else c_lit(x)


# ------------------------------------------------------------------------------------------------ forward program
def forward_source(it, standalone=True, record=False, mode="one"):
    """-> (C source of the forward ITEM + its extern "C" entry point, shared-memory bytes); standalone=False: the
    ITEM struct alone (for a combined program).  record (a spawning item): the recording forward of the tree adjoint
    -- the forward's outputs plus a record of every child (_spawn_record_code) and each root's newest child.
    mode, for Records outputs (tallymap.Records, _api.py:132-148): "one" -- one pass, a raw slot per append and the
    record's key beside it (canonicalised after the launch); "count" -- the count pass of count-then-fill: the
    per-item record counts alone (no records written, no emits); "fill" -- the fill pass: per output, the items'
    counts and canonical offsets are per-item operands after the item's own, and record k of item i goes straight to
    slot offset[i] + k while k < count[i] (an item appending a different number is seen by its count)"""
    tr = it.tr
    npi, nbc = len(it.pi), len(it.bc)
    sp = it.spawns
    rec = bool(record and sp)
    count, fill = mode == "count", mode == "fill"
    lines = [('#include "tm_spawn.cuh"' if sp else "") + PRELUDE, "namespace tmb {", "struct GenFwd {"]
    # buffer indices: per-item, broadcast, consts, order | tallies, [exact words], [records], [ring sequence and
    # control words], ctl, stats | ys, [record counts], trunc, [ring]
    recs = list(tr.records.items())         # [(name, (capacity, ((field, dtype), ...)))]
    idx = 0
    enum = []
    for j in range(npi):
        enum.append(f"kIn{j} = {idx}"); idx += 1
    if fill:
        for r in range(len(recs)):
            enum.append(f"kRCnt{r} = {idx}"); idx += 1
            enum.append(f"kROff{r} = {idx}"); idx += 1
    for k in range(nbc):
        enum.append(f"kBc{k} = {idx}"); idx += 1
    enum.append(f"kConsts = {idx}"); idx += 1
    enum.append(f"kOrder = {idx}"); idx += 1
    for t, _ in enumerate(it.specs):
        enum.append(f"kT{t} = {idx}"); idx += 1
    for t, (name, _) in enumerate(it.specs):
        if name in it.exact:
            enum.append(f"kX{t} = {idx}"); idx += 1
        elif it.acc.get(name, ("",))[0] == "wide":
            enum.append(f"kW{t} = {idx}"); idx += 1
    for r, (rname, (cap, fields)) in enumerate(recs):
        if count:
            continue
        for f in range(len(fields)):
            enum.append(f"kR{r}F{f} = {idx}"); idx += 1
        if fill:
            continue
        enum.append(f"kR{r}Cid = {idx}"); idx += 1
        enum.append(f"kR{r}K = {idx}"); idx += 1
        enum.append(f"kR{r}Ctr = {idx}"); idx += 1
    if it.claims:
        enum.append(f"kClaims = {idx}"); idx += 1
    if sp:
        enum.append(f"kSeq = {idx}"); idx += 1
        enum.append(f"kQctl = {idx}"); idx += 1
    enum.append(f"kCtl = {idx}"); idx += 1
    enum.append(f"kStats = {idx}"); idx += 1
    if rec:
        enum.append(f"kTree = {idx}"); idx += 1
    for r in range(len(tr.results)):
        enum.append(f"kY{r} = {idx}"); idx += 1
    for r in range(len(recs)):
        enum.append(f"kR{r}N = {idx}"); idx += 1
    enum.append(f"kTrunc = {idx}"); idx += 1
    if rec:
        enum.append(f"kLast = {idx}"); idx += 1
    if sp:
        enum.append(f"kQueue = {idx}"); idx += 1
    if rec:
        enum.append(f"kRecord = {idx}"); idx += 1
        enum.append(f"kRecGen = {idx}"); idx += 1
    enum.append(f"kNBuf = {idx}")
    lines.append("  enum { " + ", ".join(enum) + " };")
    if sp:
        # a child: the per-item input leaves (4 bytes each), in the order start() loads them (recording: its record
        # slot and generation too)
        lines.append("  enum { kConstM, kConstQ" + (", kConstR" if rec else "") + " };")
        lines.append("  struct Child { " + " ".join(f"{CTYPE[v.dtype]} l{m};" for m, (v, _) in enumerate(it.loads))
                     + (" i32 slot; i32 gen;" if rec else "") + " };")
        if it.post_spawns:
            lines.append("  static constexpr bool kPostSpawn = true;")
    # privatised tallies
    smem, priv = 0, {}
    for t, (name, (shape, dt)) in enumerate(it.specs):
        S = int(np.prod(shape, dtype=np.int64)) if shape else 1
        nbytes = S * 44 if name in it.exact else S * 4
        if name not in it.acc and nbytes <= (4 * PRIV_BYTES if name in it.exact else PRIV_BYTES):
            priv[name] = (t, smem, S, dt)
            smem += (nbytes + 15) // 16 * 16
    lines.append(f"  static constexpr int kSmemBytes = {max(smem, 16)};")
    # context
    ctx = ["  struct Ctx {"]
    for j, s in enumerate(it.in_specs[:npi]):
        ctx.append(f"    const {_in_ctype(s)}* in{j};")
    for k, b in enumerate(it.bc):
        ctx.append(f"    {CTYPE[b.dtype]} b{k};")       # (a table: its pointer)
    ctx.append("    i32 M;")
    ctx.append("    i32* stats;")
    tinfo = {}
    for t, (name, (shape, dt)) in enumerate(it.specs):
        S = int(np.prod(shape, dtype=np.int64)) if shape else 1
        ct = _out_ctype(it, name, dt)
        ctx.append(f"    {ct}* g{t};")
        if name in it.exact:
            ctx.append(f"    u64* x{t};")
            if name in priv:
                ctx.append(f"    u64* sx{t};")
        elif name in priv:
            ctx.append(f"    {ct}* s{t};")
        elif it.acc.get(name, ("",))[0] == "wide":
            ctx.append(f"    unsigned long long* w{t};")
        tinfo[name] = (t, S, dt, name in priv)
    for r, y in enumerate(tr.results):
        ctx.append(f"    {CTYPE[y.dtype] if y.dtype != T.BOOL else 'uint8_t'}* y{r};")
    ctx.append("    uint8_t* trunc;")
    for i in it.saved:
        ctx.append(f"    {CTYPE[it.vars[i].dtype]} p{i};")
    for r, (rname, (cap, fields)) in enumerate(recs):
        if not count:
            for f, (fname, dt) in enumerate(fields):
                ctx.append(f"    {CTYPE[dt]}* r{r}f{f};")
        if mode == "one":
            ctx += [f"    i32* r{r}cid;", f"    i32* r{r}k;", f"    unsigned long long* r{r}ctr;"]
        if fill:
            ctx += [f"    const i32* rcnt{r};", f"    const long long* roff{r};", f"    i32 rn{r};", f"    long long ro{r};"]
        ctx.append(f"    i32* r{r}n;")
    if recs:
        ctx.append("    i64 item;")
    if it.claims:
        ctx.append("    unsigned long long* claims;   // per tally: its Records slot counter")
    if rec:
        ctx += ["    i32* rec;", "    unsigned short* rgen;", "    unsigned long long* tree;", "    i32* lastout;",
                "    u64 R;"]
    ctx.append("  };")
    lines += ctx
    lines.append("  struct State {")
    lines.append("    i32 kc;")
    for j, v in enumerate(tr.carry):
        lines.append(f"    {CTYPE[v.dtype]} c{j};")
    for r in range(len(recs)):
        lines.append(f"    i32 a{r};   // records appended by the item so far")
    if rec:
        lines.append("    i32 me, gen, last;   // own record slot (-1: a root), generation, newest child's slot")
    lines.append("  };")
    # setup
    lines.append("  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {")
    for j, s in enumerate(it.in_specs[:npi]):
        lines.append(f"    c.in{j} = static_cast<const {_in_ctype(s)}*>(P.p[kIn{j}]);")
    for k, b in enumerate(it.bc):
        lines.append(_bc_setup(k, b))
    lines.append("    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));")
    lines.append("    c.stats = static_cast<i32*>(P.p[kStats]);")
    for name, (t, S, dt, pv) in tinfo.items():
        ct = _out_ctype(it, name, dt)
        lines.append(f"    c.g{t} = static_cast<{ct}*>(P.p[kT{t}]);")
        if name in it.exact:
            lines.append(f"    c.x{t} = static_cast<u64*>(P.p[kX{t}]);")
            if pv:
                lines.append(f"    c.sx{t} = reinterpret_cast<u64*>(smem + {priv[name][1]});")
        elif pv:
            lines.append(f"    c.s{t} = reinterpret_cast<{ct}*>(smem + {priv[name][1]});")
        elif it.acc.get(name, ("",))[0] == "wide":
            lines.append(f"    c.w{t} = static_cast<unsigned long long*>(P.p[kW{t}]);")
    for r, y in enumerate(tr.results):
        lines.append(f"    c.y{r} = static_cast<{CTYPE[y.dtype] if y.dtype != T.BOOL else 'uint8_t'}*>(P.p[kY{r}]);")
    lines.append("    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);")
    for r, (rname, (cap, fields)) in enumerate(recs):
        if not count:
            for f, (fname, dt) in enumerate(fields):
                lines.append(f"    c.r{r}f{f} = static_cast<{CTYPE[dt]}*>(P.p[kR{r}F{f}]);")
        if mode == "one":
            lines += [f"    c.r{r}cid = static_cast<i32*>(P.p[kR{r}Cid]);",
                      f"    c.r{r}k = static_cast<i32*>(P.p[kR{r}K]);",
                      f"    c.r{r}ctr = static_cast<unsigned long long*>(P.p[kR{r}Ctr]);"]
        if fill:
            lines += [f"    c.rcnt{r} = static_cast<const i32*>(P.p[kRCnt{r}]);",
                      f"    c.roff{r} = static_cast<const long long*>(P.p[kROff{r}]);"]
        lines.append(f"    c.r{r}n = static_cast<i32*>(P.p[kR{r}N]);")
    if it.claims:
        lines.append("    c.claims = static_cast<unsigned long long*>(P.p[kClaims]);")
    if rec:
        lines += ["    c.rec = static_cast<i32*>(P.p[kRecord]);",
                  "    c.rgen = static_cast<unsigned short*>(P.p[kRecGen]);",
                  "    c.tree = static_cast<unsigned long long*>(P.p[kTree]);",
                  "    c.lastout = static_cast<i32*>(P.p[kLast]);",
                  "    c.R = (u64)(u32)__ldg(static_cast<const i32*>(P.p[kConsts]) + kConstR);"]
    lines.append("  }")
    lines.append("  __device__ static void stage(const Params&, unsigned char*) {}")
    rindex = {rname: r for r, (rname, _) in enumerate(recs)}

    def appender_for(counter):
        def appender(rname, when_c, vals_c):
            """one record: the next raw slot of the output (one atomic, the counter keeps the true total), its
            fields and its key (item, ordinal); -0.0 is stored as +0.0 (tallymap.Records).  Count pass: the ordinal
            alone; fill pass: the fields at the canonical slot offset + ordinal, while the ordinal is below the
            item's count"""
            r = rindex[rname]
            cap, fields = tr.records[rname]
            if count:
                return f"if ({when_c}) {counter(r)} += 1;"
            if fill:
                st = [f"if ({when_c}) {{ if ({counter(r)} < c.rn{r}) {{ const long long s_ = c.ro{r} + {counter(r)};"]
                for f, ((fname, dt), v) in enumerate(zip(fields, vals_c)):
                    st.append(f" c.r{r}f{f}[s_] = {v}{' + 0.0f' if dt == T.F32 else ''};")
                st.append(f" }} {counter(r)} += 1; }}")
                return "".join(st)
            st = [f"if ({when_c}) {{ const unsigned long long o_ = atomicAdd(c.r{r}ctr, 1ull); "
                  f"if (o_ < {int(cap)}ull) {{"]
            for f, ((fname, dt), v) in enumerate(zip(fields, vals_c)):
                st.append(f" c.r{r}f{f}[o_] = {v}{' + 0.0f' if dt == T.F32 else ''};")
            st.append(f" c.r{r}cid[o_] = (i32)c.item; c.r{r}k[o_] = {counter(r)}; }} {counter(r)} += 1; }}")
            return "".join(st)
        return appender

    def claimer(e, when_c):
        """a Records slot claim (tallymap/backends/kernel/kernel.py:1052-1070): the next slot of the claimed
        tally's raw buffer, one atomic on its launch counter; -1 when not `when` or past the capacity"""
        o, t = e.outs[0].id, tinfo[e.params["tally"]][0]
        return (f"i32 v{o} = -1; if ({when_c}) {{ const unsigned long long o_ = atomicAdd(&c.claims[{t}], 1ull); "
                f"if (o_ < {int(e.params['capacity'])}ull) v{o} = (i32)o_; }}")

    def emitter(name, idx_c, v_c):
        t, S, dt, pv = tinfo[name]
        acc = it.acc.get(name)
        if acc is not None:
            drop = f"const i32 b_ = {idx_c}; if ((u32)b_ >= {S}u) atomicAdd(&c.stats[kStDroppedEmits], 1); else"
            if acc[0] == "f64":
                return f"{{ {drop} if ({v_c}) atomicAdd(&c.g{t}[b_], (double)({v_c})); }}"
            if acc[0] == "i64":
                return (f"{{ {drop} if ({v_c}) atomicAdd((unsigned long long*)&c.g{t}[b_], "
                        f"(unsigned long long)(long long)({v_c})); }}")
            return (f"{{ {drop} WideSum::emit(c.w{t}, (i32*)(c.w{t} + {S}), (u32*)(c.w{t} + {S}) + {S}, c.stats, "
                    f"b_, (double)({v_c}) * {float(acc[2])!r}); }}")
        if name in it.exact:
            return f"ExactSum<{S}>::emit({'c.sx' if pv else 'c.x'}{t}, c.stats, {idx_c}, {v_c});"
        if dt == T.F32:
            if pv:
                return f"SumPriv<{S}>::emit(c.s{t}, c.stats, {idx_c}, {v_c});"
            return (f"{{ const i32 b_ = {idx_c}; if ((u32)b_ >= {S}u) atomicAdd(&c.stats[kStDroppedEmits], 1); "
                    f"else fatom_warp_window(c.g{t}, nullptr, b_, -1, {v_c}); }}")
        tgt = f"c.s{t}" if pv else f"c.g{t}"
        return (f"{{ const i32 b_ = {idx_c}; if ((u32)b_ >= {S}u) atomicAdd(&c.stats[kStDroppedEmits], 1); "
                f"else if ({v_c}) atomicAdd(&{tgt}[b_], {v_c}); }}")

    # start: inputs, pre-loop code, the saved values, the initial carry (start_child: the same from a child's leaves)
    for head, src in [("State start(Ctx& c, i64 item)", [ld for _, ld in it.loads])] + \
            ([("State start_child(Ctx& c, const Child& ch)", [f"ch.l{m}" for m in range(len(it.loads))])]
             if sp else []):
        lines.append(f"  __device__ static {head} {{")
        names = _names_pre(it)
        for (v, _), ld in zip(it.loads, src):
            lines.append(f"    const {CTYPE[v.dtype]} v{v.id} = {ld};")
        if recs:
            # (records appended before the loop: the item's first ordinals)
            lines.append("    c.item = item;")
            lines += [f"    i32 a{r} = 0;" for r in range(len(recs))]
            if fill:
                lines += [f"    c.rn{r} = __ldg(&c.rcnt{r}[item]); c.ro{r} = __ldg(&c.roff{r}[item]);"
                          for r in range(len(recs))]
        lines += _emit_code(tr.pre, names, emitter, appender=appender_for(lambda r: f"a{r}") if recs else None,
                            skip_emits=count, claimer=claimer)
        for i in it.saved:
            lines.append(f"    c.p{i} = {names[i]};")
        lines.append("    State s;")
        lines.append("    s.kc = 0;")
        for r in range(len(recs)):
            lines.append(f"    s.a{r} = a{r};")
        if rec:
            lines.append("    s.me = ch.slot; s.gen = ch.gen; s.last = -1;" if "start_child" in head else
                         "    s.me = -1; s.gen = 0; s.last = -1;")
        for j, x in enumerate(tr.carry_in):
            lines.append(f"    s.c{j} = {_ref(x, names)};")
        lines.append("    return s;")
        lines.append("  }")
    lines += _pred_fn(it)
    lines.append("  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) {")
    lines.append("    return s.kc < c.M && pred(c, s);")
    lines.append("  }")
    split = _draw_split(it)
    if split is not None:
        # the body's draws evaluated ahead (kUnroll steps per iteration), the rest applied step by step; and the
        # state, the saved per-item context and the item index movable to another thread (end-of-launch compaction)
        dcode, rest, live = _draw_code(it, split)
        lines += dcode
        lines.append("  __device__ __forceinline__ static void apply(const Ctx& c, State& s, const Draw& d) {")
        names = _names_loop(it, tr.carry)
        for i in live:
            names[i] = f"d.d{i}"
        lines += _emit_code(rest, names, emitter, claimer=claimer)
        lines += _assign_carry(it, names)
        lines.append("  }")
        lines.append("  __device__ __forceinline__ static void step(const Ctx& c, State& s) { apply(c, s, draw(c, s, 0)); }")
    if not sp and not recs:
        lines.append("  struct Parked {")
        lines.append("    State s;")
        lines += [f"    {CTYPE[it.vars[i].dtype]} p{i};" for i in it.saved]
        lines.append("    i32 item;")
        lines.append("  };")
        lines.append("  __device__ __forceinline__ static Parked park(const Ctx& c, const State& s, i64 item) {")
        lines.append("    Parked p;")
        lines.append("    p.s = s;")
        lines += [f"    p.p{i} = c.p{i};" for i in it.saved]
        lines.append("    p.item = (i32)item;")
        lines.append("    return p;")
        lines.append("  }")
        lines.append("  __device__ __forceinline__ static State unpark(Ctx& c, const Parked& p, i64& item) {")
        lines += [f"    c.p{i} = p.p{i};" for i in it.saved]
        lines.append("    item = p.item;")
        lines.append("    return p.s;")
        lines.append("  }")
    if sp:
        lines.append("  __device__ __forceinline__ static void step(const Ctx& c, State& s, Child& o0, Child& o1, "
                     "int& n_out) {")
    elif split is None:
        lines.append("  __device__ __forceinline__ static void step(const Ctx& c, State& s) {")
    if sp or split is None:
        names = _names_loop(it, tr.carry)
        lines += _emit_code(tr.body, names, emitter, appender=appender_for(lambda r: f"s.a{r}"),
                            spawner=_spawn_record_code(it, "s.gen", "s.last") if rec else _spawn_code,
                            skip_emits=count, claimer=claimer)
        lines += _assign_carry(it, names)
        lines.append("  }")
    if not sp:
        lines.append("  __device__ static void finish(const Ctx& c, const State& s, i64 item) {")
    elif it.post_spawns:
        lines.append("  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child, Child& o0, "
                     "Child& o1, int& n_out) {")
    else:
        lines.append("  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child) {")
    names = _names_loop(it, tr.post_carry)
    for r in range(len(recs)):
        lines.append(f"    i32 a{r} = s.a{r};")
    if rec:
        lines.append("    i32 last_ = s.last;")
    lines += _emit_code(tr.post, names, emitter, appender=appender_for(lambda r: f"a{r}"),
                        spawner=_spawn_record_code(it, "s.gen", "last_") if rec else _spawn_code, skip_emits=count,
                        claimer=claimer)
    if sp:
        # a child's per-item results are discarded (tallymap/_tally.py:285-286); its truncation is counted
        lines.append("    const bool tr_ = s.kc >= c.M && pred(c, s);")
        if rec:
            # (the child's record gets its newest child: the head of its children's chain)
            lines.append(f"    if (child && s.me >= 0) c.rec[(i64)s.me * {len(it.loads) + 2} + {len(it.loads) + 1}] "
                         "= last_;")
            lines.append("    if (!child) c.lastout[item] = last_;")
        lines.append("    if (child) { if (tr_) atomicAdd(&c.stats[kStChildrenTruncated], 1); return; }")
    for r, y in enumerate(tr.results):
        lines.append(f"    c.y{r}[item] = {_ref(y, names)};")
    for r in range(len(recs)):
        lines.append(f"    c.r{r}n[item] = a{r};")
    lines.append("    c.trunc[item] = " + ("tr_ ? 1 : 0;" if sp else "(s.kc >= c.M && pred(c, s)) ? 1 : 0;"))
    lines.append("  }")
    lines.append("  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {")
    for name, (t, S, dt, pv) in tinfo.items():
        if not pv:
            continue
        if name in it.exact:
            lines.append(f"    ExactSum<{S}>::flush(c.sx{t}, c.x{t}, c.stats, tid, nth);")
        elif dt == T.F32:
            lines.append(f"    SumPriv<{S}>::flush(c.s{t}, c.g{t}, tid, nth);")
        else:
            lines.append(f"    for (int b = tid; b < {S}; b += nth) if (c.s{t}[b]) atomicAdd(&c.g{t}[b], c.s{t}[b]);")
    lines.append("  }")
    lines.append("  __device__ static void epilogue(const Ctx& c, int tid, int nth) {")
    for name, (t, S, dt, pv) in tinfo.items():
        if name in it.exact:
            lines.append(f"    ExactSum<{S}>::readout(c.x{t}, c.g{t}, c.stats, tid, nth);")
        elif it.acc.get(name, ("",))[0] == "wide":
            inv = 1.0 / float(it.acc[name][2])
            lines.append(f"    WideSum::readout(c.w{t}, (const i32*)(c.w{t} + {S}), (const u32*)(c.w{t} + {S}) + {S}, "
                         f"c.g{t}, {S}, {inv!r}, c.stats, tid, nth);")
    lines.append("  }")
    lines.append("};")
    if not standalone:
        return "\n".join(lines[2:]), max(smem, 16)
    lines.append("}  // namespace tmb")
    lines.append('extern "C" __global__ void TM_MAIN_BOUNDS tm_main(const tmb::Params P, const long long n) {')
    lines.append(f"  tmb::{'spawn_body' if sp else 'forward_body'}<tmb::GenFwd>(P, n);")
    lines.append("}")
    return "\n".join(lines), max(smem, 16)


def _out_dtype(it, name, dt):
    """the torch dtype of a Sum output"""
    acc = it.acc.get(name)
    if acc is None:
        return TDTYPE[dt]
    return {"f64": torch.float64, "i64": torch.int64}.get(acc[0]) or acc[1]


def _out_ctype(it, name, dt):
    """the C type of a Sum output's buffer: float / i32, double / long long for the wider accumulators"""
    acc = it.acc.get(name)
    if acc is None:
        return "float" if dt == T.F32 else "i32"
    if acc[0] == "f64":
        return "double"
    if acc[0] == "i64":
        return "long long"
    return {torch.float64: "double", torch.int64: "long long", torch.int32: "i32"}[acc[1]]


def _in_ctype(s):
    if s == "key":
        return "uint2"
    if isinstance(s, tuple):
        return CTYPE[s[0]]
    return CTYPE[s]


def _pred_fn(it):
    tr = it.tr
    out = ["  __device__ __forceinline__ static bool pred(const Ctx& c, const State& s) {"]
    names = _names_loop(it, tr.carry)
    out += _emit_code(tr.cond, names, None)
    out.append(f"    return {_ref(tr.cond_out, names)};")
    out.append("  }")
    return out


DRAW_UNROLL = 4      # steps drawn ahead per iteration (tm_runtime.cuh run_step) when the body's draws allow it
DRAW_LIVE_MAX = 8    # at most this many drawn values held across the unrolled steps (DRAW_UNROLL x the values a step
                     # keeps): the walk keeps two a step (8 held; the draw-ahead pays there), the photon four uniforms
                     # and more (16+ held beside a heavy step: its forward 48 -> 99 ms), so it draws step by step
_DRAW_PRIMS = ("threefry", "bits", "uniform01")


def _draw_split(it):
    """The body's equations that depend only on the per-item context (the saved pre-loop values), the broadcast
    operands, literals and the step counters (carries equal to the step index): their values at step kc + j are
    known before step kc runs, so the runtime can evaluate several steps' worth together (independent threefry
    chains; tm_runtime.cuh, run_step).  -> (draw equations, the other equations, ids of draw values the others or
    the carry update read) or None when the draws hold no threefry (nothing worth drawing ahead) or more values
    than DRAW_LIVE_MAX would hold across the unrolled steps."""
    tr = it.tr
    if it.spawns or tr.records:
        return None
    fixed = set(it.saved) | set(it.bc_ids) | {tr.carry[j].id for j in it.counter}
    draws, rest, dset = [], [], set()
    for e in tr.body:
        ok = e.prim not in ("emit", "spawn", "append", "claim", "while") and \
            all(not isinstance(x, T.Var) or x.id in fixed or x.id in dset for x in e.ins)
        if ok:
            draws.append(e)
            dset |= _ids(e.outs)
        else:
            rest.append(e)
    if not any(e.prim in _DRAW_PRIMS for e in draws):
        return None
    live = sorted(dset & (_uses(rest) | _ids(tr.body_out)))
    if DRAW_UNROLL * len(live) > DRAW_LIVE_MAX:
        return None
    return draws, rest, live


def _draw_code(it, split):
    """the ITEM's kUnroll, Draw, draw(c, s, j) and apply(c, s, d) (step == apply(draw(0)))"""
    tr = it.tr
    draws, rest, live = split
    out = [f"  static constexpr int kUnroll = {DRAW_UNROLL};", "  struct Draw {"]
    out += [f"    {CTYPE[it.vars[i].dtype]} d{i};" for i in live] or ["    int unused;"]
    out.append("  };")
    out.append("  __device__ __forceinline__ static Draw draw(const Ctx& c, const State& s, int j) {")
    names = _names_loop(it, tr.carry)
    for jc in it.counter:          # a step counter at step kc + j: its value now plus j
        names[tr.carry[jc].id] = f"(i32)((u32)s.c{jc} + (u32)j)"
    out += _emit_code(draws, names, lambda *a: "")
    out.append("    Draw d;")
    out += [f"    d.d{i} = {names[i]};" for i in live]
    out.append("    return d;")
    out.append("  }")
    return out, rest, live


def _assign_carry(it, names, state="s"):
    tr = it.tr
    out = []
    for j, x in enumerate(tr.body_out):
        out.append(f"    const {CTYPE[tr.carry[j].dtype]} n{j} = {_ref(x, names)};")
    for j in range(len(tr.body_out)):
        out.append(f"    {state}.c{j} = n{j};")
    out.append(f"    {state}.kc += 1;")
    return out


# ------------------------------------------------------------------------------------------------ compilation
_COMPILED = {}


def _headers_digest():
    """the digest of the runtime headers a lowered source includes: part of a cached cubin's key"""
    if not hasattr(_headers_digest, "d"):
        h = hashlib.sha256()
        for f in sorted(os.listdir(CSRC)):
            if f.endswith((".cuh", ".h")):
                with open(os.path.join(CSRC, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
        _headers_digest.d = h.hexdigest()
    return _headers_digest.d


def cache_dir():
    """where compiled items are kept across processes (the reference's disk cubin cache,
    backends/kernel/__init__.py:71-128): $TALLYMAP_B200_CACHE, else the package's _cache directory, beside its
    built library; "" disables it"""
    d = os.environ.get("TALLYMAP_B200_CACHE")
    return os.path.join(os.path.dirname(CSRC), "_cache") if d is None else d


MATH_MODES = ("ieee", "approx", "fast")


def options_source(math="ieee", min_blocks=None):
    """-> (the defines a call's options put before a lowered source, tm_compile flags).  math: the reference's
    cuda_math (backends/kernel/__init__.py:141-146) -- 'ieee' correctly rounded f32 division and square root (this
    backend's default: bitwise against the CPU evaluator); 'approx' div.full / sqrt.approx; 'fast' approx plus FMA
    contraction of float multiply-adds.  min_blocks: the entry point's __launch_bounds__(block, min_blocks).  The
    defaults add nothing, so a default source is unchanged."""
    if math not in MATH_MODES:
        raise ValueError(f"tallymap_b200: cuda_math must be one of {MATH_MODES}, got {math!r}")
    head = "" if math == "ieee" else f"#define TM_MATH_{math.upper()} 1\n"
    if min_blocks is not None:
        if int(min_blocks) < 1 or int(min_blocks) > 32:
            raise ValueError(f"tallymap_b200: min_blocks_per_sm must be in 1..32, got {min_blocks!r}")
        head += f"#define TM_MIN_BLOCKS {int(min_blocks)}\n"
    return head, (1 if math == "fast" else 0)


def compile_kernel(source, note, n_buffers, smem_bytes, flags=0):
    """compile `source` (its entry point `tm_main`) for sm_100a with NVRTC and register it -> kernel id.  Cached per
    process by the source's digest (the reference's structural kernel cache, backends/kernel/__init__.py:71-128) and
    on disk by the digest of the source and the runtime headers (a cubin, registered with tm_register).  flags:
    tm_compile's (1: FMA contraction); a nonzero value enters the digest."""
    digest = hashlib.sha256(source.encode() + (b"" if not flags else f"/flags={flags}".encode())).hexdigest()
    kid = int(digest[:15], 16)          # a positive int64 id
    from . import _diagnostics as diagnostics
    if kid in _COMPILED:
        diagnostics.record_kernel(dict(tag=note, kernel=kid, source_sha256=digest, buffers=n_buffers,
                                       shared_bytes=smem_bytes, compile_s=0.0, cache="process"))
        return kid
    L = _lib.lib()
    d = cache_dir()
    t0 = time.perf_counter()
    path = os.path.join(d, hashlib.sha256((digest + _headers_digest()).encode()).hexdigest() + ".cubin") if d else None
    image = None
    compiled_here = False
    if path and os.path.exists(path):
        with open(path, "rb") as fh:
            image = fh.read()
    if image is None:
        compiled_here = True
        n = ctypes.c_size_t()
        _lib.check(L.tm_compile(source.encode(), CSRC.encode(), 128, flags, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value)
        _lib.check(L.tm_compile(source.encode(), CSRC.encode(), 128, flags, buf, n.value, ctypes.byref(n)))
        image = buf.raw[:n.value]
        if path:
            try:
                os.makedirs(d, exist_ok=True)
                tmp = f"{path}.{os.getpid()}.tmp"
                with open(tmp, "wb") as fh:
                    fh.write(image)
                os.replace(tmp, path)          # (atomic: a concurrent process sees the whole file or none)
            except OSError:
                pass                           # (a read-only home: no disk cache)
    _lib.check(L.tm_register(ctypes.c_int64(kid), image, len(image), note.encode(), n_buffers, smem_bytes, 128))
    _COMPILED[kid] = note
    diagnostics.record_kernel(dict(tag=note, kernel=kid, source_sha256=digest, buffers=n_buffers,
                                   shared_bytes=smem_bytes, compile_s=round(time.perf_counter() - t0, 3),
                                   cache="none" if compiled_here else "disk"))
    from . import backend
    backend.COMPILED[kid] = n_buffers
    return kid


# ------------------------------------------------------------------------------------------------ reverse program
def _prop(eqns, act):
    """add to `act` the float results that depend on a member of it (an inner loop's: by its carries' fixpoint)"""
    for e in eqns:
        if e.prim in ("emit", "threefry", "bits", "uniform01", "inrange", "floor", "round", "stop", "gather") \
                or not e.outs:
            continue
        if e.prim == "while":
            if _uses([e]) & act:
                _, cact = _inner_active(e, act)
                act.update(o.id for o, a_ in zip(e.outs, cact) if a_)
            continue
        if any(isinstance(x, T.Var) and x.id in act for x in e.ins):
            for o in e.outs:
                if o.dtype == T.F32:
                    act.add(o.id)


def _inner_active(e, act):
    """an inner loop's activity: (the active set inside it -- `act` plus its active carries and the body values
    that depend on them or on active values outside --, per carry whether it is an active float) by a fixpoint over
    its body, as _active does for the stepping loop"""
    p = e.params
    cact = [isinstance(x, T.Var) and x.id in act and cv.dtype == T.F32 for x, cv in zip(e.ins, p["carry"])]
    while True:
        inner = set(act) | {cv.id for cv, a_ in zip(p["carry"], cact) if a_}
        _prop(p["body"], inner)
        new = [cact[j] or (isinstance(b, T.Var) and b.id in inner and p["carry"][j].dtype == T.F32)
               for j, b in enumerate(p["body_out"])]
        if new == cact:
            return inner, cact
        cact = new


def _active(it, wrt, extra=()):
    """float variables that depend on the differentiated broadcast operands (tallymap/_reverse.py:208 `_active`);
    extra: more seeds (a spawning item's float per-item inputs: a child's may carry tangents)"""
    tr = it.tr
    act = {it.bc[k].id for k in wrt if it.bc[k].dtype == T.F32} | set(extra)

    def prop(eqns):
        _prop(eqns, act)
    prop(tr.pre)
    carry_act = [isinstance(x, T.Var) and x.id in act for x in tr.carry_in]
    while True:
        for j, v in enumerate(tr.carry):
            if carry_act[j] and v.dtype == T.F32:
                act.add(v.id)
        prop(tr.body)
        new = [carry_act[j] or (isinstance(x, T.Var) and x.id in act) for j, x in enumerate(tr.body_out)]
        if new == carry_act:
            break
        carry_act = new
    for j, v in enumerate(tr.post_carry):
        if carry_act[j] and v.dtype == T.F32:
            act.add(v.id)
    prop(tr.post)
    return act, [carry_act[j] and tr.carry[j].dtype == T.F32 for j in range(len(tr.carry))]


class _Rev:
    """reverse-mode code for a straight-line equation list: cotangent locals, first contribution assigned, later ones
    added (jax's add_jaxvals order)"""

    def __init__(self, active, indent="    ", tag="g", spawn_t=None, append_t=None, append_skip=None):
        self.active, self.ct, self.lines, self.indent, self.tag = active, {}, [], indent, tag
        self.n = 0
        self.spawn_t = spawn_t      # the transpose of a spawn (the tree adjoint), else spawns have no cotangent
        self.append_t = append_t    # the transpose of a Records append, else appends have no cotangent
        self.append_skip = append_skip  # (records, when, fields) -> C: an append without a cotangent, counted

    def add(self, x, expr):
        if not isinstance(x, T.Var) or x.id not in self.active:
            return
        if x.id in self.ct:
            nm = self.ct[x.id]
            self.lines.append(f"{self.indent}{nm} = {nm} + {expr};")
        else:
            self.n += 1
            nm = f"{self.tag}{x.id}_{self.n}"
            self.lines.append(f"{self.indent}float {nm} = {expr};")
            self.ct[x.id] = nm

    def run(self, eqns, names, ct_tally):
        for e in reversed(eqns):
            if e.prim == "while":
                if _uses([e]) & self.active:
                    self.while_t(e, names, ct_tally)
                elif self.append_skip is not None and any(x.prim == "append" for x in T._walk(e.params["body"])):
                    # (the loop's records have no cotangent, but each one moves the append ordinal at which the
                    # adjoint reads the earlier records' cotangents: the loop re-run, counting them)
                    self.lines.append(f"{self.indent}{{")
                    self.lines += _emit_code([e], dict(names), None, self.indent + "  ", skip_emits=True,
                                             appender=self.append_skip)
                    self.lines.append(f"{self.indent}}}")
                continue
            if e.prim == "spawn":
                if self.spawn_t is not None:
                    self.spawn_t(self, e, names)
                continue
            if e.prim == "append":
                if self.append_t is not None:
                    self.append_t(self, e, names)
                continue
            if e.prim == "emit":
                idx, v = e.ins[:2]
                if isinstance(v, T.Var) and v.id in self.active and e.params["tally"] in ct_tally:
                    ptr, S = ct_tally[e.params["tally"]][:2]
                    i = _ref(idx, names)
                    w = f"({_ref(e.ins[2], names)}) && " if len(e.ins) > 2 else ""
                    self.add(v, f"(({w}(u32)({i}) < {S}u) ? {ptr}[{i}] : 0.0f)")
                continue
            if not e.outs or e.outs[0].id not in self.ct:
                continue
            self.rule(e, self.ct[e.outs[0].id], [_ref(x, names) for x in e.ins], names)

    def _acc(self, xid):
        """the cotangent local of outer value xid, declared (zero) here if it has none yet: an inner loop adds into
        it from inside its own scopes"""
        if xid not in self.ct:
            self.n += 1
            nm = f"{self.tag}{xid}_{self.n}"
            self.lines.append(f"{self.indent}float {nm} = 0.0f;")
            self.ct[xid] = nm
        return self.ct[xid]

    def while_t(self, e, names, ct_tally):
        """the transpose of an inner loop that reads a differentiated value (the reference differentiates every
        loop, _reverse.py:1-25): its trip count K by running it from its initial carry, then its iterations newest
        first -- each one's starting state recomputed from the initial carry (no tape: K(K-1)/2 body evaluations)
        and its body's VJP applied to the carry cotangents; the values it reads from outside gather their
        cotangents across the iterations"""
        p = e.params
        inner, cact = _inner_active(e, self.active)
        carry, ind = p["carry"], self.indent
        self.n += 1
        u = f"{self.tag}w{self.n}_"
        clos = sorted((_uses(p["body"]) | _ids(p["body_out"])) - _defs_deep(p["body"]) - _ids(carry))
        outer = [xid for xid in clos if xid in self.active]
        outer += [x.id for x, a_ in zip(e.ins, cact) if a_ and isinstance(x, T.Var) and x.id in self.active]
        for xid in dict.fromkeys(outer):
            self._acc(xid)
        ins_c = [_ref(x, names) for x in e.ins]
        L = self.lines

        def state(prefix, nm, indent):
            for j, (cv, x) in enumerate(zip(carry, ins_c)):
                L.append(f"{indent}{CTYPE[cv.dtype]} {prefix}{j} = {x};")
                nm[cv.id] = f"{prefix}{j}"

        def step(prefix, nm, indent):
            L.extend(_emit_code(p["body"], nm, None, indent, skip_emits=True))
            L.extend(f"{indent}const {CTYPE[cv.dtype]} {prefix}n{j} = {_ref(b, nm)};"
                     for j, (cv, b) in enumerate(zip(carry, p["body_out"])))
            L.extend(f"{indent}{prefix}{j} = {prefix}n{j};" for j in range(len(carry)))
        L.append(f"{ind}{{")
        i2, i3 = ind + "  ", ind + "    "
        nm = dict(names)
        state(u + "s", nm, i2)
        L.append(f"{i2}int {u}K = 0;")
        L.append(f"{i2}while (true) {{")
        L.extend(_emit_code(p["cond"], nm, None, i3, skip_emits=True))
        L.append(f"{i3}if (!({_ref(p['cond_out'], nm)})) break;")
        step(u + "s", nm, i3)
        L.append(f"{i3}++{u}K;")
        L.append(f"{i2}}}")
        for j, o in enumerate(e.outs):
            if cact[j]:
                L.append(f"{i2}float {u}c{j} = {self.ct.get(o.id, '0.0f')};")
        L.append(f"{i2}for (int {u}i = {u}K - 1; {u}i >= 0; --{u}i) {{")
        nm = dict(names)
        state(u + "r", nm, i3)
        L.append(f"{i3}for (int {u}q = 0; {u}q < {u}i; ++{u}q) {{")
        step(u + "r", dict(nm), i3 + "  ")
        L.append(f"{i3}}}")
        L.extend(_emit_code(p["body"], nm, None, i3, skip_emits=True))
        # (a Records append inside: transposed per iteration, newest first, as the forward appended them)
        sub = _Rev(inner, indent=i3, tag=u + "g", append_t=self.append_t, append_skip=self.append_skip)
        for xid in dict.fromkeys(outer):
            sub.ct[xid] = self.ct[xid]
        for j, b in enumerate(p["body_out"]):
            if cact[j]:
                sub.add(b, f"{u}c{j}")
        sub.run(p["body"], nm, ct_tally)
        L.extend(sub.lines)
        L.extend(f"{i3}{u}c{j} = {sub.ct.get(cv.id, '0.0f')};" for j, cv in enumerate(carry) if cact[j])
        L.append(f"{i2}}}")
        for j, x in enumerate(e.ins):
            if cact[j] and isinstance(x, T.Var) and x.id in self.active:
                L.append(f"{i2}{self.ct[x.id]} = {self.ct[x.id]} + {u}c{j};")
        L.append(f"{ind}}}")

    def rule(self, e, g, a, names):
        p, x = e.prim, e.ins
        out = names.get(e.outs[0].id, f"v{e.outs[0].id}")
        if p == "add":
            self.add(x[0], g)
            self.add(x[1], g)
        elif p == "sub":
            self.add(x[0], g)
            self.add(x[1], f"(-{g})")
        elif p == "mul":
            self.add(x[0], f"({g} * {a[1]})")
            self.add(x[1], f"({a[0]} * {g})")
        elif p == "div":
            self.add(x[0], f"tm_fdiv({g}, {a[1]})")
            self.add(x[1], f"(((-{g}) * {a[0]}) * tm_fdiv(1.0f, ({a[1]} * {a[1]})))")
        elif p == "neg":
            self.add(x[0], f"(-{g})")
        elif p in _DERIV:
            self.add(x[0], f"({g} * {_DERIV[p](a[0], out)})")
        elif p == "atan2":
            inv = f"tm_fdiv(1.0f, ({a[0]} * {a[0]} + {a[1]} * {a[1]}))"
            self.add(x[0], f"(({g} * {a[1]}) * {inv})")
            self.add(x[1], f"(((-{g}) * {a[0]}) * {inv})")
        elif p == "log":
            self.add(x[0], f"tm_fdiv({g}, {a[0]})")
        elif p == "exp":
            self.add(x[0], f"({g} * {out})")
        elif p == "sin":
            self.add(x[0], f"({g} * tmm::cosf({a[0]}))")
        elif p == "cos":
            self.add(x[0], f"((-{g}) * tmm::sinf({a[0]}))")
        elif p == "sqrt":
            self.add(x[0], f"({g} * tm_fdiv(0.5f, {out}))")
        elif p == "pow":
            self.add(x[0], f"({g} * ({a[1]} * tmm::powf({a[0]}, {a[1]} - 1.0f)))")
            self.add(x[1], f"({g} * (tmm::logf({a[0]}) * {out}))")
        elif p == "abs":
            self.add(x[0], f"({g} * ({a[0]} > 0.0f ? 1.0f : ({a[0]} < 0.0f ? -1.0f : 0.0f)))")
        elif p in ("max", "min"):
            # lax.max / min: the cotangent goes to the selected operand, half each on a tie (_balanced_eq)
            self.add(x[0], f"({g} * ({a[0]} == {out} ? ({a[1]} == {out} ? 0.5f : 1.0f) : 0.0f))")
            self.add(x[1], f"({g} * ({a[1]} == {out} ? ({a[0]} == {out} ? 0.5f : 1.0f) : 0.0f))")
        elif p == "select":
            self.add(x[1], f"({a[0]} ? {g} : 0.0f)")
            self.add(x[2], f"({a[0]} ? 0.0f : {g})")
        elif p == "convert":
            if x[0].dtype == T.F32 and e.outs[0].dtype == T.F32:
                self.add(x[0], g)
        elif p in ("floor", "round", "stop", "gather", "bitcast"):
            pass
        elif p == "rem":
            # lax.rem's transpose (jax: d/dx = 1, d/dy = -sign(x / y) * floor(|x / y|))
            q = f"tm_fdiv({a[0]}, {a[1]})"
            self.add(x[0], g)
            self.add(x[1], f"((-{g}) * (({q} > 0.0f ? 1.0f : ({q} < 0.0f ? -1.0f : {q})) * floorf(fabsf({q}))))")
        else:
            raise LowerError(f"tallymap_b200.lower: no reverse rule for {p}")


def _float_operands(it):
    """positions of the per-item operands whose leaves are all float32 (the ones with cotangents)"""
    out = []
    for j, x in enumerate(it.pi):
        leaves = list(x) if isinstance(x, tuple) else [x]
        if not isinstance(x, T.Key) and all(v.dtype == T.F32 for v in leaves):
            out.append(j)
    return tuple(out)


def _tree_loads(it, RS):
    """the tree adjoint's item inputs: a root's from the per-item operands, a child's from its record's words"""
    out = [f"    {CTYPE[v.dtype]} v{v.id};" for v, _ in it.loads]
    out.append("    if (c.roots) {")
    out += [f"      v{v.id} = {ld};" for v, ld in it.loads]
    out.append("    } else {")
    out.append(f"      const i32* w_ = c.rec + item * {RS};")
    out += [f"      v{v.id} = {_from_bits(f'w_[{m}]', v.dtype)};" for m, (v, _) in enumerate(it.loads)]
    out.append("    }")
    return out


def grad_source(it, wrt, standalone=True, wrt_pi=(), tree=False):
    """-> (C source of the replay ITEM for d <ct, outputs> / d bc[wrt], stored-state bytes, shared-memory bytes);
    standalone=False: the ITEM struct alone, its State the forward ITEM's (GenFwd: for the one-pass program).
    wrt_pi: per-item operands (positions among them, float32 scalars or vectors) whose per-item cotangents the
    program also writes (the reference's perturbed per-item inputs, _reverse.py vjp_prog `ip`): per-item results
    f32[N] (or f32[N, n]) before the truncation flag.
    tree (a spawning item): the adjoint launch of one generation of the tree adjoint (tallymap/_reverse_spawn.py:
    112-166, the adjoint of the "rec" program).  Its items are a generation's record slots (the claim order is the
    generation's list) or the roots (consts[kConstRoots]).  A spawn's transpose gives the spawned leaves the
    cotangents of the child's initial state, which the next-deeper generation's launch wrote to dx[slot]; the
    item's children are consumed newest first along the recorded chain, and each must hold exactly the leaves the
    replay spawns (else tree[0] counts a mismatch: _reverse_spawn.py:22-26).  At the end a child writes its own
    initial state's cotangents to dx[own slot], a root to the per-item results (every float per-item operand).
    Records outputs (tallymap/_records.py twin): per output r, the forward's per-item record counts and canonical
    offsets (the exclusive prefix sum of the counts) are per-item operands after the item's own, and each float
    field's cotangent f32[capacity] a broadcast operand after the tallies' cotangents.  An append's transpose (the
    item's appends consumed newest first) gives its float fields the cotangents at canonical slot offset + k, k its
    ordinal; a replay whose append count differs from the forward's flags the item as truncated, which poisons the
    gradient."""
    tr = it.tr
    npi, nbc, W = len(it.pi), len(it.bc), len(wrt)
    recs = list(tr.records.items()) if not tree else []
    rindex = {rname: r for r, (rname, _) in enumerate(recs)}
    if tree:
        wrt_pi = _float_operands(it)
    Lw = len(it.loads)
    RS = Lw + 2                           # a record: the child's leaves, prev, last
    fleaves = [v for v, _ in it.loads if v.dtype == T.F32]
    fpos = {v.id: f for f, v in enumerate(fleaves)}
    Lf = max(len(fleaves), 1)
    pl = []                               # (output q, the per-item operand's leaves)
    for j in wrt_pi:
        x = it.pi[j]
        leaves = list(x) if isinstance(x, tuple) else [x]
        if isinstance(x, T.Key) or any(v.dtype != T.F32 for v in leaves):
            raise LowerError("tallymap_b200.lower: only float32 per-item operands are differentiable")
        pl.append(leaves)
    act, carry_act = _active(it, wrt, extra=[v.id for leaves in pl for v in leaves])
    Wx = max(W, 1)                        # (one unused bin when only per-item operands are differentiated)
    ftal = [(t, name, shape) for t, (name, (shape, dt)) in enumerate(it.specs) if dt == T.F32]
    lines = [PRELUDE, "namespace tmb {", "struct GenGrad {"]
    idx = 0
    enum = []
    for j in range(npi):
        enum.append(f"kIn{j} = {idx}"); idx += 1
    for r in range(len(recs)):
        enum.append(f"kRCnt{r} = {idx}"); idx += 1
        enum.append(f"kROff{r} = {idx}"); idx += 1
    for k in range(nbc):
        enum.append(f"kBc{k} = {idx}"); idx += 1
    for q, (t, name, shape) in enumerate(ftal):
        enum.append(f"kCt{q} = {idx}"); idx += 1
    for r, (rname, (cap, fields)) in enumerate(recs):
        for f, (fname, dt) in enumerate(fields):
            if dt == T.F32:
                enum.append(f"kRCt{r}F{f} = {idx}"); idx += 1
    # (the tree adjoint's control words come first among its outputs: a later generation's launch zeroes them
    # alone, while the exact words sum over every launch)
    names_ = ("kRecord", "kRootLast", "kConsts", "kOrder", "kCtl", "kG", "kExact", "kStats", "kTree") if tree else \
        ("kConsts", "kOrder", "kG", "kExact", "kCtl", "kStats")
    for nm in names_:
        enum.append(f"{nm} = {idx}"); idx += 1
    for q in range(len(pl)):
        enum.append(f"kGpi{q} = {idx}"); idx += 1
    for nm in (("kDx",) if tree else ()) + ("kTrunc", "kReplay"):
        enum.append(f"{nm} = {idx}"); idx += 1
    enum.append(f"kNBuf = {idx}")
    lines.append("  enum { " + ", ".join(enum) + " };")
    lines.append("  enum { kConstM = 0, kConstC = 1, kConstThreads = 2" +
                 (", kConstRoots = 3, kConstR = 4" if tree else "") + " };")
    # output cotangents: staged in shared memory when small
    smem = f"ExactBins<{Wx}>::kSmemBytes"
    off = 0
    ct_tally = {}
    stage_lines = []
    ctx_ct = []
    for q, (t, name, shape) in enumerate(ftal):
        S = int(np.prod(shape, dtype=np.int64)) if shape else 1
        if S * 4 <= PRIV_BYTES:
            ctx_ct.append(f"    const float* ct{q};")
            stage_lines.append(f"    {{ const float* src = static_cast<const float*>(P.p[kCt{q}]); "
                               f"float* d = reinterpret_cast<float*>(smem + ExactBins<{Wx}>::kSmemBytes + {off}); "
                               f"for (int b = threadIdx.x; b < {S}; b += blockDim.x) d[b] = __ldg(&src[b]); }}")
            ct_tally[name] = (f"c.ct{q}", S, off)
            off += S * 4
        else:
            ctx_ct.append(f"    const float* ct{q};")
            ct_tally[name] = (f"c.ct{q}", S, None)
    lines.append(f"  static constexpr int kSmemBytes = {smem} + {off};")
    # (ExactBins<W>::kSmemBytes -- block words, flags, the threads' private words -- and the staged cotangents)
    smem_bytes = Wx * 5 * 8 + ((Wx * 4 + 7) // 8) * 8 + Wx * 5 * 8 * 128 + off
    ctx = ["  struct Ctx {"]
    for j, s in enumerate(it.in_specs[:npi]):
        ctx.append(f"    const {_in_ctype(s)}* in{j};")
    for k, b in enumerate(it.bc):
        ctx.append(f"    {CTYPE[b.dtype]} b{k};")       # (a table: its pointer)
    ctx += ["    i32 M;", "    i32* stats;", "    u64* gw;", "    float* g;", "    uint8_t* trunc;"]
    ctx += [f"    float* gpi{q};" for q in range(len(pl))]
    ctx += ctx_ct
    for i in it.saved:
        ctx.append(f"    {CTYPE[it.vars[i].dtype]} p{i};")
    ctx.append(f"    mutable ExactPrivS<{Wx}> pv;")
    if tree:
        ctx += ["    const i32* rec;", "    const i32* root_last;", "    float* dx;", "    u32* tree;", "    bool roots;",
                "    i64 R;", "    i32 last;   // the current item's newest child"]
    for r, (rname, (cap, fields)) in enumerate(recs):
        ctx += [f"    const i32* rcnt{r};", f"    const long long* roff{r};",
                f"    i32 rn{r};   // the current item's records in the forward", f"    long long ro{r};"]
        ctx += [f"    const float* rct{r}f{f};" for f, (fname, dt) in enumerate(fields) if dt == T.F32]
    ctx.append("  };")
    lines += ctx
    if standalone:
        lines.append("  struct State {")
        lines.append("    i32 kc;")
        for j, v in enumerate(tr.carry):
            lines.append(f"    {CTYPE[v.dtype]} c{j};")
        lines.append("  };")
    else:
        lines.append("  typedef GenFwd::State State;")
    stored = [j for j in range(len(tr.carry)) if j not in it.counter]
    lines.append("  struct Stored {")
    for j in stored:
        lines.append(f"    {CTYPE[tr.carry[j].dtype]} c{j};")
    if not stored:
        lines.append("    u32 unused;")
    lines.append("  };")
    stored_bytes = max(4, sum(4 for _ in stored))
    act_saved = [i for i in it.saved if i in act]
    lines.append("  struct Adj {")
    for j, a in enumerate(carry_act):
        if a:
            lines.append(f"    float cc{j};")
    for q in range(W):
        lines.append(f"    float cb{q};   // loop's cotangent of bc[{wrt[q]}], summed newest step first")
        lines.append(f"    float pb{q};   // the post-loop code's")
    for i in act_saved:
        lines.append(f"    float cp{i};")
    lines.append("    bool has_post;")
    if tree:
        lines.append("    i32 cur;   // the next recorded child to consume, newest first")
    for r in range(len(recs)):
        lines.append(f"    i32 ka{r};   // output {r}'s appends not yet transposed")
    lines.append("  };")
    # setup / stage
    lines.append("  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {")
    for j, s in enumerate(it.in_specs[:npi]):
        lines.append(f"    c.in{j} = static_cast<const {_in_ctype(s)}*>(P.p[kIn{j}]);")
    for k, b in enumerate(it.bc):
        lines.append(_bc_setup(k, b))
    lines.append("    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));")
    lines += ["    c.stats = static_cast<i32*>(P.p[kStats]);", "    c.gw = static_cast<u64*>(P.p[kExact]);",
              "    c.g = static_cast<float*>(P.p[kG]);", "    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);"]
    lines += [f"    c.gpi{q} = static_cast<float*>(P.p[kGpi{q}]);" for q in range(len(pl))]
    for r, (rname, (cap, fields)) in enumerate(recs):
        lines += [f"    c.rcnt{r} = static_cast<const i32*>(P.p[kRCnt{r}]);",
                  f"    c.roff{r} = static_cast<const long long*>(P.p[kROff{r}]);"]
        lines += [f"    c.rct{r}f{f} = static_cast<const float*>(P.p[kRCt{r}F{f}]);"
                  for f, (fname, dt) in enumerate(fields) if dt == T.F32]
    if tree:
        lines += ["    c.rec = static_cast<const i32*>(P.p[kRecord]);",
                  "    c.root_last = static_cast<const i32*>(P.p[kRootLast]);",
                  "    c.dx = static_cast<float*>(P.p[kDx]);", "    c.tree = static_cast<u32*>(P.p[kTree]);",
                  "    c.roots = __ldg(static_cast<const i32*>(P.p[kConsts]) + kConstRoots) != 0;",
                  "    c.R = __ldg(static_cast<const i32*>(P.p[kConsts]) + kConstR);"]
    for q, (t, name, shape) in enumerate(ftal):
        ptr, S, o = ct_tally[name]
        if o is not None:
            lines.append(f"    c.ct{q} = reinterpret_cast<const float*>(smem + ExactBins<{Wx}>::kSmemBytes + {o});")
        else:
            lines.append(f"    c.ct{q} = static_cast<const float*>(P.p[kCt{q}]);")
    lines.append(f"    c.pv.bind(smem + ExactBins<{Wx}>::kPrivOffset);")
    lines.append("  }")
    lines.append("  __device__ static void stage(const Params& P, unsigned char* smem) {")
    lines += stage_lines
    lines.append("  }")
    # start: pre-loop code without emits
    lines.append("  __device__ static State start(Ctx& c, i64 item) {")
    names = _names_pre(it)
    if tree:
        lines += _tree_loads(it, RS)
        lines.append(f"    c.last = c.roots ? __ldg(&c.root_last[item]) : c.rec[item * {RS} + {Lw + 1}];")
    else:
        for v, ld in it.loads:
            lines.append(f"    const {CTYPE[v.dtype]} v{v.id} = {ld};")
    for r in range(len(recs)):
        lines += [f"    c.rn{r} = __ldg(&c.rcnt{r}[item]);", f"    c.ro{r} = __ldg(&c.roff{r}[item]);"]
    lines += _emit_code(tr.pre, names, None, skip_emits=True)
    for i in it.saved:
        lines.append(f"    c.p{i} = {names[i]};")
    lines += ["    State s;", "    s.kc = 0;"]
    for j, x in enumerate(tr.carry_in):
        lines.append(f"    s.c{j} = {_ref(x, names)};")
    lines += ["    return s;", "  }"]
    lines += _pred_fn(it)
    lines.append("  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) {")
    lines.append("    return s.kc < c.M && pred(c, s);")
    lines.append("  }")
    lines.append(f"  __device__ static void adj_start(const Ctx&{' c' if tree or recs else ''}, Adj& a) {{")
    for j, a_ in enumerate(carry_act):
        if a_:
            lines.append(f"    a.cc{j} = 0.0f;")
    for q in range(W):
        lines.append(f"    a.cb{q} = 0.0f;")
        lines.append(f"    a.pb{q} = 0.0f;")
    for i in act_saved:
        lines.append(f"    a.cp{i} = 0.0f;")
    lines.append("    a.has_post = false;")
    if tree:
        lines.append("    a.cur = c.last;")
    for r in range(len(recs)):
        lines.append(f"    a.ka{r} = c.rn{r};")
    lines.append("  }")
    lines.append("  __device__ __forceinline__ static Stored store(const State& s) {")
    lines.append("    Stored o;")
    for j in stored:
        lines.append(f"    o.c{j} = s.c{j};")
    if not stored:
        lines.append("    o.unused = 0u;")
    lines += ["    return o;", "  }"]
    lines.append("  __device__ __forceinline__ static State restore(const Ctx&, const Stored& o, i64 step) {")
    lines += ["    State s;", "    s.kc = (i32)step;"]
    for j in range(len(tr.carry)):
        lines.append(f"    s.c{j} = {'(i32)step' if j in it.counter else f'o.c{j}'};")
    lines += ["    return s;", "  }"]
    lines.append("  __device__ __forceinline__ static void fwd(const Ctx& c, State& s) {")
    names = _names_loop(it, tr.carry)
    lines += _emit_code(tr.body, names, None, skip_emits=True)
    lines += _assign_carry(it, names)
    lines.append("  }")
    bc_pos = {it.bc[k].id: q for q, k in enumerate(wrt)}
    nsp = [0]
    nap = [0]

    def append_skip(rname, when_c, vals_c):
        return f"if ({when_c}) a.ka{rindex[rname]} -= 1;"

    def append_t(rev, e, names):
        """a Records append's transpose: its float fields' cotangents from the canonical slot offset + k"""
        nap[0] += 1
        k = nap[0]
        r = rindex[e.params["records"]]
        cap, fields = tr.records[e.params["records"]]
        when = _ref(e.ins[0], names)
        took = [(f, x) for f, ((fname, dt), x) in enumerate(zip(fields, e.ins[1:]))
                if dt == T.F32 and isinstance(x, T.Var) and x.id in rev.active]
        ind = rev.indent
        out = [f"{ind}float ra{k}_{f} = 0.0f;" for f, _ in took]
        out.append(f"{ind}if ({when}) {{")
        out.append(f"{ind}  a.ka{r} -= 1;")
        if took:
            # (an output without a capacity -- count-then-fill -- holds every slot below the item's count)
            out.append(f"{ind}  const long long s_ = c.ro{r} + (long long)a.ka{r};")
            out.append(f"{ind}  if (a.ka{r} >= 0{f' && s_ < {int(cap)}ll' if cap else ''}) {{")
            out += [f"{ind}    ra{k}_{f} = __ldg(&c.rct{r}f{f}[s_]);" for f, _ in took]
            out.append(f"{ind}  }}")
        out.append(f"{ind}}}")
        rev.lines += out
        for f, x in took:
            rev.add(x, f"ra{k}_{f}")

    def spawn_t(rev, e, names):
        """a spawn's transpose: the recorded child's initial-state cotangents into the spawned leaves"""
        nsp[0] += 1
        k = nsp[0]
        when = _ref(e.ins[0], names)
        leaves = e.ins[1:]
        vals = [_ref(x, names) for x in leaves]
        took = [(f, x) for x, (v, _) in zip(leaves, it.loads) if v.dtype == T.F32
                for f in [fpos[v.id]] if isinstance(x, T.Var) and x.id in rev.active]
        ind = rev.indent
        out = [f"{ind}float sd{k}_{f} = 0.0f;" for f, _ in took]
        same = " || ".join(f"w_[{m}] != {_bits(vals[m], v.dtype)}" for m, (v, _) in enumerate(it.loads)) or "false"
        out.append(f"{ind}if ({when}) {{")
        out.append(f"{ind}  const i32 r_ = a.cur;")
        out.append(f"{ind}  if (r_ < 0 || r_ >= c.R) {{")
        out.append(f"{ind}    atomicAdd(&c.tree[0], 1u);")
        out.append(f"{ind}  }} else {{")
        out.append(f"{ind}    const i32* w_ = c.rec + (i64)r_ * {RS};")
        out.append(f"{ind}    if ({same}) atomicAdd(&c.tree[0], 1u);")
        out.append(f"{ind}    a.cur = w_[{Lw}];")
        out += [f"{ind}    sd{k}_{f} = c.dx[(i64)r_ * {Lf} + {f}];" for f, _ in took]
        out.append(f"{ind}  }}")
        out.append(f"{ind}}}")
        rev.lines += out
        for f, x in took:
            rev.add(x, f"sd{k}_{f}")

    def finish_rev(rev, state_carry, into_carry, bc_field, extra=""):
        """after a reverse run: carry cotangents (into_carry: assign a.cc from the carry variables' cotangents),
        broadcast and saved-pre cotangents"""
        out = []
        if into_carry:
            for j, a_ in enumerate(carry_act):
                if a_:
                    v = state_carry[j]
                    out.append(f"    a.cc{j} = {rev.ct.get(v.id, '0.0f')};")
        for bid, q in bc_pos.items():
            if bid in rev.ct:
                out.append(f"    a.{bc_field}{q} = a.{bc_field}{q} + {rev.ct[bid]};")
        for i in act_saved:
            if i in rev.ct:
                out.append(f"    a.cp{i} = a.cp{i} + {rev.ct[i]};")
        return out

    # the step VJP at the state before the step
    lines.append("  __device__ __forceinline__ static void vjp(const Ctx& c, const State& at, Adj& a) {")
    names = _names_loop(it, tr.carry, "at")
    lines += _emit_code(tr.body, names, None, skip_emits=True)
    rev = _Rev(act, spawn_t=spawn_t if tree else None, append_t=append_t if recs else None,
               append_skip=append_skip if recs else None)
    for j, x in enumerate(tr.body_out):
        if carry_act[j]:
            rev.add(x, f"a.cc{j}")
    rev.run(tr.body, names, ct_tally)
    lines += rev.lines
    lines += finish_rev(rev, tr.carry, True, "cb")
    lines.append("  }")
    # the post-loop code's VJP: the loop outputs' cotangents
    lines.append("  __device__ static void post_vjp(const Ctx& c, const State& fin, Adj& a) {")
    names = _names_loop(it, tr.post_carry, "fin")
    lines += _emit_code(tr.post, names, None, skip_emits=True)
    rev = _Rev(act, spawn_t=spawn_t if tree else None, append_t=append_t if recs else None,
               append_skip=append_skip if recs else None)
    rev.run(tr.post, names, ct_tally)
    lines += rev.lines
    lines += finish_rev(rev, tr.post_carry, True, "pb")
    if any(bid in rev.ct for bid in bc_pos):
        lines.append("    a.has_post = true;")
    lines.append("  }")
    # the pre-loop code's VJP, then the item's emits
    lines.append("  __device__ static void adj_finish(const Ctx& c, const State&, const State& fin, Adj& a, i64 item) {")
    names = _names_pre(it)
    if tree:
        lines += _tree_loads(it, RS)
    else:
        for v, ld in it.loads:
            lines.append(f"    const {CTYPE[v.dtype]} v{v.id} = {ld};")
    lines += _emit_code(tr.pre, names, None, skip_emits=True)
    rev = _Rev(act, tag="h", append_t=append_t if recs else None,
               append_skip=append_skip if recs else None)
    for j, x in enumerate(tr.carry_in):
        if carry_act[j]:
            rev.add(x, f"a.cc{j}")
    for i in act_saved:
        rev.add(it.vars[i], f"a.cp{i}")
    rev.run(tr.pre, names, ct_tally)
    lines += rev.lines
    for q, k in enumerate(wrt):
        bid = it.bc[k].id
        tot = f"(a.has_post ? a.pb{q} + a.cb{q} : a.cb{q})"
        if bid in rev.ct:
            tot = f"({tot} + {rev.ct[bid]})"
        lines.append(f"    if (c.pv.emit({q}, {tot})) atomicAdd(&c.stats[kStFixedPointOverflow], 1);")
    if tree:
        # a child: its initial state's cotangents for its parent's launch, and its recorded children all consumed;
        # a truncated child counts in tree[1]
        lines.append("    if (!c.roots) {")
        lines += [f"      c.dx[item * {Lf} + {f}] = {rev.ct.get(v.id, '0.0f')};" for f, v in enumerate(fleaves)]
        lines.append("      if (a.cur != -1) atomicAdd(&c.tree[0], 1u);")
        lines.append("      if (fin.kc >= c.M && pred(c, fin)) atomicAdd(&c.tree[1], 1u);")
        lines.append("      return;")
        lines.append("    }")
        lines.append("    if (a.cur != -1) atomicAdd(&c.tree[0], 1u);")
    for q, leaves in enumerate(pl):
        # the per-item operand's cotangent: what the pre-loop VJP gathered into its leaves (+0 for an unused one)
        for e_, v in enumerate(leaves):
            lines.append(f"    c.gpi{q}[item * {len(leaves)} + {e_}] = {rev.ct.get(v.id, '0.0f')};")
    # (a replay whose appends differ in number from the forward's is flagged: its records' cotangents were misread)
    miss = "".join(f" || a.ka{r} != 0" for r in range(len(recs)))
    lines.append(f"    c.trunc[item] = ((fin.kc >= c.M && pred(c, fin)){miss}) ? 1 : 0;")
    lines.append("  }")
    lines.append("  __device__ static void adj_flush(const Ctx& c, unsigned char* smem, int tid, int) {")
    lines.append(f"    ExactBins<{Wx}>::flush(c.pv, smem, c.gw, c.stats, tid);")
    lines.append("  }")
    lines.append("  __device__ static void epilogue(const Ctx& c, int tid, int) {")
    lines.append(f"    if (tid == 0) ExactBins<{Wx}>::readout(c.gw, c.g, c.stats);")
    lines.append("  }")
    lines.append("};")
    if not standalone:
        return "\n".join(lines[2:]), stored_bytes, smem_bytes
    lines.append("}  // namespace tmb")
    lines.append('extern "C" __global__ void TM_MAIN_BOUNDS tm_main(const tmb::Params P, const long long n) {')
    lines.append("  tmb::replay_body<tmb::GenGrad, 1>(P, n);")
    lines.append("}")
    lines.append(f"static_assert(tmb::GenGrad::kSmemBytes == {smem_bytes}, \"shared-memory size\");")
    return "\n".join(lines), stored_bytes, smem_bytes


# ------------------------------------------------------------------------------------------------ one-pass value and grad
def has_active_carry(it, wrt):
    """whether a loop carry depends on the differentiated broadcast operands (else the adjoint is separable: the
    one-pass program applies)"""
    return any(_active(it, wrt)[1])


def onepass_source(it, wrt):
    """-> (C source of the one-pass value-and-grad program: the forward and reverse ITEMs combined by OnePassVG for
    forward_body, shared-memory bytes).  For an item with no active carry: each step's VJP is evaluated at the state
    the step starts from and summed, oldest step first, as the forward runs.
    Layout: [per-item][broadcast][output cotangents][consts][order] | [tallies][ct f32[W]][exact words of the
    fixed-point tallies][ct's exact words][ctl][stats] | [per-item results][truncated]."""
    tr = it.tr
    P, Bn = len(it.pi), len(it.bc)
    Q = sum(1 for _, (_, dt) in it.specs if dt == T.F32)
    Tn = len(it.specs)
    X = sum(1 for name, _ in it.specs if name in it.exact)
    R = len(tr.results)
    R0 = P + Bn + Q + 2
    f_map = list(range(P + Bn)) + [P + Bn + Q, P + Bn + Q + 1] + [R0 + t for t in range(Tn)] + \
        [R0 + Tn + 1 + x for x in range(X)] + [R0 + Tn + 2 + X, R0 + Tn + 3 + X] + \
        [R0 + Tn + 4 + X + r for r in range(R)] + [R0 + Tn + 4 + X + R]
    g_map = list(range(P + Bn + Q)) + [P + Bn + Q, P + Bn + Q + 1, R0 + Tn, R0 + Tn + 1 + X, R0 + Tn + 2 + X,
                                       R0 + Tn + 3 + X, R0 + Tn + 4 + X + R, 0]
    nbuf = R0 + Tn + 5 + X + R
    fsrc, fsmem = forward_source(it, standalone=False)
    gsrc, _, gsmem = grad_source(it, wrt, standalone=False)
    smem = (gsmem + 15) // 16 * 16 + fsmem
    lines = [PRELUDE, "namespace tmb {", fsrc, gsrc,
             "struct GenVGMap {",
             f"  enum {{ kNF = {len(f_map)}, kNG = {len(g_map)}, kNBuf = {nbuf} }};",
             "  __host__ __device__ static constexpr int f(int i) {",
             f"    constexpr int m[kNF] = {{{', '.join(map(str, f_map))}}};",
             "    return m[i];",
             "  }",
             "  __host__ __device__ static constexpr int g(int i) {",
             f"    constexpr int m[kNG] = {{{', '.join(map(str, g_map))}}};",
             "    return m[i];",
             "  }",
             "};",
             "typedef OnePassVG<GenFwd, GenGrad, GenVGMap> GenVG;",
             "static_assert(GenFwd::kNBuf == GenVGMap::kNF && GenGrad::kNBuf == GenVGMap::kNG, \"buffer maps\");",
             "}  // namespace tmb",
             'extern "C" __global__ void TM_MAIN_BOUNDS tm_main(const tmb::Params P, const long long n) {',
             "  tmb::forward_body<tmb::GenVG>(P, n);",
             "}",
             f"static_assert(tmb::GenVG::kSmemBytes == {smem}, \"shared-memory size\");"]
    return "\n".join(lines), smem, nbuf


# ------------------------------------------------------------------------------------------------ programs
def _operand(name, spec):
    from .backend import Operand
    if spec == "key":
        return Operand(name, (2,), torch.int32)
    if isinstance(spec, tuple) and spec[0] == "table":
        return Operand(name, tuple(spec[2]), TDTYPE[spec[1]])
    if isinstance(spec, tuple):
        return Operand(name, (spec[1],), TDTYPE[spec[0]])
    return Operand(name, (), TDTYPE[spec])


class Lowered:
    """a traced item's programs: the forward (compiled at construction) and its reverse programs (compiled per set
    of differentiated broadcast operands, on first use)"""

    def __init__(self, fn, in_specs, n_per_item, outputs, name=None, spawn=False, math="ieee", min_blocks=None):
        from .backend import ItemProgram, TSpec
        self.name = name or getattr(fn, "__name__", "item")
        self.head, self.flags = options_source(math, min_blocks)
        self.math, self.min_blocks = math, min_blocks
        # (a Records output without a capacity -- count-then-fill -- has capacity 0 in the one-pass program, which
        # never runs for it)
        recs = {k: (int(v[1] or 0), tuple(v[2])) for k, v in outputs.items() if v[0] == "records"}
        outputs = {k: v for k, v in outputs.items() if v[0] != "records"}
        specs = {k: (tuple(v[0]), v[1]) for k, v in outputs.items()}
        exact = [k for k, v in outputs.items() if len(v) > 2 and v[2]]
        acc = {k: v[3] for k, v in outputs.items() if len(v) > 3 and v[3]}
        self.tr = T.trace_item(fn, in_specs, n_per_item, specs, recs, spawn=spawn)
        self.it = Item(self.tr, in_specs, self.name, exact, acc)
        from . import _diagnostics as diagnostics
        tr = self.tr
        floats = sorted({float(x.value) for e in T._walk(tr.pre + tr.cond + tr.body + tr.post) for x in e.ins
                         if isinstance(x, T.Lit) and x.dtype == T.F32})
        diagnostics.record_program(dict(tag=self.name, inputs=list(in_specs), n_per_item=n_per_item,
                                        outputs={k: v[0] for k, v in outputs.items()}, records=sorted(recs),
                                        equations=dict(pre=len(tr.pre), cond=len(tr.cond), body=len(tr.body),
                                                       post=len(tr.post)),
                                        float_literals=floats[:32]))
        it = self.it
        src, smem = forward_source(it)
        self.fwd_source = src
        pi = tuple(_operand(f"in{j}", s) for j, s in enumerate(in_specs[:n_per_item]))
        bc = tuple(_operand(f"bc{k}", s) for k, s in enumerate(in_specs[n_per_item:]))
        self.pi, self.bc = pi, bc
        tallies = tuple(TSpec(nm, shape, _out_dtype(it, nm, dt), exact=nm in it.exact,
                              wide=float(it.acc[nm][2]) if it.acc.get(nm, ("",))[0] == "wide" else 0.0)
                        for nm, (shape, dt) in it.specs)
        ys = tuple(_operand(f"y{r}", y.dtype) for r, y in enumerate(self.tr.results))
        ys += tuple(_operand(f"{nm}#count", T.I32) for nm in recs)
        ys += (_operand("truncated", T.BOOL),)
        records = tuple((nm, int(cap), tuple((f, TDTYPE[dt]) for f, dt in fl)) for nm, (cap, fl) in recs.items())
        nrec = sum(len(fl) + 3 for _, _, fl in records)
        sp = it.spawns
        nbuf = len(pi) + len(bc) + 2 + len(tallies) + len(it.exact) + nrec + 2 + len(ys) + (3 if sp else 0) + \
            int(it.claims) + sum(1 for t in tallies if t.wide)
        if sp:
            # the spawn runtime's shared stack entries after the item's block (csrc/tm_spawn.cuh SpawnSmem)
            smem = (smem + 15) // 16 * 16 + SPAWN_STACK_SHARED * 4 * len(it.loads) * 128
            src += f"\nstatic_assert(tmb::SpawnSmem<tmb::GenFwd>::kBytes == {smem}, \"shared-memory size\");"
        kid = self._compile(src, self.name + "_fwd", nbuf, smem)
        self.fwd = ItemProgram(self.name + "_fwd", kid, pi=pi, bc=bc,
                               consts=("max_steps", "queue") if sp else ("max_steps",), tallies=tallies,
                               ys=ys, trunc=len(ys) - 1, records=records, spawns=sp,
                               queue_leaf_bytes=4 * len(it.loads) if sp else 0,
                               claims=len(tallies) if it.claims else 0)
        self.n_results = len(self.tr.results)
        self._fwd_nbuf = nbuf
        self.grads = {}
        self.jvps = {}
        self.vgs = {}
        self.trees = {}
        self._rec = None

    def _differentiable(self, wrt):
        """a table is read-only data of the item: no cotangent or tangent flows to it"""
        for k in wrt:
            if self.it.bc[k].dtype in T.TABLE_ELT:
                raise LowerError("tallymap_b200.lower: derivatives with respect to a broadcast table are not lowered "
                                 "(pass the differentiated parameters as scalars or a vector of at most 64)")

    def _compile(self, src, note, nbuf, smem):
        """compile one of this item's programs with the call's options (cuda_math, min_blocks_per_sm)"""
        return compile_kernel(self.head + src, note, nbuf, smem, self.flags)

    def _no_wider(self, what):
        if self.it.acc:
            raise NotImplementedError(f"tallymap_b200: {what} of an item with float64, int64 or scaled fixed-point "
                                      "Sum outputs is not lowered (grad is)")

    def jvp_program(self, wrt, lanes):
        """the forward-mode program: the forward's outputs and, per tangent lane, the tangents of its float tallies
        for tangents of bc[wrt] given per launch (an input f32[lanes, len(wrt)])"""
        self._differentiable(wrt)
        self._no_wider("forward mode")
        from .backend import ItemProgram, TSpec, Operand
        key = (tuple(wrt), int(lanes))
        if key not in self.jvps:
            for k in wrt:
                if self.bc[k].dtype != torch.float32:
                    raise LowerError("tallymap_b200.lower: only float32 broadcast operands have tangents")
            src, smem = jvp_source(self.it, list(wrt), int(lanes))
            fts = [(nm, shape) for nm, (shape, dt) in self.it.specs if dt == T.F32]
            bc = self.bc + (Operand("tangents", (int(lanes), len(wrt)), torch.float32),)
            # a fixed-point output's tangent is exact too (the same accumulator)
            tallies = self.fwd.tallies + tuple(TSpec("d_" + nm, (int(lanes),) + tuple(shape), exact=nm in self.it.exact)
                                               for nm, shape in fts)
            sp = self.it.spawns
            nx = sum(1 for t in tallies if t.exact)
            # a Records output's float fields gain one tangent field per lane ("field#d<lane>"), after the fields
            records = tuple((nm, cap, fields + tuple((f"{f}#d{l}", torch.float32) for f, dt in fields
                                                     if dt == torch.float32 for l in range(int(lanes))))
                            for nm, cap, fields in self.fwd.records)
            nrec = sum(len(fl) + 3 for _, _, fl in records)
            nbuf = len(self.pi) + len(bc) + 2 + len(tallies) + nx + nrec + 2 + len(self.fwd.ys) + (3 if sp else 0)
            kid = self._compile(src, f"{self.name}_jvp{''.join(map(str, wrt))}x{lanes}", nbuf, smem)
            self.jvps[key] = ItemProgram(f"{self.name}_jvp", kid, pi=self.pi, bc=bc,
                                         consts=("max_steps", "queue") if sp else ("max_steps",),
                                         tallies=tallies, ys=self.fwd.ys, trunc=self.fwd.trunc, spawns=sp,
                                         queue_leaf_bytes=self._child_bytes(int(lanes)) if sp else 0,
                                         records=records)
        return self.jvps[key]

    def _child_bytes(self, L):
        """bytes of a child of this spawning item in a forward-mode program: its leaves and L tangents of each float
        leaf"""
        return 4 * (len(self.it.loads) + L * sum(1 for v, _ in self.it.loads if v.dtype == T.F32))

    def vg_program(self, wrt):
        """the one-pass value-and-grad program for bc[wrt] (forward outputs, then the exact cotangent tally): with no
        active carry the step VJPs summed as the forward runs (OnePassVG); otherwise, for up to FWD_GRAD_MAX
        operands and no fixed-point output, forward mode with the tangents contracted at each emit
        (jvp_source(contract=True)); else None (the replay; also for an item with a wider accumulator)"""
        self._differentiable(wrt)
        from .backend import ItemProgram, TSpec, Operand
        wrt = tuple(wrt)
        if self.it.acc:
            return None
        if wrt not in self.vgs:
            prog = None
            sp = self.it.spawns
            if not self.fwd.records:
                for k in wrt:
                    if self.bc[k].dtype != torch.float32:
                        raise LowerError("tallymap_b200.lower: only float32 broadcast operands are differentiable")
                fts = [(nm, shape) for nm, (shape, dt) in self.it.specs if dt == T.F32]
                bc = self.bc + tuple(Operand("ct_" + nm, tuple(shape), torch.float32) for nm, shape in fts)
                tallies = self.fwd.tallies + (TSpec("ct", (len(wrt),), exact=True),)
                if not sp and not has_active_carry(self.it, list(wrt)):
                    src, smem, nbuf = onepass_source(self.it, list(wrt))
                    kid = self._compile(src, f"{self.name}_vg{''.join(map(str, wrt))}", nbuf, smem)
                elif len(wrt) <= FWD_GRAD_MAX:
                    # forward mode; through spawn, each child carries its float leaves' tangents
                    src, smem = jvp_source(self.it, list(wrt), len(wrt), contract=True)
                    nx = sum(1 for t in tallies if t.exact)
                    nbuf = len(self.pi) + len(bc) + 2 + len(tallies) + nx + 2 + len(self.fwd.ys) + (3 if sp else 0)
                    kid = self._compile(src, f"{self.name}_fg{''.join(map(str, wrt))}", nbuf, smem)
                else:
                    kid = None
                if kid is not None:
                    prog = ItemProgram(f"{self.name}_vg", kid, pi=self.pi, bc=bc,
                                       consts=("max_steps", "queue") if sp else ("max_steps",),
                                       tallies=tallies, ys=self.fwd.ys, trunc=self.fwd.trunc, spawns=sp,
                                       queue_leaf_bytes=self._child_bytes(len(wrt)) if sp else 0)
            self.vgs[wrt] = prog
        return self.vgs[wrt]

    def records_programs(self):
        """count-then-fill (Records outputs without a capacity, _api.py:138-148): (the count pass -- the per-item
        record counts, no records, no emits -- and the fill pass -- the forward's outputs, each record at its
        canonical slot from the counts and offsets given as per-item operands after the item's own).  The fill
        program's Records capacities are the placeholder 0: a call sets each to its total."""
        from .backend import ItemProgram, Operand
        if not self.fwd.records:
            raise ValueError(f"tallymap_b200: item {self.name!r} has no Records outputs")
        if getattr(self, "_rp", None) is None:
            it = self.it
            nrec = sum(len(fl) + 3 for _, _, fl in self.fwd.records)
            src, smem = forward_source(it, mode="count")
            kc = self._compile(src, self.name + "_count", self._fwd_nbuf - nrec, smem)
            cnt = ItemProgram(self.name + "_count", kc, pi=self.pi, bc=self.bc, consts=("max_steps",),
                              tallies=self.fwd.tallies, ys=self.fwd.ys, trunc=self.fwd.trunc)
            src, smem = forward_source(it, mode="fill")
            nr = len(self.fwd.records)
            kf = self._compile(src, self.name + "_fill", self._fwd_nbuf - 3 * nr + 2 * nr, smem)
            pi = self.pi + tuple(o for nm, _, _ in self.fwd.records
                                 for o in (Operand(f"{nm}#count", (), torch.int32),
                                           Operand(f"{nm}#offset", (), torch.int64)))
            fil = ItemProgram(self.name + "_fill", kf, pi=pi, bc=self.bc, consts=("max_steps",),
                              tallies=self.fwd.tallies, ys=self.fwd.ys, trunc=self.fwd.trunc,
                              records=tuple((nm, 0, fl) for nm, _, fl in self.fwd.records), records_fill=True)
            self._rp = (cnt, fil)
        return self._rp

    def jvp_fill_program(self, wrt, lanes):
        """the fill pass of count-then-fill with L tangent lanes (jvp_source mode "fill"): operands as jvp_program's
        with each Records output's counts and offsets after the per-item operands; tangent fields "field#d<lane>"
        beside the fields, every capacity the placeholder 0"""
        self._differentiable(wrt)
        self._no_wider("forward mode")
        from .backend import ItemProgram, TSpec, Operand
        key = ("fill", tuple(wrt), int(lanes))
        if key not in self.jvps:
            base = self.jvp_program(wrt, lanes)
            src, smem = jvp_source(self.it, list(wrt), int(lanes), mode="fill")
            records = tuple((nm, 0, fl) for nm, _, fl in base.records)
            nr = len(records)
            nx = sum(1 for t in base.tallies if t.exact)
            nrec = sum(len(fl) for _, _, fl in records)
            nbuf = len(self.pi) + 2 * nr + len(base.bc) + 2 + len(base.tallies) + nx + nrec + 2 + len(base.ys)
            kid = self._compile(src, f"{self.name}_jvpfill{''.join(map(str, wrt))}x{lanes}", nbuf, smem)
            pi = self.pi + tuple(o for nm, _, _ in records for o in (Operand(f"{nm}#count", (), torch.int32),
                                                                      Operand(f"{nm}#offset", (), torch.int64)))
            self.jvps[key] = dataclasses.replace(base, name=f"{self.name}_jvpfill", kernel=kid, pi=pi,
                                                 records=records, records_fill=True)
        return self.jvps[key]

    def rec_program(self):
        """the tree adjoint's recording forward (a spawning item; the reference's rec_primal): the forward's outputs,
        plus a record of every child -- its leaves, its parent's previous child and its own newest child (i32 words,
        record_bytes each) and its generation (uint16) -- and each root's newest child (the per-item result `last`)"""
        from .backend import ItemProgram, Operand
        if not self.it.spawns:
            raise ValueError(f"tallymap_b200: item {self.name!r} does not spawn")
        if self._rec is None:
            it = self.it
            src, smem = forward_source(it, record=True)
            W = len(it.loads) + 2
            smem = (smem + 15) // 16 * 16 + SPAWN_STACK_SHARED * 4 * W * 128
            src += f"\nstatic_assert(tmb::SpawnSmem<tmb::GenFwd>::kBytes == {smem}, \"shared-memory size\");"
            kid = self._compile(src, self.name + "_rec", self._fwd_nbuf + 4, smem)
            self._rec = ItemProgram(self.name + "_rec", kid, pi=self.pi, bc=self.bc,
                                    consts=("max_steps", "queue", "record"), tallies=self.fwd.tallies,
                                    ys=self.fwd.ys + (Operand("last", (), torch.int32),), trunc=self.fwd.trunc,
                                    spawns=True, queue_leaf_bytes=4 * W, record_bytes=4 * W)
        return self._rec

    def tree_program(self, wrt):
        """the tree adjoint's launch over one generation (or the roots) for d <ct, outputs> / d bc[wrt] and the roots'
        float per-item operands (grad_source(tree=True); driven by backend.tree_adjoint).  Buffers: [pi] [bc]
        [output cotangents] [record] [roots' newest child] [consts: max_steps, C, threads, roots, R] [order] |
        [ctl] [g f32[W]] [exact words] [stats] [tree u32[4]: mismatches, truncated replays] [ct_in per float
        per-item operand] [dx f32[R, float leaves]] [trunc] [replay scratch]"""
        self._differentiable(wrt)
        from .backend import ItemProgram, TSpec, Operand
        if not self.it.spawns:
            raise ValueError(f"tallymap_b200: item {self.name!r} does not spawn")
        if self.fwd.records:
            raise NotImplementedError("tallymap_b200: reverse mode of an item with Records outputs is not lowered")
        wrt = tuple(wrt)
        if wrt not in self.trees:
            for k in wrt:
                if self.bc[k].dtype != torch.float32:
                    raise LowerError("tallymap_b200.lower: only float32 broadcast operands are differentiable")
            src, stored, smem = grad_source(self.it, list(wrt), tree=True)
            fts = [(nm, shape) for nm, (shape, dt) in self.it.specs if dt == T.F32]
            bc = self.bc + tuple(Operand("ct_" + nm, tuple(shape), torch.float32) for nm, shape in fts)
            fo = _float_operands(self.it)
            ys = tuple(Operand(f"ct_in{j}", self.pi[j].shape, torch.float32) for j in fo)
            ys += (_operand("truncated", T.BOOL),)
            nbuf = len(self.pi) + len(bc) + 2 + 2 + 5 + len(fo) + 3
            tag = "".join(map(str, wrt))
            kid = self._compile(src, f"{self.name}_tree{tag}", nbuf, smem)
            self.trees[wrt] = ItemProgram(f"{self.name}_tree{tag}", kid, pi=self.pi, bc=bc,
                                          consts=("max_steps", "rev_checkpoints", "replay_threads", "roots", "record"),
                                          tallies=(TSpec("ct", (max(len(wrt), 1),), exact=True),), ys=ys,
                                          trunc=len(ys) - 1, replay_state_bytes=(stored + 3) // 4 * 4, buffers=nbuf)
        return self.trees[wrt]

    def grad_program(self, wrt, wrt_pi=()):
        """the reverse program for d <ct, outputs> / d bc[wrt] (wrt: positions among the broadcast operands) and, per
        item, d <ct, outputs> / d pi[wrt_pi] (positions among the per-item operands: per-item results before the
        truncation flag)"""
        self._differentiable(wrt)
        from .backend import ItemProgram, TSpec
        wrt, wrt_pi = tuple(wrt), tuple(wrt_pi)
        if self.it.spawns:
            raise ValueError("tallymap_b200: a spawning item's reverse mode is the tree adjoint (rec_program, "
                             "tree_program)")
        key = wrt if not wrt_pi else (wrt, wrt_pi)
        if key not in self.grads:
            for k in wrt:
                if self.bc[k].dtype != torch.float32:
                    raise LowerError("tallymap_b200.lower: only float32 broadcast operands are differentiable")
            src, stored, smem = grad_source(self.it, list(wrt), wrt_pi=wrt_pi)
            fts = [(nm, shape) for nm, (shape, dt) in self.it.specs if dt == T.F32]
            from .backend import Operand
            bc = self.bc + tuple(Operand("ct_" + nm, tuple(shape), torch.float32) for nm, shape in fts)
            # Records outputs: the forward's per-item counts and canonical offsets, and the float fields' cotangents
            pi = self.pi + tuple(o for nm, _, _ in self.fwd.records
                                 for o in (Operand(f"{nm}#count", (), torch.int32), Operand(f"{nm}#offset", (), torch.int64)))
            bc += tuple(Operand(f"ct_{nm}.{f}", (cap,), torch.float32) for nm, cap, fields in self.fwd.records
                        for f, dt in fields if dt == torch.float32)
            ys = tuple(Operand(f"ct_in{j}", self.pi[j].shape, torch.float32) for j in wrt_pi)
            ys += (_operand("truncated", T.BOOL),)
            nbuf = len(pi) + len(bc) + 2 + 4 + len(ys) + 1
            tag = "".join(map(str, wrt)) + ("_pi" + "".join(map(str, wrt_pi)) if wrt_pi else "")
            kid = self._compile(src, f"{self.name}_grad{tag}", nbuf, smem)
            self.grads[key] = ItemProgram(f"{self.name}_grad", kid, pi=pi, bc=bc,
                                          consts=("max_steps", "rev_checkpoints", "replay_threads"),
                                          tallies=(TSpec("ct", (max(len(wrt), 1),), exact=True),),
                                          ys=ys, trunc=len(ys) - 1,
                                          replay_state_bytes=(stored + 3) // 4 * 4)
        return self.grads[key]


# ------------------------------------------------------------------------------------------------ forward mode
LANES_MAX = 16        # tangent lanes of one jvp program (the reference's jacfwd lanes, LANES_MAX_LOCAL)
FWD_GRAD_MAX = 4      # value_and_grad by forward mode (one lane per operand) for items with an active carry: up to
                      # this many differentiated operands, else the replay


def _jvp_rule(e, a, d, out):
    """per-lane tangent expression of equation e's output (jax's jvp rules); a: primal input expressions, d: their
    tangent expressions (None: zero), out: the primal output expression"""
    p = e.prim
    x = d[0] if d else None
    y = d[1] if len(d) > 1 else None

    def plus(u, v):
        if u is None:
            return v
        if v is None:
            return u
        return f"({u} + {v})"
    if p == "add":
        return plus(x, y)
    if p == "sub":
        return plus(x, None if y is None else f"(-{y})")
    if p == "mul":
        return plus(None if x is None else f"({x} * {a[1]})", None if y is None else f"({a[0]} * {y})")
    if p == "div":
        return plus(None if x is None else f"tm_fdiv({x}, {a[1]})",
                    None if y is None else f"(((-{y}) * {a[0]}) * tm_fdiv(1.0f, ({a[1]} * {a[1]})))")
    if p == "neg":
        return None if x is None else f"(-{x})"
    if p in _DERIV:
        return None if x is None else f"({x} * {_DERIV[p](a[0], out)})"
    if p == "atan2":
        inv = f"tm_fdiv(1.0f, ({a[0]} * {a[0]} + {a[1]} * {a[1]}))"
        return plus(None if x is None else f"(({x} * {a[1]}) * {inv})",
                    None if y is None else f"(((-{y}) * {a[0]}) * {inv})")
    if p == "log":
        return None if x is None else f"tm_fdiv({x}, {a[0]})"
    if p == "exp":
        return None if x is None else f"({x} * {out})"
    if p == "sin":
        return None if x is None else f"({x} * tmm::cosf({a[0]}))"
    if p == "cos":
        return None if x is None else f"((-{x}) * tmm::sinf({a[0]}))"
    if p == "sqrt":
        return None if x is None else f"({x} * tm_fdiv(0.5f, {out}))"
    if p == "pow":
        return plus(None if x is None else f"({x} * ({a[1]} * tmm::powf({a[0]}, {a[1]} - 1.0f)))",
                    None if y is None else f"({y} * (tmm::logf({a[0]}) * {out}))")
    if p == "abs":
        return None if x is None else f"({x} * ({a[0]} > 0.0f ? 1.0f : ({a[0]} < 0.0f ? -1.0f : 0.0f)))"
    if p in ("max", "min"):
        return plus(None if x is None else f"({x} * ({a[0]} == {out} ? ({a[1]} == {out} ? 0.5f : 1.0f) : 0.0f))",
                    None if y is None else f"({y} * ({a[1]} == {out} ? ({a[0]} == {out} ? 0.5f : 1.0f) : 0.0f))")
    if p == "select":
        db, dc = (d[1] if len(d) > 1 else None), (d[2] if len(d) > 2 else None)
        if db is None and dc is None:
            return None
        return f"({a[0]} ? {db or '0.0f'} : {dc or '0.0f'})"
    if p == "convert":
        return x if e.outs[0].dtype == T.F32 and e.ins[0].dtype == T.F32 else None
    if p in ("floor", "round", "stop", "gather", "bitcast"):
        return None
    if p == "rem":
        q = f"tm_fdiv({a[0]}, {a[1]})"
        return plus(x, None if y is None else
                    f"((-{y}) * (({q} > 0.0f ? 1.0f : ({q} < 0.0f ? -1.0f : {q})) * floorf(fabsf({q}))))")
    raise LowerError(f"tallymap_b200.lower: no jvp rule for {p}")


def _emit_code_jvp(eqns, names, tnames, act, L, emitter, temitter, indent="    ", spawner=None, appender=None):
    """straight-line primal code with each active value's L tangents; tnames: id -> [L tangent expressions];
    spawner(when, leaves, leaf tangents): a spawn with its children's tangents; appender(records, when, fields,
    field tangents): a Records append with its float fields' tangents"""
    out = []
    for e in eqns:
        a = [names[x.id] if isinstance(x, T.Var) else c_lit(x) for x in e.ins]
        if e.prim == "while":
            act_s = set(act) | set(tnames)
            if not _uses([e]) & act_s:
                # (no tangent inside: the loop as the forward runs it; its appends carry zero field tangents)
                app = None if appender is None else (lambda rn, w, vals: appender(rn, w, vals, [None] * len(vals)))
                out += _emit_code([e], names, emitter, indent, appender=app)
                continue
            # forward mode through the loop: each active float carry's L tangents carried beside it
            p = e.params
            inner, cact = _inner_active(e, act_s)
            tn = dict(tnames)
            for j, (cv, o, x) in enumerate(zip(p["carry"], e.outs, e.ins)):
                out.append(f"{indent}{CTYPE[o.dtype]} v{o.id} = {a[j]};")
                names[o.id] = names[cv.id] = f"v{o.id}"
                if cact[j]:
                    t0 = tnames.get(x.id) if isinstance(x, T.Var) else None
                    out += [f"{indent}float dv{o.id}_{l} = {t0[l] if t0 else '0.0f'};" for l in range(L)]
                    tn[cv.id] = [f"dv{o.id}_{l}" for l in range(L)]
            out.append(f"{indent}while (true) {{")
            out += _emit_code(p["cond"], names, None, indent + "  ")
            out.append(f"{indent}  if (!({_ref(p['cond_out'], names)})) break;")
            out += _emit_code_jvp(p["body"], names, tn, inner, L, emitter, temitter, indent + "  ", spawner, appender)
            for j, (o, b) in enumerate(zip(e.outs, p["body_out"])):
                out.append(f"{indent}  const {CTYPE[o.dtype]} n{o.id} = {_ref(b, names)};")
                if cact[j]:
                    bt = tn.get(b.id) if isinstance(b, T.Var) else None
                    out += [f"{indent}  const float nd{o.id}_{l} = {bt[l] if bt else '0.0f'};" for l in range(L)]
            for j, o in enumerate(e.outs):
                out.append(f"{indent}  v{o.id} = n{o.id};")
                if cact[j]:
                    out += [f"{indent}  dv{o.id}_{l} = nd{o.id}_{l};" for l in range(L)]
            out.append(f"{indent}}}")
            for j, o in enumerate(e.outs):
                if cact[j]:
                    tnames[o.id] = [f"dv{o.id}_{l}" for l in range(L)]
            continue
        if e.prim == "spawn":
            if spawner is not None:
                tl = [tnames.get(x.id) if isinstance(x, T.Var) else None for x in e.ins[1:]]
                out.append(indent + spawner(a[0], a[1:], tl))
            continue
        if e.prim == "append":
            if appender is not None:
                tl = [tnames.get(x.id) if isinstance(x, T.Var) else None for x in e.ins[1:]]
                out.append(indent + appender(e.params["records"], a[0], a[1:], tl))
            continue
        out += _emit_code([e], names, emitter, indent)
        if e.prim == "emit":
            v = e.ins[1]
            if isinstance(v, T.Var) and v.id in tnames:
                for l in range(L):
                    st = temitter(e.params["tally"], l, a[0], tnames[v.id][l])
                    out.append(indent + (f"if ({a[2]}) {{ {st} }}" if len(a) > 2 else st))
            continue
        if not e.outs or e.outs[0].id not in act or e.outs[0].dtype != T.F32:
            continue
        o = e.outs[0]
        for l in range(L):
            d = [tnames[x.id][l] if isinstance(x, T.Var) and x.id in tnames else None for x in e.ins]
            expr = _jvp_rule(e, a, d, names[o.id])
            if expr is None:
                continue
            out.append(f"{indent}const float d{o.id}_{l} = {expr};")
            tnames.setdefault(o.id, [None] * L)[l] = f"d{o.id}_{l}"
        if o.id in tnames and any(t is None for t in tnames[o.id]):
            tnames[o.id] = [t or "0.0f" for t in tnames[o.id]]
    return out


def jvp_source(it, wrt, L, contract=False, mode="one"):
    """-> (C source of the forward ITEM with L tangent lanes of the broadcast operands bc[wrt], shared-memory bytes).
    Buffers: [per-item][broadcast][tangent seeds f32[L, W]][consts][order] | [tallies][tangent tallies f32[L, S] of
    the float tallies][ctl][stats] | [per-item results][truncated].
    contract=True: the one-pass value-and-grad by forward mode, for cotangents given up front: L = W lanes seeded
    with the identity, each tangent emit contracted with the output's cotangent at its index into a per-item sum per
    lane, the sums emitted once per item into an exact W-bin tally.  Buffers: [per-item][broadcast][output
    cotangents of the float tallies][consts][order] | [tallies][ct f32[W]][ct's exact words][ctl][stats] |
    [per-item results][truncated].
    mode="fill": Records outputs written by the fill pass of count-then-fill (forward_source's mode), the fields'
    tangents beside them at the canonical slot"""
    tr = it.tr
    npi, nbc, W = len(it.pi), len(it.bc), len(wrt)
    if contract:
        L = W
    if not 1 <= L <= LANES_MAX:
        raise LowerError(f"tallymap_b200.lower: 1..{LANES_MAX} tangent lanes")
    sp = it.spawns
    # Records outputs (forward mode proper only): each append writes its float fields' L tangents beside the fields,
    # at the same raw slot, so the canonical layout moves them with their records (tallymap/_records.py canon)
    recs = list(tr.records.items())         # [(name, (capacity, ((field, dtype), ...)))]
    fill = mode == "fill"
    if recs and contract:
        raise LowerError("tallymap_b200.lower: Records outputs have no one-pass forward-mode value-and-grad")
    # a spawning item: a child carries its float per-item inputs' tangents (fl: their positions among the leaves)
    fl = [m for m, (v, _) in enumerate(it.loads) if v.dtype == T.F32] if sp else []
    act, carry_act = _active(it, wrt, extra=[it.loads[m][0].id for m in fl])
    ftal = [(t, name, shape) for t, (name, (shape, dt)) in enumerate(it.specs) if dt == T.F32]
    lines = [('#include "tm_spawn.cuh"' if sp else "") + PRELUDE, "namespace tmb {", "struct GenJvp {"]
    idx = 0
    enum = []
    for j in range(npi):
        enum.append(f"kIn{j} = {idx}"); idx += 1
    if fill:
        for r in range(len(recs)):
            enum.append(f"kRCnt{r} = {idx}"); idx += 1
            enum.append(f"kROff{r} = {idx}"); idx += 1
    for k in range(nbc):
        enum.append(f"kBc{k} = {idx}"); idx += 1
    if contract:
        for q, _ in enumerate(ftal):
            enum.append(f"kCt{q} = {idx}"); idx += 1
    else:
        enum.append(f"kTan = {idx}"); idx += 1
    enum.append(f"kConsts = {idx}"); idx += 1
    enum.append(f"kOrder = {idx}"); idx += 1
    for t, _ in enumerate(it.specs):
        enum.append(f"kT{t} = {idx}"); idx += 1
    # fixed-point outputs (Sum(fixed_point=True)): exact words after every tally (the primal's, then -- forward
    # mode proper -- their tangents', which use the same exact accumulator: the reference's same-scale tangent)
    ex = [(t, name) for t, (name, _) in enumerate(it.specs) if name in it.exact]
    if contract:
        enum.append(f"kG = {idx}"); idx += 1
        for t, _ in ex:
            enum.append(f"kX{t} = {idx}"); idx += 1
        enum.append(f"kExact = {idx}"); idx += 1
    else:
        for q, _ in enumerate(ftal):
            enum.append(f"kD{q} = {idx}"); idx += 1
        for t, _ in ex:
            enum.append(f"kX{t} = {idx}"); idx += 1
        for t, _ in ex:
            enum.append(f"kDX{t} = {idx}"); idx += 1
    for r, (rname, (cap, fields)) in enumerate(recs):
        for f in range(len(fields)):
            enum.append(f"kR{r}F{f} = {idx}"); idx += 1
        for f, (fname, dt) in enumerate(fields):
            if dt == T.F32:
                for l in range(L):
                    enum.append(f"kR{r}D{f}_{l} = {idx}"); idx += 1
        if fill:
            continue
        enum.append(f"kR{r}Cid = {idx}"); idx += 1
        enum.append(f"kR{r}K = {idx}"); idx += 1
        enum.append(f"kR{r}Ctr = {idx}"); idx += 1
    if sp:
        enum.append(f"kSeq = {idx}"); idx += 1
        enum.append(f"kQctl = {idx}"); idx += 1
    enum.append(f"kCtl = {idx}"); idx += 1
    enum.append(f"kStats = {idx}"); idx += 1
    for r in range(len(tr.results)):
        enum.append(f"kY{r} = {idx}"); idx += 1
    for r in range(len(recs)):
        enum.append(f"kR{r}N = {idx}"); idx += 1
    enum.append(f"kTrunc = {idx}"); idx += 1
    if sp:
        enum.append(f"kQueue = {idx}"); idx += 1
    enum.append(f"kNBuf = {idx}")
    lines.append("  enum { " + ", ".join(enum) + " };")
    if sp:
        lines.append("  enum { kConstM, kConstQ };")
        fields = [f"{CTYPE[v.dtype]} l{m};" for m, (v, _) in enumerate(it.loads)]
        fields += [f"float d{m}_{l};" for m in fl for l in range(L)]
        lines.append("  struct Child { " + " ".join(fields) + " };")
        if it.post_spawns:
            lines.append("  static constexpr bool kPostSpawn = true;")
    smem, priv = 0, {}
    if contract:
        # the exact cotangent bins with the threads' private words first, then the staged output cotangents
        smem = (W * 5 * 8 + ((W * 4 + 7) // 8) * 8 + W * 5 * 8 * 128 + 15) // 16 * 16
        for q, (t, name, shape) in enumerate(ftal):
            S = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if S * 4 <= PRIV_BYTES:
                priv[("c", name)] = smem
                smem += (S * 4 + 15) // 16 * 16
    for t, (name, (shape, dt)) in enumerate(it.specs):
        S = int(np.prod(shape, dtype=np.int64)) if shape else 1
        nb = S * 44 if name in it.exact else S * 4
        if nb <= (4 * PRIV_BYTES if name in it.exact else PRIV_BYTES):
            priv[("p", name)] = smem
            smem += (nb + 15) // 16 * 16
    for q, (t, name, shape) in enumerate(ftal):
        S = int(np.prod(shape, dtype=np.int64)) if shape else 1
        nb = L * S * 44 if name in it.exact else L * S * 4
        if not contract and nb <= (4 * PRIV_BYTES if name in it.exact else PRIV_BYTES):
            priv[("d", name)] = smem
            smem += (nb + 15) // 16 * 16
    lines.append(f"  static constexpr int kSmemBytes = {max(smem, 16)};")
    ctx = ["  struct Ctx {"]
    for j, s in enumerate(it.in_specs[:npi]):
        ctx.append(f"    const {_in_ctype(s)}* in{j};")
    for k, b in enumerate(it.bc):
        ctx.append(f"    {CTYPE[b.dtype]} b{k};")       # (a table: its pointer)
    for q, k in enumerate(wrt):
        for l in range(L):
            ctx.append(f"    float db{k}_{l};")
    ctx += ["    i32 M;", "    i32* stats;", "    uint8_t* trunc;"]
    sizes = {}
    for t, (name, (shape, dt)) in enumerate(it.specs):
        S = int(np.prod(shape, dtype=np.int64)) if shape else 1
        sizes[name] = S
        ct = "float" if dt == T.F32 else "i32"
        ctx.append(f"    {ct}* g{t};")
        if name in it.exact:
            ctx.append(f"    u64* x{t};")
            if ("p", name) in priv:
                ctx.append(f"    u64* sx{t};")
            if not contract:
                ctx.append(f"    u64* dx{t};")
                if ("d", name) in priv:
                    ctx.append(f"    u64* sdx{t};")
        elif ("p", name) in priv:
            ctx.append(f"    {ct}* s{t};")
    for q, (t, name, shape) in enumerate(ftal):
        if contract:
            ctx.append(f"    const float* ct{t};")
            continue
        ctx.append(f"    float* gd{t};")
        if ("d", name) in priv and name not in it.exact:
            ctx.append(f"    float* sd{t};")
    if contract:
        ctx += ["    u64* gw;", "    float* g;", f"    mutable ExactPrivS<{W}> pv;"]
    for r, y in enumerate(tr.results):
        ctx.append(f"    {CTYPE[y.dtype] if y.dtype != T.BOOL else 'uint8_t'}* y{r};")
    act_saved = [i for i in it.saved if i in act]
    for i in it.saved:
        ctx.append(f"    {CTYPE[it.vars[i].dtype]} p{i};")
    for i in act_saved:
        for l in range(L):
            ctx.append(f"    float dp{i}_{l};")
    for r, (rname, (cap, fields)) in enumerate(recs):
        for f, (fname, dt) in enumerate(fields):
            ctx.append(f"    {CTYPE[dt]}* r{r}f{f};")
            if dt == T.F32:
                ctx += [f"    float* r{r}d{f}_{l};" for l in range(L)]
        if fill:
            ctx += [f"    const i32* rcnt{r};", f"    const long long* roff{r};", f"    i32 rn{r};", f"    long long ro{r};"]
        else:
            ctx += [f"    i32* r{r}cid;", f"    i32* r{r}k;", f"    unsigned long long* r{r}ctr;"]
        ctx.append(f"    i32* r{r}n;")
    if recs:
        ctx.append("    i64 item;")
    ctx.append("  };")
    lines += ctx
    lines.append("  struct State {")
    lines.append("    i32 kc;")
    for j, v in enumerate(tr.carry):
        lines.append(f"    {CTYPE[v.dtype]} c{j};")
        if carry_act[j]:
            for l in range(L):
                lines.append(f"    float d{j}_{l};")
    if contract:
        for l in range(L):
            lines.append(f"    float a{l};   // the item's cotangent of bc[{wrt[l]}] so far")
    for r in range(len(recs)):
        lines.append(f"    i32 rc{r};   // records appended by the item so far")
    lines.append("  };")
    tidx = {name: t for t, (name, _) in enumerate(it.specs)}
    lines.append("  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {")
    for j, s in enumerate(it.in_specs[:npi]):
        lines.append(f"    c.in{j} = static_cast<const {_in_ctype(s)}*>(P.p[kIn{j}]);")
    for k, b in enumerate(it.bc):
        lines.append(_bc_setup(k, b))
    for q, k in enumerate(wrt):
        for l in range(L):
            if contract:
                lines.append(f"    c.db{k}_{l} = {'1.0f' if l == q else '0.0f'};")
            else:
                lines.append(f"    c.db{k}_{l} = __ldg(static_cast<const float*>(P.p[kTan]) + {l * W + q});")
    lines += ["    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));",
              "    c.stats = static_cast<i32*>(P.p[kStats]);", "    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);"]
    for t, (name, (shape, dt)) in enumerate(it.specs):
        ct = "float" if dt == T.F32 else "i32"
        lines.append(f"    c.g{t} = static_cast<{ct}*>(P.p[kT{t}]);")
        if name in it.exact:
            lines.append(f"    c.x{t} = static_cast<u64*>(P.p[kX{t}]);")
            if ("p", name) in priv:
                lines.append(f"    c.sx{t} = reinterpret_cast<u64*>(smem + {priv[('p', name)]});")
            if not contract:
                lines.append(f"    c.dx{t} = static_cast<u64*>(P.p[kDX{t}]);")
                if ("d", name) in priv:
                    lines.append(f"    c.sdx{t} = reinterpret_cast<u64*>(smem + {priv[('d', name)]});")
        elif ("p", name) in priv:
            lines.append(f"    c.s{t} = reinterpret_cast<{ct}*>(smem + {priv[('p', name)]});")
    for q, (t, name, shape) in enumerate(ftal):
        if contract:
            if ("c", name) in priv:
                lines.append(f"    c.ct{t} = reinterpret_cast<const float*>(smem + {priv[('c', name)]});")
            else:
                lines.append(f"    c.ct{t} = static_cast<const float*>(P.p[kCt{q}]);")
            continue
        lines.append(f"    c.gd{t} = static_cast<float*>(P.p[kD{q}]);")
        if ("d", name) in priv and name not in it.exact:
            lines.append(f"    c.sd{t} = reinterpret_cast<float*>(smem + {priv[('d', name)]});")
    if contract:
        lines += ["    c.gw = static_cast<u64*>(P.p[kExact]);", "    c.g = static_cast<float*>(P.p[kG]);",
                  f"    c.pv.bind(smem + ExactBins<{W}>::kPrivOffset);"]
    for r, y in enumerate(tr.results):
        lines.append(f"    c.y{r} = static_cast<{CTYPE[y.dtype] if y.dtype != T.BOOL else 'uint8_t'}*>(P.p[kY{r}]);")
    for r, (rname, (cap, fields)) in enumerate(recs):
        for f, (fname, dt) in enumerate(fields):
            lines.append(f"    c.r{r}f{f} = static_cast<{CTYPE[dt]}*>(P.p[kR{r}F{f}]);")
            if dt == T.F32:
                lines += [f"    c.r{r}d{f}_{l} = static_cast<float*>(P.p[kR{r}D{f}_{l}]);" for l in range(L)]
        if fill:
            lines += [f"    c.rcnt{r} = static_cast<const i32*>(P.p[kRCnt{r}]);",
                      f"    c.roff{r} = static_cast<const long long*>(P.p[kROff{r}]);"]
        else:
            lines += [f"    c.r{r}cid = static_cast<i32*>(P.p[kR{r}Cid]);",
                      f"    c.r{r}k = static_cast<i32*>(P.p[kR{r}K]);",
                      f"    c.r{r}ctr = static_cast<unsigned long long*>(P.p[kR{r}Ctr]);"]
        lines.append(f"    c.r{r}n = static_cast<i32*>(P.p[kR{r}N]);")
    lines.append("  }")
    if contract:
        lines.append("  __device__ static void stage(const Params& P, unsigned char* smem) {")
        for q, (t, name, shape) in enumerate(ftal):
            if ("c", name) in priv:
                S = int(np.prod(shape, dtype=np.int64)) if shape else 1
                lines.append(f"    {{ const float* src = static_cast<const float*>(P.p[kCt{q}]); "
                             f"float* d = reinterpret_cast<float*>(smem + {priv[('c', name)]}); "
                             f"for (int b = threadIdx.x; b < {S}; b += blockDim.x) d[b] = __ldg(&src[b]); }}")
        lines.append("  }")
    else:
        lines.append("  __device__ static void stage(const Params&, unsigned char*) {}")
    acc = {"p": "a"}

    def emitter(name, idx_c, v_c):
        t, S, dt = tidx[name], sizes[name], it.tr.specs[name][1]
        pv = ("p", name) in priv
        if name in it.exact:
            return f"ExactSum<{S}>::emit({'c.sx' if pv else 'c.x'}{t}, c.stats, {idx_c}, {v_c});"
        if dt == T.F32:
            if pv:
                return f"SumPriv<{S}>::emit(c.s{t}, c.stats, {idx_c}, {v_c});"
            return (f"{{ const i32 b_ = {idx_c}; if ((u32)b_ >= {S}u) atomicAdd(&c.stats[kStDroppedEmits], 1); "
                    f"else fatom_warp_window(c.g{t}, nullptr, b_, -1, {v_c}); }}")
        tgt = f"c.s{t}" if pv else f"c.g{t}"
        return (f"{{ const i32 b_ = {idx_c}; if ((u32)b_ >= {S}u) atomicAdd(&c.stats[kStDroppedEmits], 1); "
                f"else if ({v_c}) atomicAdd(&{tgt}[b_], {v_c}); }}")

    def temitter(name, l, idx_c, dv_c):
        t, S = tidx[name], sizes[name]
        if contract:
            # the tangent emit contracted with the cotangent at its index (an out-of-range index adds nothing)
            a_ = f"{acc['p']}{l}"
            return f"{{ const i32 b_ = {idx_c}; if ((u32)b_ < {S}u) {a_} = {a_} + c.ct{t}[b_] * {dv_c}; }}"
        if name in it.exact:
            w_ = f"c.sdx{t}" if ("d", name) in priv else f"c.dx{t}"
            return (f"{{ const i32 b_ = {idx_c}; if ((u32)b_ < {S}u) ExactSum<{L * S}>::emit({w_}, c.stats, "
                    f"{l * S} + b_, {dv_c}); }}")
        tgt = f"c.sd{t}" if ("d", name) in priv else f"c.gd{t}"
        # (an out-of-range index is counted once, by the primal emit)
        return f"{{ const i32 b_ = {idx_c}; if ((u32)b_ < {S}u) fatom(&{tgt}[{l * S} + b_], {dv_c}); }}"

    bc_t = {it.bc[k].id: [f"c.db{k}_{l}" for l in range(L)] for k in wrt}
    rindex = {rname: r for r, (rname, _) in enumerate(recs)}

    def appender_for(counter):
        def appender(rname, when_c, vals_c, vals_t):
            """one record at the next raw slot (as the forward's), its float fields' tangents beside it; -0.0 is
            stored as +0.0 (its tangent unchanged)"""
            r = rindex[rname]
            cap, fields = tr.records[rname]
            if fill:
                st = [f"if ({when_c}) {{ if ({counter(r)} < c.rn{r}) {{ const long long o_ = c.ro{r} + {counter(r)};"]
            else:
                st = [f"if ({when_c}) {{ const unsigned long long o_ = atomicAdd(c.r{r}ctr, 1ull); "
                      f"if (o_ < {int(cap)}ull) {{"]
            for f, ((fname, dt), v) in enumerate(zip(fields, vals_c)):
                st.append(f" c.r{r}f{f}[o_] = {v}{' + 0.0f' if dt == T.F32 else ''};")
                if dt == T.F32:
                    for l in range(L):
                        tv = vals_t[f][l] if vals_t[f] is not None else "0.0f"
                        st.append(f" c.r{r}d{f}_{l}[o_] = {tv};")
            if fill:
                st.append(f" }} {counter(r)} += 1; }}")
            else:
                st.append(f" c.r{r}cid[o_] = (i32)c.item; c.r{r}k[o_] = {counter(r)}; }} {counter(r)} += 1; }}")
            return "".join(st)
        return appender

    def spawner(when_c, leaves_c, leaf_t):
        """a child's leaves and, for its float leaves, their tangents"""
        st = [f"if ({when_c}) {{ Child& o_ = n_out == 0 ? o0 : o1;"]
        st += [f" o_.l{m} = {v};" for m, v in enumerate(leaves_c)]
        for m in fl:
            for l in range(L):
                st.append(f" o_.d{m}_{l} = {leaf_t[m][l] if leaf_t[m] is not None else '0.0f'};")
        st.append(" ++n_out; }")
        return "".join(st)
    # start (a root: its inputs carry no tangent) and start_child (a child's leaves and their tangents)
    heads = [("State start(Ctx& c, i64 item)", [ld for _, ld in it.loads], {})]
    if sp:
        heads.append(("State start_child(Ctx& c, const Child& ch)", [f"ch.l{m}" for m in range(len(it.loads))],
                      {it.loads[m][0].id: [f"ch.d{m}_{l}" for l in range(L)] for m in fl}))
    for head, src_, tin in heads:
        lines.append(f"  __device__ static {head} {{")
        names = _names_pre(it)
        tn = dict(bc_t)
        tn.update(tin)
        if contract:
            acc["p"] = "a"
            for l in range(L):
                lines.append(f"    float a{l} = 0.0f;")
        for (v, _), ld in zip(it.loads, src_):
            lines.append(f"    const {CTYPE[v.dtype]} v{v.id} = {ld};")
        if recs:
            lines.append("    c.item = item;")
            lines += [f"    i32 rc{r} = 0;" for r in range(len(recs))]
            if fill:
                lines += [f"    c.rn{r} = __ldg(&c.rcnt{r}[item]); c.ro{r} = __ldg(&c.roff{r}[item]);"
                          for r in range(len(recs))]
        lines += _emit_code_jvp(tr.pre, names, tn, act, L, emitter, temitter,
                                appender=appender_for(lambda r: f"rc{r}") if recs else None)
        for i in it.saved:
            lines.append(f"    c.p{i} = {names[i]};")
        for i in act_saved:
            for l in range(L):
                lines.append(f"    c.dp{i}_{l} = {tn[i][l] if i in tn else '0.0f'};")
        lines += ["    State s;", "    s.kc = 0;"]
        if recs:
            lines += [f"    s.rc{r} = rc{r};" for r in range(len(recs))]
        if contract:
            for l in range(L):
                lines.append(f"    s.a{l} = a{l};")
        for j, x in enumerate(tr.carry_in):
            lines.append(f"    s.c{j} = {_ref(x, names)};")
            if carry_act[j]:
                for l in range(L):
                    tv = tn[x.id][l] if isinstance(x, T.Var) and x.id in tn else "0.0f"
                    lines.append(f"    s.d{j}_{l} = {tv};")
        lines += ["    return s;", "  }"]
    lines += _pred_fn(it)
    lines.append("  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) {")
    lines.append("    return s.kc < c.M && pred(c, s);")
    lines.append("  }")

    def loop_tn(carry, state):
        tn = dict(bc_t)
        for i in act_saved:
            tn[i] = [f"c.dp{i}_{l}" for l in range(L)]
        for j, v in enumerate(carry):
            if carry_act[j]:
                tn[v.id] = [f"{state}.d{j}_{l}" for l in range(L)]
        return tn
    if sp:
        lines.append("  __device__ __forceinline__ static void step(const Ctx& c, State& s, Child& o0, Child& o1, "
                     "int& n_out) {")
    else:
        lines.append("  __device__ __forceinline__ static void step(const Ctx& c, State& s) {")
    names = _names_loop(it, tr.carry)
    tn = loop_tn(tr.carry, "s")
    acc["p"] = "s.a"
    lines += _emit_code_jvp(tr.body, names, tn, act, L, emitter, temitter, spawner=spawner,
                            appender=appender_for(lambda r: f"s.rc{r}"))
    for j, x in enumerate(tr.body_out):
        lines.append(f"    const {CTYPE[tr.carry[j].dtype]} n{j} = {_ref(x, names)};")
        if carry_act[j]:
            for l in range(L):
                tv = tn[x.id][l] if isinstance(x, T.Var) and x.id in tn else "0.0f"
                lines.append(f"    const float nd{j}_{l} = {tv};")
    for j in range(len(tr.body_out)):
        lines.append(f"    s.c{j} = n{j};")
        if carry_act[j]:
            for l in range(L):
                lines.append(f"    s.d{j}_{l} = nd{j}_{l};")
    lines += ["    s.kc += 1;", "  }"]
    if not sp:
        lines.append("  __device__ static void finish(const Ctx& c, const State& s, i64 item) {")
    elif it.post_spawns:
        lines.append("  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child, Child& o0, "
                     "Child& o1, int& n_out) {")
    else:
        lines.append("  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child) {")
    names = _names_loop(it, tr.post_carry)
    tn = loop_tn(tr.post_carry, "s")
    if contract:
        acc["p"] = "a"
        for l in range(L):
            lines.append(f"    float a{l} = s.a{l};")
    for r in range(len(recs)):
        lines.append(f"    i32 rc{r} = s.rc{r};")
    lines += _emit_code_jvp(tr.post, names, tn, act, L, emitter, temitter, spawner=spawner,
                            appender=appender_for(lambda r: f"rc{r}"))
    if contract:
        for l in range(L):
            lines.append(f"    if (c.pv.emit({l}, a{l})) atomicAdd(&c.stats[kStFixedPointOverflow], 1);")
    if sp:
        # a child's per-item results are discarded (tallymap/_tally.py:285-286); its truncation is counted
        lines.append("    const bool tr_ = s.kc >= c.M && pred(c, s);")
        lines.append("    if (child) { if (tr_) atomicAdd(&c.stats[kStChildrenTruncated], 1); return; }")
    for r, y in enumerate(tr.results):
        lines.append(f"    c.y{r}[item] = {_ref(y, names)};")
    for r in range(len(recs)):
        lines.append(f"    c.r{r}n[item] = rc{r};")
    lines.append("    c.trunc[item] = " + ("tr_ ? 1 : 0;" if sp else "(s.kc >= c.M && pred(c, s)) ? 1 : 0;"))
    lines.append("  }")
    lines.append("  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {")
    if contract:
        lines.append(f"    ExactBins<{W}>::flush(c.pv, const_cast<unsigned char*>(smem), c.gw, c.stats, tid);")
    for t, (name, (shape, dt)) in enumerate(it.specs):
        S = sizes[name]
        if name in it.exact:
            if ("p", name) in priv:
                lines.append(f"    ExactSum<{S}>::flush(c.sx{t}, c.x{t}, c.stats, tid, nth);")
            if ("d", name) in priv:
                lines.append(f"    ExactSum<{L * S}>::flush(c.sdx{t}, c.dx{t}, c.stats, tid, nth);")
            continue
        if ("p", name) in priv:
            if dt == T.F32:
                lines.append(f"    SumPriv<{S}>::flush(c.s{t}, c.g{t}, tid, nth);")
            else:
                lines.append(f"    for (int b = tid; b < {S}; b += nth) if (c.s{t}[b]) atomicAdd(&c.g{t}[b], c.s{t}[b]);")
    for q, (t, name, shape) in enumerate(ftal):
        if ("d", name) in priv and name not in it.exact:
            lines.append(f"    SumPriv<{L * sizes[name]}>::flush(c.sd{t}, c.gd{t}, tid, nth);")
    lines.append("  }")
    lines.append("  __device__ static void epilogue(const Ctx& c, int tid, int nth) {")
    if contract:
        lines.append(f"    if (tid == 0) ExactBins<{W}>::readout(c.gw, c.g, c.stats);")
    for t, name in ex:
        lines.append(f"    ExactSum<{sizes[name]}>::readout(c.x{t}, c.g{t}, c.stats, tid, nth);")
        if not contract:
            lines.append(f"    ExactSum<{L * sizes[name]}>::readout(c.dx{t}, c.gd{t}, c.stats, tid, nth);")
    lines.append("  }")
    lines.append("};")
    lines.append("}  // namespace tmb")
    lines.append('extern "C" __global__ void TM_MAIN_BOUNDS tm_main(const tmb::Params P, const long long n) {')
    lines.append(f"  tmb::{'spawn_body' if sp else 'forward_body'}<tmb::GenJvp>(P, n);")
    lines.append("}")
    lines.append(f"static_assert(tmb::GenJvp::kSmemBytes == {max(smem, 16)}, \"shared-memory size\");")
    total = max(smem, 16)
    if sp:
        # the spawn runtime's shared stack entries after the item's block (csrc/tm_spawn.cuh SpawnSmem)
        total = (total + 15) // 16 * 16 + SPAWN_STACK_SHARED * 4 * (len(it.loads) + len(fl) * L) * 128
        lines.append(f"static_assert(tmb::SpawnSmem<tmb::GenJvp>::kBytes == {total}, \"shared-memory size\");")
    return "\n".join(lines), total
