"""The user-facing layer over the backend: `vmap(item, outputs, in_axes, max_steps)` returning `Result`, its
reverse mode (`grad`, `value_and_grad`) and forward mode (`jvp`, `jacfwd`), with the reference's result contract
(tallymap/_api.py:180-195, 681-698, 898-958):

  * outputs: the Sums (and Records); EVERY float output is NaN when a resource limit intervened (an item hit
    max_steps, counted in stats['n_truncated']; a spawned child hit max_steps or did not fit the Queue, counted in
    stats['children_truncated'] / ['children_dropped']; a Records output overflowed: _api.py:898-915); integer
    outputs and per-item results are never poisoned;
  * per_item: the item's per-item results; truncated: bool[N];
  * stats: spawned, children_dropped, children_truncated, fixed_point_overflow, dropped_emits, n_truncated (and
    appended / records_dropped for Records).

A gradient is a replay launch (the adjoint program recomputes every item from its inputs: _api.py:951-958) whose own
truncation flags poison the cotangent (_primitive.py:586-594); `value_and_grad` with cotangents given up front is one
fused launch where the item has a pipelined value-and-grad program; through spawn it is the tree adjoint.

An item is either a Python function written against tallymap_b200.lang -- traced, lowered to CUDA and compiled on
its first call (MappedFn) -- or the name of a hand-lowered family ("quickstart", "walk1d", "photon", "lorenz",
"shower": Mapped).  JAX is not a dependency.
"""
import dataclasses
from typing import Any, NamedTuple

import numpy as np
import torch

from . import backend as B
from . import trace as T
from .trace import TallyError, UnsupportedError  # noqa: F401  (the reference's public exception types)


@dataclasses.dataclass(frozen=True)
class Sum:
    """a summed output of a fixed shape (tallymap.Sum, _api.py:55-84), of dtype float32, int32, float64 or int64 (a
    float64 output sums the item's float32 values in float64, an int64 one its int32 values in int64).
    fixed_point=True with float32 (items traced from Python functions): EXACT -- each bin is the correctly rounded
    float32 of the exact sum of its emits, bitwise independent of their order (run to run, launch order, number of
    GPUs); a non-finite emit or an accumulator overflow makes the bin NaN, counted in stats['fixed_point_overflow'].
    fixed_point=True with another dtype: each emit adds round(v * scale) to an int64 word whose signed carry is kept
    beside it, so a bin's total is exact and order-independent past 2^63; it is read out as total / scale in the
    output's dtype.  An emit with |v * scale| >= 9.2e18 is dropped, counted in 'fixed_point_overflow', and makes a
    float bin NaN; a total that does not fit the dtype is counted there too (a float bin is NaN)."""
    shape: tuple
    dtype: torch.dtype = torch.float32
    fixed_point: bool = False
    scale: float = 2.0 ** 32

    def __post_init__(self):
        shape = (self.shape,) if isinstance(self.shape, (int, np.integer)) else self.shape
        object.__setattr__(self, "shape", tuple(int(s) for s in shape))
        if self.dtype not in (torch.float32, torch.int32, torch.float64, torch.int64):
            raise TypeError("tallymap_b200: a Sum of float32, int32, float64 or int64")
        if not (float(self.scale) > 0.0 and np.isfinite(float(self.scale))):
            raise ValueError("tallymap_b200: a fixed-point Sum's scale is a positive finite number")

    def accumulator(self):
        """None (a plain float32 / int32 sum, or the exact float32 one), ("f64",), ("i64",) or ("wide", dtype,
        scale) (the scaled fixed-point sum)"""
        if self.fixed_point and self.dtype != torch.float32:
            return ("wide", self.dtype, float(self.scale))
        if self.dtype == torch.float64:
            return ("f64",)
        if self.dtype == torch.int64:
            return ("i64",)
        return None


@dataclasses.dataclass(frozen=True)
class Queue:
    """the spawn queue of a spawning item (tallymap.Queue, _api.py:88-98): a ring of `capacity` slots for children
    shared between threads.  Each thread runs the children it spawns depth-first from a private stack and shares
    through the ring only what idle threads wait for, so the ring holds at most about one child per idle thread; a
    child that finds it full is dropped, counted in stats['children_dropped'], and poisons every float output."""
    capacity: int

    def __post_init__(self):
        if not 1 <= int(self.capacity) <= 2 ** 31 - 1:
            raise ValueError("tallymap_b200.Queue: capacity in [1, 2^31 - 1]")
        object.__setattr__(self, "capacity", int(self.capacity))


@dataclasses.dataclass(frozen=True)
class Records:
    """a Records output (tallymap.Records, _api.py:98-170): Records({field: dtype}, capacity=C) or
    Records({field: dtype}) (capacity None).  Items append with t = t.append(name, {field: value}, when=...);
    Result.outputs[name] is {field: tensor}: record k of item i at slot offset[i] + k (offset the exclusive prefix sum
    of the per-item counts); stats['appended'][name] the true total.
      capacity C (one pass, _records.py): tensors of C slots, those past the last record zero.  More than C records
        poisons the call: float fields and every float Sum NaN, integer fields -1, stats['records_dropped'][name]
        the excess.
      capacity None (count-then-fill, _api.py:138-148): the items run twice, a count pass (each item's record count)
        and the fill pass (every output; record k of item i written straight to offset[i] + k): tensors of exactly
        the total.  An item whose fill appends a different number of records than its count poisons the call like
        an overflow, counted in stats['records_mismatch'][name]."""
    fields: tuple
    capacity: Any

    def __init__(self, *args, fields=None, capacity=None):
        for a in args:             # (the reference's Records(fields, capacity) in either order)
            if isinstance(a, dict):
                if fields is not None:
                    raise TypeError("tallymap_b200.Records: fields given twice")
                fields = a
            elif a is None or isinstance(a, (int, np.integer)):
                capacity = a
            else:
                raise TypeError(f"tallymap_b200.Records(fields, capacity): unexpected argument {a!r}")
        fl = []
        for f, dt in sorted((fields or {}).items()):
            if dt not in (torch.float32, torch.int32):
                raise TypeError(f"tallymap_b200.Records: field {f!r}: float32 or int32")
            fl.append((f, dt))
        if not fl:
            raise TypeError("tallymap_b200.Records needs fields")
        if capacity is not None and not 1 <= int(capacity) <= 2 ** 31 - 1:
            raise ValueError("tallymap_b200.Records: capacity in [1, 2^31 - 1] or None")
        object.__setattr__(self, "fields", tuple(fl))
        object.__setattr__(self, "capacity", None if capacity is None else int(capacity))


class Result(NamedTuple):
    outputs: dict
    per_item: Any
    truncated: Any
    stats: dict


@dataclasses.dataclass(frozen=True)
class Family:
    """an item program in its forward and reverse forms.  in_axes: the item's (0 | None) per argument (the
    per-item operands first, then broadcast ones, as the programs lay them out); grads: broadcast operand index ->
    its adjoint program; ys: which per-item results the item returns (besides the truncation flag)."""
    name: str
    fwd: B.ItemProgram
    grads: dict          # tuple of broadcast operand indices -> the adjoint program giving their cotangents
    in_axes: tuple
    default_max_steps: int
    fused: dict = dataclasses.field(default_factory=dict)   # the same keys -> value-and-grad program (one launch)
    onepass: dict = dataclasses.field(default_factory=dict)  # the same keys -> one-pass value-and-grad (no active
                                                              # carry: step VJPs summed as the forward runs)
    onepass_grad: bool = False   # grad(exact_order=False) runs the one-pass launch: it is forward mode, while the
                                 # replay re-runs the forward
    claim_order: object = None   # pi -> an int32 permutation of the items, the order the launch claims them in (a
                                 # scheduling hint: it moves no result to another item or tally)


FAMILIES = {
    "quickstart": Family("quickstart", B.Q1_FWD, {(0,): B.Q1_GRAD}, (0, 0, None), 100, {(0,): B.Q1_VG},
                         {(0,): B.Q1_VG1}),
    "walk1d": Family("walk1d", B.RW_FWD, {(0,): B.RW_GRAD}, (0, 0, None), 20000, {(0,): B.RW_VG},
                     {(0,): B.RW_VG1}),
    "photon": Family("photon", B.PH_FWD, {(0, 1): B.PH_GRAD}, (0, None, None), 100000, {}, {(0, 1): B.PH_VG1},
                     onepass_grad=True),
    "lorenz": Family("lorenz", B.OD_FWD, {(0,): B.OD_GRAD}, (0, 0, 0, 0, None), 50000, {}, {(0,): B.OD_VG1},
                     onepass_grad=True),
    # reverse mode through spawn: the tree adjoint (backend.tree_grad), w.r.t. X0 and the roots' E and depth
    # (roots claimed largest energy first: a root's subtree grows with its energy, so the launch's tail is small trees)
    "shower": Family("shower", B.SH_FWD, {"tree": B.tree_grad}, (0, 0, 0, None), 100000, onepass_grad=True,
                     claim_order=lambda pi: B.energy_order(pi[0])),
}


def _limits(p, stats):
    """did a resource limit intervene (_api.py:898-912, _limits)?  An item hit max_steps; for a spawning program
    also a child that did not fit the queue or hit max_steps.  -> a bool tensor on the device"""
    bad = stats["n_truncated"] > 0
    if p.spawns:
        bad = bad | (stats["children_dropped"] > 0) | (stats["children_truncated"] > 0)
    return bad


def _f32(c):
    """a cotangent as float32 (a float64 output's cotangent enters the float32 adjoint)"""
    return c.to(torch.float32) if isinstance(c, torch.Tensor) and c.dtype != torch.float32 else c


def _poison(outs, bad):
    """NaN for every float output when `bad` (a select, so a clean call is bitwise unchanged: _api.py:916-925)."""
    return {n: (torch.where(bad, torch.full_like(v, float("nan")), v) if v.is_floating_point() else v)
            for n, v in outs.items()}


def _poison_records(rec, bad):
    """a Records output's fields when it overflowed or its fill disagreed with its count: float fields NaN, integer
    fields -1 (as the one-pass canonical layout poisons)"""
    return {n: torch.where(bad, torch.full_like(v, float("nan") if v.is_floating_point() else -1), v)
            for n, v in rec.items()}


class Mapped:
    """tallymap.vmap(item, outputs, in_axes, max_steps) over a lowered item family."""

    def __init__(self, fam, outputs, in_axes, max_steps, spawn=None, opts=None):
        self.fam = fam
        self.opts = opts or options()
        if spawn is not None and not fam.fwd.spawns:
            raise ValueError(f"tallymap_b200: item {fam.name!r} does not spawn")
        self.queue = spawn.capacity if spawn is not None else None
        names = [t.name for t in fam.fwd.tallies]
        if sorted(outputs) != sorted(names):
            raise KeyError(f"tallymap_b200: item {fam.name!r} writes outputs {names}, got {sorted(outputs)}")
        for t in fam.fwd.tallies:
            o = outputs[t.name]
            if tuple(o.shape) != tuple(t.shape) and "N" not in t.shape or o.dtype != t.dtype:
                raise TypeError(f"tallymap_b200: output {t.name!r} is Sum({t.shape}, {t.dtype}) in this item, got "
                                f"Sum({o.shape}, {o.dtype})")
        if tuple(in_axes) != tuple(fam.in_axes):
            raise ValueError(f"tallymap_b200: item {fam.name!r} maps in_axes={fam.in_axes}, got {tuple(in_axes)}")
        self.max_steps = int(fam.default_max_steps if max_steps is None else max_steps)
        if self.max_steps < 1:
            raise ValueError("tallymap_b200: max_steps must be >= 1")

    def _split(self, args):
        if len(args) != len(self.fam.in_axes):
            raise TypeError(f"tallymap_b200: item {self.fam.name!r} takes {len(self.fam.in_axes)} arguments")
        pi = [a for a, ax in zip(args, self.fam.in_axes) if ax == 0]
        bc = [a for a, ax in zip(args, self.fam.in_axes) if ax is None]
        return pi, bc

    def __call__(self, *args, n_active=None):
        """the forward launch; n_active: only items i < n_active run (_api.py:466-469)"""
        pi, bc = self._split(args)
        p = self.fam.fwd
        order = None
        if self.fam.claim_order is not None and n_active is None:
            # (the first per-item operand moved once, here: run takes the device tensor as it is)
            pi = [B._dev(pi[0], torch.device("cuda", torch.cuda.current_device()), torch.float32)] + pi[1:]
            order = self.fam.claim_order(pi)
        out = B.run(p, pi, bc, consts=(self.max_steps,), queue=self.queue, n_active=n_active, order=order)
        nt = len(p.tallies)
        tallies = {t.name: v for t, v in zip(p.tallies, out[:nt])}
        stats_raw = out[nt]
        ys = out[nt + 1:]
        trunc = ys[p.trunc].bool()
        per = [y for i, y in enumerate(ys) if i != p.trunc]
        n_tr = trunc.sum(dtype=torch.int32)
        stats = {n: stats_raw[i] for i, n in enumerate(B.STATS)}
        stats["n_truncated"] = n_tr
        outs = _poison(tallies, _limits(p, stats))
        return Result(outs, per[0] if len(per) == 1 else (tuple(per) or None), trunc, stats)

    def value_and_grad(self, *args, wrt, cotangents, fused=True, exact_order=False):
        """(Result, gradient of <cotangents, outputs>) with the inputs moved to the device once.  The cotangents are
        given up front, so where the item has a fused program this is ONE launch.  An item with no active carry (its
        loop state does not depend on `wrt`: the walkers) runs the one-pass program: each step's VJP is summed as the
        forward runs, oldest step first, so the gradient equals the reverse program's within the float tolerance
        (not bitwise: f32 summation order); the photon's one-pass program is forward mode (its one active carry's
        tangent travels with the state), again within the float tolerance.  With exact_order=True, or for other items, the fused program is the
        replay whose count pass is the forward pass, emitting the forward's tallies while it stores the states the
        step VJPs then read (bitwise the separate forward and replay; tests/test_fused_gpu.py).  Otherwise (or
        fused=False) one forward and one replay launch; the replay claims items longest first by the forward's trip
        counts (an LPT schedule: the replay of an item costs a known function of its trip count), which balances the
        threads' work and keeps a warp's lanes in the same replay phase; it changes no result (the cotangent tally is
        exact, per-item results are indexed by item)."""
        dev = torch.device("cuda", torch.cuda.current_device())
        moved = []
        for a, ax in zip(args, self.fam.in_axes):
            if ax == 0:
                t = a if isinstance(a, torch.Tensor) else torch.from_numpy(B._host(a))
                moved.append(t.to(dev, non_blocking=True))
            else:
                moved.append(a)
        if fused and "tree" in self.fam.grads and not exact_order:
            return self._onepass_tree(moved, wrt, cotangents)
        if fused:
            r = self._fused(moved, wrt, cotangents, onepass=not exact_order)
            if r is not None:
                return r
        res = self(*moved)
        order = None
        if "tree" not in self.fam.grads and isinstance(res.per_item, torch.Tensor) and \
                res.per_item.dtype == torch.int32:
            order = longest_first(res.per_item)
        return res, self.grad(*moved, wrt=wrt, cotangents=cotangents, order=order)

    def grad(self, *args, wrt, cotangents, order=None, exact_order=True):
        """d <cotangents, outputs> / d args[wrt] for broadcast operand(s) `wrt` (an argument index or a tuple of
        them): ONE replay launch (for the shower: the tree adjoint).  cotangents: {output name: array of the output's
        shape}; missing outputs get zero cotangents.  -> a scalar for one index, a vector for a tuple; NaN when an
        item's replay hit max_steps.  exact_order=False: where the family's one-pass program is forward mode (the
        photon, the Lorenz ensemble, the shower), that launch instead, its forward outputs discarded -- faster than
        the replay, which re-runs the forward, and equal to it within the float tolerance."""
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        if not exact_order and self.fam.onepass_grad:
            return self.value_and_grad(*args, wrt=wrt, cotangents=cotangents)[1]
        if "tree" in self.fam.grads:
            return self._tree_grad(args, idx, cotangents, wrt)
        if any(self.fam.in_axes[w] is not None for w in idx):
            raise ValueError("tallymap_b200: grad with respect to a per-item operand is not built for this item")
        bpos = tuple(sum(1 for ax in self.fam.in_axes[:w] if ax is None) for w in idx)
        prog, sel = None, None
        for key, g in self.fam.grads.items():
            if all(b in key for b in bpos):
                prog, sel = g, [key.index(b) for b in bpos]
                break
        if prog is None:
            raise NotImplementedError(f"tallymap_b200: item {self.fam.name!r} has no adjoint for arguments {idx}")
        pi, bc = self._split(args)
        cts = []
        for t in self.fam.fwd.tallies:
            c = cotangents.get(t.name)
            n = int(pi[0].shape[0]) if pi else 0
            cts.append(torch.zeros(t.dims(n), dtype=t.dtype) if c is None else c)
        out = B.run(prog, pi, list(bc) + cts, consts=(self.max_steps,), order=order,
                    rev_checkpoints=self.opts["rev_checkpoints"])
        ct = out[0].reshape(-1)[sel]
        trunc = out[len(prog.tallies) + 1 + prog.trunc]
        ct = torch.where(trunc.bool().any(), torch.full_like(ct, float("nan")), ct)
        return ct.reshape(()) if isinstance(wrt, int) else ct


    def _cotangents(self, n, cotangents):
        return [torch.zeros(t.dims(n), dtype=t.dtype) if cotangents.get(t.name) is None else cotangents[t.name]
                for t in self.fam.fwd.tallies]

    def _fused(self, args, wrt, cotangents, onepass=True):
        """(Result, gradient) from the family's one-pass (when `onepass`) or fused value-and-grad program, or None
        when it has none for `wrt`"""
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        if any(self.fam.in_axes[w] is not None for w in idx):
            return None
        bpos = tuple(sum(1 for ax in self.fam.in_axes[:w] if ax is None) for w in idx)
        prog, sel = None, None
        for progs in ((self.fam.onepass,) if onepass else ()) + (self.fam.fused,):
            for key, g in progs.items():
                if all(b in key for b in bpos):
                    prog, sel = g, [key.index(b) for b in bpos]
                    break
            if prog is not None:
                break
        if prog is None or (prog.replay_state_bytes and not B.pipelined(prog, self.max_steps)):
            return None
        pi, bc = self._split(args)
        n = int(pi[0].shape[0]) if pi else 0
        out = B.run(prog, pi, list(bc) + self._cotangents(n, cotangents), consts=(self.max_steps,),
                    rev_checkpoints=self.opts["rev_checkpoints"])
        p = self.fam.fwd
        nt = len(p.tallies)
        tallies = {t.name: v for t, v in zip(p.tallies, out[:nt])}
        ct = out[nt].reshape(-1)[sel]
        stats_raw = out[nt + 1]
        ys = out[nt + 2:]
        trunc = ys[p.trunc].bool()
        per = [y for i, y in enumerate(ys) if i != p.trunc]
        n_tr = trunc.sum(dtype=torch.int32)
        stats = {nm: stats_raw[i] for i, nm in enumerate(B.STATS)}
        stats["n_truncated"] = n_tr
        bad = n_tr > 0
        res = Result(_poison(tallies, bad), per[0] if len(per) == 1 else (tuple(per) or None), trunc, stats)
        ct = torch.where(bad, torch.full_like(ct, float("nan")), ct)
        return res, (ct.reshape(()) if isinstance(wrt, int) else ct)

    def _onepass_tree(self, args, wrt, cotangents):
        """(Result, gradient) of the shower in one spawn launch: forward mode through spawn (backend.sh_value_and_grad),
        the gradient within the float tolerance of the tree adjoint's; NaN when a limit intervened"""
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        pi, bc = self._split(args)
        c = cotangents.get("dep")
        ct = torch.zeros(512, dtype=torch.float32) if c is None else c
        order = self.fam.claim_order(pi) if self.fam.claim_order is not None else None
        r = B.sh_value_and_grad(pi, bc[0], ct, max_steps=self.max_steps, queue=self.queue, order=order)
        p = self.fam.fwd
        trunc = r["trunc"].bool()
        n_tr = trunc.sum(dtype=torch.int32)
        stats = {nm: r["stats"][i] for i, nm in enumerate(B.STATS)}
        stats["n_truncated"] = n_tr
        bad = _limits(p, stats)
        res = Result(_poison({"dep": r["dep"], "count": r["count"]}, bad), r["k"], trunc, stats)
        by_arg = {0: r["g_E"], 1: r["g_depth"], 3: r["g_X0"].reshape(())}
        if any(w not in by_arg for w in idx):
            raise ValueError(f"tallymap_b200: item {self.fam.name!r} is differentiable in arguments {sorted(by_arg)}")
        g = tuple(torch.where(bad, torch.full_like(by_arg[w], float("nan")), by_arg[w]) for w in idx)
        return res, (g[0] if isinstance(wrt, int) else g)

    def _tree_grad(self, args, idx, cotangents, wrt):
        """the gradient of a spawning item through its children (tallymap/_reverse_spawn.py:233-336): the recording
        forward, then one adjoint launch per generation, deepest first, and one over the roots.  Differentiable
        arguments: the roots' float per-item operands (-> f32[N]) and the broadcast X0 (-> a scalar)."""
        pi, bc = self._split(args)
        c = cotangents.get("dep")
        ct = torch.zeros(512, dtype=torch.float32) if c is None else c
        r = self.fam.grads["tree"](pi, bc[0], ct, max_steps=self.max_steps,
                                   rev_checkpoints=self.opts["rev_checkpoints"])
        by_arg = {0: r["ct_E"], 1: r["ct_depth"], 3: r["ct_X0"].reshape(())}
        if any(w not in by_arg for w in idx):
            raise ValueError(f"tallymap_b200: item {self.fam.name!r} is differentiable in arguments {sorted(by_arg)}")
        self.last_tree = r["info"]
        g = tuple(by_arg[w] for w in idx)
        return g[0] if isinstance(wrt, int) else g


def longest_first(k):
    """the claim order that runs items with the largest trip counts first (a stable descending sort on device)"""
    return torch.argsort(k, descending=True, stable=True).to(torch.int32)


class MappedFn:
    """tallymap.vmap over a Python item function: traced (tallymap_b200.trace) on its first call with a given
    operand signature, lowered to CUDA and compiled for sm_100a at run time (tallymap_b200.lower, NVRTC); the reverse
    programs are lowered and compiled on the first gradient request for each set of differentiated operands."""

    def __init__(self, fn, outputs, in_axes, max_steps, spawn=None, opts=None):
        self.fn = fn
        self.opts = opts or options()
        if spawn is not None and not isinstance(spawn, Queue):
            raise TypeError("tallymap_b200: spawn= takes a tallymap_b200.Queue(capacity)")
        self.spawn = spawn
        self.outputs = {}
        for name, o in outputs.items():
            if isinstance(o, Records):
                self.outputs[name] = ("records", o.capacity,
                                      tuple((f, "f32" if dt == torch.float32 else "i32") for f, dt in o.fields))
                continue
            # (shape, the item's value type, exact float32 sum, the wider accumulator or None)
            acc = o.accumulator()
            self.outputs[name] = (tuple(o.shape), "f32" if o.dtype in (torch.float32, torch.float64) else "i32",
                                  bool(o.fixed_point) and o.dtype == torch.float32, acc)
        if in_axes == 0:
            import inspect
            ps = list(inspect.signature(fn).parameters.values())[1:]
            if any(q.kind in (q.VAR_POSITIONAL, q.VAR_KEYWORD) for q in ps):
                raise TypeError("tallymap_b200: an item with *args takes in_axes as a tuple (0 or None per argument)")
            in_axes = (0,) * len(ps)
        self.in_axes = tuple(in_axes)
        if any(ax not in (0, None) for ax in self.in_axes):
            raise ValueError("tallymap_b200: in_axes entries are 0 (per item) or None (broadcast)")
        self.max_steps = int(2 ** 31 - 1 if max_steps is None else max_steps)
        if self.max_steps < 1:
            raise ValueError("tallymap_b200: max_steps must be >= 1")
        self._lowered = {}
        self.last_lowered = None
        self.last_tree = None       # a spawning item's last tree adjoint: its counters (backend.tree_adjoint info)

    @staticmethod
    def _spec(a, per_item):
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(B._host(a))
        dt = {torch.float32: "f32", torch.int32: "i32", torch.uint32: "u32"}.get(t.dtype)
        if dt is None:
            raise TypeError(f"tallymap_b200: operand dtype {t.dtype} (float32, int32 or uint32 key data)")
        shape = tuple(t.shape[1:]) if per_item else tuple(t.shape)
        if shape == ():
            return dt if dt != "u32" else "i32"
        if per_item and shape == (2,) and dt in ("i32", "u32"):
            return "key"                      # uint32[N, 2] key data (int32 bits on torch)
        if per_item and len(shape) == 1 and dt == "f32":
            return ("f32", shape[0])
        if not per_item and len(shape) == 1 and dt == "f32" and 1 <= shape[0] <= BC_VECTOR_MAX:
            return (dt, shape[0])             # a broadcast vector: that many broadcast scalars
        if not per_item and 1 <= len(shape) <= 2 and dt in ("f32", "i32") and 0 < int(np.prod(shape)) < 2 ** 31:
            return ("table", dt, shape)       # a broadcast table, read by index (lang: t[i], t[i, j])
        raise TypeError(f"tallymap_b200: operand of {'per-item ' if per_item else ''}shape {shape} and dtype {dt} "
                        "is not lowered")

    def lowered(self, args):
        from . import lower
        if len(args) != len(self.in_axes):
            raise TypeError(f"tallymap_b200: the item takes {len(self.in_axes)} arguments, got {len(args)}")
        pis = [self._spec(a, True) for a, ax in zip(args, self.in_axes) if ax == 0]
        bcs = [self._spec(a, False) for a, ax in zip(args, self.in_axes) if ax is None]
        key = (tuple(pis), tuple(bcs))
        if key not in self._lowered:
            order = [ax for ax in self.in_axes]
            # the item's arguments in their declared order; the lowering wants per-item first
            perm = [i for i, ax in enumerate(order) if ax == 0] + [i for i, ax in enumerate(order) if ax is None]
            bargs = [i for i, ax in enumerate(order) if ax is None]
            # a broadcast vector is lowered as consecutive broadcast scalars: argument -> (first, n or None)
            groups, leaves = {}, []
            for i, sp in zip(bargs, bcs):
                vec = isinstance(sp, tuple) and sp[0] != "table"
                groups[i] = (len(leaves), sp[1] if vec else None)
                leaves += [sp[0]] * sp[1] if vec else [sp]
            npi = len(pis)

            def item(t, *xs):
                vals = list(xs[:npi])
                for i in bargs:
                    f, n = groups[i]
                    vals.append(xs[npi + f] if n is None else T.Vec(xs[npi + f:npi + f + n]))
                args_ = [None] * len(vals)
                for pos, x in zip(perm, vals):
                    args_[pos] = x
                return self.fn(t, *args_)
            item.__name__ = getattr(self.fn, "__name__", "item")
            L = lower.Lowered(item, pis + leaves, npi, self.outputs, spawn=self.spawn is not None,
                              math=self.opts["math"], min_blocks=self.opts["min_blocks"])
            L.bc_groups = groups
            if self.opts["schedule"] == "step" and isinstance(L.tr.cond_out, T.Lit):
                raise UnsupportedError(f"tallymap_b200: schedule='step' needs an item with exactly one top-level "
                                       f"while loop; {item.__name__} has none")
            self._lowered[key] = L
        self.last_lowered = self._lowered[key]
        return self._lowered[key]

    def _split(self, args):
        """(per-item operands, broadcast scalars): a broadcast vector gives one scalar per element"""
        pi = [a for a, ax in zip(args, self.in_axes) if ax == 0]
        bc = []
        for a, ax in zip(args, self.in_axes):
            if ax is None:
                t = a if isinstance(a, torch.Tensor) else B._host(a)
                vec = t.ndim == 1 and 1 <= t.shape[0] <= BC_VECTOR_MAX and str(t.dtype).endswith("float32")
                bc += [t[i] for i in range(t.shape[0])] if vec else [a]
        return pi, bc

    @staticmethod
    def _per_item(L, ys):
        """the flat per-item results regrouped as the item returned them: a vector -> one tensor (N, n); -> the
        Result's per_item (one value, a tuple, or None)"""
        groups = L.tr.result_groups or [(j, None) for j in range(len(ys))]
        per = [ys[f] if n is None else torch.stack(list(ys[f:f + n]), dim=1) for f, n in groups]
        return per[0] if len(per) == 1 else (tuple(per) or None)

    def _bleaves(self, L, idx):
        """-> (the broadcast scalar positions of broadcast arguments idx, in order; argument -> (its first position
        among them, n for a vector or None for a scalar))"""
        pos, where = [], {}
        for w in idx:
            f, n = L.bc_groups[w]
            where[w] = (len(pos), n)
            pos += [f] if n is None else list(range(f, f + n))
        return tuple(pos), where

    @staticmethod
    def _per_arg(ct, where, wrt, idx):
        """a broadcast gradient vector (one entry per scalar position) -> one gradient per argument: a scalar for
        a scalar argument, f32[n] for a vector; the flat vector itself for a tuple of scalar arguments"""
        if all(n is None for _, n in where.values()) and not isinstance(wrt, int):
            return ct
        got = {w: ct[q].reshape(()) if n is None else ct[q:q + n] for w, (q, n) in where.items()}
        return got[wrt] if isinstance(wrt, int) else tuple(got[w] for w in idx)

    def __call__(self, *args, n_active=None):
        """the forward launch; n_active: only items i < n_active run, the others emit nothing, are never truncated
        and their per-item results are zero (_api.py:466-469)"""
        L = self.lowered(args)
        pi, bc = self._split(args)
        p = L.fwd
        if p.records and self._fill_needed():
            # count-then-fill: the count pass, then the fill pass with every record at its canonical slot
            cnts, offs, tots = self._counts(L, pi, bc, n_active)
            fprog = self._sized(L.records_programs()[1], tots)
            out = B.run(fprog, self._with_counts(pi, cnts, offs), bc, consts=(self.max_steps,), n_active=n_active)
            return self._result(L, fprog, out, B.run.last["results"], fill=(cnts, tots))
        out = B.run(p, pi, bc, consts=(self.max_steps,), queue=self.spawn.capacity if self.spawn else None,
                    n_active=n_active)
        return self._result(L, p, out, B.run.last["results"])

    def _fill_needed(self):
        """whether a Records output has no capacity (count-then-fill)"""
        return any(o[0] == "records" and o[1] is None for o in self.outputs.values())

    def _counts(self, L, pi, bc, n_active=None):
        """the count pass: per Records output (L.fwd.records' order) the items' record counts int32[N], their
        canonical offsets int64[N] (the exclusive prefix sum) and the total (host ints: one synchronisation)"""
        cprog = L.records_programs()[0]
        out = B.run(cprog, pi, bc, consts=(self.max_steps,), n_active=n_active)
        ys = out[len(cprog.tallies) + 1:]
        cnts = [ys[L.n_results + r].clone() for r in range(len(L.fwd.records))]
        offs = [torch.cumsum(c.to(torch.int64), 0) - c.to(torch.int64) for c in cnts]
        tots = [int(t) for t in torch.stack([c.to(torch.int64).sum() for c in cnts]).cpu().tolist()]
        return cnts, offs, tots

    @staticmethod
    def _sized(prog, tots):
        """a fill program with each Records output's buffers sized to its total"""
        return dataclasses.replace(prog, records=tuple((nm, max(t, 1), fl) for (nm, _, fl), t in zip(prog.records, tots)))

    @staticmethod
    def _with_counts(pi, cnts, offs):
        return list(pi) + [x for c, o in zip(cnts, offs) for x in (c, o)]

    def _fill_records(self, L, raw, ys, cnts, tots, lanes=0):
        """a fill launch's Records outputs (raw: its buffers by name): ({name: {field: tensor}} -- the declared
        capacity's slots, zeros past the last record, or the exact total without one --, {name: {float field:
        tangent (lanes, size)}}, stats additions, a device bool: an output overflowed or an item's fill appended a
        different number of records than its count)"""
        recs, tans = {}, {}
        st = {"appended": {}, "records_dropped": {}, "records_mismatch": {}}
        bad = torch.zeros((), dtype=torch.bool, device=ys[0].device)
        for r, (nm, _, fields) in enumerate(L.fwd.records):
            cap, tot = self.outputs[nm][1], tots[r]
            size = tot if cap is None else cap
            keep = min(tot, size)

            def take(buf, dt):
                o = torch.zeros(size, dtype=dt, device=buf.device)
                o[:keep] = buf[:keep]
                return o
            recs[nm] = {f: take(raw[f"{nm}.{f}"], dt) for f, dt in fields}
            if lanes:
                tans[nm] = {f: torch.stack([take(raw[f"{nm}.{f}#d{l}"], torch.float32) for l in range(lanes)])
                            for f, dt in fields if dt == torch.float32}
            mis = (ys[L.n_results + r] != cnts[r]).sum(dtype=torch.int32)
            st["appended"][nm] = torch.tensor(tot, dtype=torch.int64, device=mis.device)
            st["records_dropped"][nm] = torch.tensor(max(tot - size, 0), dtype=torch.int64, device=mis.device)
            st["records_mismatch"][nm] = mis
            bad = bad | (mis > 0) | (tot > size)
        return recs, tans, st, bad

    def _result(self, L, p, out, raw, fill=None):
        """the Result of a forward launch's outputs (run()'s list; raw: its buffers by name); fill: (counts, totals)
        of a count-then-fill launch"""
        nt = len(p.tallies)
        tallies = {t.name: v for t, v in zip(p.tallies, out[:nt])}
        stats_raw = out[nt]
        ys = out[nt + 1:]
        trunc = ys[p.trunc].bool()
        per = list(ys[:L.n_results])
        n_tr = trunc.sum(dtype=torch.int32)
        stats = {n: stats_raw[i] for i, n in enumerate(B.STATS)}
        stats["n_truncated"] = n_tr
        bad = _limits(p, stats)
        recs = None
        if p.records and fill is not None:
            recs, _, st, over = self._fill_records(L, raw, ys, fill[0], fill[1])
            stats.update(st)
            bad = bad | over
            recs = {nm: _poison_records(rec, over) for nm, rec in recs.items()}
        elif p.records:
            counts = {nm: ys[L.n_results + r] for r, (nm, _, _) in enumerate(p.records)}
            cr = B.canonical_records(p, raw, counts)
            recs = {nm: rec for nm, (rec, _) in cr.items()}
            tots = {nm: tot for nm, (_, tot) in cr.items()}
            stats["appended"] = tots
            stats["records_dropped"] = {nm: torch.clamp(tots[nm] - cap, min=0) for nm, cap, _ in p.records}
            over = any(int(v) > 0 for v in stats["records_dropped"].values())
            bad = bad | over
        outs = _poison(tallies, bad)
        if recs is not None:
            for nm, rec in recs.items():
                outs[nm] = rec if not bool(n_tr > 0) else _poison(rec, n_tr > 0)
        return Result(outs, self._per_item(L, per[:L.n_results]), trunc, stats)

    def grad(self, *args, wrt, cotangents, order=None, n_active=None):
        """d <cotangents, outputs> / d args[wrt] for float32 operand(s) `wrt`: ONE replay launch of the generated
        adjoint.  A broadcast operand's cotangent is summed over the items (exactly); a per-item operand's is per
        item (shape (N,) or (N, n)).  -> one cotangent for one index, a tuple in `wrt`'s order for a tuple (for
        broadcast operands only: a vector, as before); NaN when an item's replay hit max_steps.  A spawning item:
        reverse mode through spawn, the recording forward and one launch per generation (_tree).  Records outputs:
        cotangents[name] = {float field: f32[capacity]} in the canonical layout; a forward launch gives the adjoint
        each item's record count and offset first; NaN when a Records output overflowed its capacity or a replay
        appended a different number of records."""
        L = self.lowered(args)
        if L.it.spawns:
            if order is not None or n_active is not None:
                raise ValueError("tallymap_b200: the tree adjoint of a spawning item takes no claim order or n_active")
            return self._tree(L, args, wrt, cotangents)[1]
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        bidx = [w for w in idx if self.in_axes[w] is None]
        pidx = [w for w in idx if self.in_axes[w] == 0]
        bpos, where = self._bleaves(L, bidx)
        ppos = tuple(sum(1 for ax in self.in_axes[:w] if ax == 0) for w in pidx)
        prog = L.grad_program(bpos, ppos)
        pi, bc = self._split(args)
        n = int((pi[0] if isinstance(pi[0], torch.Tensor) else B._host(pi[0])).shape[0]) if pi else 0
        cts = []
        for name, o in self.outputs.items():
            if o[0] == "records" or o[1] != "f32":
                continue
            c = cotangents.get(name)
            cts.append(torch.zeros(o[0], dtype=torch.float32) if c is None else _f32(c))
        over = False
        if L.fwd.records:
            # (a Records output's cotangents sit at its canonical slots: the adjoint needs each item's record count
            # and offset, so the count pass runs first -- the reference's fill twin reads the primal's counts)
            cnts, offs, tots = self._counts(L, pi, bc, n_active)
            pi = self._with_counts(pi, cnts, offs)
            sizes = {}
            for r, (nm, _, fields) in enumerate(L.fwd.records):
                cap = self.outputs[nm][1]
                sizes[nm] = tots[r] if cap is None else cap
                over = over or (cap is not None and tots[r] > cap)
            for nm, _, fields in L.fwd.records:
                given = cotangents.get(nm) or {}
                for f, dt in fields:
                    if dt == torch.float32:
                        c = given.get(f)
                        cts.append(torch.zeros(sizes[nm], dtype=torch.float32) if c is None else c)
            # (an output without a capacity: its cotangents have the call's total records)
            prog = dataclasses.replace(prog, bc=tuple(
                dataclasses.replace(o, shape=(sizes[o.name[3:].split(".")[0]],))
                if o.name.startswith("ct_") and "." in o.name and o.name[3:].split(".")[0] in sizes else o
                for o in prog.bc))
        out = B.run(prog, pi, list(bc) + cts, consts=(self.max_steps,), order=order,
                    rev_checkpoints=self.opts["rev_checkpoints"], n_active=n_active)
        ct = out[0].reshape(-1)
        ys = out[2:]
        bad = ys[prog.trunc].bool().any() | over
        nan = lambda v: torch.where(bad, torch.full_like(v, float("nan")), v)
        if not pidx:
            return self._per_arg(nan(ct), where, wrt, idx)
        got = {w: nan(ct[q]).reshape(()) if n is None else nan(ct[q:q + n]) for w, (q, n) in where.items()}
        got.update({w: nan(ys[q]) for q, w in enumerate(pidx)})
        return got[wrt] if isinstance(wrt, int) else tuple(got[w] for w in idx)

    def jvp(self, *args, wrt, tangents, n_active=None):
        """forward mode (tallymap's jvp of a mapped call, _api.py:305-345): ONE launch of the generated tangent program.
        wrt: float32 broadcast argument index or tuple of indices, W scalars in all (a broadcast vector counts its n
        elements, in order); tangents: W values (one tangent lane) or an
        array [L, W] (L <= 16 lanes, the reference's dual lanes).  -> (Result, {output name: tangent}), a tangent of
        shape (*output.shape) for one lane, (L, *output.shape) for L lanes; a Records output's tangent is {float
        field: its tangent in the canonical layout, (capacity,) or (L, capacity)}; NaN when an item hit max_steps."""
        from . import lower
        L_ = self.lowered(args)
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        if any(self.in_axes[w] is not None for w in idx):
            raise ValueError("tallymap_b200: tangents of per-item operands are not lowered")
        bpos, _ = self._bleaves(L_, idx)
        tan = torch.as_tensor(np.asarray(tangents, np.float32) if not isinstance(tangents, torch.Tensor)
                              else tangents, dtype=torch.float32)
        lanes_given = tan.dim() == 2
        tan = tan.reshape(-1, len(bpos))
        L = int(tan.shape[0])
        if L > lower.LANES_MAX:
            raise ValueError(f"tallymap_b200: at most {lower.LANES_MAX} tangent lanes per launch")
        prog = L_.jvp_program(bpos, L)
        pi, bc = self._split(args)
        fill = None
        if prog.records and self._fill_needed():
            # count-then-fill: the count pass, then the fill pass with the tangents beside the records
            cnts, offs, tots = self._counts(L_, pi, bc, n_active)
            fill = (cnts, tots)
            prog = self._sized(L_.jvp_fill_program(bpos, L), tots)
            pi = self._with_counts(pi, cnts, offs)
        out = B.run(prog, pi, list(bc) + [tan], consts=(self.max_steps,),
                    queue=self.spawn.capacity if self.spawn else None, n_active=n_active)
        raw = B.run.last["results"]
        nf = len(L_.fwd.tallies)
        nt = len(prog.tallies)
        tallies = {t.name: v for t, v in zip(prog.tallies[:nf], out[:nf])}
        dts = {t.name[2:]: v for t, v in zip(prog.tallies[nf:], out[nf:nt])}
        stats_raw = out[nt]
        ys = out[nt + 1:]
        trunc = ys[prog.trunc].bool()
        per = [y for i, y in enumerate(ys) if i != prog.trunc]
        n_tr = trunc.sum(dtype=torch.int32)
        stats = {n: stats_raw[i] for i, n in enumerate(B.STATS)}
        stats["n_truncated"] = n_tr
        bad = _limits(prog, stats)
        rec_out, rec_t = {}, {}
        if fill is not None:
            rec_out, rec_t, st, over = self._fill_records(L_, raw, ys, fill[0], fill[1], lanes=L)
            stats.update(st)
            bad = bad | over
            rec_out = {nm: _poison_records(rec, over) for nm, rec in rec_out.items()}
        elif prog.records:
            # the records and their fields' tangents in the canonical layout (moved together, _records.py canon);
            # a Records output past its capacity poisons every float output and tangent, as in the forward
            counts = {nm: ys[L_.n_results + r] for r, (nm, _, _) in enumerate(prog.records)}
            recs = B.canonical_records(prog, raw, counts)
            stats["appended"] = {nm: tot for nm, (_, tot) in recs.items()}
            stats["records_dropped"] = {nm: torch.clamp(tot - cap, min=0)
                                        for (nm, cap, _), (_, tot) in zip(prog.records, recs.values())}
            if any(int(v) > 0 for v in stats["records_dropped"].values()):
                bad = bad | True
            for nm, cap, fields in L_.fwd.records:
                rec = recs[nm][0]
                rec_out[nm] = {f: rec[f] for f, _ in fields}
                rec_t[nm] = {f: torch.stack([rec[f"{f}#d{l}"] for l in range(L)]) for f, dt in fields
                             if dt == torch.float32}
        outs = _poison(tallies, bad)
        for nm, rec in rec_out.items():
            outs[nm] = rec if not bool(n_tr > 0) else _poison(rec, n_tr > 0)
        res = Result(outs, self._per_item(L_, per[:L_.n_results]), trunc, stats)
        dts = _poison(dts, bad)
        dts.update({nm: _poison(t, bad) for nm, t in rec_t.items()})
        if not lanes_given:
            dts = {k: ({f: t[0] for f, t in v.items()} if isinstance(v, dict) else v[0]) for k, v in dts.items()}
        return res, dts

    def jacfwd(self, *args, wrt):
        """the Jacobian of every float output w.r.t. the broadcast operands `wrt` by forward mode: one lane per
        operand -> {output name: array (W, *output.shape)}"""
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        W = len(self._bleaves(self.lowered(args), idx)[0])
        _, dts = self.jvp(*args, wrt=idx, tangents=np.eye(W, dtype=np.float32))
        return dts

    def value_and_grad(self, *args, wrt, cotangents, exact_order=False):
        """(Result, gradient).  An item whose loop carries do not depend on `wrt` runs ONE generated one-pass launch
        (each step's VJP summed as the forward runs, oldest step first: the gradient within the float tolerance of
        the replay's); otherwise, or with exact_order=True, the forward launch and the generated replay launch."""
        dev = torch.device("cuda", torch.cuda.current_device())
        moved = [(a if isinstance(a, torch.Tensor) else torch.from_numpy(B._host(a))).to(dev, non_blocking=True)
                 if ax == 0 else a for a, ax in zip(args, self.in_axes)]
        if not exact_order:
            L = self.lowered(moved)
            idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
            if all(self.in_axes[w] is None for w in idx):
                bpos, where = self._bleaves(L, idx)
                prog = L.vg_program(bpos)
                if prog is not None:
                    res, ct = self._onepass(L, prog, moved, (), cotangents)
                    return res, self._per_arg(ct, where, wrt, idx)
        L = self.lowered(moved)
        if L.it.spawns:
            return self._tree(L, moved, wrt, cotangents)
        return self(*moved), self.grad(*moved, wrt=wrt, cotangents=cotangents)

    def _tree(self, L, args, wrt, cotangents):
        """(Result, gradient) of a spawning item by reverse mode through spawn (tallymap/_reverse_spawn.py:233-336):
        the recording forward (its outputs are the Result), then one adjoint launch per generation, deepest first,
        and one over the roots (backend.tree_record, backend.tree_adjoint).  Differentiable: float32 broadcast
        operands (their cotangents summed over every particle, exactly) and the roots' float32 per-item operands (a
        cotangent per root).  Every gradient is NaN when the record is incomplete (a child dropped or beyond the
        record's capacity, a tree deeper than backend.TREE_MAX_GEN generations), when a replay disagrees with the
        record, or when a particle hit max_steps.  The counters of the last call: self.last_tree.  (With
        cuda_math='fast' the recording and the adjoint kernels may contract multiply-adds differently, so a replay
        can disagree with the record: a NaN gradient, never a wrong one.)"""
        from . import lower
        idx = (wrt,) if isinstance(wrt, int) else tuple(wrt)
        bidx = [w for w in idx if self.in_axes[w] is None]
        pidx = [w for w in idx if self.in_axes[w] == 0]
        bpos, where = self._bleaves(L, bidx)
        fo = lower._float_operands(L.it)
        ppos = [sum(1 for ax in self.in_axes[:w] if ax == 0) for w in pidx]
        for w, q in zip(pidx, ppos):
            if q not in fo:
                raise lower.LowerError(f"tallymap_b200: argument {w} is not a float32 per-item operand (no cotangent)")
        adj = L.tree_program(bpos)
        rec = L.rec_program()
        pi, bc = self._split(args)
        t = B.tree_record(rec, pi, bc, max_steps=self.max_steps, queue=self.spawn.capacity if self.spawn else None)
        cts = []
        for name, o in self.outputs.items():
            if o[1] != "f32":
                continue
            c = cotangents.get(name)
            cts.append(torch.zeros(o[0], dtype=torch.float32) if c is None else _f32(c))
        r = B.tree_adjoint(adj, t, cts, max_steps=self.max_steps, rev_checkpoints=self.opts["rev_checkpoints"])
        self.last_tree = r["info"]
        out = t["forward"]
        res = self._result(L, rec, out[:len(out) - 1], t["results"])     # (without the roots' newest child)
        bad = r["poisoned"]
        nan = lambda v: torch.where(bad, torch.full_like(v, float("nan")), v)
        ct = r["g"].reshape(-1)
        got = {w: nan(ct[q]).reshape(()) if n is None else nan(ct[q:q + n]) for w, (q, n) in where.items()}
        got.update({w: nan(r["ct_in"][fo.index(q)]) for w, q in zip(pidx, ppos)})
        return res, (got[wrt] if isinstance(wrt, int) else tuple(got[w] for w in idx))

    def _onepass(self, L, prog, args, wrt, cotangents):
        pi, bc = self._split(args)
        cts = []
        for name, o in self.outputs.items():
            if o[0] == "records" or o[1] != "f32":
                continue
            c = cotangents.get(name)
            cts.append(torch.zeros(o[0], dtype=torch.float32) if c is None else _f32(c))
        out = B.run(prog, pi, list(bc) + cts, consts=(self.max_steps,),
                    queue=self.spawn.capacity if self.spawn else None)
        nt = len(L.fwd.tallies)
        tallies = {t.name: v for t, v in zip(L.fwd.tallies, out[:nt])}
        ct = out[nt].reshape(-1)
        stats_raw = out[nt + 1]
        ys = out[nt + 2:]
        trunc = ys[prog.trunc].bool()
        per = list(ys[:L.n_results])
        n_tr = trunc.sum(dtype=torch.int32)
        stats = {n: stats_raw[i] for i, n in enumerate(B.STATS)}
        stats["n_truncated"] = n_tr
        bad = _limits(prog, stats)
        res = Result(_poison(tallies, bad), self._per_item(L, per[:L.n_results]), trunc, stats)
        ct = torch.where(bad, torch.full_like(ct, float("nan")), ct)
        return res, (ct.reshape(()) if isinstance(wrt, int) else ct)


OPTIONS = ("cuda_math", "schedule", "min_blocks_per_sm", "xla_batch_size", "rev_checkpoints", "rev_stats")
BC_VECTOR_MAX = 64      # a broadcast vector of at most this many elements is lowered as that many broadcast scalars
BACKENDS = ("auto", "xla")


def options(backend="auto", **opts):
    """the call options of tallymap.vmap (_api.py:414-425, 493-507), validated -> dict(math, schedule, min_blocks,
    rev_checkpoints).
      cuda_math          'ieee' (this backend's default: correctly rounded f32 division and square root, bitwise
                         against the CPU evaluator and across GPU counts) | 'approx' (the reference's default:
                         div.full / sqrt.approx) | 'fast' (approx plus FMA contraction of float multiply-adds;
                         statistical only).  Lowered items only: the built-in families are compiled ahead of time
                         with 'ieee'
      schedule           'item' | 'step': both run this runtime's step-granular refill (a warp runs the item loop
                         while every lane steps and refills a lane whose item ended); 'step' also demands an item
                         with exactly one top-level while loop, as the reference's does
      min_blocks_per_sm  None | N in 1..32: the lowered entry point's __launch_bounds__(block, N)
      rev_checkpoints    'auto' (default) | C >= 1: the replay adjoint's states per checkpoint buffer
      rev_stats          accepted; the tree adjoint's counters are always kept (Mapped.last_tree)
      xla_batch_size     accepted for the reference's xla backend, which this build does not have
    backend: 'auto' (the kernel backend) | 'xla' (the reference's plain-JAX interpreter: UnsupportedError here)"""
    from . import lower
    bad = sorted(set(opts) - set(OPTIONS))
    if bad:
        raise ValueError(f"tallymap_b200: unknown option(s) {bad}; options are {', '.join(OPTIONS)}")
    if backend not in BACKENDS:
        raise ValueError(f"tallymap_b200: unknown backend {backend!r}; backends are {', '.join(BACKENDS)}")
    if backend == "xla":
        raise UnsupportedError("tallymap_b200: backend='xla' is the reference's plain-JAX interpreter, which needs "
                               "JAX; this package is the kernel backend (backend='auto')")
    math = opts.get("cuda_math") or "ieee"
    if math not in lower.MATH_MODES:
        raise ValueError(f"tallymap_b200: cuda_math must be 'ieee', 'approx' or 'fast', got {math!r}")
    schedule = opts.get("schedule", "item")
    if schedule not in ("item", "step"):
        raise ValueError(f"tallymap_b200: schedule must be 'item' or 'step', got {schedule!r}")
    mb = opts.get("min_blocks_per_sm")
    if mb is not None and (isinstance(mb, bool) or not isinstance(mb, (int, np.integer)) or not 1 <= int(mb) <= 32):
        raise ValueError(f"tallymap_b200: min_blocks_per_sm must be None or an integer in 1..32, got {mb!r}")
    rc = opts.get("rev_checkpoints", "auto")
    if rc == "auto" or rc is None:
        rc = None
    elif isinstance(rc, bool) or not isinstance(rc, (int, np.integer)) or int(rc) < 1:
        raise ValueError(f"tallymap_b200: rev_checkpoints must be 'auto' or an integer >= 1, got {rc!r}")
    return dict(math=math, schedule=schedule, min_blocks=None if mb is None else int(mb),
                rev_checkpoints=None if rc is None else int(rc))


def vmap(fn=None, *, outputs, in_axes=0, max_steps=None, spawn=None, backend="auto", **opts):
    """tallymap.vmap (_api.py:428-507): `fn` is a Python function written against tallymap_b200.lang (traced,
    lowered and compiled on first call) or the name of a built-in lowered family ("quickstart", "walk1d", "photon",
    "lorenz", "shower"); with fn=None, a decorator.  in_axes: 0 (every argument per item), or 0 / None per argument.
    spawn: a Queue, for an item that spawns children with t.spawn (_api.py:88-98, 426-433).  opts: see options()."""
    if fn is None:
        return lambda f: vmap(f, outputs=outputs, in_axes=in_axes, max_steps=max_steps, spawn=spawn,
                              backend=backend, **opts)
    o = options(backend, **opts)
    # a bare shape stands for Sum(shape) (_api.py:509)
    outputs = {k: (v if isinstance(v, (Sum, Records)) else Sum(v)) for k, v in outputs.items()}
    if callable(fn) and not isinstance(fn, Family):
        return MappedFn(fn, outputs, in_axes, max_steps, spawn, o)
    fam = FAMILIES[fn] if isinstance(fn, str) else fn
    if o["math"] != "ieee" or o["min_blocks"] is not None:
        raise UnsupportedError(f"tallymap_b200: the built-in item {fam.name!r} is compiled ahead of time with "
                               "cuda_math='ieee' and its own launch bounds (cuda_math / min_blocks_per_sm apply to "
                               "lowered items)")
    return Mapped(fam, outputs, fam.in_axes if in_axes == 0 else in_axes, max_steps, spawn, o)
