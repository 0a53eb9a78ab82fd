"""The kernel-backend driver: `run(p, pi, bc, ...)`, the B200 counterpart of the reference's KB.run
(tallymap/backends/kernel/__init__.py:135-185), and the item programs it can launch.

An ItemProgram here describes one lowered item program and its buffer layout.  `run` marshals the operands the way
KB.run does -- [per-item operands] [broadcast operands] [hoisted constants] -- allocates the results
[sum tallies] [scratch accumulators] [control words] [stats int32[5]] [per-item results], lets the launcher zero the
first n_zero of them, launches through the C ABI on the current CUDA stream, and returns, in the reference's output
order (backends/kernel/__init__.py:177-185, _primitive._abstract): [sum tallies] + [stats] + [per-item results].
Keys enter as uint32[..., 2] key data (__init__.py:131-132).

Also here: replay_plan (the replay's checkpoint count C, sized from device memory), tree_grad (reverse mode through
spawn: the recording forward, the generation lists and one adjoint launch per generation) and canonical_records (the
Records layout after a launch).

Everything runs on the GPU through libtm_b200.so; there is no CPU path.  Device memory and streams come from torch.
"""
import ctypes
import dataclasses
from typing import Tuple

import numpy as np
import torch

from . import _lib

STATS = ("spawned", "children_dropped", "children_truncated", "fixed_point_overflow", "dropped_emits")
CTL_WORDS = 8
EXACT_WORDS = 5
QCTL_WORDS = 6 * 32         # the spawn ring's control words, one 128-byte line each
QUEUE_DEFAULT = 1 << 22     # ring slots of a spawning program (64 MiB of leaves for the shower)


@dataclasses.dataclass(frozen=True)
class TSpec:
    """a Sum tally of the program (tallymap/_api.py:204-220): flat size S, dtype; exact: the f32 sum is kept as 5
    carry-save int64 words per bin (a scratch buffer) and read out correctly rounded."""
    name: str
    shape: Tuple[int, ...]
    dtype: torch.dtype = torch.float32
    exact: bool = False
    f64: bool = False      # accumulated in an f64 shadow (a scratch result), rounded once to the f32 output
    wide: float = 0.0      # nonzero: a scaled fixed-point sum of this scale (lo / carry / flag words per bin)

    def dims(self, N=None):
        """the shape with a leading "N" (a tally indexed by item id) resolved to the launch's item count"""
        return tuple(N if d == "N" else d for d in self.shape)

    def size(self, N=None):
        return int(np.prod(self.dims(N), dtype=np.int64)) if self.shape else 1

    @property
    def S(self):
        return self.size()


@dataclasses.dataclass(frozen=True)
class Operand:
    name: str
    shape: Tuple[int, ...]          # per-item operands: the shape of ONE item's value
    dtype: torch.dtype


@dataclasses.dataclass(frozen=True)
class ItemProgram:
    """one lowered program: its kernel and its operand / result layout.
    pi: per-item operands; bc: broadcast operands (for an adjoint: then the output cotangents); consts: hoisted
    int32 constants (max_steps); tallies: sum outputs; ys: per-item results; trunc: index of the truncation flag in
    ys (None: no max_steps cap); grad_of: for an adjoint, the (forward program name, broadcast operand index) it
    differentiates."""
    name: str
    kernel: str
    pi: Tuple[Operand, ...]
    bc: Tuple[Operand, ...]
    consts: Tuple[str, ...]
    tallies: Tuple[TSpec, ...]
    ys: Tuple[Operand, ...]
    trunc: int = None
    spawns: bool = False
    replay_state_bytes: int = 0     # an adjoint: bytes of one stored loop state in its replay scratch
    queue_leaf_bytes: int = 0       # a spawning program: bytes of one child's leaves in the ring
    record_bytes: int = 0           # a recording spawning program: bytes of one child's record (tree adjoint)
    buffers: int = 0                # nonzero: launched by its own driver with this many buffers (not by run())
    vg_fallback: str = None         # a pipelined value-and-grad program: its kernel needs C >= max_steps (two heads
                                    # per thread); with a smaller C the launch uses this fused replay kernel instead
    records: tuple = ()             # Records outputs: ((name, capacity, ((field, torch dtype), ...)), ...)
    records_fill: bool = False      # the fill pass of count-then-fill: records go straight to their canonical slots
                                    # (offset + k from per-item operands), so the fields alone, sized by `capacity`
    claims: int = 0                 # Records slot claims of a reference jaxpr (tallymap_claim): one u64 launch counter
                                    # per tally (zeroed), after the Records buffers

    @property
    def n_args(self):
        return len(self.pi) + len(self.bc) + 2     # + hoisted constants + the optional claim order

    def result_layout(self, N, replay_bytes=0, queue=0, record=0):
        """[(name, nbytes, torch dtype, shape)] of the results, in buffer order, and n_zero.  An adjoint's replay
        scratch (replay_bytes, from replay_plan) comes last and is not zeroed; a spawning program's ring of `queue`
        slots: its sequence and control words are zeroed (an empty ring), its leaves come last, not zeroed; a
        recording program's tree counters are zeroed and its `record` slots come after the ring, not zeroed."""
        out = []
        for t in self.tallies:
            out.append((t.name, t.size(N) * _itemsize(t.dtype), t.dtype, t.dims(N)))
        for t in self.tallies:
            S = t.size(N)
            if t.f64:
                out.append((t.name + ".f64", S * 8, torch.float64, (S,)))
            if t.exact:
                # EXACT_WORDS int64 words per bin, then one u32 flag word per bin (rounded up to whole u64s)
                n64 = S * EXACT_WORDS + (S + 1) // 2
                out.append((t.name + ".exact", n64 * 8, torch.int64, (n64,)))
            if t.wide:
                # per bin: an int64 low word, then an i32 carry and a u32 flag (csrc/tm_tally.cuh WideSum)
                out.append((t.name + ".wide", S * 16, torch.int64, (2 * S,)))
        for name, cap, fields in self.records:
            # the raw records (a slot per append, in claim order), their keys (item, ordinal) and the slot counter;
            # a fill pass: the fields alone, in the canonical layout
            for f, dt in fields:
                out.append((f"{name}.{f}", cap * 4, dt, (cap,)))
            if self.records_fill:
                continue
            # (internal buffers are named with '#': a field may be called 'k')
            out.append((f"{name}#cid", cap * 4, torch.int32, (cap,)))
            out.append((f"{name}#k", cap * 4, torch.int32, (cap,)))
            out.append((f"{name}#ctr", 8, torch.int64, (1,)))
        if self.claims:
            out.append(("claims", 8 * self.claims, torch.int64, (self.claims,)))
        if self.queue_leaf_bytes:
            out.append(("queue.seq", max(queue, 1) * 4, torch.int32, (max(queue, 1),)))
            out.append(("queue.ctl", QCTL_WORDS * 4, torch.int32, (QCTL_WORDS,)))
        out.append(("ctl", CTL_WORDS * 4, torch.int32, (CTL_WORDS,)))
        out.append(("stats", len(STATS) * 4, torch.int32, (len(STATS),)))
        if self.record_bytes:
            out.append(("tree", 4 * 8, torch.int64, (4,)))
        n_zero = len(out)
        for y in self.ys:
            out.append((y.name, N * int(np.prod(y.shape, dtype=np.int64)) * _itemsize(y.dtype), y.dtype,
                        (N,) + tuple(y.shape)))
        if self.replay_state_bytes:
            n = max(1, (replay_bytes + 15) // 16)
            out.append(("replay", n * 16, torch.int32, (n * 4,)))
        if self.queue_leaf_bytes:
            n = max(queue, 1) * self.queue_leaf_bytes // 4
            out.append(("queue.ring", n * 4, torch.int32, (n,)))
        if self.record_bytes:
            n = max(record, 1) * self.record_bytes // 4
            out.append(("record", n * 4, torch.int32, (n,)))
            out.append(("record.gen", max(record, 1) * 2, torch.int16, (max(record, 1),)))
        return out, n_zero


_LAYOUTS = {}


def _layout(p, N, replay_bytes, queue, record):
    """p.result_layout, remembered per (program, sizes): it is a pure function of them, and a launch-bound call
    (small N) otherwise spends a large part of its host time recomputing it"""
    key = (id(p), int(N), int(replay_bytes), int(queue), int(record))
    hit = _LAYOUTS.get(key)
    if hit is None or hit[0] is not p:
        if len(_LAYOUTS) > 4096:
            _LAYOUTS.clear()
        hit = (p, p.result_layout(N, replay_bytes, queue, record))   # (p kept alive: its id stays its own)
        _LAYOUTS[key] = hit
    return hit[1]


def _itemsize(dt):
    return torch.empty((), dtype=dt).element_size()


def canonical_records(p, results, counts):
    """the reference's one-pass Records layout (tallymap/_records.py:35-62 canon): record k of item i moves from its
    raw slot to slot offset[i] + k, offset the exclusive prefix sum of the per-item counts of the same launch; slots
    past the last record are zero.  results: the launch's buffers by name; counts: name -> int32[N].
    -> {name: ({field: tensor[capacity]}, total appended)}; a total beyond the capacity poisons (float fields NaN,
    integer fields -1), as a full Queue does"""
    out = {}
    for name, cap, fields in p.records:
        cnt = counts[name].to(torch.int64)
        total = cnt.sum()
        off = torch.cumsum(cnt, 0) - cnt
        n = int(min(int(total), cap))
        cid = results[f"{name}#cid"][:n].to(torch.int64)
        pos = off[cid] + results[f"{name}#k"][:n].to(torch.int64) if n else cid
        keep = pos < cap
        over = int(total) > cap
        rec = {}
        for f, dt in fields:
            o = torch.zeros(cap, dtype=dt, device=cnt.device)
            if n:
                o[pos[keep]] = results[f"{name}.{f}"][:n][keep]
            if over:
                o.fill_(float("nan") if dt.is_floating_point else -1)
            rec[f] = o
        out[name] = (rec, total)
    return out


_U32 = torch.int32   # uint32 key data travels as int32 bits (torch has no full uint32 arithmetic; bits only)

# -------------------------------------------------------------------------------------------------- programs
# The benchmark items (benchmark configurations 1 and 2), forward and reverse.  Buffer layouts: csrc/items_walks.cuh.
_F32 = torch.float32
KEY = Operand("key", (2,), _U32)

Q1_FWD = ItemProgram("q1_fwd", "q1_fwd", pi=(Operand("x", (), _F32), KEY), bc=(Operand("theta", (), _F32),),
                     consts=("max_steps",), tallies=(TSpec("hist", (16,)),),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8)), trunc=1)
Q1_GRAD = ItemProgram("q1_grad", "q1_grad", pi=(Operand("x", (), _F32), KEY),
                      bc=(Operand("theta", (), _F32), Operand("ct_hist", (16,), _F32)),
                      consts=("max_steps", "rev_checkpoints", "replay_threads"),
                      tallies=(TSpec("ct_theta", (1,), exact=True),),
                      ys=(Operand("truncated", (), torch.uint8),), trunc=0, replay_state_bytes=4)
RW_FWD = ItemProgram("rw_fwd", "rw_fwd", pi=(Operand("x", (), _F32), KEY), bc=(Operand("drift", (), _F32),),
                     consts=("max_steps",), tallies=(TSpec("hist", (256,)), TSpec("side", (2,))),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8)), trunc=1)
RW_GRAD = ItemProgram("rw_grad", "rw_grad", pi=(Operand("x", (), _F32), KEY),
                      bc=(Operand("drift", (), _F32), Operand("ct_hist", (256,), _F32), Operand("ct_side", (2,), _F32)),
                      consts=("max_steps", "rev_checkpoints", "replay_threads"),
                      tallies=(TSpec("ct_drift", (1,), exact=True),),
                      ys=(Operand("truncated", (), torch.uint8),), trunc=0, replay_state_bytes=4)

# value and gradient in one launch (FusedVG: the replay's count pass is the forward pass, emitting its tallies), for
# cotangents given up front: the forward's tallies, then the gradient's exact tally; the forward's per-item results
Q1_VG = ItemProgram("q1_vg", "q1_vg", pi=Q1_GRAD.pi, bc=Q1_GRAD.bc, consts=Q1_GRAD.consts,
                    tallies=Q1_FWD.tallies + Q1_GRAD.tallies, ys=Q1_FWD.ys, trunc=1, replay_state_bytes=4,
                    vg_fallback="q1_vg_replay")
RW_VG = ItemProgram("rw_vg", "rw_vg", pi=RW_GRAD.pi, bc=RW_GRAD.bc, consts=RW_GRAD.consts,
                    tallies=RW_FWD.tallies + RW_GRAD.tallies, ys=RW_FWD.ys, trunc=1, replay_state_bytes=4,
                    vg_fallback="rw_vg_replay")
# the one-pass value and grad (OnePassVG: items with no active carry sum each step's VJP as the forward runs; the
# per-item cotangent is summed oldest step first, so the gradient equals the reverse program's within the float
# tolerance, not bitwise): the fused layouts without the replay scratch
Q1_VG1 = ItemProgram("q1_vg_onepass", "q1_vg_onepass", pi=Q1_GRAD.pi, bc=Q1_GRAD.bc, consts=("max_steps",),
                     tallies=Q1_FWD.tallies + Q1_GRAD.tallies, ys=Q1_FWD.ys, trunc=1)
RW_VG1 = ItemProgram("rw_vg_onepass", "rw_vg_onepass", pi=RW_GRAD.pi, bc=RW_GRAD.bc, consts=("max_steps",),
                     tallies=RW_FWD.tallies + RW_GRAD.tallies, ys=RW_FWD.ys, trunc=1)

# benchmark configuration 3, the photon slab (csrc/items_photon.cuh)
PH_FWD = ItemProgram("ph_fwd", "ph_fwd", pi=(KEY,), bc=(Operand("mu_a", (), _F32), Operand("mu_s", (), _F32)),
                     consts=("max_steps",), tallies=(TSpec("dep", (64, 64, 64)),),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8)), trunc=1)
PH_GRAD = ItemProgram("ph_grad", "ph_grad", pi=(KEY,),
                      bc=(Operand("mu_a", (), _F32), Operand("mu_s", (), _F32), Operand("ct_dep", (64, 64, 64), _F32)),
                      consts=("max_steps", "rev_checkpoints", "replay_threads"),
                      tallies=(TSpec("ct_mu", (2,), exact=True),),
                      ys=(Operand("truncated", (), torch.uint8),), trunc=0, replay_state_bytes=32)

# benchmark configuration 4, the Lorenz RK45 ensemble (csrc/items_ode.cuh); "bins3": the final tally's 3N bins
OD_PI = (Operand("sigma", (), _F32), Operand("rho", (), _F32), Operand("y0", (3,), _F32),
         Operand("item_id", (), torch.int32))
OD_FWD = ItemProgram("od_fwd", "od_fwd", pi=OD_PI, bc=(Operand("beta", (), _F32),), consts=("max_steps", "bins3"),
                     tallies=(TSpec("final", ("N", 3)), TSpec("mean_z", ())),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8)), trunc=1)
OD_GRAD = ItemProgram("od_grad", "od_grad", pi=OD_PI,
                      bc=(Operand("beta", (), _F32), Operand("ct_final", ("N", 3), _F32), Operand("ct_mean", (), _F32)),
                      consts=("max_steps", "rev_checkpoints", "replay_threads", "bins3"),
                      tallies=(TSpec("ct_beta", (1,), exact=True),),
                      ys=(Operand("truncated", (), torch.uint8),), trunc=0, replay_state_bytes=32)
# the Lorenz ensemble's value and grad w.r.t. beta in one forward pass by forward mode (the tangents of y and k1
# carried with the state; csrc/items_ode.cuh ODVG1): within the float tolerance of the replay's gradient
OD_VG1 = ItemProgram("od_vg_onepass", "od_vg_onepass", pi=OD_PI, bc=OD_GRAD.bc, consts=("max_steps", "bins3"),
                     tallies=OD_FWD.tallies + OD_GRAD.tallies, ys=OD_FWD.ys, trunc=1)

# benchmark configuration 5, the branching shower (csrc/items_shower.cuh): a spawning program with a ring of Q slots
SH_FWD = ItemProgram("sh_fwd", "sh_fwd", pi=(Operand("E", (), _F32), Operand("depth", (), _F32), KEY),
                     bc=(Operand("X0", (), _F32),), consts=("max_steps", "queue"),
                     tallies=(TSpec("dep", (512,)), TSpec("count", (1,), torch.int32)),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8)), trunc=1, spawns=True,
                     queue_leaf_bytes=16)

# its reverse mode (the tree adjoint): the recording forward (the forward's outputs plus every child's record and
# each root's newest child) and the per-generation adjoint, launched by tree_grad
SH_PI = (Operand("E", (), _F32), Operand("depth", (), _F32), KEY)
# the shower's value and gradient w.r.t. the roots' E0 in one spawn launch, by forward mode through spawn (each particle
# carries d E / d E0 of its root; csrc/items_shower.cuh SHVG1): per-root exact sums, read out by sh_value_and_grad
SH_VG1 = ItemProgram("sh_vg_onepass", "sh_vg_onepass", pi=SH_PI,
                     bc=(Operand("X0", (), _F32), Operand("ct_dep", (512,), _F32)), consts=("max_steps", "queue", "items"),
                     tallies=(TSpec("dep", (512,)), TSpec("count", (1,), torch.int32), TSpec("g_E", ("N",), exact=True),
                              TSpec("steps", (1,), torch.int64)),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8)), trunc=1, spawns=True,
                     queue_leaf_bytes=24)
SH_REC = ItemProgram("sh_rec", "sh_rec", pi=SH_PI, bc=(Operand("X0", (), _F32),), consts=("max_steps", "queue", "record"),
                     tallies=(TSpec("dep", (512,)), TSpec("count", (1,), torch.int32)),
                     ys=(Operand("k", (), torch.int32), Operand("truncated", (), torch.uint8),
                         Operand("last", (), torch.int32)), trunc=1, spawns=True, queue_leaf_bytes=24,
                     record_bytes=32)
SH_GRAD = ItemProgram("sh_grad", "sh_grad", pi=SH_PI,
                      bc=(Operand("X0", (), _F32), Operand("ct_dep", (512,), _F32)),
                      consts=("max_steps", "rev_checkpoints", "replay_threads", "roots", "record"),
                      tallies=(TSpec("ct_X0", (1,), exact=True),), ys=(), replay_state_bytes=4, buffers=18)

# the photon's value and grad in one forward pass by forward mode (w's tangent w.r.t. albedo carried with the state;
# csrc/items_photon.cuh PHVG1): within the float tolerance of the replay's gradient
PH_VG1 = ItemProgram("ph_vg_onepass", "ph_vg_onepass", pi=PH_GRAD.pi, bc=PH_GRAD.bc, consts=("max_steps",),
                     tallies=PH_FWD.tallies + PH_GRAD.tallies, ys=PH_FWD.ys, trunc=1)

PROGRAMS = {p.name: p for p in (Q1_FWD, Q1_GRAD, Q1_VG, Q1_VG1, RW_FWD, RW_GRAD, RW_VG, RW_VG1, PH_FWD, PH_GRAD, PH_VG1,
                                OD_FWD, OD_GRAD, SH_FWD, SH_REC, SH_GRAD, SH_VG1)}


# -------------------------------------------------------------------------------------------------- run
COMPILED = {}      # kernel id of a program compiled at run time (tallymap_b200.lower) -> its buffer count


def kernel_ref(kernel):
    """(kernel id, buffer count) of a built-in kernel name or of a run-time compiled kernel id"""
    if isinstance(kernel, int):
        if kernel not in COMPILED:
            raise _lib.TallymapError(f"tallymap_b200: kernel id {kernel} was not compiled in this process")
        return kernel, COMPILED[kernel]
    return _lib.kernel_id(kernel)


def _host(x):
    """a numpy operand as a contiguous array torch accepts (uint32 key data travels as int32 bits)"""
    a = np.asarray(x)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return a if a.flags.c_contiguous else np.ascontiguousarray(a)    # (ascontiguousarray makes 0-d arrays 1-d)


def _dev(x, device, dtype):
    if isinstance(x, torch.Tensor):
        t = x
    else:
        t = torch.from_numpy(_host(x))
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.to(device, non_blocking=True).contiguous()


# The replay's checkpoint count C (the reference's rev_checkpoints option, tallymap/_reverse.py:116-134).  Any C gives
# bitwise the same cotangents; C only trades memory for replay work.  The reference picks C from the logical state
# size (16 for small steps, a 64 KiB budget per thread) and notes that the right rule sizes C against device memory;
# here, with HBM to spare: C = max_steps when every resident thread's head of max_steps + 1 states fits in
# REV_BUDGET_FRACTION of the free device memory (no item then needs a checkpoint pass or a refill: the replay is
# one forward evaluation and one VJP per step), else the largest power of two up to REV_C_POW2_MAX whose 3C + 1
# states per thread fit.
REV_BUDGET_FRACTION = 0.2
REV_C_MIN = 16
REV_C_POW2_MAX = 4096      # (the checkpointed fallback: beyond this C the replay's refill work is < 2% of K)


_PLANS = {}


def replay_plan(p, max_steps, rev_checkpoints=None, device=None):
    """-> (C, threads, scratch bytes) of adjoint program p's replay on the current device (decided once per program,
    device, max_steps and option, so repeated launches keep their C and reuse their buffers)."""
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    # (keyed by the kernel and its state size, not the program's name: lowered items of the same name, or one item's
    # programs for different operands, are different kernels whose resident threads and scratch differ)
    key = (p.kernel, p.replay_state_bytes, p.vg_fallback, dev, int(max_steps), rev_checkpoints)
    if key not in _PLANS:
        _PLANS[key] = _replay_plan(p, max_steps, rev_checkpoints, device)
    return _PLANS[key]


def replay_scratch_states(C, max_steps, pipelined=False):
    """compact states per thread of the replay scratch: the head alone when C >= max_steps (for a pipelined
    value-and-grad kernel: its ring tape of C + 1 states), else head + checkpoints + tape (the replay kernel's
    layout)"""
    if C >= max_steps:
        return C + 1
    return 3 * C + 1


def pipelined(p, max_steps, device=None):
    """whether fused value-and-grad program p runs its pipelined kernel at max_steps on this device (its ring tape of
    every resident thread fits), rather than the fused checkpointed replay, which is slower than a forward launch and
    a replay launch (a warp pays for its counting and its sweeping lanes at once)"""
    if p.vg_fallback is None:
        return False
    C = replay_plan(p, max_steps, None, device)[0]
    return C + 1 == ring_states(max_steps)


def ring_states(max_steps):
    """the ring tape of a pipelined value-and-grad kernel: the smallest power of two >= max_steps + 2 states"""
    T = 1
    while T < int(max_steps) + 2:
        T *= 2
    return T


def _replay_plan(p, max_steps, rev_checkpoints, device):
    kid, _ = kernel_ref(p.kernel)
    info = _lib.kernel_info(kid)
    threads = info["sms"] * info["blocks_per_sm"] * info["block"]
    M = int(max_steps)
    per = lambda C: replay_scratch_states(C, M, p.vg_fallback is not None) * p.replay_state_bytes
    if rev_checkpoints is not None:
        C = int(rev_checkpoints)
        if C < 1:
            raise ValueError("tallymap_b200: rev_checkpoints must be >= 1")
    else:
        torch.cuda.empty_cache()             # (blocks cached by earlier calls count as free)
        free, _ = torch.cuda.mem_get_info(device)
        budget = REV_BUDGET_FRACTION * free
        pipelined = p.vg_fallback is not None
        Ch = ring_states(M) - 1 if pipelined and M <= 2 ** 29 else M
        if M <= 2 ** 29 and threads * per(Ch) <= budget:
            C = max(Ch, 1)
        else:
            C = REV_C_MIN
            while C * 2 < M and C * 2 <= REV_C_POW2_MAX and threads * per(C * 2) <= budget:
                C *= 2
    return C, threads, threads * per(C)


def run(p, pi, bc, consts=(), target="cuda", ndev=1, stream=None, out=None, rev_checkpoints=None, order=None,
        queue=None, record=None, n_active=None, **_):
    """Launch program `p` over the items of `pi` (per-item operands, leading axis N) with broadcast operands `bc`
    and hoisted int32 constants `consts` (max_steps).  -> [sum tallies] + [stats int32[5]] + [per-item results]
    as torch tensors on the current CUDA device, and the raw control words as the attribute-free last element
    of `run.last` (for tm_check_status).  target must be 'cuda' (no CPU fallback, as the reference's kernel
    backend never falls back: _primitive.py:189-194).  out: optional preallocated result buffers (as returned by
    alloc_results), reused without reallocation.  order: optional int32[N] permutation, the order in which the
    kernel's threads claim items (e.g. longest first, from a primal call's trip counts); it changes no result.
    n_active: optional item count <= N (the reference's n_active, _api.py:466-469): only items i < n_active run; the
    others emit nothing, are never truncated and their per-item results are zero (the launch zeroes them); refused
    for a spawning program, as the reference refuses it (_api.py:530-532: a child's item index would reach beyond
    the active count)."""
    if n_active is not None and p.spawns:
        raise ValueError("tallymap: n_active with spawn is not supported")
    if target != "cuda":
        raise NotImplementedError("tallymap_b200 runs on CUDA devices only (no CPU fallback)")
    if not torch.cuda.is_available():
        raise RuntimeError("tallymap_b200: no CUDA device")
    dev = torch.device("cuda", torch.cuda.current_device())
    if len(pi) != len(p.pi) or len(bc) != len(p.bc):
        raise TypeError(f"{p.name}: expected {len(p.pi)} per-item and {len(p.bc)} broadcast operands, "
                        f"got {len(pi)} and {len(bc)}")
    args = [_dev(x, dev, o.dtype) for x, o in zip(pi, p.pi)]
    N = int(args[0].shape[0]) if args else 0
    for a, o in zip(args, p.pi):
        if tuple(a.shape) != (N,) + tuple(o.shape):
            raise TypeError(f"{p.name}: per-item operand {o.name} has shape {tuple(a.shape)}, expected "
                            f"{(N,) + tuple(o.shape)}")
    if N > 2 ** 31 - 1:
        raise ValueError("tallymap_b200: at most 2^31 - 1 items per call (tallymap/_api.py:540-542)")
    for x, o in zip(bc, p.bc):
        t = _dev(x, dev, o.dtype)
        want = tuple(N if d == "N" else d for d in o.shape)
        if tuple(t.shape) != want:
            raise TypeError(f"{p.name}: broadcast operand {o.name} has shape {tuple(t.shape)}, expected {want}")
        args.append(t)
    replay_bytes = 0
    Q = int(queue or QUEUE_DEFAULT) if p.queue_leaf_bytes else 0
    R = record_capacity(N, record, dev, record_slot_bytes(p)) if p.record_bytes else 0
    known = {"max_steps": int(consts[0]) if consts else 0, "bins3": 3 * N, "queue": Q, "record": R, "items": N}
    if p.replay_state_bytes:
        C, threads, replay_bytes = replay_plan(p, known["max_steps"], rev_checkpoints, dev)
        known.update(rev_checkpoints=C, replay_threads=threads)
    consts = tuple(known[c] for c in p.consts)
    args.append(_consts(consts or (0,), dev))
    n_items = N
    if n_active is not None:
        n_items = int(n_active)
        if not 0 <= n_items <= N:
            raise ValueError(f"{p.name}: n_active must be in [0, {N}], got {n_active}")
        if order is not None:
            raise ValueError(f"{p.name}: a claim order and n_active together are not supported")
    if order is not None:
        order = _dev(order, dev, torch.int32)
        if tuple(order.shape) != (N,):
            raise TypeError(f"{p.name}: order has shape {tuple(order.shape)}, expected {(N,)}")
    args.append(order)
    layout, n_zero = _layout(p, N, replay_bytes, Q, R)
    res = out if out is not None else alloc_results(p, N, dev, replay_bytes, Q, R)
    if any(t.numel() * t.element_size() < nb for t, (_, nb, _, _) in zip(res, layout)):
        raise ValueError(f"{p.name}: preallocated results are smaller than the launch needs")
    kernel = p.kernel
    if p.vg_fallback is not None and (known["rev_checkpoints"] + 1 != ring_states(known["max_steps"])):
        kernel = p.vg_fallback          # (items may outgrow the head: the fused replay's checkpointed schedule)
    kid, nbuf = kernel_ref(kernel)
    ptrs = [0 if t is None else t.data_ptr() for t in args] + [t.data_ptr() for t in res]
    if len(ptrs) != nbuf:
        raise _lib.TallymapError(f"{p.name}: layout has {len(ptrs)} buffers, kernel {kernel} takes {nbuf}")
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    flags = (4 if p.spawns else 0) | 8
    # (with n_active < N the per-item results, which follow the zeroed buffers, are zeroed too)
    nz = n_zero + (len(p.ys) if n_items < N else 0)
    _lib.launch(kid, st, ptrs, len(args), [nb for _, nb, _, _ in layout], nz, n_items, flags=flags)
    names = [n for n, _, _, _ in layout]
    tallies = [res[names.index(t.name)] for t in p.tallies]
    ys = res[n_zero:n_zero + len(p.ys)]
    run.last = dict(ctl=res[names.index("ctl")], args=args, consts=consts, results=dict(zip(names, res)),
                    kernel=kernel)
    return tallies + [res[names.index("stats")]] + list(ys)


# The record of a spawning program's reverse mode holds every child ever spawned (a slot is never reused, the
# reference's condition for a complete record: tallymap/_reverse_spawn.py:30-33).  Its capacity R is the user's
# `record`, else RECORD_PER_ROOT slots per root (at least RECORD_MIN), at most what RECORD_BUDGET_FRACTION of the free
# device memory holds at RECORD_SLOT_BYTES per slot (the record, its compact generation, the generation lists and the
# children's cotangents), below 2^31.  A tree with more children than R is not recorded in full: its gradient is NaN.
RECORD_PER_ROOT = 16384
RECORD_MIN = 1 << 20
RECORD_BUDGET_FRACTION = 0.5
RECORD_SLOT_BYTES = 32 + 2 + 4 + 8
_RECORD = {}


def record_slot_bytes(p):
    """device bytes a recorded child costs recording program p: its record, its compact generation, its place in
    the generation lists and its initial state's cotangents (a float per float leaf)"""
    fl = sum(int(np.prod(o.shape, dtype=np.int64)) for o in p.pi if o.dtype == _F32)
    return p.record_bytes + 2 + 4 + 4 * fl


def record_capacity(N, record=None, device=None, slot_bytes=RECORD_SLOT_BYTES):
    if record is not None:
        R = int(record)
        if not 1 <= R < 2 ** 31:
            raise ValueError("tallymap_b200: record capacity must be in [1, 2^31)")
        return R
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    key = (int(N), dev.index, int(slot_bytes))
    if key not in _RECORD:
        torch.cuda.empty_cache()             # (blocks cached by earlier calls count as free)
        free, _ = torch.cuda.mem_get_info(dev)
        _RECORD[key] = int(max(1, min(2 ** 31 - 1, max(RECORD_MIN, RECORD_PER_ROOT * int(N)),
                                      RECORD_BUDGET_FRACTION * free // int(slot_bytes))))
    return _RECORD[key]


TREE_MAX_GEN = 1024     # generations the tree adjoint takes (deeper trees: NaN gradient, counted)


def sh_value_and_grad(pi, X0, ct_dep, max_steps=100000, queue=None, stream=None, out=None, order=None):
    """the shower's forward outputs and the gradient of <ct_dep, dep> in ONE spawn launch (forward mode through
    spawn, SH_VG1), then the per-root readout of the exact words (tm_exact_combine).  d/d depth0 and d/d X0 are
    zero: depth and X0 reach the outputs only through the integer bin index (the tree adjoint gives the same +0).
    -> dict(dep, count, stats, k, trunc, g_E, g_depth, g_X0, steps: every particle's steps, the launch's work
    count) as device tensors (g_E NaN for a root whose sum overflowed; the caller poisons on truncation and dropped
    children).  order: an optional root claim order (an int32 permutation), e.g. largest energy first
    (energy_order): it changes which thread runs a root when, no result."""
    st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    res = run(SH_VG1, pi, [X0, ct_dep], consts=(max_steps,), queue=queue, stream=st, out=out, order=order)
    dep, count, g_E, steps, stats, k, tr = res
    N = int(k.shape[0])
    if N:
        words = run.last["results"]["g_E.exact"]
        _lib.check(_lib.lib().tm_exact_combine(ctypes.c_void_p(st), ctypes.c_void_p(words.data_ptr()), 1, N,
                                               ctypes.c_void_p(g_E.data_ptr()), ctypes.c_void_p(stats.data_ptr())))
    return dict(dep=dep, count=count, stats=stats, k=k, trunc=tr, g_E=g_E, g_depth=torch.zeros_like(g_E),
                g_X0=torch.zeros(1, dtype=torch.float32, device=g_E.device), steps=steps)


def energy_order(E0):
    """the shower's roots, largest primary energy first (int32, on E0's device): a root's subtree is proportional to
    its energy, so claiming the largest first leaves small trees for the end of the launch (longest-processing-time
    first, with the energy as the cost estimate); the order changes no result"""
    E0 = E0 if isinstance(E0, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(E0, np.float32))
    return torch.argsort(E0, descending=True).to(torch.int32)


def tree_record(p, pi, bc, max_steps=100000, queue=None, record=None, stream=None):
    """the first half of reverse mode through spawn (tallymap/_reverse_spawn.py:85-109 rec_primal and :255-283, the
    generation order): recording program p's launch (the forward's outputs, every child's record and generation,
    each root's newest child), then the generation lists (tm_tree_generations).  With the default record capacity
    too small for the tree, the (deterministic) recording runs once more with exactly the children it counted, when
    they fit in device memory.  -> dict(forward: run()'s outputs, args, results (by name), stats, ctl, N, R (the
    capacity), total (children spawned), n_rec (recorded), counts (host: records per generation, the last entry
    the generations beyond TREE_MAX_GEN), offs, lists (device: record slots by generation), G (the deepest
    generation), incomplete (a child dropped, not recorded, or too deep: the gradient is NaN))"""
    import ctypes
    dev = torch.device("cuda", torch.cuda.current_device())
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    slot = record_slot_bytes(p)
    for attempt in range(2):
        fwd = run(p, pi, bc, consts=(max_steps,), queue=queue, record=record, stream=st)
        last = run.last
        res, args = last["results"], last["args"]
        R = int(last["consts"][p.consts.index("record")])
        N = int(args[0].shape[0])
        rec, stats = res["record"], res["stats"]
        head = torch.cat([res["tree"][:1], stats.to(torch.int64)]).cpu()        # (one sync)
        total, dropped = int(head[0]), int(head[1 + STATS.index("children_dropped")])
        if total <= R or record is not None or attempt == 1 or total >= 2 ** 31:
            break
        # the default capacity was short: the recording is deterministic, so record again with exactly the children
        # it counted, when they fit beside what is allocated (and keep that capacity for later calls with N roots)
        free, _ = torch.cuda.mem_get_info(dev)
        if total * slot > 0.9 * (free + rec.numel() * rec.element_size()):
            break
        del fwd, last, res, rec, stats
        run.last = None
        torch.cuda.empty_cache()
        _RECORD[(N, dev.index, slot)] = total
        record = total
    n_rec = min(total, R)
    L = _lib.lib()
    counts = torch.empty(TREE_MAX_GEN + 1, dtype=torch.int64, device=dev)
    cursor = torch.empty_like(counts)
    lists = torch.empty(max(n_rec, 1), dtype=torch.int32, device=dev)
    gens = res["record.gen"]                # (the records' generations, u16: 2 bytes a record to read)
    _lib.check(L.tm_tree_generations(ctypes.c_void_p(st), ctypes.c_void_p(gens.data_ptr()), n_rec, 2, 0, 2,
                                     TREE_MAX_GEN, ctypes.c_void_p(counts.data_ptr()),
                                     ctypes.c_void_p(cursor.data_ptr()), ctypes.c_void_p(lists.data_ptr())))
    cnt = counts.cpu().numpy()                                              # (second sync)
    offs = np.concatenate([[0], np.cumsum(cnt)])
    nz = np.nonzero(cnt[:TREE_MAX_GEN])[0]
    G = int(nz.max()) if len(nz) else 0
    incomplete = total > R or dropped > 0 or cnt[TREE_MAX_GEN] > 0
    return dict(forward=fwd, args=args, results=res, stats=stats, ctl=last["ctl"], N=N, R=R, total=total,
                n_rec=n_rec, counts=cnt, offs=offs, lists=lists, G=G, incomplete=bool(incomplete))


def tree_adjoint(adj, t, cts, max_steps=100000, rev_checkpoints=None, stream=None):
    """the second half of reverse mode through spawn for a lowered item (tallymap/_reverse_spawn.py:285-336): over a
    recorded tree t (tree_record of the item's recording program), one launch of the adjoint program adj
    (Lowered.tree_program) per generation, deepest first, each child's initial-state cotangents going to its
    parent's launch, then one launch over the roots.  cts: the output cotangents (adj's operands after the item's
    broadcast operands).  -> dict(g: f32[W], the broadcast operands' cotangents summed over every particle (exact
    sums); ct_in: [f32[N, ...] per float per-item operand], the roots' cotangents; poisoned: a device bool -- the
    record incomplete, a replay that disagreed with the record (tree[0]) or hit max_steps (tree[1]), or an item
    truncated or a child dropped in the forward; the caller NaN-poisons; words, stats, info)"""
    dev = torch.device("cuda", torch.cuda.current_device())
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    args, res, N, n_rec = t["args"], t["results"], t["N"], t["n_rec"]
    npi = len(adj.pi)
    nbc = len(adj.bc) - len(cts)
    ins = list(args[:npi + nbc])
    for c, o in zip(cts, adj.bc[nbc:]):
        x = _dev(c, dev, _F32)
        if tuple(x.shape) != tuple(o.shape):
            raise TypeError(f"{adj.name}: cotangent {o.name} has shape {tuple(x.shape)}, expected {tuple(o.shape)}")
        ins.append(x)
    ins += [res["record"], res["last"]]
    C, threads, replay_bytes = replay_plan(adj, max_steps, rev_checkpoints, dev)
    W = adj.tallies[0].S
    n64 = W * EXACT_WORDS + (W + 1) // 2
    fl = sum(int(np.prod(o.shape, dtype=np.int64)) for o in adj.pi if o.dtype == _F32)
    outs = [torch.empty(CTL_WORDS, dtype=torch.int32, device=dev), torch.empty(W, dtype=_F32, device=dev),
            torch.empty(n64, dtype=torch.int64, device=dev), torch.empty(len(STATS), dtype=torch.int32, device=dev),
            torch.empty(4, dtype=torch.int32, device=dev)]
    outs += [torch.zeros((N,) + tuple(o.shape), dtype=_F32, device=dev) for o in adj.ys[:-1]]
    outs += [torch.empty(max(n_rec, 1) * max(fl, 1), dtype=_F32, device=dev),
             torch.zeros(N, dtype=torch.uint8, device=dev),
             torch.empty(max(1, (replay_bytes + 15) // 16) * 4, dtype=torch.int32, device=dev)]
    nbytes = [x.numel() * x.element_size() for x in outs]
    kid, nbuf = kernel_ref(adj.kernel)
    cnt, offs, lists = t["counts"], t["offs"], t["lists"]
    launches = 0
    if not t["incomplete"]:
        for g in list(range(t["G"], 0, -1)) + [0]:
            n = N if g == 0 else int(cnt[g])
            if n == 0:
                continue
            cst = _consts((int(max_steps), C, threads, 1 if g == 0 else 0, max(n_rec, 1)), dev)
            order = 0 if g == 0 else lists.data_ptr() + 4 * int(offs[g])
            ptrs = [x.data_ptr() for x in ins] + [cst.data_ptr(), order] + [x.data_ptr() for x in outs]
            if len(ptrs) != nbuf or nbuf != adj.buffers:
                raise _lib.TallymapError(f"{adj.name}: {len(ptrs)} buffers for a kernel of {nbuf}")
            # (the first launch zeroes the control words, the gradient's exact words, stats and tree counters; later
            # launches only their control words: the exact words sum over every generation)
            _lib.launch(kid, st, ptrs, len(ins) + 2, nbytes, 5 if launches == 0 else 1, n, flags=8)
            launches += 1
    if launches == 0:
        for x in outs[:5]:
            x.zero_()
    g_out, tree = outs[1], outs[4]
    fstats = t["stats"]
    bad = (tree[0] > 0) | (tree[1] > 0) | (fstats[STATS.index("children_truncated")] > 0) | \
        (fstats[STATS.index("children_dropped")] > 0) | outs[-2].bool().any() | bool(t["incomplete"])
    tree_adjoint.last = dict(ctl=outs[0], fwd_ctl=t["ctl"])
    info = dict(children=t["total"], generations=t["G"], launches=launches + 2, kernels=launches + 4, record=t["R"],
                poisoned=bad, mismatch=tree[0], replay_truncated=tree[1], generation_sizes=cnt[:t["G"] + 1].tolist())
    tree_adjoint.last_info = info
    return dict(g=g_out, ct_in=outs[5:5 + len(adj.ys) - 1], poisoned=bad, words=outs[2], stats=outs[3], info=info)


def tree_grad(pi, X0, ct_dep, max_steps=100000, queue=None, record=None, rev_checkpoints=None, stream=None):
    """Reverse mode through spawn for the shower (tallymap/_reverse_spawn.py:233-336, tree_vjp): the recording
    forward (rec_primal), the generation lists (tm_tree_generations), then one adjoint launch per generation,
    deepest first, and one over the roots.  Each adjoint item replays its particle and injects its children's
    initial-state cotangents (from the previous launch) at the spawn step.
    -> dict(forward=[dep, count, stats, k, truncated] as run() returns them, ct_X0 f32[1], ct_E f32[N],
            ct_depth f32[N], words (ct_X0's exact scratch words, for a cross-GPU combine), info={children,
            generations, launches (the reference's count: the recording primal + one per generation + the roots'),
            kernels (launches of this backend's kernels), record, poisoned (device bool), ...})
    Every cotangent is NaN when the record is incomplete (a child dropped or past the record's capacity, a
    generation deeper than TREE_MAX_GEN), when a replay disagrees with the record, or when any particle hit
    max_steps."""
    dev = torch.device("cuda", torch.cuda.current_device())
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    rt = tree_record(SH_REC, pi, [X0], max_steps=max_steps, queue=queue, record=record, stream=st)
    fwd, args, res, stats = rt["forward"], rt["args"], rt["results"], rt["stats"]
    rec, root_last = res["record"], res["last"]
    N, R, n_rec, total, G = rt["N"], rt["R"], rt["n_rec"], rt["total"], rt["G"]
    cnt, offs, lists, incomplete = rt["counts"], rt["offs"], rt["lists"], rt["incomplete"]

    # the adjoint launches: [E0, depth0, keys, X0, ct_dep, record, last, consts, order] | [ctl, ct_X0, exact words,
    # stats, tree counters, ct_E, ct_depth, dx, replay scratch]
    C, threads, replay_bytes = replay_plan(SH_GRAD, max_steps, rev_checkpoints, dev)
    x0 = args[3]
    ctd = _dev(ct_dep, dev, _F32).reshape(-1)
    if ctd.numel() != 512:
        raise TypeError("tallymap_b200: ct_dep must have 512 elements")
    outs = [torch.empty(CTL_WORDS, dtype=torch.int32, device=dev), torch.empty(1, dtype=_F32, device=dev),
            torch.empty(EXACT_WORDS + 1, dtype=torch.int64, device=dev),
            torch.empty(len(STATS), dtype=torch.int32, device=dev), torch.empty(4, dtype=torch.int32, device=dev),
            torch.empty(N, dtype=_F32, device=dev), torch.empty(N, dtype=_F32, device=dev),
            torch.empty(max(n_rec, 1) * 2, dtype=_F32, device=dev),
            torch.empty(max(1, (replay_bytes + 15) // 16) * 4, dtype=torch.int32, device=dev)]
    nbytes = [t.numel() * t.element_size() for t in outs]
    kid, nbuf = _lib.kernel_id(SH_GRAD.kernel)
    base = [args[0], args[1], args[2], x0, ctd, rec, root_last]
    launches = 0
    if not incomplete:
        for g in list(range(G, 0, -1)) + [0]:
            n = N if g == 0 else int(cnt[g])
            if n == 0:
                continue
            # (the adjoint bounds child slots by the recorded count, not the capacity: no slot past it was written)
            cst = _consts((int(max_steps), C, threads, 1 if g == 0 else 0, max(n_rec, 1)), dev)
            order = 0 if g == 0 else lists.data_ptr() + 4 * int(offs[g])
            ptrs = [t.data_ptr() for t in base] + [cst.data_ptr(), order] + [t.data_ptr() for t in outs]
            assert len(ptrs) == nbuf == SH_GRAD.buffers
            _lib.launch(kid, st, ptrs, 9, nbytes, 5 if launches == 0 else 1, n, flags=8)
            launches += 1
    if launches == 0:
        for t in outs[:5]:
            t.zero_()
    ctX, ctE, ctD, tree = outs[1], outs[5], outs[6], outs[4]
    trunc = fwd[4]
    bad = (tree[0] > 0) | (tree[1] > 0) | (stats[2] > 0) | trunc.bool().any() | bool(incomplete)
    nan = lambda v: torch.where(bad, torch.full_like(v, float("nan")), v)
    tree_grad.last = dict(ctl=outs[0], fwd_ctl=rt["ctl"])
    return dict(forward=fwd[:5], ct_X0=nan(ctX), ct_E=nan(ctE), ct_depth=nan(ctD),
                words=outs[2], stats=outs[3],
                info=dict(children=total, generations=G, launches=launches + 2, kernels=launches + 4, record=R,
                          poisoned=bad,
                          mismatch=tree[0], replay_truncated=tree[1], generation_sizes=cnt[:G + 1].tolist()))


_CONSTS = {}


def _consts(vals, dev):
    """the hoisted-constant buffer, made once per (values, device): no host copy on the launch path"""
    key = (vals, dev.index)
    t = _CONSTS.get(key)
    if t is None:
        t = torch.tensor(vals, dtype=torch.int32).to(dev)
        _CONSTS[key] = t
    return t


def alloc_results(p, N, device=None, replay_bytes=None, queue=None, record=None, max_steps=None):
    """result buffers for N items (an adjoint's replay scratch as planned on `device` for `max_steps` unless given; a
    spawning program's ring of `queue` slots; a recording program's `record` slots)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    if replay_bytes is None and p.replay_state_bytes:
        replay_bytes = replay_plan(p, max_steps or 2 ** 31 - 1, None, device)[2]
    Q = int(queue or QUEUE_DEFAULT) if p.queue_leaf_bytes else 0
    R = record_capacity(N, record, device, record_slot_bytes(p)) if p.record_bytes else 0
    layout, n_zero = _layout(p, N, replay_bytes or 0, Q, R)
    # the zeroed results (tallies, scratch accumulators, control words, stats) share ONE allocation, each at a
    # 16-byte aligned offset in layout order: Sum tallies of one dtype that follow each other in the layout are then
    # one contiguous range, which the multi-GPU step all_reduces in place with no packing copy
    # (parallel.all_reduce_sums)
    offs, o = [], 0
    for _, nb, _, _ in layout[:n_zero]:
        offs.append(o)
        o += (nb + 15) // 16 * 16
    blob = torch.empty(max(o, 16), dtype=torch.uint8, device=device)
    out = [blob[a:a + nb].view(dt).view(shape) for a, (_, nb, dt, shape) in zip(offs, layout[:n_zero])]
    return out + [torch.empty(shape, dtype=dt, device=device) for _, _, dt, shape in layout[n_zero:]]


def check_status(ctl):
    """raise if a finished launch's device error word (ctl[3]) is set (a device wait gave up, a bounds check)."""
    import ctypes
    w = np.ascontiguousarray(ctl.detach().cpu().numpy().view(np.uint32))
    _lib.check(_lib.lib().tm_check_status(w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))))
