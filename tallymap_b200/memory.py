"""Device memory of a call's outputs on this backend: output_memory (a slope and a fixed term), cell_bytes,
call_memory and max_cells, the counterparts of tallymap.output_memory / cell_bytes / call_memory / max_cells
(tallymap/_memory.py:155-260) for a caller that sizes its outputs from the free device memory.

The reference's numbers model its two backends and add what XLA's buffer assignment measured on top; here they are
the structural bytes of this backend's own buffers, exactly as backend.ItemProgram.result_layout allocates them:

  Sum float32 / int32          the output (4 B per cell)
  Sum float64 / int64          the output (8 B)
  Sum(fixed_point=True) f32    5 int64 carry-save words + a u32 flag + the output (48 B)
  Sum(fixed_point=True, other) an int64 word, an i32 carry, a u32 flag + the output (16 B + the output's itemsize)
  Records (per slot)           one pass: each field (4 B), the key (item, ordinal: 8 B), and the canonical copy of
                               each field; count-then-fill: each field, written once at its canonical slot

and, per derivative, the tangent tallies of a jvp (a float output's: a float32 or an exact tally per lane), the
cotangent a grad / vjp reads (4 B per float cell; a vjp also holds the forward output).  The fixed term is the
launch's own zeroed control and stats words.  NOT included, as in the reference: the items' inputs, per-item results
and per-item state (the replay's scratch, per thread, sized by backend.replay_plan), the spawn ring, and the CUDA
caching allocator's rounding of each buffer."""
import math
from typing import NamedTuple

import torch

from .api import Records, Sum
from .backend import CTL_WORDS, EXACT_WORDS, STATS

MAX_CELLS = (1 << 31) - 1            # cells are indexed with int32 (tally indices, emits)
DERIVATIVES = ("forward", "jvp", "vjp", "grad")
_LAUNCH = 4 * CTL_WORDS + 4 * len(STATS)


class OutputMemory(NamedTuple):
    """device memory of one output in a call: per_cell * cells + fixed bytes"""
    per_cell: float
    fixed: int

    def total(self, cells):
        return self.per_cell * cells + self.fixed


def _size(output):
    if isinstance(output, Records):
        return output.capacity
    shape = output.shape if isinstance(output, Sum) else output
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return int(math.prod(shape)) if shape else 1


def _derivative(d):
    d = "forward" if d is None else d
    if d not in DERIVATIVES:
        raise ValueError(f"tallymap_b200: derivative must be None or one of {DERIVATIVES}, got {d!r}")
    return d


def _per_cell(output, derivative, lanes):
    """bytes per cell of one output under `derivative`"""
    if isinstance(output, Records):
        nf = len(output.fields)
        nfloat = sum(1 for _, dt in output.fields if dt == torch.float32)
        per = 4 * nf + (0 if output.capacity is None else 8 + 4 * nf)
        if derivative == "jvp":
            per += 4 * nfloat * lanes * (1 if output.capacity is None else 2)
        elif derivative in ("grad", "vjp"):
            per += 4 * nfloat
        return per
    if not isinstance(output, Sum):
        output = Sum(output)
    item = torch.empty((), dtype=output.dtype).element_size()
    acc = output.accumulator()
    isfloat = output.dtype.is_floating_point
    if output.fixed_point and acc is None:
        per = 8 * EXACT_WORDS + 4 + item
    elif acc is not None and acc[0] == "wide":
        per = 16 + item
    else:
        per = item
    if derivative == "jvp" and isfloat:
        if acc is not None:
            raise ValueError("tallymap_b200: forward mode of a float64 or scaled fixed-point Sum is not lowered")
        per += lanes * ((8 * EXACT_WORDS + 4 + 4) if output.fixed_point else 4)
    elif derivative in ("grad", "vjp") and isfloat:
        per = 4 if derivative == "grad" else per + 4
    elif derivative in ("grad",):
        per = 0
    return per


def _args(output, derivative, cells, who):
    d = _derivative(derivative)
    S = _size(output) if cells is None else int(cells)
    if S is None:
        raise ValueError(f"tallymap_b200.{who}: a Records output with capacity=None needs cells=")
    if not 1 <= S <= MAX_CELLS:
        raise ValueError(f"tallymap_b200.{who}: cells must be in [1, 2^31 - 1], got {S}")
    return d, S


def output_memory(output, derivative=None, *, cells=None, lanes=1):
    """device memory one output of a tallymap_b200.vmap call holds while the call runs: OutputMemory(per_cell,
    fixed).  output: a Sum, a Records (per slot) or a shape (a float32 Sum); derivative: None / 'forward' | 'jvp'
    (`lanes` tangent lanes) | 'vjp' | 'grad'; cells: the cell count (default: the output's own size)."""
    d, _ = _args(output, derivative, cells, "output_memory")
    return OutputMemory(float(_per_cell(output, d, int(lanes))), _LAUNCH)


def cell_bytes(output, derivative=None, *, cells=None, lanes=1):
    """device memory per cell of one output at `cells` cells (default: its own size), the fixed term included"""
    d, S = _args(output, derivative, cells, "cell_bytes")
    return (_per_cell(output, d, int(lanes)) * S + _LAUNCH) / S


def call_memory(outputs, derivative=None, *, lanes=1):
    """device memory, in bytes, the outputs of ONE call hold: each output's per-cell bytes times its size, plus the
    launch's fixed words once.  outputs: the outputs= dict of tallymap_b200.vmap, or a list"""
    outs = list(outputs.values()) if isinstance(outputs, dict) else list(outputs)
    tot = 0
    for o in outs:
        d, S = _args(o, derivative, None, "call_memory")
        tot += _per_cell(o, d, int(lanes)) * S
    return int(math.ceil(tot + _LAUNCH))


def max_cells(output, derivative=None, *, memory=None, lanes=1):
    """the largest cell count of one output: 2^31 - 1 (int32 indices), and with memory= (bytes) the largest count
    whose output_memory(...).total(count) fits it"""
    d = _derivative(derivative)
    if memory is None:
        return MAX_CELLS
    per = _per_cell(output, d, int(lanes))
    if memory < _LAUNCH + per:
        return 0
    return int(min(MAX_CELLS, (memory - _LAUNCH) // per)) if per else MAX_CELLS
