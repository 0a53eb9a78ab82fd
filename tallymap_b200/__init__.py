"""tallymap_b200: a B200-native (sm_100a) kernel backend for tallymap.

Layers (top down):
  api.vmap / Result      the tallymap result contract (poisoning, stats) over lowered item programs
  lang, trace, lower     Python item functions: traced to a scalar IR, lowered to CUDA, compiled at run time (NVRTC)
  backend.run            the kernel-backend driver, the counterpart of tallymap/backends/kernel/__init__.py:135 run
  _lib                   ctypes binding of libtm_b200.so, the C ABI of include/tallymap_b200.h
  csrc/                  the persistent-thread runtime and item programs, CUDA for sm_100a
  prng                   jax.random key arithmetic on the host (numpy), for inputs made without JAX
  parallel               items sharded over GPUs, tallies combined with NCCL
"""
from . import lang, prng
from ._lib import TallymapError, build
from .api import FAMILIES, Queue, Records, Result, Sum, TallyError, UnsupportedError, vmap
from .backend import PROGRAMS, STATS, ItemProgram, TSpec, run
from ._diagnostics import diagnostics, history
from .trace import TallyToken as Tally      # the item's tally handle (tallymap.Tally): t.add / t.append / t.spawn
from .memory import OutputMemory, call_memory, cell_bytes, max_cells, output_memory

__version__ = "0.1.0"
__all__ = ["FAMILIES", "PROGRAMS", "STATS", "ItemProgram", "OutputMemory", "Queue", "Records", "Result", "Sum", "TSpec",
           "Tally", "TallyError", "TallymapError", "UnsupportedError", "build", "call_memory", "cell_bytes",
           "diagnostics",
           "history", "lang", "max_cells", "output_memory", "prng", "run", "supported_primitives", "vmap"]


def supported_primitives():
    """the jaxpr primitives the jaxpr front end lowers (tallymap.supported_primitives): the sorted names of
    tallymap_b200.from_jaxpr's table"""
    from . import from_jaxpr
    return from_jaxpr.supported_primitives()
