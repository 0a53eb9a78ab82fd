"""tallymap_b200.diagnostics(): what to look at when something is wrong, and what a bug report should contain (the
counterpart of tallymap.diagnostics / history, tallymap/_diagnostics.py:1-53, for this backend).

    tm.diagnostics()              versions, environment, device, compiler and cache, the last lowered item programs
                                  and compiled kernels -- with each kernel's resources (registers and local memory per
                                  thread, shared memory, resident blocks per SM) when a GPU is present -- and the last
                                  tree adjoint's counters
    tm.diagnostics(reset=True)    the same, then the history cleared
    tm.history()                  cheap: the last item programs and kernel records, nothing probed

Kernel records come from lower.compile_kernel (tag, kernel id, source digest, compile seconds, the cache that held it),
program records from lower.Lowered (item name, equations per part, input specs, outputs, the float constants the
item closed over -- a derivative cannot reach them: what you differentiate must be an argument)."""
import collections
import os
import platform
import sys

HISTORY = 16
PROGRAMS = collections.deque(maxlen=HISTORY)
KERNELS = collections.deque(maxlen=HISTORY)


def record_kernel(rec):
    KERNELS.append(dict(rec))


def record_program(rec):
    PROGRAMS.append(dict(rec))


def history():
    """-> dict(programs=[...], kernels=[...]): the last HISTORY lowered item programs and compiled kernels, oldest
    first"""
    return dict(programs=[dict(r) for r in PROGRAMS], kernels=[dict(r) for r in KERNELS])


def _platform():
    import torch
    d = dict(torch=torch.__version__, cuda_available=torch.cuda.is_available())
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        d.update(gpu=p.name, compute_capability=f"{p.major}.{p.minor}", sms=p.multi_processor_count,
                 memory_gib=round(p.total_memory / 2 ** 30, 1), devices=torch.cuda.device_count())
    return d


def _resources(kid):
    from . import _lib
    try:
        return _lib.kernel_info(kid)
    except Exception as e:                    # noqa: BLE001 -- no GPU (the resources need a context): say so
        return dict(unavailable=str(e).splitlines()[0][:120])


def diagnostics(reset=False):
    """-> dict(versions, env, platform, cuda, programs, kernels, tree); reset: clear the history after reading it"""
    import numpy as np

    from . import __version__, _lib, backend, lower
    plat = _platform()
    out = dict(
        versions=dict(tallymap_b200=__version__, numpy=np.__version__, python=sys.version.split()[0]),
        env={k: os.environ[k] for k in ("TALLYMAP_B200_CACHE", "CUDA_VISIBLE_DEVICES") if k in os.environ},
        machine=platform.machine(),
        platform=plat,
        cuda=dict(library=_lib.LIB, library_built=os.path.exists(_lib.LIB), cache_dir=lower.cache_dir() or None,
                  arch="sm_100a"),
        programs=[dict(r) for r in PROGRAMS],
        kernels=[dict(r, resources=_resources(r["kernel"])) if plat["cuda_available"] else dict(r) for r in KERNELS],
        tree={k: (v.item() if hasattr(v, "item") and getattr(v, "numel", lambda: 0)() == 1 else v)
              for k, v in (getattr(backend.tree_adjoint, "last_info", None) or {}).items()},
    )
    if reset:
        PROGRAMS.clear()
        KERNELS.clear()
    return out
