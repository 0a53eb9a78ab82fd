"""Loader and build step of libtm_b200.so, the C-ABI CUDA library (include/tallymap_b200.h).

There is no CPU fallback: every entry point of this package that computes goes through this library, and loading
it fails loudly when it has not been built.  `build()` compiles it in-tree for sm_100a with nvcc (it cross-compiles
on a machine without a GPU).
"""
import ctypes
import os
import subprocess
import sys
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libtm_b200.so")
INCLUDE = os.path.join(ROOT, "include")

# sm_100a only; --fmad=false: every f32 + - * is one IEEE rounding (the reference compiles its kernels with
# -fmad=false, tallymap/backends/kernel/compile.py:27); -lineinfo for profiler source attribution.
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "--fmad=false", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared"]

_LOCK = threading.Lock()
_HANDLE = None

TM_OK, TM_EINVAL, TM_ECUDA, TM_EDEVICE = 0, 1, 2, 3


class TallymapError(RuntimeError):
    """an error reported by libtm_b200 (the reference's ffi::Error)."""


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h", ".cc"))) + [
        os.path.join(INCLUDE, "tallymap_b200.h")]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def xla_ffi_include():
    """-I flags for XLA's FFI headers when JAX is importable (jax.ffi.include_dir()), else none: the XLA FFI handler
    (csrc/tm_ffi.cc) is then left out of the build and tm_ffi_available() returns 0"""
    d = os.environ.get("TM_XLA_FFI_INCLUDE")
    if not d:
        r = subprocess.run([sys.executable, "-c", "import jax; print(jax.ffi.include_dir())"], capture_output=True,
                           text=True)
        d = r.stdout.strip() if r.returncode == 0 else ""
    return ["-I", d] if d and os.path.isdir(d) else []


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force=False, verbose=False):
    """compile libtm_b200.so for sm_100a (in-tree, so it travels with the repository) -> its path."""
    with _LOCK:
        if not force and not stale():
            return LIB
        os.makedirs(LIBDIR, exist_ok=True)
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + xla_ffi_include() + [
            "-o", tmp, os.path.join(CSRC, "tm_capi.cu"), os.path.join(CSRC, "tm_ffi.cc")]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise TallymapError("nvcc failed building libtm_b200.so:\n" + r.stdout + r.stderr)
        os.replace(tmp, LIB)
        if verbose:
            print(r.stdout + r.stderr)
        return LIB


def lib():
    """the loaded library (ctypes.CDLL); raises when it is missing: there is no fallback."""
    global _HANDLE
    with _LOCK:
        if _HANDLE is not None:
            return _HANDLE
        if not os.path.exists(LIB):
            raise TallymapError(f"libtm_b200.so is not built ({LIB}); run tallymap_b200._lib.build() or "
                                "`python -c 'import __graft_entry__ as g; g.build()'` first")
        L = ctypes.CDLL(LIB)
        P, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        L.tm_abi_version.restype = ctypes.c_int
        L.tm_last_error.restype = ctypes.c_char_p
        L.tm_kernel_id.argtypes = [ctypes.c_char_p, ctypes.POINTER(i64), ctypes.POINTER(i32)]
        L.tm_kernel_name.argtypes = [i32, ctypes.POINTER(ctypes.c_char_p)]
        L.tm_register.argtypes = [i64, P, ctypes.c_size_t, ctypes.c_char_p, i32, i32, i32]
        L.tm_kernel_info.argtypes = [i64, ctypes.POINTER(ctypes.c_longlong)]
        L.tm_kernel_state_bytes.argtypes = [i64, ctypes.POINTER(i32)]
        L.tm_launch.argtypes = [i64, P, ctypes.POINTER(P), i32, i32, ctypes.POINTER(ctypes.c_size_t), i32, i32, i64,
                                ctypes.POINTER(i32)]
        L.tm_check_status.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        L.tm_exact_combine.argtypes = [P, P, i32, i32, P, P]
        L.tm_exact_scatter.argtypes = [P, P, P, i64, i32, P, P, P]
        L.tm_exact_scatter_noalloc.argtypes = [P, P, P, i64, i32, P, P]
        L.tm_math_eval.argtypes = [P, i32, P, P, P, i64]
        L.tm_probe_threefry.argtypes = [P, i32, P, i64, ctypes.POINTER(i64)]
        L.tm_ffi_available.restype = ctypes.c_int
        L.tm_probe_issue.argtypes = [P, i32, i32, P, i64, ctypes.POINTER(i64)]
        L.tm_tree_generations.argtypes = [P, P, i64, i32, i32, i32, i32, P, P, P]
        L.tm_compile_register.argtypes = [i64, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, i32, i32, i32]
        L.tm_compile.argtypes = [ctypes.c_char_p, ctypes.c_char_p, i32, i32, P, ctypes.c_size_t,
                                 ctypes.POINTER(ctypes.c_size_t)]
        _HANDLE = L
        return L


def check(rc):
    if rc != TM_OK:
        raise TallymapError(lib().tm_last_error().decode(errors="replace"))


# the symbols include/tallymap_b200.h declares (tests check the library exports each one)
EXPORTS = ("tm_abi_version", "tm_last_error", "tm_kernel_id", "tm_kernel_name", "tm_register", "tm_kernel_info",
           "tm_kernel_state_bytes",
           "tm_launch", "tm_check_status", "tm_exact_combine", "tm_exact_scatter", "tm_exact_scatter_noalloc",
           "tm_probe_threefry", "tm_probe_issue", "tm_ffi_available", "tm_math_eval", "tm_tree_generations",
           "tm_compile_register", "tm_compile")


PROBE_THREEFRY, PROBE_FP32, PROBE_ODE_STEP, PROBE_ODE_STEP_VJP, PROBE_PHOTON_STEP, PROBE_ODE_STEP_JVP = 0, 1, 2, 3, 4, 5


def probe_rate(kind, iters, stream, device, reps=3):
    """iterations per second of tm_probe_issue's probe `kind` at full occupancy on `device` (CUDA events on
    `stream`, the best of `reps` launches) -> (rate, threads)"""
    import torch
    out = torch.empty(148 * 2048 * 2, dtype=torch.int32, device=device)
    used = ctypes.c_int64()
    best = None
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        check(lib().tm_probe_issue(ctypes.c_void_p(stream.cuda_stream), kind, iters, ctypes.c_void_p(out.data_ptr()),
                                   out.numel(), ctypes.byref(used)))
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    return used.value * iters / (best / 1e3), used.value


def kernel_id(name):
    i = ctypes.c_int64()
    nb = ctypes.c_int32()
    check(lib().tm_kernel_id(name.encode(), ctypes.byref(i), ctypes.byref(nb)))
    return i.value, nb.value


def kernel_names():
    out, i = [], 0
    while True:
        p = ctypes.c_char_p()
        check(lib().tm_kernel_name(i, ctypes.byref(p)))
        if p.value is None:
            return out
        out.append(p.value.decode())
        i += 1


def kernel_info(kid):
    out = (ctypes.c_longlong * 7)()
    check(lib().tm_kernel_info(kid, out))
    keys = ("registers", "local_bytes", "shared_bytes", "blocks_per_sm", "sms", "threads_per_sm", "block")
    return dict(zip(keys, list(out)))


def launch(kid, stream, ptrs, n_args, ret_bytes, n_zero, n_items, flags=0):
    """tm_launch over raw device pointers (ints); raises TallymapError on failure."""
    n = len(ptrs)
    arr = (ctypes.c_void_p * n)(*ptrs)
    rb = (ctypes.c_size_t * max(1, len(ret_bytes)))(*ret_bytes)
    st = ctypes.c_int32()
    check(lib().tm_launch(kid, ctypes.c_void_p(stream), arr, n_args, n - n_args, rb, n_zero, flags, n_items,
                          ctypes.byref(st)))
