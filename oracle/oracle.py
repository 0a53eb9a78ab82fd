"""TEST INFRASTRUCTURE ONLY: ctypes front end of the CPU oracle (a C++/OpenMP restatement of the reference's CPU
kernel target for the benchmark item programs; see oracle_core.h, oracle_run.h, programs.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this module, and only as
the checker or the timed CPU baseline: the product (tallymap_b200) never calls it.

The library is built with -march=native, so it is built per host CPU (the GPU box's host differs from the build
container's): one .so per CPU model under oracle/_build/.
"""
import ctypes
import hashlib
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LOCK = threading.Lock()
_LIB = None


def _cpu_tag():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith(("model name", "flags")):
                    model += ln
    except OSError:
        pass
    return hashlib.sha256(model.encode()).hexdigest()[:12]


def lib_path():
    return os.path.join(HERE, "_build", f"liboracle-{_cpu_tag()}.so")


def build(force=False):
    """compile the oracle for this host's CPU (make; a few seconds) -> path of the .so."""
    path = lib_path()
    srcs = [os.path.join(HERE, f) for f in os.listdir(HERE) if f.endswith((".cpp", ".h"))]
    srcs.append(os.path.join(HERE, "..", "tallymap_b200", "csrc", "tm_math.h"))     # (the shared math it includes)
    if not force and os.path.exists(path) and all(os.path.getmtime(s) <= os.path.getmtime(path) for s in srcs):
        return path
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    os.replace(os.path.join(HERE, "_build", "liboracle.so"), path)
    return path


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            L = ctypes.CDLL(build())
            P = ctypes.c_void_p
            i64, i32, f32, u32 = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_uint32
            L.or_num_threads.restype = ctypes.c_int
            L.or_threefry2x32.argtypes = [u32, u32, u32, u32, P]
            L.or_split.argtypes = [u32, u32, i64, P]
            L.or_uniform.argtypes = [u32, u32, i64, f32, f32, P]
            L.or_exact_sum.argtypes = [P, P, i64, ctypes.c_int, P, P]
            L.or_exact_words.argtypes = [P, P, i64, ctypes.c_int, P]
            L.or_exact_read.argtypes = [P, P]
            L.or_exact_read.restype = f32
            L.or_q1_fwd.argtypes = [i64, P, P, f32, i32, ctypes.c_int, P, P, P, P, ctypes.c_int]
            L.or_q1_grad.argtypes = [i64, P, P, f32, P, i32, ctypes.c_int, ctypes.c_int, P, P, P]
            L.or_rw_fwd.argtypes = [i64, P, P, f32, i32, ctypes.c_int, P, P, P, P, P, ctypes.c_int]
            L.or_rw_grad.argtypes = [i64, P, P, f32, P, i32, ctypes.c_int, ctypes.c_int, P, P, P]
            L.or_ph_fwd.argtypes = [i64, P, f32, f32, i32, ctypes.c_int, P, P, P, P, ctypes.c_int, ctypes.c_int]
            L.or_ph_grad.argtypes = [i64, P, f32, f32, P, i32, ctypes.c_int, ctypes.c_int, P, P, P, ctypes.c_int]
            L.or_math.argtypes = [ctypes.c_int, P, P, P, i64]
            L.or_od_fwd.argtypes = [i64, P, P, P, P, f32, i32, ctypes.c_int, P, P, P, P, P, ctypes.c_int]
            L.or_sh_fwd.argtypes = [i64, P, P, P, f32, i32, ctypes.c_int, P, P, P, P, P, ctypes.c_int]
            L.or_od_grad.argtypes = [i64, P, P, P, P, f32, P, P, i32, ctypes.c_int, ctypes.c_int, P, P, P]
            L.or_od_vg1.argtypes = [i64, P, P, P, P, f32, P, P, i32, ctypes.c_int, P, P, P, P]
            L.or_sh_grad.argtypes = [i64, P, P, P, f32, P, i32, ctypes.c_int, P, P, P, P]
            L.or_sh_vg1.argtypes = [i64, P, P, P, f32, P, i32, ctypes.c_int, P, P]
            _LIB = L
    return _LIB


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def num_threads():
    return lib().or_num_threads()


# ----------------------------------------------------------------------------------------------- RNG / exact sum
def threefry2x32(k0, k1, c0, c1):
    out = np.zeros(2, np.uint32)
    lib().or_threefry2x32(int(k0), int(k1), int(c0), int(c1), _p(out))
    return int(out[0]), int(out[1])


def split(key, n):
    out = np.zeros((n, 2), np.uint32)
    lib().or_split(int(key[0]), int(key[1]), n, _p(out))
    return out


def uniform(key, n, lo=0.0, hi=1.0):
    out = np.zeros(n, np.float32)
    lib().or_uniform(int(key[0]), int(key[1]), n, lo, hi, _p(out))
    return out


def exact_sum(vals, bins, nb):
    vals = np.ascontiguousarray(vals, np.float32)
    bins = np.ascontiguousarray(bins, np.int32)
    out = np.zeros(nb, np.float32)
    stats = np.zeros(5, np.int32)
    lib().or_exact_sum(_p(vals), _p(bins), len(vals), nb, _p(out), _p(stats))
    return out, stats


def exact_words(vals, bins, nb):
    vals = np.ascontiguousarray(vals, np.float32)
    bins = np.ascontiguousarray(bins, np.int32)
    w = np.zeros((nb, 5), np.int64)
    lib().or_exact_words(_p(vals), _p(bins), len(vals), nb, _p(w))
    return w


def exact_read(words):
    w = np.ascontiguousarray(words, np.int64)
    bad = np.zeros(1, np.int32)
    o = lib().or_exact_read(_p(w), _p(bad))
    return np.float32(o), bool(bad[0])


# ----------------------------------------------------------------------------------------------- programs
def q1_fwd(x0, keys, theta, max_steps=100, nthreads=1, f64acc=True):
    """f64acc: f32 tallies accumulated in f64 and rounded once (the checker); False: the reference host target's f32
    partials (the timed CPU baseline)."""
    x0 = np.ascontiguousarray(x0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    n = len(x0)
    hist = np.zeros(16, np.float32)
    k = np.zeros(n, np.int32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_q1_fwd(n, _p(x0), _p(keys), float(theta), max_steps, nthreads, _p(hist), _p(k), _p(tr), _p(st),
                    int(f64acc))
    return dict(hist=hist, k=k, trunc=tr.astype(bool), stats=st)


def q1_grad(x0, keys, theta, ct, max_steps=100, C=16, nthreads=1):
    x0 = np.ascontiguousarray(x0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    ct = np.ascontiguousarray(ct, np.float32)
    n = len(x0)
    g = np.zeros(1, np.float32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_q1_grad(n, _p(x0), _p(keys), float(theta), _p(ct), max_steps, C, nthreads, _p(g), _p(tr), _p(st))
    return dict(g=g, trunc=tr.astype(bool), stats=st)


def rw_fwd(x0, keys, drift, max_steps=20000, nthreads=1, f64acc=True):
    x0 = np.ascontiguousarray(x0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    n = len(x0)
    hist = np.zeros(256, np.float32)
    side = np.zeros(2, np.float32)
    k = np.zeros(n, np.int32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_rw_fwd(n, _p(x0), _p(keys), float(drift), max_steps, nthreads, _p(hist), _p(side), _p(k), _p(tr),
                    _p(st), int(f64acc))
    return dict(hist=hist, side=side, k=k, trunc=tr.astype(bool), stats=st)


def rw_grad(x0, keys, drift, ct, max_steps=20000, C=16, nthreads=1):
    x0 = np.ascontiguousarray(x0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    ct = np.ascontiguousarray(ct, np.float32)
    n = len(x0)
    g = np.zeros(1, np.float32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_rw_grad(n, _p(x0), _p(keys), float(drift), _p(ct), max_steps, C, nthreads, _p(g), _p(tr), _p(st))
    return dict(g=g, trunc=tr.astype(bool), stats=st)


def ph_fwd(keys, mu_a=0.1, mu_s=10.0, max_steps=100000, nthreads=0, f64acc=True, libm=False):
    keys = np.ascontiguousarray(keys, np.uint32)
    n = len(keys)
    dep = np.zeros(64 ** 3, np.float32)
    k = np.zeros(n, np.int32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_ph_fwd(n, _p(keys), mu_a, mu_s, max_steps, nthreads, _p(dep), _p(k), _p(tr), _p(st), int(f64acc),
                    int(libm))
    return dict(dep=dep.reshape(64, 64, 64), k=k, trunc=tr.astype(bool), stats=st)


def ph_grad(keys, mu_a=0.1, mu_s=10.0, ct=None, max_steps=100000, C=16, nthreads=0, libm=False):
    keys = np.ascontiguousarray(keys, np.uint32)
    ct = np.ones(64 ** 3, np.float32) if ct is None else np.ascontiguousarray(ct, np.float32).reshape(-1)
    n = len(keys)
    g = np.zeros(2, np.float32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_ph_grad(n, _p(keys), mu_a, mu_s, _p(ct), max_steps, C, nthreads, _p(g), _p(tr), _p(st), int(libm))
    return dict(g=g, trunc=tr.astype(bool), stats=st)


MATH_FN = {"log": 0, "exp": 1, "sin": 2, "cos": 3, "pow": 4, "atan": 5, "atan2": 6, "asin": 7, "acos": 8, "tan": 9,
           "sinh": 10, "cosh": 11, "asinh": 12, "acosh": 13, "atanh": 14, "exp2": 15, "log2": 16, "cbrt": 17,
           "erf": 18, "erfc": 19, "erfinv": 20, "nextafter": 21, "lgamma": 22}


def math(fn, x, y=None):
    """the backend's shared f32 math evaluated on the host"""
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(np.zeros_like(x) if y is None else y, np.float32)
    out = np.zeros_like(x)
    lib().or_math(MATH_FN[fn], _p(x), _p(y), _p(out), len(x))
    return out


def od_inputs(n, seed=3):
    """benchmark configuration 4's synthetic inputs: sigma ~ U(9, 11), rho ~ U(26, 30), y0 ~ N((1, 1, 1), 0.1^2), f32"""
    rng = np.random.default_rng(seed)
    sigma = rng.uniform(9, 11, n).astype(np.float32)
    rho = rng.uniform(26, 30, n).astype(np.float32)
    y0 = (1.0 + 0.1 * rng.standard_normal((n, 3))).astype(np.float32)
    return sigma, rho, y0, np.arange(n, dtype=np.int32)


def od_fwd(sigma, rho, y0, item_id, beta=8.0 / 3.0, max_steps=50000, nthreads=0, f64acc=True):
    sigma, rho = np.ascontiguousarray(sigma, np.float32), np.ascontiguousarray(rho, np.float32)
    y0, item_id = np.ascontiguousarray(y0, np.float32), np.ascontiguousarray(item_id, np.int32)
    n = len(sigma)
    fin = np.zeros(3 * n, np.float32)
    mean = np.zeros(1, np.float32)
    k = np.zeros(n, np.int32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_od_fwd(n, _p(sigma), _p(rho), _p(y0), _p(item_id), np.float32(beta), max_steps, nthreads, _p(fin),
                    _p(mean), _p(k), _p(tr), _p(st), int(f64acc))
    return dict(final=fin.reshape(n, 3), mean=mean, k=k, trunc=tr.astype(bool), stats=st)


def od_grad(sigma, rho, y0, item_id, beta=8.0 / 3.0, ct_final=None, ct_mean=1.0, max_steps=50000, C=16, nthreads=0):
    sigma, rho = np.ascontiguousarray(sigma, np.float32), np.ascontiguousarray(rho, np.float32)
    y0, item_id = np.ascontiguousarray(y0, np.float32), np.ascontiguousarray(item_id, np.int32)
    n = len(sigma)
    ctf = np.ones(3 * n, np.float32) if ct_final is None else np.ascontiguousarray(ct_final, np.float32).reshape(-1)
    ctm = np.array([ct_mean], np.float32)
    g = np.zeros(1, np.float32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_od_grad(n, _p(sigma), _p(rho), _p(y0), _p(item_id), np.float32(beta), _p(ctf), _p(ctm), max_steps, C,
                     nthreads, _p(g), _p(tr), _p(st))
    return dict(g=g, trunc=tr.astype(bool), stats=st)


def od_vg1(sigma, rho, y0, item_id, beta=8.0 / 3.0, ct_final=None, ct_mean=1.0, max_steps=50000, nthreads=0):
    """forward mode w.r.t. beta in the backend's one-pass order (programs.cpp OdVG1): the exact gradient g f32[1],
    the trip counts and truncation flags"""
    sigma, rho = np.ascontiguousarray(sigma, np.float32), np.ascontiguousarray(rho, np.float32)
    y0, item_id = np.ascontiguousarray(y0, np.float32), np.ascontiguousarray(item_id, np.int32)
    n = len(sigma)
    ctf = np.ones(3 * n, np.float32) if ct_final is None else np.ascontiguousarray(ct_final, np.float32).reshape(-1)
    ctm = np.array([ct_mean], np.float32)
    g = np.zeros(1, np.float32)
    k = np.zeros(n, np.int32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_od_vg1(n, _p(sigma), _p(rho), _p(y0), _p(item_id), np.float32(beta), _p(ctf), _p(ctm), max_steps,
                    nthreads, _p(g), _p(k), _p(tr), _p(st))
    return dict(g=g, k=k, trunc=tr.astype(bool), stats=st)


def sh_inputs(n, seed=5):
    """benchmark configuration 5's primaries: E0 = exp(U(0, ln 1000)) (numpy default_rng(5)), depth 0, keys split(PRNGKey(5))"""
    import sys
    import os
    sys.path.insert(0, os.path.dirname(HERE))
    from tallymap_b200 import prng
    rng = np.random.default_rng(seed)
    E0 = np.exp(rng.uniform(0.0, np.log(1000.0), n)).astype(np.float32)
    return E0, np.zeros(n, np.float32), prng.split(prng.PRNGKey(5), n)


def sh_fwd(E0, d0, keys, X0=1.0, max_steps=100000, nthreads=0, f64acc=True):
    E0, d0 = np.ascontiguousarray(E0, np.float32), np.ascontiguousarray(d0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    n = len(E0)
    dep = np.zeros(512, np.float32)
    count = np.zeros(1, np.int32)
    k = np.zeros(n, np.int32)
    tr = np.zeros(n, np.uint8)
    st = np.zeros(5, np.int32)
    lib().or_sh_fwd(n, _p(E0), _p(d0), _p(keys), X0, max_steps, nthreads, _p(dep), _p(count), _p(k), _p(tr), _p(st),
                    int(f64acc))
    return dict(dep=dep, count=count, k=k, trunc=tr.astype(bool), stats=st)


def sh_vg1(E0, d0, keys, X0=1.0, ct_dep=None, max_steps=100000, nthreads=0):
    """the one-pass shower gradient (forward mode through spawn, exact per-root sums): g_E[n]"""
    E0, d0 = np.ascontiguousarray(E0, np.float32), np.ascontiguousarray(d0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    n = len(E0)
    ct = np.ones(512, np.float32) if ct_dep is None else np.ascontiguousarray(ct_dep, np.float32)
    gE = np.zeros(n, np.float32)
    st = np.zeros(5, np.int32)
    lib().or_sh_vg1(n, _p(E0), _p(d0), _p(keys), X0, _p(ct), max_steps, nthreads, _p(gE), _p(st))
    return dict(g_E=gE, stats=st)


def sh_grad(E0, d0, keys, X0=1.0, ct_dep=None, max_steps=100000, nthreads=0):
    """the shower's tree adjoint: d <ct_dep, dep> / d (X0, E0, depth0)"""
    E0, d0 = np.ascontiguousarray(E0, np.float32), np.ascontiguousarray(d0, np.float32)
    keys = np.ascontiguousarray(keys, np.uint32)
    n = len(E0)
    ct = np.ones(512, np.float32) if ct_dep is None else np.ascontiguousarray(ct_dep, np.float32)
    gx = np.zeros(1, np.float32)
    gE = np.zeros(n, np.float32)
    gD = np.zeros(n, np.float32)
    st = np.zeros(5, np.int32)
    lib().or_sh_grad(n, _p(E0), _p(d0), _p(keys), X0, _p(ct), max_steps, nthreads, _p(gx), _p(gE), _p(gD), _p(st))
    return dict(g_X0=gx, g_E=gE, g_depth=gD, stats=st)
