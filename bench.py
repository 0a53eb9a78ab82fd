#!/usr/bin/env python
"""Benchmark of the tallymap B200 backend on benchmark configuration 2: the 1-D random walk, N = 4,194,304 items per GPU.

One STEP = the forward outputs plus the reverse-mode gradient (w.r.t. the broadcast `drift`, cotangent ones on the
hist tally) over the step's items: "Mitems/s fwd & grad".  The step is timed as the ONE value-and-grad launch that
value_and_grad runs where the item has one: for an item with no active carry (the walkers) the one-pass program,
which sums each step's VJP as the forward runs (the gradient within the float tolerance of the reverse program's;
--exact-order times the fused replay instead, bitwise the reverse program's summation order), else the fused
replay whose count pass is the forward; otherwise (--unfused, or items without one) a forward launch then the
replay launch, whose threads claim items longest first by the forward's trip counts (a device argsort inside the
step); the separate forward and gradient (replay) times are reported too (fwd_ms, grad_ms).  Inputs (x0 ~ U(0,1) from PRNGKey(1)'s first subkey, per-item keys split from the
second) are synthetic, made with jax.random's algorithm on the host (tallymap_b200.prng).  Weak scaling: each rank
runs its own 4,194,304 items (a contiguous slice of the global item set) and the partial tallies are combined with
one NCCL collective step (all_reduce of the f32 / i32 tallies, all_gather + on-device combine of the exact gradient
words).

  python bench.py [--gpus N --steps K --warmup W]            # this backend (N > 1: under torchrun)
  python bench.py --impl reference [...]                    # the reference's CPU path, timed on the host cores

Timing: W untimed warm-up steps; K timed steps, each bracketed by CUDA events on the launching stream, L2 flushed
(a 256 MiB write) between steps outside the events; barrier + synchronize around the timed loop; the max over ranks.
`e2e` repeats the step through the public API (tallymap_b200.vmap(...).value_and_grad) from pinned host inputs,
copies and the result read-back inside the timed region.  `roofline`: the walkers are integer-issue bound (two
threefry2x32 per step, 79 INT32 ops each, dominate); the peak is the same device's measured threefry2x32 rate at
full occupancy (tm_probe_threefry), so frac = the fraction of issue-rate speed of light the kernel reaches.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ITEMS = 4194304
MAX_STEPS = 20000
TF_OPS = 79          # INT32 ops per threefry2x32 (2 XOR + 2 ADD + 20 x (ADD, ROTL, XOR) + 5 x 3 ADD)
METRIC = "Mitems/s fwd & grad at N=4M, 1/2/4/8 B200, % of roofline vs host CPU"
WARM_S = 0.25        # seconds of untimed warm-up work at least (the GPU's clock ramps up over the first few ms)
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per item of one launch, from the ncu captures summarised
# under profiles/ (kernel -> (bytes per item, items in the capture)); the bench scales them to its own launch
TRAFFIC = {
    "rw_vg_onepass": ((13003008 + 0) / 1048576, 1048576),
    "ph_vg_onepass": ((9116416 + 512) / 1048576, 1048576),
    "rw_vg": ((38916657408 + 37082540288) / 4194304, 4194304),
    "rw_grad": ((5.241173e9 + 6.034955e9) / 1048576, 1048576),
    "rw_fwd": ((53075712 + 3524096) / 4194304, 4194304),
    "ph_fwd": ((10.557440e6 + 0.0) / 1048576, 1048576),
    "od_grad": ((3.060892e9 + 3.133417e9) / 262144, 262144),
    "od_fwd": ((0.009466e9 + 0.0) / 262144, 262144),
    "od_vg_onepass": ((12634368 + 0) / 262144, 262144),
}


def rw_inputs(n, start=0, total=None):
    from tallymap_b200 import prng
    kx, ks = prng.split(prng.PRNGKey(1), 2)
    return prng.uniform(kx, n, start=start), prng.split(ks, n, start=start)


def q1_inputs(n, start=0, total=None):
    from tallymap_b200 import prng
    total = total or start + n
    return (np.linspace(0.1, 0.99, total, dtype=np.float32)[start:start + n].copy(),
            prng.split(prng.PRNGKey(0), n, start=start))


def od_inputs(n, start=0, total=None):
    """benchmark configuration 4: sigma ~ U(9, 11), rho ~ U(26, 30), y0 ~ N((1, 1, 1), 0.1^2) (numpy default_rng(3), as the
    reference's benchmarks make host inputs), item_id = the global item index"""
    total = total or start + n
    rng = np.random.default_rng(3)
    sigma = rng.uniform(9, 11, total).astype(np.float32)[start:start + n]
    rho = rng.uniform(26, 30, total).astype(np.float32)[start:start + n]
    y0 = (1.0 + 0.1 * rng.standard_normal((total, 3))).astype(np.float32)[start:start + n]
    return sigma.copy(), rho.copy(), y0.copy(), np.arange(start, start + n, dtype=np.int32)


def sh_inputs(n, start=0, total=None):
    """benchmark configuration 5: E0 = exp(U(0, ln 1000)) (numpy default_rng(5)), depth 0, keys split(PRNGKey(5))"""
    from tallymap_b200 import prng
    total = total or start + n
    rng = np.random.default_rng(5)
    E0 = np.exp(rng.uniform(0.0, np.log(1000.0), total)).astype(np.float32)[start:start + n]
    return E0.copy(), np.zeros(n, np.float32), prng.split(prng.PRNGKey(5), n, start=start)


def ph_inputs(n, start=0, total=None):
    from tallymap_b200 import prng
    return (prng.split(prng.PRNGKey(2), n, start=start),)


class Cfg:
    """one benchmark configuration: programs, inputs, and the threefry2x32 count of a forward step (tf) and of a
    replay step VJP (tf_vjp)."""

    def __init__(self, name, fwd, grad, inputs, bc, ct, tallies, max_steps, tf, tf_vjp, items, workload):
        self.name, self.fwd, self.grad, self.inputs, self.bc, self.ct = name, fwd, grad, inputs, bc, ct
        self.tallies, self.max_steps, self.tf, self.tf_vjp, self.items = tallies, max_steps, tf, tf_vjp, items
        self.workload = workload


def configs(B):
    return {
        "rw": Cfg("rw", B.RW_FWD, B.RW_GRAD, rw_inputs, [1.0], [np.ones(256, np.float32), np.zeros(2, np.float32)],
                  ["hist", "side"], 20000, 2, 0, N_ITEMS,
                  "1-D random walk (benchmark configuration 2): forward + grad w.r.t. drift"),
        "ph": Cfg("ph", B.PH_FWD, B.PH_GRAD, ph_inputs, [0.1, 10.0], [np.ones((64, 64, 64), np.float32)], ["dep"],
                  100000, 5, 3, N_ITEMS,
                  "photon slab (benchmark configuration 3): forward + grad w.r.t. (mu_a, mu_s)"),
        "q1": Cfg("q1", B.Q1_FWD, B.Q1_GRAD, q1_inputs, [2.0], [np.ones(16, np.float32)], ["hist"], 100, 2, 0, 10000,
                  "quickstart walker (benchmark configuration 1): forward + grad w.r.t. theta"),
        "od": Cfg("od", B.OD_FWD, B.OD_GRAD, od_inputs, [8.0 / 3.0], ["ones(N,3)", np.float32(1.0)],
                  ["final", "mean_z"], 50000, 0, 0, 1048576,
                  "Lorenz RK45 ensemble (benchmark configuration 4): forward + replay grad w.r.t. beta"),
        # the separate gradient is the tree adjoint: the recording forward, the generation lists, one adjoint launch
        # per generation and one over the roots (backend.tree_grad); the step is the one-pass spawn launch (forward
        # mode through spawn) unless --exact-order
        "sh": Cfg("sh", B.SH_FWD, B.SH_GRAD, sh_inputs, [1.0], [np.ones(512, np.float32)], ["dep", "count"], 100000,
                  0, 0, 1048576,
                  "branching shower (benchmark configuration 5): forward + grad w.r.t. the roots' E0 and X0 (items = roots)"),
    }


FAM = {"rw": "walk1d", "ph": "photon", "q1": "quickstart", "od": "lorenz", "sh": "shower"}


OD_FP32_OPS = 255     # f32 add / mul / min / max / abs / compare of one Lorenz RK45 trial step (+ 3 div, 1 sqrt, 1 pow)


def od_roofline(_lib, stream, dev, steps, micro, f_ms, g_ms, grad_kernel, fwd_kernel, v_ms=None, vg_kernel=None):
    """The Lorenz ensemble's roofline: its bound is the issue rate of its own instruction mix (six stage
    evaluations, the error norm, an f32 pow in the shared double-precision math, the accept decision), so the peaks
    are tm_probe_issue's probes of that mix at full occupancy: P0 trial steps/s (kind 2) and P1 (trial step + step
    VJP)/s (kind 3).  The forward runs `steps` trial steps; the replay `micro` forward step evaluations (count,
    checkpoint and fill passes) and one step VJP per trial step.  Ideal times: forward steps / P0; replay
    steps / P1 + (micro - steps) / P0.  achieved is in forward-step equivalents (a VJP pair counts P0 / P1), so
    frac = ideal time / measured time.  `micro` is replay_micro_steps: the forward evaluations of the count,
    checkpoint and fill passes plus one per step VJP, so the forward evaluations alone are micro - steps, of which
    `steps` pair with the VJPs (the probe's kind 3 iteration: a trial step and a step VJP).  Beside it the FP32 pipe:
    the trial steps' algorithmic f32 operations over the forward time against the probe's FP32 instruction rate
    (kind 1).  With the one-pass forward-mode launch timed (v_ms): its peak P2 = (trial step + stage tangents)/s
    (kind 5), ideal time steps / P2, and it is the headline entry (the step the bench times)."""
    p0, _ = _lib.probe_rate(_lib.PROBE_ODE_STEP, 512, stream, dev)
    p1, _ = _lib.probe_rate(_lib.PROBE_ODE_STEP_VJP, 256, stream, dev)
    pf, _ = _lib.probe_rate(_lib.PROBE_FP32, 8192, stream, dev)
    pf *= 16
    g_s, f_s = g_ms / 1e3, f_ms / 1e3
    ideal_g = steps / p1 + max(micro - 2 * steps, 0) / p0
    ideal_f = steps / p0
    eq = ideal_g * p0
    if v_ms is not None:
        p2, _ = _lib.probe_rate(_lib.PROBE_ODE_STEP_JVP, 256, stream, dev)
        v_s = v_ms / 1e3
        r = od_roofline(_lib, stream, dev, steps, micro, f_ms, g_ms, grad_kernel, fwd_kernel)
        r["modes"]["vg"] = {"kernel": vg_kernel, "achieved": round(steps / v_s / 1e9, 4),
                            "frac": round(steps / p2 / v_s, 4)}
        r.update({"kernel": vg_kernel, "achieved": round(steps / v_s / 1e9, 4), "peak": round(p2 / 1e9, 4),
                  "unit": "G trial steps with tangents/s", "frac": round(steps / p2 / v_s, 4),
                  "peak_source": "measured: tm_probe_issue kind 5 (the item's trial step with its stages' tangents at "
                                 "full occupancy, no divergence or memory) on this GPU",
                  "work": f"{steps} trial steps (accepted + rejected), each with its stages' tangents"})
        r["probe"]["p2_step_jvp_per_s"] = round(p2, 1)
        return r
    return {"bound": "issue", "kernel": grad_kernel, "achieved": round(eq / g_s / 1e9, 4), "peak": round(p0 / 1e9, 4),
            "unit": "G trial-step equivalents/s", "frac": round(ideal_g / g_s, 4), "traffic": None,
            "peak_source": "measured: tm_probe_issue kind 2 (the item's trial step at full occupancy, no "
                           "divergence or memory) and kind 3 (trial step + step VJP) on this GPU",
            "work": f"{steps} trial steps (accepted + rejected); the replay: {micro - steps} forward step "
                    f"evaluations (count, checkpoint, fill) and one step VJP per trial step",
            "probe": {"p0_steps_per_s": round(p0, 1), "p1_step_vjp_per_s": round(p1, 1)},
            "modes": {"fwd": {"kernel": fwd_kernel, "achieved": round(steps / f_s / 1e9, 4),
                              "frac": round(ideal_f / f_s, 4)},
                      "grad": {"kernel": grad_kernel, "achieved": round(eq / g_s / 1e9, 4),
                               "frac": round(ideal_g / g_s, 4)},
                      "step": {"frac": round((ideal_f + ideal_g) / (f_s + g_s), 4)}},
            "fp32": {"ops_per_trial_step": OD_FP32_OPS, "kernel": fwd_kernel,
                     "achieved_tops": round(steps * OD_FP32_OPS / f_s / 1e12, 3), "peak_tops": round(pf / 1e12, 3),
                     "frac": round(steps * OD_FP32_OPS / f_s / pf, 4),
                     "peak_source": "measured: tm_probe_issue kind 1 (independent f32 multiply and add chains)"}}


def replay_micro_steps(K, C):
    """loop-step evaluations of the checkpointed replay (count, checkpoint, advance + fill, sweep) for trip counts K,
    summed: the schedule of tallymap/_reverse.py:343-440."""
    ks, cnt = np.unique(np.asarray(K, np.int64), return_counts=True)
    m = np.maximum(C, (ks + C - 1) // C)
    ns = (ks + m - 1) // m
    tot = ks + np.where(ns > 1, (ns - 1) * m, 0)           # count pass + checkpoint pass
    for s in range(C):
        L = np.clip(ks - s * m, 0, m)
        live = (s < ns) & (L > 0)
        nsub = (L + C - 1) // C
        for u in range(int(nsub.max()) if live.any() else 0):
            LL = np.clip(L - u * C, 0, C)
            ok = live & (u < nsub)
            first = (s == 0) & (u == 0)
            fill = np.where(first, 0, u * C + LL - 1)
            tot = tot + np.where(ok, fill + LL, 0)
    return int((tot * cnt).sum())


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region (SM clock, throttle reasons)."""
    Q = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus = bus_id          # the PCI bus number of this rank's device (torch), or None
        self.rows, self.proc, self.err = [], None, None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError as e:
            self.err = str(e)

    def _read(self):
        for ln in self.proc.stdout:
            self.rows.append([c.strip() for c in ln.split(",")])

    def stop(self):
        # a timed region shorter than nvidia-smi's start-up and sampling interval (Q1's: well under a millisecond a
        # step) ends before the first sample: then wait for one, taken right after the region, and say so
        late = False
        if self.proc and not self.rows:
            late = True
            t_end = time.time() + 3.0
            while not self.rows and time.time() < t_end and self.proc.poll() is None:
                time.sleep(0.01)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        def bus(r):
            try:
                return int(r[1].split(":")[1], 16)
            except (IndexError, ValueError):
                return None
        rows = [r for r in self.rows if len(r) >= 10]
        mine = [r for r in rows if self.bus is not None and bus(r) == self.bus] or rows
        if not mine:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": self.err or "nvidia-smi unavailable"}
        sm = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in mine for n, v in zip(names, r[6:10]) if v.strip().lower() == "active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None,
               "sm_max_mhz": float(mine[0][3]) if mine[0][3].replace(".", "").isdigit() else None,
               "reasons": reasons, "samples": len(mine)}
        if late:
            out["note"] = "timed region shorter than the sampling interval: sampled right after it"
        return out


# ------------------------------------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle
    oracle.build()
    from tallymap_b200 import backend as B
    cfg = configs(B)[args.config]
    nth = len(os.sched_getaffinity(0))
    os.environ.setdefault("OMP_PROC_BIND", "close")
    host = cfg.inputs(args.items or cfg.items, 0)
    n, dt, _ = cpu_rate(cfg, host, 2.0, nth)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle_step(cfg, host, n, nth)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    v = n / (ms / 1e3) / 1e6
    sample = (f"first {n} of the {len(host[0])} items per step (fwd + grad), the reference host target's model (f32 "
              f"tallies, libm), {nth} OpenMP threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "Mitems/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32+u32", "data": "synthetic (jax.random algorithm, host)",
        "config": {"workload": cfg.workload, "items_per_gpu": len(host[0]), "max_steps": cfg.max_steps,
                   "sample_items": n},
        "cpu_baseline": {"value": round(v, 4), "unit": "Mitems/s", "cores": nth, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "Mitems/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference (JAX) cannot run on this image (jax is not installed, no network): this is the "
                "oracle/ C++ restatement of its CPU kernel target"}), flush=True)


# ------------------------------------------------------------------------------------------------ our arm
def oracle_step(cfg, host, n, nth):
    """one fwd + grad of the first n items on the host cores: the oracle in the reference host target's mode (f32
    tallies; libm transcendentals)"""
    from oracle import oracle
    if cfg.name == "rw":
        oracle.rw_fwd(host[0][:n], host[1][:n], 1.0, nthreads=nth, f64acc=False)
        oracle.rw_grad(host[0][:n], host[1][:n], 1.0, np.ones(256, np.float32), nthreads=nth)
    elif cfg.name == "q1":
        oracle.q1_fwd(host[0][:n], host[1][:n], 2.0, nthreads=nth, f64acc=False)
        oracle.q1_grad(host[0][:n], host[1][:n], 2.0, np.ones(16, np.float32), nthreads=nth)
    elif cfg.name == "od":
        h = [a[:n] for a in host]
        oracle.od_fwd(*h, nthreads=nth, f64acc=False)
        oracle.od_grad(*h, nthreads=nth)
    elif cfg.name == "sh":
        h = [a[:n] for a in host]
        oracle.sh_fwd(*h, nthreads=nth, f64acc=False)
        oracle.sh_grad(*h, nthreads=nth)
    else:
        oracle.ph_fwd(host[0][:n], nthreads=nth, f64acc=False, libm=True)
        oracle.ph_grad(host[0][:n], nthreads=nth, libm=True)


def oracle_check(cfg, pre, nth):
    """the oracle in its checker mode (the backend's shared math, f64 tally partials) on the items `pre` -> dict with
    the per-item k and trunc"""
    from oracle import oracle
    if cfg.name == "rw":
        return oracle.rw_fwd(pre[0], pre[1], 1.0, max_steps=cfg.max_steps, nthreads=nth)
    if cfg.name == "q1":
        return oracle.q1_fwd(pre[0], pre[1], 2.0, max_steps=cfg.max_steps, nthreads=nth)
    if cfg.name == "ph":
        return oracle.ph_fwd(pre[0], max_steps=cfg.max_steps, nthreads=nth)
    if cfg.name == "od":
        return oracle.od_fwd(*pre, max_steps=cfg.max_steps, nthreads=nth)
    return oracle.sh_fwd(*pre, max_steps=cfg.max_steps, nthreads=nth)


def parity_block(cfg, host, runs, nth, prefix=262144, longest=1024):
    """Per-item parity of the timed launches against the oracle: the first `prefix` items and the `longest` items
    with the most steps (gathered by index: the heavy tail near max_steps), per-item trip counts and truncation
    flags bitwise.  runs: {launch name: (k, trunc) host arrays of the whole launch}.  Items are independent, so a
    prefix or a gathered subset has the same per-item results as the whole launch."""
    N = len(host[0])
    k0 = next(iter(runs.values()))[0]
    tail = np.sort(np.argsort(k0, kind="stable")[::-1][:min(longest, N)])
    idx = np.union1d(np.arange(min(prefix, N)), tail)
    t0 = time.perf_counter()
    ref = oracle_check(cfg, [np.ascontiguousarray(h[idx]) for h in host], nth)
    out = {"items": int(len(idx)), "of": N, "prefix": int(min(prefix, N)), "longest": int(len(tail)),
           "max_steps_compared": int(ref["k"].max()) if len(idx) else 0,
           "truncated_compared": int(ref["trunc"].sum()),
           "checker": "oracle/ (shared f32 math, f64 tally partials)", "host_s": None}
    for name, (k, tr) in runs.items():
        out[name] = {"k_bitwise": bool(np.array_equal(k[idx], ref["k"])),
                     "trunc_bitwise": bool(np.array_equal(tr[idx].astype(bool), ref["trunc"]))}
    out["host_s"] = round(time.perf_counter() - t0, 1)
    out["ok"] = all(v["k_bitwise"] and v["trunc_bitwise"] for v in out.values() if isinstance(v, dict))
    return out


def oracle_split(cfg, host, n, nth):
    """the CPU step's parts on the first n items, timed separately (seconds): the forward, the gradient in the
    reference's order (its checkpointed replay / tree adjoint), and -- where the GPU step runs a one-pass program --
    the gradient by the same one-pass algorithm, so the GPU-to-CPU ratio of like algorithms can be read off"""
    from oracle import oracle
    h = [a[:n] for a in host]
    parts = {}

    def timed(name, f):
        t0 = time.perf_counter()
        f()
        parts[name] = time.perf_counter() - t0
    if cfg.name == "rw":
        timed("fwd", lambda: oracle.rw_fwd(h[0], h[1], 1.0, nthreads=nth, f64acc=False))
        timed("grad", lambda: oracle.rw_grad(h[0], h[1], 1.0, np.ones(256, np.float32), nthreads=nth))
        timed("grad_onepass", lambda: oracle.rw_grad(h[0], h[1], 1.0, np.ones(256, np.float32), C=-1,
                                                     nthreads=nth))
    elif cfg.name == "q1":
        timed("fwd", lambda: oracle.q1_fwd(h[0], h[1], 2.0, nthreads=nth, f64acc=False))
        timed("grad", lambda: oracle.q1_grad(h[0], h[1], 2.0, np.ones(16, np.float32), nthreads=nth))
        timed("grad_onepass", lambda: oracle.q1_grad(h[0], h[1], 2.0, np.ones(16, np.float32), C=-1, nthreads=nth))
    elif cfg.name == "ph":
        timed("fwd", lambda: oracle.ph_fwd(h[0], nthreads=nth, f64acc=False, libm=True))
        timed("grad", lambda: oracle.ph_grad(h[0], nthreads=nth, libm=True))
        timed("grad_onepass", lambda: oracle.ph_grad(h[0], C=-1, nthreads=nth, libm=True))
    elif cfg.name == "od":
        timed("fwd", lambda: oracle.od_fwd(*h, nthreads=nth, f64acc=False))
        timed("grad", lambda: oracle.od_grad(*h, nthreads=nth))
        timed("grad_onepass", lambda: oracle.od_vg1(*h, nthreads=nth))
    else:
        timed("fwd", lambda: oracle.sh_fwd(*h, nthreads=nth, f64acc=False))
        timed("grad", lambda: oracle.sh_grad(*h, nthreads=nth))
        timed("grad_onepass", lambda: oracle.sh_vg1(*h, nthreads=nth))
    return {k + "_mitems_s": round(n / v / 1e6, 4) for k, v in parts.items()}


def cpu_rate(cfg, host, target_s, nth):
    """-> (items, seconds, Mitems/s) of oracle_step on a prefix of the items sized to about target_s seconds"""
    n = min(4096, len(host[0]))
    while True:
        t0 = time.perf_counter()
        oracle_step(cfg, host, n, nth)
        dt = time.perf_counter() - t0
        if dt >= target_s or n >= len(host[0]):
            return n, dt, n / dt / 1e6
        n = min(len(host[0]), max(n * 2, int(n * target_s / max(dt, 1e-3) * 0.9)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="rw", choices=["rw", "ph", "q1", "od", "sh"])
    ap.add_argument("--items", type=int, default=None, help="items per GPU (default: the configuration's N)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the per-item parity check against the oracle")
    ap.add_argument("--index-order", action="store_true",
                    help="(the shower) claim roots in index order instead of largest energy first (the argsort "
                         "value_and_grad and the forward run inside the timed step)")
    ap.add_argument("--unfused", action="store_true", help="time the step as a forward and a replay launch")
    ap.add_argument("--exact-order", action="store_true",
                    help="time the fused replay (the reverse program's summation order, bitwise) instead of the "
                         "one-pass value-and-grad of an item with no active carry")
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.warmup < 3:
        raise SystemExit("bench.py: at least 3 warm-up steps")
    if world > 1:
        # NCCL's communicator setup on the log (its INIT lines show every rank joining the one communicator); set
        # before torch loads NCCL, which reads them once
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")

    import torch
    import torch.distributed as dist

    import tallymap_b200 as tm
    from tallymap_b200 import _lib
    from tallymap_b200 import backend as B
    from tallymap_b200 import parallel
    from tallymap_b200.api import longest_first

    cfg = configs(B)[args.config]
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    N = args.items or cfg.items
    host = cfg.inputs(N, rank * N, N * world)
    pi = [torch.from_numpy(h.view(np.int32) if h.dtype == np.uint32 else h).to(dev) for h in host]
    bc = [torch.tensor(v, dtype=torch.float32, device=dev) for v in cfg.bc]
    ct = [torch.ones((N, 3), device=dev) if isinstance(c, str) else torch.tensor(c, device=dev) for c in cfg.ct]
    tree = cfg.name == "sh"
    fo = B.alloc_results(cfg.fwd, N, dev)
    go = None if tree else B.alloc_results(cfg.grad, N, dev, max_steps=cfg.max_steps)
    nb = cfg.grad.tallies[0].S
    g_all = torch.zeros(nb, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    gnames = None if tree else [n for n, _, _, _ in cfg.grad.result_layout(N)[0]]
    ntal = len(cfg.fwd.tallies)
    tree_info = {}

    # the claim order the public API gives the launch (the shower: roots largest energy first), computed every step
    claim = None if args.index_order else tm.FAMILIES[FAM[cfg.name]].claim_order

    def fwd():
        out = B.run(cfg.fwd, pi, bc, consts=(cfg.max_steps,), out=fo, order=claim(pi) if claim else None)
        if world > 1:
            parallel.all_reduce_sums(out[:ntal + 1])
        return out

    def grad():
        if tree:
            r = B.tree_grad(pi, bc[0], ct[0], max_steps=cfg.max_steps)
            tree_info.update(r["info"])
            if world > 1:
                parallel.combine_exact(r["words"], nb, g_all, r["stats"])
            return r
        # the replay claims items longest first by the forward's trip counts (as value_and_grad does)
        order = longest_first(fo[-2])
        out = B.run(cfg.grad, pi, bc + ct, consts=(cfg.max_steps,), out=go, order=order)
        if world > 1:
            parallel.combine_exact(go[gnames.index(cfg.grad.tallies[0].name + ".exact")], nb, g_all,
                                   go[gnames.index("stats")])
        return out

    # the value-and-grad launch value_and_grad runs for cotangents given up front, when the item has one: the one-pass
    # program for an item with no active carry (unless --exact-order), else the pipelined fused replay
    wkey = (0,) if len(cfg.bc) == 1 else tuple(range(len(cfg.bc)))
    fam_ = tm.FAMILIES[FAM[cfg.name]]
    fused = None if (tree or args.unfused) else (None if args.exact_order else fam_.onepass.get(wkey))
    if fused is None and not (tree or args.unfused):
        fused = fam_.fused.get(wkey)
        if fused is not None and not B.pipelined(fused, cfg.max_steps, dev):
            fused = None              # (as value_and_grad: the fused replay would be slower than two launches)
    # the shower's one spawn launch (forward mode through spawn), what value_and_grad runs for it
    sh_vg = tree and not (args.unfused or args.exact_order)
    if sh_vg:
        fused = B.SH_VG1
    vo = None if fused is None else B.alloc_results(fused, N, dev, max_steps=cfg.max_steps)
    vnames = None if fused is None else [n for n, _, _, _ in fused.result_layout(N)[0]]

    def vg():
        if sh_vg:
            r = B.sh_value_and_grad(pi, bc[0], ct[0], max_steps=cfg.max_steps, out=vo,
                                    order=claim(pi) if claim else None)
            if world > 1:
                parallel.all_reduce_sums([r["dep"], r["count"], r["stats"]])
            return r
        out = B.run(fused, pi, bc + ct, consts=(cfg.max_steps,), out=vo)
        if world > 1:
            parallel.all_reduce_sums(out[:ntal] + [out[ntal + 1]])
            parallel.combine_exact(vo[vnames.index(fused.tallies[-1].name + ".exact")], nb, g_all,
                                   vo[vnames.index("stats")])
        return out

    def warm():
        fwd()
        grad()
        if fused is not None:
            vg()

    for _ in range(args.warmup):
        warm()
    torch.cuda.synchronize()
    # then more (untimed) warm-up steps, about WARM_S of work: a configuration whose step is well under a millisecond
    # (Q1) otherwise times its steps while the GPU's clock is still ramping up (0.26 ms a step after 3 warm-up steps,
    # 0.05 ms after 20).  The count from one more step's time (the first ones include one-time set-up), the same on
    # every rank (their steps hold collectives).
    t_w = time.perf_counter()
    warm()
    torch.cuda.synchronize()
    per = time.perf_counter() - t_w
    extra = max(0, min(10000, int(WARM_S / max(per, 1e-6))))
    if world > 1:
        te = torch.tensor([extra], dtype=torch.int64, device=dev)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        extra = int(te.item())
    for _ in range(extra):
        warm()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = Clocks(getattr(torch.cuda.get_device_properties(dev), "pci_bus_id", None))
    clocks.start()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    evf = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # (1) the step as two launches: the forward, then the gradient (replay) alone -- the reference's two numbers
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        fwd()
        ev[i][1].record(stream)
        grad()
        ev[i][2].record(stream)
    # (2) the step as one fused value-and-grad launch
    if fused is not None:
        for i in range(args.steps):
            flush.zero_()
            evf[i][0].record(stream)
            vg()
            evf[i][1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    f_ms = sum(e[0].elapsed_time(e[1]) for e in ev)
    g_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    v_ms = sum(e[0].elapsed_time(e[1]) for e in evf) if fused is not None else 0.0
    t = torch.tensor([f_ms + g_ms, f_ms, g_ms, v_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    sep_ms, f_ms, g_ms, v_ms = (float(v) / args.steps for v in t.tolist())
    tot_ms = v_ms if fused is not None else sep_ms
    value = N * world / (tot_ms / 1e3) / 1e6

    # ---- e2e: the public API from pinned host inputs, H2D + both launches + result read-back timed
    fam = FAM[cfg.name]
    F = tm.FAMILIES[fam]
    f = tm.vmap(fam, outputs={t.name: tm.Sum(t.dims(N), t.dtype) for t in F.fwd.tallies}, in_axes=F.in_axes,
                max_steps=cfg.max_steps)
    pinned = [p.cpu().pin_memory() for p in pi]
    wrt = tuple(i for i, ax in enumerate(F.in_axes) if ax is None)
    cts = {t.name: c for t, c in zip(F.fwd.tallies, ct)}
    d2h = [0]

    def e2e_step():
        r, g = f.value_and_grad(*pinned, *bc, wrt=wrt if len(wrt) > 1 else wrt[0], cotangents=cts)
        outs = [r.outputs[t.name] for t in F.fwd.tallies] + [r.stats["n_truncated"].reshape(1), g.reshape(-1)]
        if world > 1:
            parallel.all_reduce_sums(outs[:-1])
        host_out = [o.to("cpu") for o in outs]
        d2h[0] = sum(h.numel() * h.element_size() for h in host_out)
        return host_out

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_ms = 0.0
    for i in range(args.steps):
        flush.zero_()
        e0.record(stream)
        e2e_step()
        e1.record(stream)
        e1.synchronize()
        e2e_ms += e0.elapsed_time(e1)
    te = torch.tensor([e2e_ms / args.steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = N * world / (float(te.item()) / 1e3) / 1e6

    # ---- roofline of the dominant kernel: threefry2x32 evaluations per second against the probe's
    fnames = [n for n, _, _, _ in cfg.fwd.result_layout(N, 0, B.QUEUE_DEFAULT if tree else 0)[0]]
    kk = fo[fnames.index("k")].to("cpu").numpy()
    steps_total = int(kk.astype(np.int64).sum())
    tf_fwd = cfg.tf * steps_total
    C_used = B.replay_plan(cfg.grad, cfg.max_steps, None, dev)[0]
    # the replay evaluates forward steps in its count, checkpoint and fill passes (cfg.tf threefry2x32 each) and one
    # step VJP per step (cfg.tf_vjp each)
    tf_grad = cfg.tf * (replay_micro_steps(kk, C_used) - steps_total) + cfg.tf_vjp * steps_total
    import ctypes
    pout = torch.empty(148 * 2048 * 2, dtype=torch.int32, device=dev)
    used = ctypes.c_int64()
    pe = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    iters = 4096
    for rep in range(3):
        pe[0].record(stream)
        _lib.check(_lib.lib().tm_probe_threefry(ctypes.c_void_p(stream.cuda_stream), iters,
                                                ctypes.c_void_p(pout.data_ptr()), pout.numel(), ctypes.byref(used)))
        pe[1].record(stream)
    torch.cuda.synchronize()
    peak = used.value * iters / (pe[0].elapsed_time(pe[1]) / 1e3) / 1e9
    dom = (cfg.grad.kernel, tf_grad, g_ms) if g_ms >= f_ms else (cfg.fwd.kernel, tf_fwd, f_ms)
    if fused is not None and not fused.replay_state_bytes:
        # the one-pass launch: each forward step once (cfg.tf threefry2x32); its gradient part draws nothing
        dom = (fused.kernel, cfg.tf * steps_total, v_ms)
    elif fused is not None:
        # the fused launch: the replay's schedule, its count pass being the forward (cfg.tf threefry2x32 per
        # evaluation), plus the step VJPs
        C_vg = B.replay_plan(fused, cfg.max_steps, None, dev)[0]
        tf_vg = cfg.tf * (replay_micro_steps(kk, C_vg) - steps_total) + cfg.tf_vjp * steps_total
        dom = (fused.kernel, tf_vg, v_ms)
    if sh_vg:
        # the shower's one spawn launch: every particle step draws 4 threefry2x32 (fold_in and three uniforms), every
        # split 2 more (fold_in of the step key for each of its two children: one per child spawned); the steps and
        # children counted by the launch itself
        r_last = B.sh_value_and_grad(pi, bc[0], ct[0], max_steps=cfg.max_steps, out=vo)   # (this rank's own counts)
        torch.cuda.synchronize()
        n_steps = int(r_last["steps"][0].item())
        n_spawned = int(r_last["stats"][0].item())
        dom = (fused.kernel, 4 * n_steps + n_spawned, v_ms)
    achieved = dom[1] / (dom[2] / 1e3) / 1e9
    tr = TRAFFIC.get(dom[0])
    traffic = None if tr is None else int(round(tr[0] * N))
    roofline = {"bound": "issue", "kernel": dom[0], "achieved": round(achieved, 2), "peak": round(peak, 2),
                "unit": "Gthreefry/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                "traffic_source": None if tr is None else
                f"ncu dram bytes read+write of one launch at N={tr[1]}, scaled by items to N={N}",
                "peak_source": "measured: tm_probe_threefry at full occupancy on this GPU",
                "achieved_int32_tops": round(achieved * TF_OPS / 1e3, 3),
                "work": (f"{dom[1]} threefry2x32 per launch (4 per particle step over {n_steps} steps, 1 per child "
                         f"-- 2 per split -- over {n_spawned} children; counted by the launch)") if sh_vg else
                        (f"{dom[1]} threefry2x32 per launch ({cfg.tf} per forward step, "
                         f"{0 if fused is not None and not fused.replay_state_bytes else cfg.tf_vjp} per step VJP; "
                         "steps from the per-item trip counts and the replay schedule)")} if (cfg.tf or sh_vg) else None
    if cfg.name == "od":
        roofline = od_roofline(_lib, stream, dev, steps_total, replay_micro_steps(kk, C_used), f_ms, g_ms,
                               cfg.grad.kernel, cfg.fwd.kernel, v_ms if fused is not None else None,
                               fused.kernel if fused is not None else None)
        # (the replay: its head buffer, every trial step's state written in the count pass and read in the sweep; the
        # one-pass launch: the inputs once)
        tr = TRAFFIC.get(fused.kernel if fused is not None else cfg.grad.kernel)
        if tr is not None:
            mp = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
            hbm = json.load(open(mp)).get("hbm_gbs") if os.path.exists(mp) else None
            roofline["traffic"] = int(round(tr[0] * N))
            roofline["traffic_source"] = f"ncu dram bytes read+write of one launch at N={tr[1]}, scaled by items to N={N}"
            gbs = roofline["traffic"] / ((v_ms if fused is not None else g_ms) / 1e3) / 1e9
            roofline["hbm"] = {"achieved": round(gbs, 2), "unit": "GB/s", "peak": hbm,
                               "frac": round(gbs / hbm, 4) if hbm else None,
                               "peak_source": "measured: MEASURED_PEAKS.json hbm_gbs" if hbm else None}
    if roofline is not None and not tree and cfg.name != "od":
        # per mode (the separate launches): the forward and the replay gradient against the same probe
        roofline["modes"] = {
            "fwd": {"kernel": cfg.fwd.kernel, "achieved": round(tf_fwd / (f_ms / 1e3) / 1e9, 2),
                    "frac": round(tf_fwd / (f_ms / 1e3) / 1e9 / peak, 4)},
            "grad": {"kernel": cfg.grad.kernel, "achieved": round(tf_grad / (g_ms / 1e3) / 1e9, 2),
                     "frac": round(tf_grad / (g_ms / 1e3) / 1e9 / peak, 4)}}
    if cfg.name == "ph" and roofline is not None:
        # the photon's step mixes threefry with the shared math (log, sincos, sqrt in double) and f32 work, so its
        # own speed of light is the probe of that step (tm_probe_issue kind 4); the threefry view stays beside it
        p4, _ = _lib.probe_rate(_lib.PROBE_PHOTON_STEP, 1024, stream, dev)
        tf_view = dict(roofline)
        ms = dom[2]
        roofline = {"bound": "issue", "kernel": dom[0], "achieved": round(steps_total / (ms / 1e3) / 1e9, 4),
                    "peak": round(p4 / 1e9, 4), "unit": "G photon steps/s",
                    "frac": round(steps_total / (ms / 1e3) / p4, 4), "traffic": traffic,
                    "traffic_source": tf_view.get("traffic_source"),
                    "peak_source": "measured: tm_probe_issue kind 4 (the photon step at full occupancy, deposit in a "
                                   "register, no divergence from claims, no memory) on this GPU",
                    "work": f"{steps_total} photon steps (from the per-item trip counts)",
                    "modes": {"fwd": {"kernel": cfg.fwd.kernel,
                                      "frac": round(steps_total / (f_ms / 1e3) / p4, 4)}},
                    "threefry": {k: tf_view[k] for k in ("achieved", "peak", "unit", "frac", "achieved_int32_tops",
                                                         "work")}}
    if roofline is not None and traffic is not None:
        # the memory side of the roofline: the kernel's measured DRAM bytes per launch over its time, against the
        # measured copy bandwidth (MEASURED_PEAKS.json): how far from memory-bound the path is
        mp = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
        hbm = json.load(open(mp)).get("hbm_gbs") if os.path.exists(mp) else None
        gbs = traffic / (dom[2] / 1e3) / 1e9
        roofline["hbm"] = {"achieved": round(gbs, 2), "unit": "GB/s", "peak": hbm,
                           "frac": round(gbs / hbm, 5) if hbm else None,
                           "peak_source": "measured: MEASURED_PEAKS.json hbm_gbs" if hbm else None}

    parity = None
    if rank == 0 and not args.no_parity:
        # the timed launches' per-item outputs (this rank's items) against the oracle on a prefix + the longest items
        runs = {"forward": (kk, fo[fnames.index("truncated")].to("cpu").numpy())}
        if fused is not None and not sh_vg:
            runs["value_and_grad"] = (vo[vnames.index("k")].to("cpu").numpy(),
                                      vo[vnames.index("truncated")].to("cpu").numpy())
        elif sh_vg:
            runs["value_and_grad"] = (r_last["k"].to("cpu").numpy(), r_last["trunc"].to("cpu").numpy())
        parity = parity_block(cfg, host, runs, len(os.sched_getaffinity(0)))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        nth = len(os.sched_getaffinity(0))
        n, dt, v = cpu_rate(cfg, host, 10.0, nth)
        cpu = {"value": round(v, 4), "unit": "Mitems/s", "cores": nth, "kind": "port",
               "sample": f"oracle port (the reference CPU kernel target's model: f32 tallies, libm): fwd + grad of "
                         f"the first {n} items, {dt:.1f} s on {nth} OpenMP threads",
               # the parts on the same items: forward, the reference-order gradient (the value's), and the one-pass
               # gradient the GPU step uses (the like-for-like algorithm)
               "split": oracle_split(cfg, host, n, nth)}
    info = _lib.kernel_info(_lib.kernel_id((fused or cfg.grad).kernel)[0])
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "Mitems/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "clock_warmup_steps": extra, "ms_per_step": round(tot_ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32+u32", "data": "synthetic (jax.random algorithm on the host)",
        "config": {"workload": cfg.workload, "items_per_gpu": N, "items_total": N * world,
                   "max_steps": cfg.max_steps, "rev_checkpoints": C_used,
                   "parallelism": f"items sharded over {world} GPU(s)",
                   "l2": "flushed between timed steps (256 MiB write)"},
        "step": ("one value-and-grad launch (" + fused.kernel + (": the one-pass program, the gradient accumulated "
                 "as the forward runs" if not fused.replay_state_bytes else ": the replay whose count pass is the "
                 "forward")
                 + ")") if fused is not None else "a forward launch, then the gradient launch(es)",
        "fwd_ms": round(f_ms, 3), "grad_ms": round(g_ms, 3), "separate_ms": round(sep_ms, 3),
        "fused_ms": round(v_ms, 3) if fused is not None else None,
        "fwd_mitems_s": round(N * world / (f_ms / 1e3) / 1e6, 3),
        "grad_mitems_s": round(N * world / (g_ms / 1e3) / 1e6, 3),
        "mean_trip_count": round(steps_total / N, 2),
        **({"particles_per_gpu": int(fo[fnames.index("count")][0].item()),
            "particles_mnodes_s": round(int(fo[fnames.index("count")][0].item()) * world / (tot_ms / 1e3) / 1e6, 3),
            "tree_generations": tree_info.get("generations"), "tree_adjoint_launches": tree_info.get("launches")}
           if tree else {}),
        "e2e": {"value": round(e2e_val, 3), "unit": "Mitems/s",
                "h2d_bytes_per_step": int(sum(h.nbytes for h in host)), "d2h_bytes_per_step": int(d2h[0])},
        # (the shower's one-pass step: the spawn launch and the per-root readout of the exact words)
        "gpu_launches": args.steps * ((2 if sh_vg else 1 + tree_info["kernels"]) if tree else
                                      ((1 if fused is not None else 2) + (1 if world > 1 else 0))),
        "roofline": roofline,
        "clocks": clk,
        "kernel_resources": info,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if parity is not None:
        line["parity"] = parity
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
