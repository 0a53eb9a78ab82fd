"""The lowering on the CPU: tracing item functions to the scalar IR, generating the forward and reverse ITEM
sources, and compiling them for sm_100a with NVRTC (which needs no GPU).  Launches are in test_lower_gpu.py."""
import numpy as np
import pytest

import tallymap_b200 as tm
from tallymap_b200 import lang as tl
from tallymap_b200 import lower, prng
from tallymap_b200 import trace as T

from items_lang import mixer, quickstart, walk


def _args_walk(n=16):
    kx, ks = prng.split(prng.PRNGKey(1), 2)
    return prng.uniform(kx, n), prng.split(ks, n), np.float32(1.0)


def test_trace_walk_structure():
    tr = T.trace_item(walk, ["f32", "key", "f32"], 2, {"hist": ((256,), "f32"), "side": ((2,), "f32")})
    assert len(tr.carry) == 2 and [v.dtype for v in tr.carry] == ["i32", "f32"]
    assert any(e.prim == "emit" and e.params["tally"] == "hist" for e in tr.body)
    assert any(e.prim == "emit" and e.params["tally"] == "side" for e in tr.post)
    assert sum(e.prim == "threefry" for e in tr.body) == 1 and sum(e.prim == "uniform01" for e in tr.body) == 1


def test_lowered_programs_compile():
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    L = f.lowered(_args_walk())
    assert isinstance(L.fwd.kernel, int) and L.fwd.kernel > 0
    g = L.grad_program((0,))
    assert g.replay_state_bytes == 4          # the step counter k is the step index: only x is stored
    assert L.it.counter == {0}
    # the generated step VJP is the hand-lowered one's expression: ct_drift += ct_hist[bin] * x
    src = lower.grad_source(L.it, [0])[0]
    assert "a.cb0 = a.cb0 + g" in src


def test_mixer_compiles_with_all_primitives():
    kx = prng.split(prng.PRNGKey(3), 8)
    f = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), tm.api.torch.int32),
                                "end": tm.Sum(())},
                in_axes=(0, 0, 0, None, None), max_steps=64)
    pos = np.zeros((8, 3), np.float32)
    L = f.lowered((pos, kx, np.full(8, 5, np.int32), np.float32(0.3), np.float32(1.7)))
    g = L.grad_program((0, 1))
    assert g.tallies[0].shape == (2,)


def test_trace_errors():
    def two_loops(t, x, key, d):
        x = tl.while_loop(lambda c: c > 0.0, lambda c: c - 1.0, x)
        x = tl.while_loop(lambda c: c > 0.0, lambda c: c - 1.0, x)
        return t, x
    with pytest.raises(T.TraceError, match="one top-level"):
        T.trace_item(two_loops, ["f32", "key", "f32"], 2, {})

    def no_loop(t, x, key, d):
        return t, x
    with pytest.raises(T.TraceError, match="no while_loop"):
        T.trace_item(no_loop, ["f32", "key", "f32"], 2, {})

    def mixed(t, x, key, d):
        def body(c):
            return c + (c > 0.0).astype(tl.int32)
        x = tl.while_loop(lambda c: c > 0.0, body, x)
        return t, x
    with pytest.raises(T.TraceError, match="convert"):
        T.trace_item(mixed, ["f32", "key", "f32"], 2, {})


def test_compile_error_reports_nvrtc_log(tmlib):
    with pytest.raises(tmlib.TallymapError, match="NVRTC failed"):
        lower.compile_kernel("this is not CUDA", "broken", 3, 16)


def test_fixed_point_sum_lowers_to_exact_bins():
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,), fixed_point=True), "side": tm.Sum((2,))},
                in_axes=(0, 0, None), max_steps=20000)
    L = f.lowered(_args_walk())
    assert [t.exact for t in L.fwd.tallies] == [True, False]
    assert "ExactSum<256>::emit(c.sx0" in L.fwd_source and "ExactSum<256>::readout" in L.fwd_source
    with pytest.raises(NotImplementedError):
        tm.Sum((4,), tm.api.torch.int32, fixed_point=True)


def test_jvp_programs_compile():
    kx = prng.split(prng.PRNGKey(3), 8)
    f = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), tm.api.torch.int32),
                                "end": tm.Sum(())},
                in_axes=(0, 0, 0, None, None), max_steps=64)
    L = f.lowered((np.zeros((8, 3), np.float32), kx, np.full(8, 5, np.int32), np.float32(0.3), np.float32(1.7)))
    p = L.jvp_program((0, 1), 2)
    assert [t.name for t in p.tallies] == ["dep", "hits", "end", "d_dep", "d_end"]
    assert p.tallies[3].shape == (2, 8, 8, 8) and p.tallies[4].shape == (2,)
    with pytest.raises(lower.LowerError):
        L.jvp_program((0,), 17)


def test_records_lower_and_compile():
    from items_lang import walk_records
    outs = {"hist": tm.Sum((256,)), "hits": tm.Records({"k": tm.api.torch.int32, "x": tm.api.torch.float32},
                                                       capacity=1024),
            "exit": tm.Records({"k": tm.api.torch.int32, "side": tm.api.torch.int32}, capacity=16)}
    f = tm.vmap(walk_records, outputs=outs, in_axes=(0, 0, None), max_steps=20000)
    L = f.lowered(_args_walk())
    names = [n for n, _, _, _ in L.fwd.result_layout(16)[0]]
    assert names[:3] == ["hist", "hits.k", "hits.x"] and "exit#ctr" in names and "hits#count" in names
    assert "atomicAdd(c.r0ctr, 1ull)" in L.fwd_source
    with pytest.raises(NotImplementedError):
        L.grad_program((0,))


def test_ir_evaluator_matches_the_oracle(orc):
    """the IR evaluator (the lowering's oracle) against the hand-written oracle on the traced walk and quickstart"""
    from oracle.ir_eval import Evaluator
    kx, ks = prng.split(prng.PRNGKey(1), 2)
    x, k = prng.uniform(kx, 40), prng.split(ks, 40)
    tr = T.trace_item(walk, ["f32", "key", "f32"], 2, {"hist": ((256,), "f32"), "side": ((2,), "f32")})
    r = Evaluator(tr, 20000).run([x, k], [1.0])
    ref = orc.rw_fwd(x, k, 1.0)
    assert np.array_equal(r["results"][0], ref["k"]) and np.array_equal(r["trunc"], ref["trunc"])
    assert np.array_equal(r["stats"], ref["stats"])
    assert np.abs(r["sums"]["hist"] - ref["hist"]).max() <= 1e-6 * np.abs(ref["hist"]).max()
    xq = np.linspace(0.1, 0.99, 50, dtype=np.float32)
    kq = prng.split(prng.PRNGKey(0), 50)
    trq = T.trace_item(quickstart, ["f32", "key", "f32"], 2, {"hist": ((16,), "f32")})
    rq = Evaluator(trq, 100).run([xq, kq], [2.0])
    refq = orc.q1_fwd(xq, kq, 2.0)
    assert np.array_equal(rq["results"][0], refq["k"])
    assert np.abs(rq["sums"]["hist"] - refq["hist"]).max() <= 1e-6 * np.abs(refq["hist"]).max()
