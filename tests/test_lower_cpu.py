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
    def two_loops(t, x, key, d):          # (the second loop, after the stepping loop, is an inner loop)
        x = tl.while_loop(lambda c: c > 0.0, lambda c: c - 1.0, x)
        x = tl.while_loop(lambda c: c > 0.0, lambda c: c - 1.0, x)
        return t, x
    tr2 = T.trace_item(two_loops, ["f32", "key", "f32"], 2, {})
    assert [e.prim for e in tr2.post] == ["while"]

    def no_loop(t, x, key, d):        # (a loop-free item: a loop of zero steps, its code after it)
        return t, x
    tr0 = T.trace_item(no_loop, ["f32", "key", "f32"], 2, {})
    assert tr0.carry == [] and tr0.body == [] and not tr0.cond_out.value

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
    # (another dtype with fixed_point: the scaled fixed-point sum; a dtype beyond float32 / int32 / float64 / int64
    # and a scale that is not a positive finite number are refused)
    assert tm.Sum((4,), tm.api.torch.int32, fixed_point=True).accumulator() == ("wide", tm.api.torch.int32, 2.0 ** 32)
    with pytest.raises(TypeError):
        tm.Sum((4,), tm.api.torch.float16)
    with pytest.raises(ValueError):
        tm.Sum((4,), tm.api.torch.float64, fixed_point=True, scale=0.0)


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
    # reverse mode: the forward's per-item counts and offsets become per-item operands, the float fields'
    # cotangents broadcast operands; forward mode: a tangent field per float field and lane
    g = L.grad_program((0,))
    assert [o.name for o in g.pi] == ["in0", "in1", "hits#count", "hits#offset", "exit#count", "exit#offset"]
    assert [o.name for o in g.bc] == ["bc0", "ct_hist", "ct_hits.x"]
    j = L.jvp_program((0,), 2)
    assert [f for f, _ in dict((nm, fl) for nm, _, fl in j.records)["hits"]] == ["k", "x", "x#d0", "x#d1"]


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


def _sh_specs():
    return {"dep": ((512,), "f32"), "count": ((1,), "i32")}


def test_spawn_traces_and_lowers():
    """t.spawn lowers onto the spawn runtime: a Child of the per-item leaves, step with two child slots, a
    start_child and the ring buffers; post-loop spawns take the finish form with child slots"""
    from items_lang import shower, spawn_walk
    tr = T.trace_item(shower, ["f32", "f32", "key", "f32"], 3, _sh_specs(), spawn=True)
    assert sum(e.prim == "spawn" for e in tr.body) == 2 and len(tr.body[-1].ins) >= 1
    f = tm.vmap(shower, outputs={"dep": tm.Sum((512,)), "count": tm.Sum((1,), tm.api.torch.int32)},
                in_axes=(0, 0, 0, None), max_steps=100000, spawn=tm.Queue(4096))
    from oracle import oracle as orc
    E0, d0, keys = orc.sh_inputs(8)
    L = f.lowered((E0, d0, keys, np.float32(1.0)))
    assert L.fwd.spawns and L.fwd.queue_leaf_bytes == 16 and L.fwd.consts == ("max_steps", "queue")
    src = L.fwd_source
    assert "struct Child { float l0; float l1; u32 l2; u32 l3; };" in src
    assert "start_child(Ctx& c, const Child& ch)" in src and "spawn_body<tmb::GenFwd>" in src
    names = [n for n, _, _, _ in L.fwd.result_layout(8, queue=4096)[0]]
    assert names == ["dep", "count", "queue.seq", "queue.ctl", "ctl", "stats", "y0", "truncated", "queue.ring"]
    with pytest.raises(ValueError, match="tree adjoint"):
        L.grad_program((0,))
    # reverse mode through spawn: the recording forward (a record of 4 leaves + prev + last per child) and the
    # per-generation adjoint (cotangents of the float per-item operands E and depth)
    rec = L.rec_program()
    assert rec.record_bytes == 24 and rec.queue_leaf_bytes == 24 and rec.consts == ("max_steps", "queue", "record")
    names = [n for n, _, _, _ in rec.result_layout(8, queue=4096, record=64)[0]]
    assert names == ["dep", "count", "queue.seq", "queue.ctl", "ctl", "stats", "tree", "y0", "truncated", "last",
                     "queue.ring", "record", "record.gen"]
    adj = L.tree_program((0,))
    assert [y.name for y in adj.ys] == ["ct_in0", "ct_in1", "truncated"] and adj.buffers == 19
    src = lower.grad_source(L.it, [0], tree=True)[0]
    assert "kNBuf = 19" in src and src.count("a.cur = w_[4];") == 2 and "c.dx[item * 2 + 1]" in src
    fw = tm.vmap(spawn_walk, outputs={"Q": tm.Sum((16,)), "C": tm.Sum((16,), tm.api.torch.int32)},
                 in_axes=(0, 0, 0), max_steps=100, spawn=tm.Queue(1024))
    Lw = fw.lowered((np.zeros(4, np.int32), np.ones(4, np.float32), prng.split(prng.PRNGKey(2), 4)))
    assert "static constexpr bool kPostSpawn = true;" in Lw.fwd_source


def test_spawn_trace_errors():
    from items_lang import shower
    with pytest.raises(T.TraceError, match="needs a Queue"):
        T.trace_item(shower, ["f32", "f32", "key", "f32"], 3, _sh_specs())

    def bad_structure(t, E, depth, key, X0):
        def body(c):
            k, t = c
            t = t.spawn((E, key), when=k > 1)
            return k + 1, t
        k, t = tl.while_loop(lambda c: c[0] < 3, body, (0, t))
        return t, k
    with pytest.raises(T.TraceError, match="structure"):
        T.trace_item(bad_structure, ["f32", "f32", "key", "f32"], 3, _sh_specs(), spawn=True)

    def before_loop(t, E, depth, key, X0):
        t = t.spawn((E, depth, key), when=E > 1.0)
        k, t = tl.while_loop(lambda c: c[0] < 3, lambda c: (c[0] + 1, c[1]), (0, t))
        return t, k
    with pytest.raises(T.TraceError, match="before the loop"):
        T.trace_item(before_loop, ["f32", "f32", "key", "f32"], 3, _sh_specs(), spawn=True)


def test_ir_evaluator_shower_matches_the_oracle(orc):
    """the evaluator runs spawned children: the traced shower against the hand-written oracle (particle count and
    per-root trip counts bitwise, the deposit within the float-sum tolerance)"""
    from items_lang import shower
    from oracle.ir_eval import Evaluator
    E0, d0, keys = orc.sh_inputs(6)
    tr = T.trace_item(shower, ["f32", "f32", "key", "f32"], 3, _sh_specs(), spawn=True)
    r = Evaluator(tr, 100000).run([E0, d0, keys], [1.0])
    ref = orc.sh_fwd(E0, d0, keys, 1.0)
    assert int(r["sums"]["count"][0]) == int(ref["count"][0])
    assert np.array_equal(r["results"][0], ref["k"]) and np.array_equal(r["trunc"], ref["trunc"])
    assert int(r["stats"][0]) == int(ref["stats"][0]) and int(r["stats"][4]) == int(ref["stats"][4])
    assert np.abs(r["sums"]["dep"] - ref["dep"]).max() <= 1e-5 * np.abs(ref["dep"]).max()


def test_onepass_program_for_items_without_active_carry():
    """the walk's carries do not depend on drift: a one-pass value-and-grad program (OnePassVG over the generated
    forward and reverse ITEMs) compiles; the mixer's carries depend on a and b: forward mode instead"""
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    L = f.lowered(_args_walk())
    p = L.vg_program((0,))
    assert p is not None and [t.name for t in p.tallies] == ["hist", "side", "ct"] and p.tallies[-1].exact
    names = [n for n, _, _, _ in p.result_layout(16)[0]]
    assert names == ["hist", "side", "ct", "ct.exact", "ctl", "stats", "y0", "truncated"]
    src = lower.onepass_source(L.it, [0])[0]
    assert "OnePassVG<GenFwd, GenGrad, GenVGMap>" in src and "typedef GenFwd::State State;" in src
    kx = prng.split(prng.PRNGKey(3), 8)
    fm = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), tm.api.torch.int32),
                                 "end": tm.Sum(())},
                 in_axes=(0, 0, 0, None, None), max_steps=64)
    Lm = fm.lowered((np.zeros((8, 3), np.float32), kx, np.full(8, 5, np.int32), np.float32(0.3), np.float32(1.7)))
    assert lower.has_active_carry(Lm.it, [0, 1]) and "_fg" in lower._COMPILED[Lm.vg_program((0, 1)).kernel]
    fq = tm.vmap(quickstart, outputs={"hist": tm.Sum((16,), fixed_point=True)}, in_axes=(0, 0, None), max_steps=100)
    Lq = fq.lowered((np.linspace(0.1, 0.9, 8, dtype=np.float32), prng.split(prng.PRNGKey(0), 8), np.float32(2.0)))
    pq = Lq.vg_program((0,))
    assert [n for n, _, _, _ in pq.result_layout(8)[0]][:4] == ["hist", "ct", "hist.exact", "ct.exact"]


def test_forward_mode_value_and_grad_program_for_active_carries():
    """the mixer's carries depend on a and b: value_and_grad's one-pass program is forward mode (the identity's two
    tangent lanes contracted with the cotangents at each emit, exact per-item sums)"""
    kx = prng.split(prng.PRNGKey(3), 8)
    fm = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8)), "hits": tm.Sum((4,), tm.api.torch.int32),
                                 "end": tm.Sum(())},
                 in_axes=(0, 0, 0, None, None), max_steps=64)
    Lm = fm.lowered((np.zeros((8, 3), np.float32), kx, np.full(8, 5, np.int32), np.float32(0.3), np.float32(1.7)))
    p = Lm.vg_program((0, 1))
    assert p is not None and [t.name for t in p.tallies] == ["dep", "hits", "end", "ct"]
    names = [n for n, _, _, _ in p.result_layout(8)[0]]
    assert names == ["dep", "hits", "end", "ct", "ct.exact", "ctl", "stats", "y0", "truncated"]
    src = lower.jvp_source(Lm.it, [0, 1], 2, contract=True)[0]
    assert "c.pv.emit(1, a1)" in src and "c.db1_1 = 1.0f;" in src and "c.db1_0 = 0.0f;" in src


def test_forward_mode_through_spawn_lowers():
    """a spawning item's forward-mode programs: the child carries its float leaves' tangents"""
    from items_lang import spawn_decay
    f = tm.vmap(spawn_decay, outputs={"Q": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=10,
                spawn=tm.Queue(4096))
    L = f.lowered((np.zeros(4, np.int32), np.ones(4, np.float32), prng.split(prng.PRNGKey(2), 4), np.float32(1.1)))
    p = L.vg_program((0,))
    assert p.spawns and p.queue_leaf_bytes == 4 * (4 + 1) and p.consts == ("max_steps", "queue")
    src = lower.jvp_source(L.it, [0], 1, contract=True)[0]
    assert "float d1_0;" in src and "start_child(Ctx& c, const Child& ch)" in src and "spawn_body<tmb::GenJvp>" in src
    j = L.jvp_program((0,), 2)
    assert j.spawns and j.queue_leaf_bytes == 4 * (4 + 2)


def test_loop_free_item_lowers_and_evaluates(orc):
    """a loop-free item lowers (forward, one-pass value-and-grad, replay) and the evaluator runs it"""
    from items_lang import scatter
    from oracle.ir_eval import Evaluator
    f = tm.vmap(scatter, outputs={"h": tm.Sum((8,)), "s": tm.Sum(())}, in_axes=(0, 0, None))
    args = _args_walk(32)
    L = f.lowered(args)
    assert L.vg_program((0,)) is not None and L.grad_program((0,)).replay_state_bytes == 4
    tr = T.trace_item(scatter, ["f32", "key", "f32"], 2, {"h": ((8,), "f32"), "s": ((), "f32")})
    r = Evaluator(tr, 100).run(list(args[:2]), [1.0])
    assert not r["trunc"].any() and r["sums"]["s"][0] > 0


def test_per_item_operand_gradient_program():
    """grad w.r.t. a per-item operand: the generated replay writes each item's cotangent before the flag"""
    from items_lang import affine
    f = tm.vmap(affine, outputs={"h": tm.Sum((8,))}, in_axes=(0, 0, None), max_steps=10)
    L = f.lowered(_args_walk(16))
    p = L.grad_program((0,), (0,))
    assert [y.name for y in p.ys] == ["ct_in0", "truncated"] and p.trunc == 1
    p0 = L.grad_program((), (0,))
    assert p0.tallies[0].shape == (1,)
    src = lower.grad_source(L.it, [0], wrt_pi=(0,))[0]
    assert "c.gpi0[item * 1 + 0] =" in src


def test_forward_mode_of_fixed_point_outputs():
    """jvp and the forward-mode value_and_grad of an item with a fixed-point output: its tangent is exact too"""
    f = tm.vmap(mixer, outputs={"dep": tm.Sum((8, 8, 8), fixed_point=True), "hits": tm.Sum((4,), tm.api.torch.int32),
                                "end": tm.Sum(())},
                in_axes=(0, 0, 0, None, None), max_steps=64)
    kx = prng.split(prng.PRNGKey(3), 8)
    L = f.lowered((np.zeros((8, 3), np.float32), kx, np.full(8, 5, np.int32), np.float32(0.3), np.float32(1.7)))
    p = L.jvp_program((0, 1), 2)
    assert [(t.name, t.exact) for t in p.tallies] == [("dep", True), ("hits", False), ("end", False),
                                                       ("d_dep", True), ("d_end", False)]
    names = [n for n, _, _, _ in p.result_layout(8)[0]]
    assert names[:7] == ["dep", "hits", "end", "d_dep", "d_end", "dep.exact", "d_dep.exact"]
    v = L.vg_program((0, 1))
    assert [n for n, _, _, _ in v.result_layout(8)[0]][:6] == ["dep", "hits", "end", "ct", "dep.exact", "ct.exact"]


def test_compiled_items_disk_cache(monkeypatch):
    """a compiled item is kept on disk by the digest of its source and the runtime headers, and a later process
    (here: a cleared in-process cache) registers the cached cubin instead of compiling again"""
    import os
    import shutil
    d = os.path.join(os.path.dirname(lower.CSRC), "_cache", f"test-{os.getpid()}")
    monkeypatch.setenv("TALLYMAP_B200_CACHE", d)
    try:
        def walk3(t, x, key, drift):          # (a source no other test compiles in this process)
            def body(c):
                k, x, t = c
                u = tl.random.uniform(tl.random.fold_in(key, k))
                return k + 1, x + 0.03 * (2 * u - 1), t.add("hist", (x * 256).astype(tl.int32), drift * x)
            k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
            return t, k
        f = tm.vmap(walk3, outputs={"hist": tm.Sum((256,))}, in_axes=(0, 0, None), max_steps=20000)
        L = f.lowered(_args_walk())
        cached = os.listdir(d)
        assert len(cached) >= 1 and all(p.endswith(".cubin") for p in cached)
        kid = L.fwd.kernel
        lower._COMPILED.pop(kid)
        calls = []
        monkeypatch.setattr(lower._lib.lib(), "tm_compile", lambda *a: calls.append(a) or 1)
        assert lower.compile_kernel(L.fwd_source, "walk_fwd", 12, 16) == kid
        assert not calls
    finally:
        shutil.rmtree(d, ignore_errors=True)


def test_vector_compositions_trace():
    """cumsum and searchsorted over a per-item vector trace to the expected scalar equations"""
    def item(t, p, key, a):
        c = tl.cumsum(p)
        i = tl.searchsorted(c, a)
        t = t.add("h", i, 1)
        return t, c[2]
    tr = T.trace_item(item, [("f32", 3), "key", "f32"], 2, {"h": ((4,), "i32")})
    prims = [e.prim for e in tr.post]
    assert prims.count("add") >= 2 + 2 and prims.count("lt") == 3 and prims.count("emit") == 1
    from oracle.ir_eval import Evaluator
    p = np.float32([[0.1, 0.2, 0.3], [0.5, 0.5, 0.5]])
    r = Evaluator(tr, 10).run([p, prng.split(prng.PRNGKey(0), 2)], [0.45])
    assert list(r["sums"]["h"]) == [1, 0, 1, 0]        # cumsums (0.1, 0.3, 0.6) and (0.5, 1, 1.5) against 0.45
    assert np.allclose(r["results"][0], [0.6, 1.5])


def test_vmap_options_validated():
    """tallymap.vmap's options (_api.py:414-425, 493-507): unknown names, bad values and backend='xla' raise"""
    outs = {"hist": tm.Sum((256,)), "side": tm.Sum((2,))}
    for bad in ({"cuda_math": "exact"}, {"schedule": "warp"}, {"min_blocks_per_sm": 0}, {"min_blocks_per_sm": 33},
                {"min_blocks_per_sm": True}, {"rev_checkpoints": 0}, {"rev_checkpoints": "some"}, {"fill": 1}):
        with pytest.raises(ValueError):
            tm.vmap(walk, outputs=outs, in_axes=(0, 0, None), **bad)
    with pytest.raises(ValueError):
        tm.vmap(walk, outputs=outs, in_axes=(0, 0, None), backend="cuda")
    with pytest.raises(tm.UnsupportedError) as e:
        tm.vmap(walk, outputs=outs, in_axes=(0, 0, None), backend="xla")
    assert isinstance(e.value, NotImplementedError)
    with pytest.raises(tm.UnsupportedError):      # the built-in families are compiled ahead of time with 'ieee'
        tm.vmap("walk1d", outputs=outs, in_axes=(0, 0, None), cuda_math="approx")
    f = tm.vmap(walk, outputs=outs, in_axes=(0, 0, None), cuda_math="approx", schedule="step", min_blocks_per_sm=4,
                rev_checkpoints=8, rev_stats=True, xla_batch_size=1024)
    assert f.opts == dict(math="approx", schedule="step", min_blocks=4, rev_checkpoints=8)


def test_vmap_decorator_and_default_in_axes():
    """@tm.vmap(outputs=..., ...) as a decorator; in_axes=0 maps every argument after the tally"""
    @tm.vmap(outputs={"h": tm.Sum((8,))}, max_steps=10)
    def item(t, x, key):
        return t.add("h", (x * 8).astype(tl.int32), 1.0)
    assert isinstance(item, tm.api.MappedFn) and item.in_axes == (0, 0)
    g = tm.vmap("walk1d", outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, max_steps=100)
    assert g.fam.in_axes == (0, 0, None)


def test_cuda_math_and_min_blocks_sources():
    """cuda_math='approx' / 'fast' put div.full / sqrt.approx behind tm_fdiv / tm_fsqrt (and 'fast' compiles with FMA
    contraction); min_blocks_per_sm sets the entry point's launch bounds; the default source is unchanged"""
    def item(t, x, key, a):
        def body(c):
            k, x, t = c
            u = tl.random.uniform(tl.random.fold_in(key, k))
            return k + 1, x + a * tl.sqrt(u) / (1.0 + x), t.add("h", (x * 8).astype(tl.int32), x / a)
        k, x, t = tl.while_loop(lambda c: c[1] < 1.0, body, (0, x, t))
        return t, k
    outs = {"h": tm.Sum((8,))}
    args = _args_walk()
    ids = {}
    for math, mb in (("ieee", None), ("approx", None), ("fast", None), ("ieee", 4)):
        f = tm.vmap(item, outputs=outs, in_axes=(0, 0, None), max_steps=100, cuda_math=math, min_blocks_per_sm=mb)
        L = f.lowered(args)
        body = L.fwd_source.split("struct GenFwd")[1]
        assert "tm_fdiv(" in body and "tm_fsqrt(" in body and " / " not in body
        assert L.head == lower.options_source(math, mb)[0] and L.flags == (math == "fast")
        g = L.grad_program((0,))
        ids[(math, mb)] = (L.fwd.kernel, g.kernel)
    assert len({v for v in ids.values()}) == 4
    assert lower.options_source("ieee") == ("", 0)
    assert lower.options_source("approx", 2)[0] == "#define TM_MATH_APPROX 1\n#define TM_MIN_BLOCKS 2\n"


def test_schedule_step_needs_a_loop():
    """schedule='step' raises UnsupportedError for an item with no top-level while loop (_api.py:447-452)"""
    def flat(t, x):
        return t.add("h", 0, x)
    f = tm.vmap(flat, outputs={"h": tm.Sum((1,))}, in_axes=(0,), schedule="step")
    with pytest.raises(tm.UnsupportedError):
        f.lowered((np.float32([1.0, 2.0]),))
    g = tm.vmap(flat, outputs={"h": tm.Sum((1,))}, in_axes=(0,), schedule="item")
    assert g.lowered((np.float32([1.0, 2.0]),)).fwd.kernel > 0


def test_error_types():
    """the reference's exception types: a Tally read as a value is a TallyError (_rewrite.py:31), a construct the
    kernel backend does not lower an UnsupportedError (a NotImplementedError, _api.py:198); both TraceErrors here"""
    def reads(t, x):
        return t, x + t
    def nested(t, x):                     # (a spawn inside an inner loop: a step pushes at most two children)
        def body(c):
            i, t = c
            j, t = tl.while_loop(lambda d: d[0] < 2, lambda d: (d[0] + 1, d[1].spawn((x,))), (0, t))
            return i + j, t
        i, t = tl.while_loop(lambda c: c[0] < 4, body, (0, t))
        return t, i
    def drops(t, x):
        return x
    specs = {"h": ((1,), "f32")}
    with pytest.raises(tm.TallyError):
        T.trace_item(reads, ["f32"], 1, specs)
    with pytest.raises(tm.TallyError):
        T.trace_item(drops, ["f32"], 1, specs)
    with pytest.raises(tm.UnsupportedError) as e:
        T.trace_item(nested, ["f32"], 1, specs, spawn=True)
    assert isinstance(e.value, NotImplementedError) and isinstance(e.value, T.TraceError)
    assert issubclass(lower.LowerError, tm.UnsupportedError)


def test_broadcast_vector_operands():
    """a broadcast float32[n] operand (n <= 64) is lowered as n broadcast scalars: the item sees a tuple; grad, jvp
    and value_and_grad address it as one argument (its gradient f32[n])"""
    from items_lang import walk_theta, walk_theta_scalars
    outs = {"hist": tm.Sum((64,))}
    x, k, _ = _args_walk()
    f = tm.vmap(walk_theta, outputs=outs, in_axes=(0, 0, None), max_steps=1000)
    g = tm.vmap(walk_theta_scalars, outputs=outs, in_axes=(0, 0, None, None, None), max_steps=1000)
    th = np.float32([0.5, 0.03, 0.1])
    L = f.lowered((x, k, th))
    Ls = g.lowered((x, k, *th))
    assert L.bc_groups == {2: (0, 3)} and len(L.fwd.bc) == 3
    assert L.fwd_source.split("struct GenFwd")[1] == Ls.fwd_source.split("struct GenFwd")[1]
    pi, bc = f._split((x, k, th))
    assert len(pi) == 2 and len(bc) == 3 and float(bc[1]) == np.float32(0.03)
    assert f._bleaves(L, (2,)) == ((0, 1, 2), {2: (0, 3)})
    ct = np.arange(3, dtype=np.float32)
    assert np.array_equal(f._per_arg(ct, {2: (0, 3)}, 2, (2,)), ct)
    assert f._per_arg(ct, {3: (0, None), 4: (1, None), 2: (2, None)}, (3, 4, 2), (3, 4, 2)) is ct
    assert L.grad_program((0, 1, 2)).kernel > 0
    big = (x, k, np.zeros(65, np.float32))           # past 64 elements: a table, read by index, not differentiable
    Lb = f.lowered(big)
    assert Lb.bc_groups == {2: (0, None)} and Lb.fwd.bc[0].shape == (65,)
    with pytest.raises(tm.UnsupportedError):
        Lb.grad_program((0,))


def test_broadcast_tables():
    """a broadcast array larger than a parameter vector (or any int32 array, or a 2-D array) is a table read by
    traced indices with jax.numpy's semantics (negative counts from the end, then clamped); the IR evaluator agrees
    with numpy's clip-mode take; derivatives with respect to a table raise UnsupportedError"""
    from items_lang import lookup, neighbours
    from oracle.ir_eval import Evaluator
    rng = np.random.default_rng(0)
    x, k, _ = _args_walk(64)
    xs = rng.uniform(0.5, 1.5, 100).astype(np.float32)
    pairs = rng.uniform(-1, 1, (100, 2)).astype(np.float32)
    f = tm.vmap(lookup, outputs={"h": tm.Sum((16,), fixed_point=True)}, in_axes=(0, 0, None, None, None),
                max_steps=20000)
    L = f.lowered((x, k, xs, pairs, np.float32(0.7)))
    assert [o.shape for o in L.fwd.bc] == [(100,), (100, 2), ()]
    assert "__ldg(&c.b0[" in L.fwd_source and "__ldg(&c.b1[" in L.fwd_source
    assert L.grad_program((2,)).kernel > 0 and L.grad_program((), (0,)).kernel > 0
    with pytest.raises(tm.UnsupportedError):
        L.grad_program((0,))
    with pytest.raises(tm.UnsupportedError):
        L.jvp_program((1,), 1)
    ref = Evaluator(L.tr, 20000, ("h",)).run([x, k], [xs, pairs, np.float32(0.7)])
    kk = ref["results"][0]
    assert np.array_equal(ref["results"][1], xs[-1] + pairs[np.clip(kk, 0, 99), 1])
    # the cell-list item: neighbour counts equal a brute-force count
    N = 128
    pos = rng.uniform(0, 8, (N, 2)).astype(np.float32)
    cell = np.clip((pos[:, 1] / 2).astype(int), 0, 3) * 4 + np.clip((pos[:, 0] / 2).astype(int), 0, 3)
    order = np.argsort(cell, kind="stable").astype(np.int32)
    start = np.searchsorted(cell[order], np.arange(17)).astype(np.int32)
    g = tm.vmap(neighbours, outputs={"u": tm.Sum((4,))}, in_axes=(0, None, None, None, None), max_steps=1 << 14)
    ii = np.arange(N, dtype=np.int32)
    L2 = g.lowered((ii, order, start, pos, np.float32([1.0, 0.5])))
    assert L2.bc_groups[4] == (3, 2) and [o.shape for o in L2.fwd.bc][:3] == [(N,), (17,), (N, 2)]
    r = Evaluator(L2.tr, 1 << 14).run([ii], [order, start, pos, 1.0, 0.5])
    d = (pos[:, None, :] - pos[None, :, :] + 12.0) % 8.0 - 4.0
    nb = (((d ** 2).sum(-1) < 4.0) & ~np.eye(N, dtype=bool)).sum(1)
    assert np.array_equal(r["results"][0], nb)


def test_vector_traced_index():
    """a float32 vector read by a traced index: a chain of selects (differentiable), the index wrapped and clamped"""
    def item(t, p, key, a):
        i = (a * 10).astype(tl.int32) - 2
        return t.add("h", 0, p[i] + p[-1]), p[i]
    tr = T.trace_item(item, [("f32", 3), "key", "f32"], 2, {"h": ((1,), "f32")})
    from oracle.ir_eval import Evaluator
    p = np.float32([[1, 2, 3], [4, 5, 6]])
    keys = prng.split(prng.PRNGKey(0), 2)
    for a, want in ((0.0, [2, 5]), (0.25, [1, 4]), (0.35, [2, 5]), (0.99, [3, 6]), (-1.0, [1, 4])):
        r = Evaluator(tr, 10).run([p, keys], [np.float32(a)])
        assert list(r["results"][0]) == want, (a, r["results"][0])


def test_special_math_trace_and_compile():
    """the inverse trigonometric, hyperbolic, exp2 / log2 / cbrt and erf family lower to the shared math; the
    evaluator's values track numpy / scipy within float32 rounding; random.normal is sqrt(2) erfinv of jax's
    uniform on (nextafter(-1, 0), 1)"""
    from scipy import special as sp
    from items_lang import special
    from oracle.ir_eval import Evaluator
    n = 64
    x = np.random.default_rng(2).uniform(-1, 1, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(8), n)
    f = tm.vmap(special, outputs={"h": tm.Sum((8,))}, in_axes=(0, 0, None), max_steps=100)
    L = f.lowered((x, keys, np.float32(0.8)))
    body = L.fwd_source.split("struct GenFwd")[1]
    for fn in ("atanf", "atan2f", "asinf", "acosf", "tanf", "sinhf", "coshf", "asinhf", "acoshf", "atanhf", "exp2f",
               "log2f", "cbrtf", "erff", "erfcf", "erfinvf"):
        assert f"tmm::{fn}(" in body, fn
    assert L.grad_program((0,)).kernel > 0 and L.jvp_program((0,), 2).kernel > 0
    r = Evaluator(L.tr, 100).run([x, keys], [np.float32(0.8)])
    assert np.isfinite(r["results"][0]).all() and (r["results"][1] == 1).all()
    # random.normal against its definition through numpy/scipy in float64, rounded
    def item(t, key):
        return t, tl.random.normal(key)
    tr = T.trace_item(item, ["key"], 1, {})
    z = Evaluator(tr, 1).run([keys], [])["results"][0]
    assert abs(float(np.mean(z))) < 0.5 and 0.5 < float(np.std(z)) < 1.5
    from tallymap_b200 import prng as pr
    bits = np.array([pr.threefry2x32(np.uint32(k[0]), np.uint32(k[1]), np.uint32(0), np.uint32(0)) for k in keys])
    b = (bits[:, 0] ^ bits[:, 1]).astype(np.uint32)
    f01 = ((b >> 9) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)
    lo = np.nextafter(np.float32(-1), np.float32(0))
    uu = np.maximum(lo, f01 * np.float32(2.0) + lo)
    want = (np.float32(np.sqrt(2)) * sp.erfinv(uu.astype(np.float64)).astype(np.float32)).astype(np.float32)
    assert np.array_equal(z.astype(np.float32), want)


def test_cond_switch_fori():
    """lax.cond / switch of value branches become selects (both traced, jax's semantics under vmap);
    fori_loop with static bounds unrolls; branches that use the tally differently raise TallyError"""
    from oracle.ir_eval import Evaluator

    def item(t, x, key, a):
        y = tl.cond(x > 0.5, lambda v: (v * a, v + 1.0), lambda v: (v - a, v * 2.0), x)
        s = tl.switch((x * 4).astype(tl.int32), [lambda v: v, lambda v: -v, lambda v: v * v], x)
        z = tl.fori_loop(0, 3, lambda i, c: c * 0.5 + i, x)
        return t.add("h", 0, y[0] + y[1] + s + z), y[0], s, z
    tr = T.trace_item(item, ["f32", "key", "f32"], 2, {"h": ((1,), "f32")})
    xs = np.float32([0.1, 0.3, 0.6, 0.9])
    r = Evaluator(tr, 10).run([xs, prng.split(prng.PRNGKey(0), 4)], [np.float32(2.0)])
    a = np.float32(2.0)
    assert np.array_equal(r["results"][0], np.where(xs > 0.5, xs * a, xs - a).astype(np.float32))
    idx = np.clip((xs * 4).astype(np.int32), 0, 2)
    assert np.array_equal(r["results"][1], np.choose(idx, [xs, -xs, xs * xs]).astype(np.float32))
    z = xs
    for i in range(3):
        z = (z * np.float32(0.5) + np.float32(i)).astype(np.float32)
    assert np.array_equal(r["results"][2], z)

    def bad(t, x):
        t, y = tl.cond(x > 0.5, lambda tt: (tt.add("h", 0, 1.0), x), lambda tt: (x, tt), t)
        return t
    with pytest.raises(tm.TallyError, match="the same way"):
        T.trace_item(bad, ["f32"], 1, {"h": ((1,), "f32")})
    f = tm.vmap(item, outputs={"h": tm.Sum((1,))}, in_axes=(0, 0, None), max_steps=10)
    L = f.lowered((xs, prng.split(prng.PRNGKey(0), 4), np.float32(2.0)))
    assert L.grad_program((0,)).kernel > 0


def test_vector_semantics():
    """small vectors with jax.numpy's elementwise semantics: arithmetic, broadcasting, comparisons, where, math,
    integer powers by binary powering, reductions; a walk-on-spheres item written with them traces, evaluates to
    its scalar restatement and compiles with its gradient"""
    from oracle.ir_eval import Evaluator
    from items_lang import spheres

    def item(t, p, key, a):
        v = tl.array([a, 2.0 * a, 3.0])
        w = (p + v) * 2.0 - v / a
        z = tl.where(w > 4.0, w ** 2, -w) + tl.sqrt(tl.abs(p))
        return t.add("h", 0, tl.sum(z) + tl.dot(p, v)), tl.max(z), (w ** -3)[0], tl.sum(tl.sign(p - 0.5))
    tr = T.trace_item(item, [("f32", 3), "key", "f32"], 2, {"h": ((1,), "f32")})
    p = np.float32([[0.1, 0.9, 2.0], [1.0, -2.0, 0.5]])
    a = np.float32(1.5)
    r = Evaluator(tr, 10).run([p, prng.split(prng.PRNGKey(0), 2)], [a])
    f32 = np.float32
    v = np.array([[a, f32(2.0) * a, f32(3.0)]], np.float32)
    w = ((p + v) * f32(2.0) - v / a).astype(np.float32)
    z = (np.where(w > 4.0, w * w, -w) + np.sqrt(np.abs(p))).astype(np.float32)
    assert np.array_equal(r["results"][0], z.max(1))
    assert np.array_equal(r["results"][1], (f32(1.0) / (w[:, 0] * (w[:, 0] * w[:, 0]))).astype(np.float32))
    assert np.array_equal(r["results"][2], np.sign(p - f32(0.5)).sum(1).astype(np.float32))
    with pytest.raises(T.TraceError):
        T.trace_item(lambda t, p, k, a: (t, tl.sum(p + tl.array([1.0, 2.0]))), [("f32", 3), "key", "f32"], 2, {})
    n = 32
    rng = np.random.default_rng(0)
    x0 = rng.uniform(0.1, 0.9, (n, 2)).astype(np.float32)
    point = np.arange(n, dtype=np.int32) % 8
    keys = prng.split(prng.PRNGKey(4), n)
    th = np.float32([1.0, 3.0, 0.2, 0.1])
    f = tm.vmap(spheres, outputs={"u": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=4096)
    L = f.lowered((x0, point, keys, th))
    assert L.grad_program((0, 1, 2, 3)).kernel > 0
    out = Evaluator(L.tr, 4096).run([x0, point, keys], list(th))
    assert (out["results"][0] > 0).all() and np.isfinite(out["sums"]["u"]).all()


def test_add_vectors():
    """t.add with a vector index and a vector or scalar value: one emit per element (the reference's array emit,
    _tally.py:248-282), out-of-range elements dropped and counted"""
    from oracle.ir_eval import Evaluator

    def item(t, p, key, a):
        b = (p * 4.0).astype(tl.int32)
        t = t.add("h", b, p * a)
        t = t.add("g", (b, tl.array([0, 1, 2])), 1)
        return t, tl.sum(b)
    tr = T.trace_item(item, [("f32", 3), "key", "f32"], 2, {"h": ((4,), "f32"), "g": ((4, 3), "i32")})
    p = np.float32([[0.1, 0.6, 0.9], [1.2, 0.3, 0.3]])
    r = Evaluator(tr, 10).run([p, prng.split(prng.PRNGKey(0), 2)], [np.float32(2.0)])
    h = np.zeros(4, np.float32)
    g = np.zeros((4, 3), np.int64)
    dropped = 0
    for row in p:
        for j, v in enumerate(row):
            b = int(np.float32(v) * np.float32(4.0))
            if 0 <= b < 4:
                h[b] += np.float32(v) * np.float32(2.0)
                g[b, j] += 1
            else:
                dropped += 2
    assert np.allclose(r["sums"]["h"], h) and np.array_equal(r["sums"]["g"].reshape(4, 3), g)
    assert r["stats"][4] == dropped == 2



def test_numpy_compositions():
    """jax.numpy functions formed from the lowered primitives, against numpy in float32 on ordinary and awkward
    values: prod, mean, argmax / argmin (NaN wins, first index), cumprod / cummax / cummin, isnan / isinf,
    nan_to_num, logaddexp, hypot, norm"""
    from oracle.ir_eval import Evaluator

    def item(t, p, key):
        v = tl.array(p)
        return (t, tl.prod(v), tl.mean(v), tl.argmax(v), tl.argmin(v), tl.cumprod(v)[2], tl.cummax(v)[1],
                tl.cummin(v)[2], tl.isnan(v[0]).astype(tl.int32), tl.isinf(v[1]).astype(tl.int32),
                tl.nan_to_num(v[1]), tl.logaddexp(v[0], v[1]), tl.hypot(v[1], v[2]), tl.norm(v))
    tr = T.trace_item(item, [("f32", 3), "key"], 2, {})
    inf, nan = np.float32(np.inf), np.float32(np.nan)
    p = np.float32([[0.5, 2.0, -3.0], [1.0, 1.0, 1.0], [nan, 1.0, 2.0], [1.0, inf, 0.0], [-inf, -inf, 4.0],
                    [0.0, 0.0, 0.0], [1e30, 1e30, 3.0]])
    r = Evaluator(tr, 1).run([p, prng.split(prng.PRNGKey(0), len(p))], [])["results"]
    f = np.float32
    with np.errstate(all="ignore"):
        want = [p[:, 0] * p[:, 1] * p[:, 2], (p[:, 0] + p[:, 1] + p[:, 2]) / f(3), np.argmax(p, 1), np.argmin(p, 1),
                np.cumprod(p, 1)[:, 2], np.maximum.accumulate(p, 1)[:, 1], np.minimum.accumulate(p, 1)[:, 2],
                np.isnan(p[:, 0]), np.isinf(p[:, 1]), np.nan_to_num(p[:, 1]), np.logaddexp(p[:, 0], p[:, 1]),
                np.hypot(p[:, 1], p[:, 2]), np.sqrt((p * p).sum(1))]
    for j, (got, w) in enumerate(zip(r, want)):
        w = np.asarray(w)
        if w.dtype.kind == "f":
            w = w.astype(np.float32)
            ok = np.allclose(got, w, rtol=2e-7, atol=0, equal_nan=True) and np.array_equal(np.isnan(got), np.isnan(w))
        else:
            ok = np.array_equal(got, w.astype(np.int64))
        assert ok, (j, got, w)


def test_outputs_shorthand():
    """a bare shape in outputs is Sum(shape) (_api.py:509); Sum takes an int shape"""
    from items_lang import walk
    f = tm.vmap(walk, outputs={"hist": (256,), "side": tm.Sum(2)}, in_axes=(0, 0, None))
    assert f.outputs == {"hist": ((256,), "f32", False, None), "side": ((2,), "f32", False, None)}
    assert tm.Sum(4).shape == (4,) and tm.Sum(()).shape == ()


def test_vector_results():
    """an item returning a vector: one flat per-item result per element, regrouped into an (N, n) array"""
    import torch
    from oracle.ir_eval import Evaluator
    from items_lang import drift2d
    n = 16
    x0 = np.random.default_rng(1).uniform(0.3, 0.7, (n, 2)).astype(np.float32)
    keys = prng.split(prng.PRNGKey(2), n)
    f = tm.vmap(drift2d, outputs={"exits": tm.Sum((4,))}, in_axes=(0, 0, None), max_steps=10000)
    L = f.lowered((x0, keys, np.float32(0.1)))
    assert L.tr.result_groups == [(0, 2), (2, None)] and L.n_results == 3
    r = Evaluator(L.tr, 10000).run([x0, keys], [np.float32(0.1)])
    ys = [torch.from_numpy(np.asarray(v)) for v in r["results"]]
    xy, k = f._per_item(L, ys)
    assert tuple(xy.shape) == (n, 2) and tuple(k.shape) == (n,)
    assert ((xy <= 0) | (xy >= 1)).any(dim=1).all()


def test_randint_gumbel_categorical():
    """random.randint (in [minval, maxval), equal to its arithmetic restated in numpy on the same bits; minval when
    maxval <= minval), random.gumbel (-log(-log u)) and random.categorical (the Gumbel-max choice: frequencies near
    softmax(logits))"""
    from oracle.ir_eval import Evaluator

    def item(t, key):
        return (t, tl.random.randint(key, (), -3, 10), tl.random.randint(key, (2,), 5, 5)[1],
                tl.random.categorical(key, tl.array([0.0, 1.0, -1.0, 0.5])), tl.random.gumbel(key),
                tl.random.randint(key, (), 0, 100000), tl.random.randint(key, (), -70000, 2 ** 31 - 1))
    tr = T.trace_item(item, ["key"], 1, {})
    n = 4000
    keys = prng.split(prng.PRNGKey(21), n)
    r = Evaluator(tr, 1).run([keys], [])["results"]
    ri, same, cat, g, big, huge = r
    assert ri.min() == -3 and ri.max() == 9 and (same == 5).all()
    k1 = np.array([prng.threefry2x32(np.uint32(k[0]), np.uint32(k[1]), np.uint32(0), np.uint32(0)) for k in keys])
    k2 = np.array([prng.threefry2x32(np.uint32(k[0]), np.uint32(k[1]), np.uint32(0), np.uint32(1)) for k in keys])
    bits = lambda kk: np.array([np.bitwise_xor(*prng.threefry2x32(np.uint32(a), np.uint32(b), np.uint32(0),
                                                                  np.uint32(0))) for a, b in kk], np.uint64)
    span = 13
    mult = (65536 % span) ** 2 % span
    want = (((bits(k1) % span) * mult + bits(k2) % span) % (2 ** 32) % span).astype(np.int64) - 3
    assert np.array_equal(ri, want)
    # spans above 2^16: jax's multiplier (2^16 mod span)^2 mod span is formed in uint32, where the square wraps
    for span, lo, got in ((100000, 0, big), (2 ** 31 - 1 + 70000, -70000, huge)):
        m32 = (((65536 % span) ** 2) & 0xFFFFFFFF) % span
        want = ((((bits(k1) % span) * m32) & 0xFFFFFFFF) + bits(k2) % span) & 0xFFFFFFFF
        want = (want % span).astype(np.int64) + lo
        assert np.array_equal(got.astype(np.int64), want)
    assert (((65536 % 100000) ** 2) & 0xFFFFFFFF) % 100000 == 0      # the wrap that an exact product would miss
    p = np.exp([0.0, 1.0, -1.0, 0.5])
    p /= p.sum()
    freq = np.bincount(cat, minlength=4) / n
    assert np.abs(freq - p).max() < 0.03
    assert abs(float(np.mean(g)) - 0.5772) < 0.06


def test_scan():
    """lax.scan with a static length, unrolled: the final carry and the stacked outputs"""
    from oracle.ir_eval import Evaluator

    def item(t, p, key):
        c, ys = tl.scan(lambda c, x: (c * 0.5 + x, c + x), 0.0, p)
        c2, (a, b) = tl.scan(lambda c, _: (c + 1.0, (c, c * c)), 1.0, length=3)
        return t, c, ys[2], tl.sum(a) + tl.sum(b) + c2
    tr = T.trace_item(item, [("f32", 3), "key"], 1, {})
    p = np.float32([[1.0, 2.0, 4.0], [0.5, -1.0, 3.0]])
    r = Evaluator(tr, 1).run([p, prng.split(prng.PRNGKey(0), 2)], [])["results"]
    for row, c, y2 in zip(p, r[0], r[1]):
        cc, ys = np.float32(0), []
        for x in row:
            ys.append(cc + x)
            cc = cc * np.float32(0.5) + x
        assert c == cc and y2 == ys[2]
    assert (r[2] == np.float32(1 + 2 + 3 + 1 + 4 + 9 + 4)).all()


def test_constant_vector_lookup():
    """a constant vector (numpy or Python numbers) read by a traced index, as a Gillespie item's state-change table
    jnp.array([1, -1, 1, -1])[r]: a chain of selects of literals, clamped as jax.numpy clamps"""
    from oracle.ir_eval import Evaluator

    def item(t, x, key):
        r = (x * 4.0).astype(tl.int32)
        dx = tl.array(np.array([1, -1, 1, -1], np.int32))[r]
        w = tl.array([0.5, 1.5, 2.5, 3.5])[r - 1]
        return t, dx, w
    tr = T.trace_item(item, ["f32", "key"], 1, {})
    xs = np.float32([0.0, 0.3, 0.6, 0.9, 2.0, -1.0])
    r = Evaluator(tr, 1).run([xs, prng.split(prng.PRNGKey(0), len(xs))], [])["results"]
    idx = (xs * 4).astype(np.int32)
    tab = np.array([1, -1, 1, -1])
    assert np.array_equal(r[0], tab[np.clip(np.where(idx < 0, idx + 4, idx), 0, 3)])
    w = np.float32([0.5, 1.5, 2.5, 3.5])
    j = idx - 1
    assert np.array_equal(r[1], w[np.clip(np.where(j < 0, j + 4, j), 0, 3)])


def test_random_choice():
    """random.choice with replacement: with p, the inverse-CDF index searchsorted(cumsum(p), total (1 - u)) (restated
    in numpy on the same uniforms) and frequencies near p; without p, randint(0, n); values taken from a vector"""
    from oracle.ir_eval import Evaluator
    p = [0.1, 0.6, 0.3]

    def item(t, key):
        return (t, tl.random.choice(key, 3, p=tl.array(p)), tl.random.choice(key, tl.array([2.0, 4.0, 8.0])),
                tl.random.uniform(key))
    tr = T.trace_item(item, ["key"], 1, {})
    n = 3000
    r = Evaluator(tr, 1).run([prng.split(prng.PRNGKey(9), n)], [])["results"]
    pc = np.cumsum(np.float32(p), dtype=np.float32)
    want = np.searchsorted(pc, (pc[-1] * (np.float32(1) - r[2])).astype(np.float32), side="left")
    assert np.array_equal(r[0], want)
    assert np.abs(np.bincount(r[0], minlength=3) / n - np.array(p)).max() < 0.03
    assert set(np.unique(r[1])) <= {2.0, 4.0, 8.0}


def test_laplace_rademacher():
    """random.laplace (sign(u) log1p(-|u|): symmetric, mean |x| near 1) and random.rademacher (+-1, balanced)"""
    from oracle.ir_eval import Evaluator

    def item(t, key):
        return t, tl.random.laplace(key), tl.random.rademacher(key, (2,))[1]
    tr = T.trace_item(item, ["key"], 1, {})
    n = 4000
    r = Evaluator(tr, 1).run([prng.split(prng.PRNGKey(10), n)], [])["results"]
    assert abs(float(np.mean(r[0]))) < 0.1 and abs(float(np.mean(np.abs(r[0]))) - 1.0) < 0.08
    assert set(np.unique(r[1])) == {-1, 1} and abs(float(np.mean(r[1]))) < 0.06


def test_truncated_normal():
    """random.truncated_normal: inside (lower, upper), the standard normal's mean on [-1, 2] (about 0.2297)"""
    from oracle.ir_eval import Evaluator

    def item(t, key):
        return t, tl.random.truncated_normal(key, -1.0, 2.0)
    tr = T.trace_item(item, ["key"], 1, {})
    r = Evaluator(tr, 1).run([prng.split(prng.PRNGKey(11), 4000)], [])["results"][0]
    assert r.min() > -1.0 and r.max() < 2.0 and abs(float(r.mean()) - 0.2297) < 0.05


def test_interp_and_table_search():
    """searchsorted over a sorted table (an unrolled binary search) equals numpy's; interp over a vector and over
    tables equals its float32 formula and is close to numpy's float64 interp"""
    from oracle.ir_eval import Evaluator
    xp = np.float32([0.0, 0.1, 0.1, 0.4, 1.0, 2.5, 3.0])
    fp = np.float32([1.0, 2.0, 3.0, -1.0, 0.5, 4.0, 4.5])

    def item(t, x, key, txp, tfp):
        return (t, tl.searchsorted(txp, x), tl.searchsorted(txp, x, side="right"), tl.interp(x, txp, tfp),
                tl.interp(x, tl.array(list(xp)), tl.array(list(fp)), left=-9.0))
    tr = T.trace_item(item, ["f32", "key", ("table", "f32", (7,)), ("table", "f32", (7,))], 2, {})
    x = np.float32([-1.0, 0.0, 0.05, 0.1, 0.2, 0.4, 2.0, 2.9999, 3.0, 5.0])
    r = Evaluator(tr, 1).run([x, prng.split(prng.PRNGKey(0), len(x))], [xp, fp])["results"]
    assert np.array_equal(r[0], np.searchsorted(xp, x, "left"))
    assert np.array_equal(r[1], np.searchsorted(xp, x, "right"))
    i = np.clip(np.searchsorted(xp, x, "right"), 1, 6)
    dx = xp[i] - xp[i - 1]
    want = np.where(dx == 0, fp[i - 1], fp[i - 1] + ((x - xp[i - 1]) / np.where(dx == 0, 1, dx)) * (fp[i] - fp[i - 1]))
    want = np.where(x < xp[0], fp[0], np.where(x > xp[-1], fp[-1], want)).astype(np.float32)
    assert np.array_equal(r[2], want)
    assert np.allclose(r[2], np.interp(x, xp, fp), rtol=1e-5, atol=1e-6)
    assert np.array_equal(r[3], np.where(x < 0, np.float32(-9), want))


def test_lgamma_nextafter():
    """lang.lgamma (the shared double-precision lgamma, rounded once) against scipy's gammaln rounded to float32, and
    lang.nextafter against numpy, both through the IR evaluator (which runs the shared math of the device); neither
    has a derivative rule (the reference's op table has no digamma), so differentiating through them raises"""
    from oracle.ir_eval import Evaluator
    import scipy.special as sp

    def item(t, x, y):
        return t, tl.lgamma(x), tl.nextafter(x, y)
    tr = T.trace_item(item, ["f32", "f32"], 2, {})
    rng = np.random.default_rng(418)
    x = np.concatenate([rng.uniform(-12, 12, 3000), np.exp(rng.uniform(-30, 80, 2000)),
                        [0.0, -0.0, 1.0, 2.0, -3.0, 0.5, -2.5, np.inf, -np.inf, np.nan, 1e-45]]).astype(np.float32)
    y = np.where(rng.random(len(x)) < 0.5, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
    y[:5] = x[:5]
    r = Evaluator(tr, 1).run([x, y], [])["results"]
    lg, na = np.asarray(r[0], np.float32), np.asarray(r[1], np.float32)
    with np.errstate(all="ignore"):
        want = sp.gammaln(x.astype(np.float64)).astype(np.float32)
    want = np.where(np.isneginf(x), np.float32(np.inf), want)         # (C's lgamma(-inf) = +inf)
    ok = ~np.isnan(want)
    assert np.array_equal(np.isnan(lg), np.isnan(want))
    assert np.array_equal(lg[ok].view(np.uint32), want[ok].view(np.uint32))
    wn = np.nextafter(x, y)
    assert np.array_equal(np.isnan(na), np.isnan(wn))
    assert np.array_equal(na[~np.isnan(wn)].view(np.uint32), wn[~np.isnan(wn)].view(np.uint32))
    import tallymap_b200 as tm

    def walk(t, x, key, a):
        def body(c):
            k, x, t = c
            t = t.add("s", 0, tl.lgamma(a + x))
            return k + 1, x + 1.0, t
        k, x, t = tl.while_loop(lambda c: c[0] < 3, body, (0, x, t))
        return t, k
    f = tm.vmap(walk, outputs={"s": tm.Sum(())}, in_axes=(0, 0, None), max_steps=10)
    L = f.lowered((np.float32([1.0, 2.0]), prng.split(prng.PRNGKey(0), 2), np.float32(0.5)))
    assert "tmm::lgammaf" in L.fwd_source
    with pytest.raises(lower.LowerError, match="lgamma"):
        L.grad_program((0,))


def test_n_active_with_spawn_is_refused():
    """n_active with a spawning program raises, as the reference's mapped call does (_api.py:530-532)"""
    from tallymap_b200 import backend as B
    E, d, k = np.ones(4, np.float32), np.zeros(4, np.float32), prng.split(prng.PRNGKey(0), 4)
    with pytest.raises(ValueError, match="n_active with spawn is not supported"):
        B.run(B.SH_FWD, [E, d, k], [np.float32(1.0)], consts=(100,), n_active=2)


def test_sort_argsort():
    """sort / argsort of a vector (a sorting network of compare-exchanges): ascending, NaNs last, stable (numpy's
    stable sort on the same values, the signed zeros kept in their input order)"""
    from oracle.ir_eval import Evaluator

    def item(t, p, key):
        s, a = tl.sort(p), tl.argsort(p)
        return (t,) + tuple(s) + tuple(a)
    tr = T.trace_item(item, [("f32", 5), "key"], 2, {})
    nan = np.float32(np.nan)
    p = np.float32([[3.0, 1.0, 2.0, 1.0, -5.0], [nan, 0.0, -0.0, 2.0, nan], [4.0, 3.0, 2.0, 1.0, 0.0],
                    [1.0, 1.0, 1.0, 1.0, 1.0]])
    r = Evaluator(tr, 1).run([p, prng.split(prng.PRNGKey(0), len(p))], [])["results"]
    got_s = np.stack(r[:5], 1).astype(np.float32)
    got_a = np.stack(r[5:], 1)
    want_a = np.argsort(p, axis=1, kind="stable")
    assert np.array_equal(got_a, want_a)
    want_s = np.take_along_axis(p, want_a, 1)
    assert np.array_equal(got_s.view(np.uint32)[~np.isnan(got_s)], want_s.view(np.uint32)[~np.isnan(want_s)])
    assert np.array_equal(np.isnan(got_s), np.isnan(want_s))

    # a vector mixing Python-float constants with traced values: NaNs last whichever side holds the constant
    def mixed(t, p, key):
        v = tl.array([2.0, p[0], 0.5, p[1], float("nan"), p[2]])
        s, a = tl.sort(v), tl.argsort(v)
        return (t,) + tuple(s) + tuple(a)
    tr = T.trace_item(mixed, [("f32", 3), "key"], 2, {})
    q = np.float32([[nan, 1.0, 3.0], [-1.0, nan, nan], [0.5, 0.5, -0.0]])
    r = Evaluator(tr, 1).run([q, prng.split(prng.PRNGKey(0), len(q))], [])["results"]
    full = np.float32([[2.0, a, 0.5, b, nan, c] for a, b, c in q])
    want_a = np.argsort(full, axis=1, kind="stable")
    assert np.array_equal(np.stack(r[6:], 1), want_a)
    got_s = np.stack(r[:6], 1).astype(np.float32)
    want_s = np.take_along_axis(full, want_a, 1)
    assert np.array_equal(np.isnan(got_s), np.isnan(want_s))
    assert np.array_equal(got_s[~np.isnan(got_s)].view(np.uint32), want_s[~np.isnan(want_s)].view(np.uint32))


def test_records_argument_forms():
    """tallymap.Records(fields, capacity) in either order, capacity None (count-then-fill) by default; bad forms
    raise"""
    f32 = tm.api.torch.float32
    assert tm.Records({"a": f32}, 5).capacity == 5 and tm.Records(5, {"a": f32}).capacity == 5
    assert tm.Records({"a": f32}).capacity is None and tm.Records(fields={"a": f32}, capacity=None).capacity is None
    for bad in (lambda: tm.Records({"a": f32}, 0), lambda: tm.Records({}, 4), lambda: tm.Records({"a": f32}, "x"),
                lambda: tm.Records({"a": tm.api.torch.float64}, 4), lambda: tm.Records({"a": f32}, fields={"b": f32})):
        with pytest.raises((TypeError, ValueError)):
            bad()


def test_cond_branches_write_the_tally():
    """t.add / t.append / t.spawn inside lax.cond and lax.switch branches (nested too) are made by the taken branch
    only (tallymap/_rewrite.py:573-598): each effect carries its branch's predicate; the IR evaluator's sums, records
    and results equal those of the same item written with selects, and the forward, reverse, forward-mode and
    Records programs compile"""
    from oracle.ir_eval import Evaluator
    from items_lang import branch_writes, branch_writes_where, spawn_decay, spawn_decay_cond
    n = 300
    x = np.random.default_rng(3).uniform(0, 1, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(5), n)
    specs = {"h": ((5,), "f32")}
    recs = {"low": (1 << 14, (("k", "i32"), ("x", "f32")))}
    tr = T.trace_item(branch_writes, ["f32", "key", "f32"], 2, specs, recs)
    tw = T.trace_item(branch_writes_where, ["f32", "key", "f32"], 2, specs, recs)
    emits = [e for e in tr.body if e.prim == "emit"]
    assert len(emits) == 4 and all(len(e.ins) == 3 for e in emits)
    assert [e for e in tr.body if e.prim == "append"][0].ins[0].dtype == T.BOOL
    r = Evaluator(tr, 100).run([x, keys], [np.float32(1.3)])
    w = Evaluator(tw, 100).run([x, keys], [np.float32(1.3)])
    assert np.array_equal(r["sums"]["h"], w["sums"]["h"]) and r["sums"]["h"].min() > 0
    assert r["records"]["low"] == w["records"]["low"] and len(r["records"]["low"]) > 0
    assert np.array_equal(r["results"][0], w["results"][0])
    f = tm.vmap(branch_writes, outputs={"h": tm.Sum((5,)), "low": tm.Records({"k": tm.api.torch.int32,
                                                                        "x": tm.api.torch.float32})},
                in_axes=(0, 0, None), max_steps=100)
    L = f.lowered((x, keys, np.float32(1.3)))
    assert L.fwd.kernel > 0 and L.grad_program((0,)).kernel > 0 and L.jvp_program((0,), 1).kernel > 0
    assert all(p.kernel > 0 for p in L.records_programs())
    src = lower.forward_source(L.it)[0]
    assert src.count("if (v") >= 4
    # a spawn inside a cond branch: the same tree as spawn_decay's `when`
    g = np.zeros(50, np.int32)
    wv = np.random.default_rng(1).uniform(0.5, 1.5, 50).astype(np.float32)
    k2 = prng.split(prng.PRNGKey(13), 50)
    specs = ["i32", "f32", "key", "f32"]
    outs = {"Q": ((8,), "f32")}
    ra, rb = (Evaluator(T.trace_item(fn, specs, 3, outs, spawn=True), 10).run([g, wv, k2], [np.float32(1.1)])
              for fn in (spawn_decay_cond, spawn_decay))
    assert np.array_equal(ra["sums"]["Q"], rb["sums"]["Q"]) and ra["stats"][0] == rb["stats"][0] == 100


def _host_rejection(x0, key, a):
    """the rejection item (items_lang.rejection) restated with the host PRNG, one item: (h bins, tries, k, n, s)"""
    f = np.float32
    h, tries = np.zeros(9), [0, 0]
    k, x = 0, f(x0)
    while k < 200 and 0.0 < x < 1.0:
        kk = prng.fold_in(key, k)
        j, u, v = 0, f(1.0), f(1.0)
        while j < 64 and f(f(u * u) + f(v * v)) >= 1.0:
            kj = prng.fold_in(kk, j)
            u = f(f(2.0) * prng.uniform(prng.fold_in(kj, 0), 1)[0] - f(1.0))
            v = f(f(2.0) * prng.uniform(prng.fold_in(kj, 1), 1)[0] - f(1.0))
            j += 1
            tries[0] += 1
        if x > 0.5:
            tries[1] += 3
        x = f(x + f(f(0.05) * u))
        b = int(f(x * f(8.0)))
        if 0 <= b < 9:
            h[b] += float(f(a * x))
        k += 1
    y, n = f(abs(x)), 0
    while n < 32 and y > 0.01:
        n, y = n + 1, f(y * f(0.5))
    h[8] += float(f(a * y))
    return h, tries, k, n, sum(range(k % 5))


def test_inner_while_loops():
    """inner while loops -- inside the stepping loop's body (reading the step's key from outside, writing the tally
    inside), inside a cond branch (iterating only where the branch is taken), after the stepping loop, and a
    fori_loop with a traced bound -- trace to nested "while" equations that the IR evaluator runs as the host
    restatement does, bitwise; the forward, reverse, one-pass and forward-mode programs compile, inner loops that
    read a differentiated value included"""
    from oracle.ir_eval import Evaluator
    from items_lang import newton, rejection, rejection_active
    specs = {"h": ((9,), "f32"), "tries": ((2,), "i32")}
    tr = T.trace_item(rejection, ["f32", "key", "f32"], 2, specs)
    assert sum(e.prim == "while" for e in tr.body) == 2 and sum(e.prim == "while" for e in tr.post) == 2
    n = 24
    x0 = np.random.default_rng(6).uniform(0.2, 0.8, n).astype(np.float32)
    keys = prng.split(prng.PRNGKey(17), n)
    a = np.float32(1.25)
    r = Evaluator(tr, 1000).run([x0, keys], [a])
    h, tries = np.zeros(9), np.zeros(2, np.int64)
    for i in range(n):
        hi, ti, k, nn, s_ = _host_rejection(x0[i], keys[i], a)
        h += hi
        tries += ti
        assert (r["results"][0][i], r["results"][1][i], r["results"][2][i]) == (k, nn, s_), i
    assert np.array_equal(r["sums"]["tries"], tries) and tries[0] > 0 and tries[1] > 0
    assert np.abs(r["sums"]["h"] - h).max() <= 1e-9 * np.abs(h).max()
    f = tm.vmap(rejection, outputs={"h": tm.Sum((9,)), "tries": tm.Sum((2,), tm.api.torch.int32)},
                in_axes=(0, 0, None), max_steps=1000)
    L = f.lowered((x0, keys, a))
    src = L.fwd_source
    assert src.count("while (true)") >= 4
    assert L.grad_program((0,)).kernel > 0 and L.jvp_program((0,), 1).kernel > 0
    assert L.vg_program((0,)).kernel > 0
    # inner loops that read the differentiated value: reverse mode transposes them (trip count, then the iterations
    # newest first from recomputed states), forward mode carries their tangents
    for item in (rejection_active, newton):
        g = tm.vmap(item, outputs={"h": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=10)
        La = g.lowered((x0, keys, a))
        assert La.fwd.kernel > 0 and La.grad_program((0,)).kernel > 0 and La.jvp_program((0,), 2).kernel > 0
        assert La.vg_program((0,)).kernel > 0
        assert "for (int gw" in lower.grad_source(La.it, [0])[0]


def _acc_outputs():
    import torch
    return {"f64": tm.Sum((4,), torch.float64), "i64": tm.Sum((4,), torch.int64),
            "w64": tm.Sum((4,), torch.float64, fixed_point=True, scale=2.0 ** 20),
            "wi32": tm.Sum((4,), torch.int32, fixed_point=True, scale=1.0),
            "wbig": tm.Sum((4,), torch.float64, fixed_point=True, scale=2.0 ** 50)}


def test_wider_accumulators_lower_and_evaluate():
    """Sum outputs of float64 and int64 and scaled fixed-point Sums (tallymap/_api.py:55-84) lower to float64 /
    int64 atomics and to the carry-word accumulator read out by the launch's last block; grad compiles (their
    cotangents enter the float32 adjoint), value_and_grad falls back to it, forward mode refuses them; the IR
    evaluator's scaled sums are exact integers (wbig: totals far past 2^63)"""
    import torch
    from oracle.ir_eval import Evaluator
    from items_lang import accumulators
    outs = _acc_outputs()
    f = tm.vmap(accumulators, outputs=outs, in_axes=(0, 0, None), max_steps=200)
    x0 = np.random.default_rng(1).uniform(0.3, 0.7, 64).astype(np.float32)
    keys = prng.split(prng.PRNGKey(2), 64)
    L = f.lowered((x0, keys, np.float32(1.5)))
    assert [t.dtype for t in L.fwd.tallies] == [torch.float64, torch.int64, torch.float64, torch.int32, torch.float64]
    assert [t.wide for t in L.fwd.tallies] == [0.0, 0.0, 2.0 ** 20, 1.0, 2.0 ** 50]
    assert "WideSum::readout" in L.fwd_source and "(unsigned long long*)&c.g1" in L.fwd_source
    assert L.grad_program((0,)).kernel > 0 and L.vg_program((0,)) is None
    with pytest.raises(NotImplementedError, match="forward mode"):
        L.jvp_program((0,), 1)
    wide = {"w64": ("f64", 2.0 ** 20), "wi32": ("i32", 1.0), "wbig": ("f64", 2.0 ** 50)}
    specs = {k: ((4,), "f32" if k in ("f64", "w64", "wbig") else "i32") for k in outs}
    tr = T.trace_item(accumulators, ["f32", "key", "f32"], 2, specs)
    r = Evaluator(tr, 200, wide=wide).run([x0, keys], [np.float32(1.5)])
    assert r["sums"]["i64"].dtype == np.int64 and r["sums"]["wi32"].dtype == np.int64
    assert r["sums"]["wbig"].min() > 2.0 ** 63 / 2.0 ** 50 and not r["stats"][3]
    assert np.abs(r["sums"]["w64"] - r["sums"]["f64"]).max() <= 64 * 100 * 2.0 ** -21


def test_memory_model_matches_the_layout():
    """tallymap_b200.output_memory / cell_bytes / call_memory / max_cells (tallymap/_memory.py:155-260): the per-cell
    bytes of each Sum kind equal what the forward program's result layout allocates for that output (the output and
    its accumulator words); derivatives add the tangent tallies or the cotangent; supported_primitives lists the jaxpr
    front end's table"""
    from items_lang import accumulators
    outs = dict(_acc_outputs(), f64=tm.Sum((4,), tm.api.torch.float64))
    f = tm.vmap(accumulators, outputs=outs, in_axes=(0, 0, None), max_steps=200)
    x0 = np.float32([0.5, 0.4])
    L = f.lowered((x0, prng.split(prng.PRNGKey(2), 2), np.float32(1.5)))
    layout, _ = L.fwd.result_layout(2)
    for nm, o in outs.items():
        allocated = sum(nb for name, nb, _, _ in layout if name == nm or name.startswith(nm + "."))
        assert tm.output_memory(o).per_cell * 4 == allocated, nm
    ex = tm.Sum((1000,), fixed_point=True)
    assert tm.output_memory(ex).per_cell == 48 and tm.output_memory(ex, "jvp", lanes=2).per_cell == 48 + 2 * 48
    assert tm.output_memory(tm.Sum(8), "grad").per_cell == 4 and tm.output_memory(tm.Sum(8), "vjp").per_cell == 8
    assert tm.cell_bytes(ex, cells=10) == (48 * 10 + tm.memory._LAUNCH) / 10
    assert tm.call_memory({"a": tm.Sum((4,)), "b": ex}) == 4 * 4 + 48 * 1000 + tm.memory._LAUNCH
    assert tm.max_cells(tm.Sum(1)) == 2 ** 31 - 1 and tm.max_cells(ex, memory=48 * 100 + tm.memory._LAUNCH) == 100
    with pytest.raises(ValueError):
        tm.output_memory(tm.Sum(4, tm.api.torch.float64), "jvp")
    prims = tm.supported_primitives()
    assert {"while", "cond", "scan", "tallymap_emit", "tallymap_claim", "gather", "sort", "exp"} <= set(prims)
    assert "fft" not in prims and prims == sorted(prims)


def test_diagnostics_and_history():
    """tallymap_b200.diagnostics / history (tallymap/_diagnostics.py:1-53): the last lowered item programs (their
    equation counts and the float literals they closed over) and compiled kernels (tag, id, source digest, compile
    time or the disk cache), the environment and the device; reset clears the history"""
    tm.diagnostics(reset=True)
    f = tm.vmap(walk, outputs={"hist": tm.Sum((256,)), "side": tm.Sum((2,))}, in_axes=(0, 0, None), max_steps=20000)
    f.lowered(_args_walk())
    h = tm.history()
    assert h["programs"][-1]["tag"] == "walk" and h["programs"][-1]["equations"]["body"] > 0
    assert 0.02 in h["programs"][-1]["float_literals"]
    assert any(k["tag"] == "walk_fwd" and len(k["source_sha256"]) == 64 for k in h["kernels"])
    d = tm.diagnostics(reset=True)
    assert d["versions"]["tallymap_b200"] and d["cuda"]["arch"] == "sm_100a" and "cuda_available" in d["platform"]
    assert d["programs"] and not tm.history()["programs"]


def test_vector_at_updates():
    """x.at[i].set / add / multiply / min / max / get on a per-item vector, static and traced indices (negative
    from the end; out of range dropped by default, clamped with mode='clip'): the IR evaluator against numpy"""
    from oracle.ir_eval import Evaluator

    def item(t, v, i, y):
        a = v.at[i].set(y)
        b = v.at[i].add(y, mode="clip")
        c = v.at[-1].multiply(y)
        d = v.at[i].max(y)
        e = v.at[7].set(y)
        return t, a, b, c, d, e, v.at[i].get()
    tr = T.trace_item(item, [("f32", 4), "i32", "f32"], 3, {})
    n = 40
    rng = np.random.default_rng(5)
    vs = rng.normal(size=(n, 4)).astype(np.float32)
    ii = rng.integers(-6, 7, n).astype(np.int32)
    ys = rng.normal(size=n).astype(np.float32)
    res = [np.asarray(r) for r in Evaluator(tr, 1).run([vs, ii, ys], [])["results"]]
    for q in range(n):
        v, k, y = vs[q], int(ii[q]), ys[q]
        kk = k + 4 if k < 0 else k
        a = v.copy()
        if 0 <= kk < 4:
            a[kk] = y
        b = v.copy()
        b[min(max(kk, 0), 3)] += y
        c = v.copy()
        c[3] *= y
        d = v.copy()
        if 0 <= kk < 4:
            d[kk] = max(d[kk], y)
        want = np.concatenate([a, b, c, d, v, [v[min(max(kk, 0), 3)]]]).astype(np.float32)
        got = np.float32([res[j][q] for j in range(21)])
        assert np.array_equal(got, want), q


def test_bit_counts():
    """lax.population_count and lax.clz of int32 / uint32 (lang and the jaxpr front end): the IR evaluator against
    Python's bit counts of the 32-bit pattern, the lowering through __popc / __clz"""
    from oracle.ir_eval import Evaluator

    def item(t, x, u):
        return t, tl.population_count(x), tl.clz(x), tl.population_count(u), tl.clz(u)
    tr = T.trace_item(item, ["i32", "u32"], 2, {})
    xs = np.int32([0, 1, -1, 2 ** 31 - 1, -(2 ** 31), 12345, -7])
    us = np.uint32([0, 1, 2 ** 32 - 1, 2 ** 31, 255, 65536, 3])
    r = [np.asarray(v) for v in Evaluator(tr, 1).run([xs, us], [])["results"]]
    pc = lambda v: bin(int(v) & 0xFFFFFFFF).count("1")
    cz = lambda v: 32 - (int(v) & 0xFFFFFFFF).bit_length()
    assert list(r[0]) == [pc(v) for v in xs] and list(r[1]) == [cz(v) for v in xs]
    assert list(r[2]) == [pc(v) for v in us] and list(r[3]) == [cz(v) for v in us]
    src = lower.forward_source(lower.Item(tr, ["i32", "u32"], "bits"))[0]
    assert "__popc((unsigned)" in src and "__clz((int)" in src
    f = tm.vmap(lambda t, x: (t, tl.population_count(x) + tl.clz(x)), outputs={}, in_axes=(0,))
    assert f.lowered((xs,)).fwd.kernel > 0
    assert {"population_count", "clz", "lgamma"} <= set(tm.supported_primitives())


def test_inner_loop_carries_keys_and_vectors():
    """an inner loop whose carry holds a key (re-derived each iteration) and a vector: traced, evaluated as the
    host's loop with the host PRNG, and compiled"""
    from oracle.ir_eval import Evaluator

    def item(t, x, key):
        def body(d):
            j, kk, v = d
            k2 = tl.random.fold_in(kk, j)
            u = tl.random.uniform(k2)
            return j + 1, k2, tl.array([v[1], v[0] + u])
        n = tl.while_loop(lambda c: c < 1, lambda c: c + 1, 0)          # (the stepping loop: the next is inner)
        j, kk, v = tl.while_loop(lambda d: d[0] < 3 * n, body, (0, key, tl.array([x, 0.0])))
        return t, v[0], v[1]
    tr = T.trace_item(item, ["f32", "key"], 2, {})
    assert [e.prim for e in tr.post] == ["while"]
    xs = np.float32([0.5, -1.0, 2.0])
    keys = prng.split(prng.PRNGKey(4), 3)
    r = Evaluator(tr, 1).run([xs, keys], [])["results"]
    for i in range(3):
        kk, v = keys[i], [xs[i], np.float32(0.0)]
        for j in range(3):
            kk = prng.fold_in(kk, j)
            u = prng.uniform(kk, 1)[0]
            v = [v[1], np.float32(v[0] + u)]
        assert (np.float32(r[0][i]), np.float32(r[1][i])) == (v[0], v[1]), i
    f = tm.vmap(item, outputs={}, in_axes=(0, 0))
    assert f.lowered((xs, keys)).fwd.kernel > 0
