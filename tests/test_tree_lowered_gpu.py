"""GPU parity of reverse mode through spawn for traced items: the tree adjoint (tallymap/_reverse_spawn.py:233-336)
lowered from any spawning item -- the recording forward, one adjoint launch per generation, deepest first, and one
over the roots.  Checked against the oracle's tree adjoint of the shower (oracle sh_grad), against the hand-lowered
shower's (backend.tree_grad), against forward mode through spawn and against central differences of the IR
evaluator (items whose outputs are polynomials in the differentiated value); and the poisoning paths of
_reverse_spawn.py:28-33 -- a record that misses children, a replay that disagrees with the record (the reference's
negative control: a perturbed record), truncation and dropped children."""
import numpy as np
import pytest
import torch

import tallymap_b200 as tm
from tallymap_b200 import backend as B
from tallymap_b200 import prng

pytestmark = pytest.mark.gpu


def near_roots(a, b, rel=1e-5, ab=1e-6):
    """per root: within `rel` relative, or `ab` absolute for near-zero roots (the float tolerance)"""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= np.maximum(rel * np.abs(b), ab)))


def _shower(Q=1 << 22, M=100000):
    from items_lang import shower
    return tm.vmap(shower, outputs={"dep": tm.Sum((512,)), "count": tm.Sum((1,), torch.int32)},
                   in_axes=(0, 0, 0, None), max_steps=M, spawn=tm.Queue(Q))


@pytest.mark.parametrize("n", [1, 777, 20000])
def test_traced_shower_tree_adjoint_matches_oracle(cuda, orc, n):
    """the traced shower's tree adjoint w.r.t. the roots' E0 and depth0 and the broadcast X0: per root within the
    float tolerance of the oracle's tree adjoint; the forward outputs (from the recording launch) as the oracle's
    forward; no replay mismatch"""
    E0, d0, keys = orc.sh_inputs(n)
    ct = np.random.default_rng(n).normal(size=512).astype(np.float32)
    f = _shower()
    r, (gE, gD, gX) = f.value_and_grad(E0, d0, keys, np.float32(1.0), wrt=(0, 1, 3),
                                       cotangents={"dep": torch.from_numpy(ct)})
    torch.cuda.synchronize()
    B.check_status(B.tree_adjoint.last["fwd_ctl"])
    B.check_status(B.tree_adjoint.last["ctl"])
    info = f.last_tree
    assert int(info["mismatch"]) == 0 and int(info["replay_truncated"]) == 0 and not bool(info["poisoned"])
    ref = orc.sh_grad(E0, d0, keys, ct_dep=ct)
    assert near_roots(gE.cpu().numpy(), ref["g_E"])
    assert near_roots(gD.cpu().numpy(), ref["g_depth"])
    assert float(gX) == float(ref["g_X0"][0]) == 0.0
    fw = orc.sh_fwd(E0, d0, keys)
    assert np.array_equal(r.outputs["count"].cpu().numpy(), fw["count"])
    assert np.array_equal(r.per_item.cpu().numpy(), fw["k"])
    assert info["children"] == int(fw["stats"][0])


def test_traced_shower_tree_adjoint_matches_hand_lowered(cuda, orc):
    """2^16 roots (~6e7 particles): the traced tree adjoint against the hand-lowered one, per root; the same
    generations; bitwise repeatable"""
    E0, d0, keys = orc.sh_inputs(1 << 16)
    ct = np.random.default_rng(4).normal(size=512).astype(np.float32)
    f = _shower()
    gE, gD = f.grad(E0, d0, keys, np.float32(1.0), wrt=(0, 1), cotangents={"dep": torch.from_numpy(ct)})
    info = f.last_tree
    h = B.tree_grad([E0, d0, keys], np.float32(1.0), ct)
    torch.cuda.synchronize()
    assert info["generations"] == h["info"]["generations"] and info["children"] == h["info"]["children"]
    assert info["generation_sizes"] == h["info"]["generation_sizes"]
    assert near_roots(gE.cpu().numpy(), h["ct_E"].cpu().numpy())
    assert near_roots(gD.cpu().numpy(), h["ct_depth"].cpu().numpy())
    gE2, _ = f.grad(E0, d0, keys, np.float32(1.0), wrt=(0, 1), cotangents={"dep": torch.from_numpy(ct)})
    assert torch.equal(gE.view(torch.int32), gE2.view(torch.int32))


def _decay(M=10, Q=1 << 16):
    from items_lang import spawn_decay
    return tm.vmap(spawn_decay, outputs={"Q": tm.Sum((8,))}, in_axes=(0, 0, 0, None), max_steps=M,
                   spawn=tm.Queue(Q))


def _decay_args(n):
    rng = np.random.default_rng(12)
    return (np.zeros(n, np.int32), rng.uniform(0.5, 1.5, n).astype(np.float32), prng.split(prng.PRNGKey(13), n))


def _eval(fn, specs, outs, per_item, bc, M):
    from oracle.ir_eval import Evaluator
    from tallymap_b200 import trace as T
    tr = T.trace_item(fn, specs, 3, outs, spawn=True)
    return Evaluator(tr, M).run(list(per_item), list(bc))


def test_traced_tree_adjoint_broadcast_and_roots(cuda):
    """a post-loop spawn two generations deep (spawn_decay, polynomial in a and in each root's w): the broadcast
    cotangent against forward mode through spawn and a central difference of the IR evaluator; each root's
    cotangent of w against a central difference of that root's tree alone"""
    from items_lang import spawn_decay
    args = _decay_args(3000)
    a, h = 1.1, 1.1e-2
    ct = np.linspace(-1.0, 2.0, 8).astype(np.float32)
    f = _decay()
    r, (gw, ga) = f.value_and_grad(*args, np.float32(a), wrt=(1, 3), cotangents={"Q": torch.from_numpy(ct)})
    torch.cuda.synchronize()
    B.check_status(B.tree_adjoint.last["ctl"])
    assert f.last_tree["generations"] == 2 and f.last_tree["children"] == 2 * 3000
    assert int(f.last_tree["mismatch"]) == 0
    # forward mode (one launch, the tangent carried by each child)
    _, gf = f.value_and_grad(*args, np.float32(a), wrt=3, cotangents={"Q": torch.from_numpy(ct)})
    torch.cuda.synchronize()
    assert abs(float(ga) - float(gf)) <= 1e-5 * abs(float(gf))
    specs, outs = ["i32", "f32", "key", "f32"], {"Q": ((8,), "f32")}
    q = lambda aa, per=args: _eval(spawn_decay, specs, outs, per, [np.float32(aa)], 10)["sums"]["Q"]
    c64 = ct.astype(np.float64)
    want = float(np.dot(c64, (q(a + h) - q(a - h)) / (2 * h)))
    assert abs(float(ga) - want) <= 1e-3 * abs(want)
    # per root: that root's tree alone, w moved by +-hw
    gw = gw.cpu().numpy()
    hw = 1e-2
    for i in [0, 1, 17, 2999]:
        one = lambda dw: (args[0][i:i + 1], np.array([args[1][i] + dw], np.float32), args[2][i:i + 1])
        d = float(np.dot(c64, (q(a, one(hw)) - q(a, one(-hw))) / (2 * hw)))
        assert abs(float(gw[i]) - d) <= 1e-3 * max(abs(d), 1e-3), (i, float(gw[i]), d)
    assert near_roots(r.outputs["Q"].cpu().numpy(), q(a), rel=1e-5, ab=1e-4)


def test_traced_tree_adjoint_post_loop_walk(cuda):
    """spawn_walk: an integer generation leaf, a float weight leaf and a key, one child after the loop while g < 3
    (three generations): each root's cotangent of x against a central difference of its tree alone (where the
    difference is smooth); the gradient through the public grad()"""
    from items_lang import spawn_walk
    n = 2000
    rng = np.random.default_rng(9)
    g = np.zeros(n, np.int32)
    x = rng.uniform(0.5, 1.5, n).astype(np.float32)
    x[np.abs(x - 1.0) < 0.05] = 0.8                     # (away from the root's trip-count step at x = 1)
    keys = prng.split(prng.PRNGKey(11), n)
    f = tm.vmap(spawn_walk, outputs={"Q": tm.Sum((16,)), "C": tm.Sum((16,), torch.int32)}, in_axes=(0, 0, 0),
                max_steps=100, spawn=tm.Queue(4096))
    ct = np.random.default_rng(2).normal(size=16).astype(np.float32)
    gx = f.grad(g, x, keys, wrt=1, cotangents={"Q": torch.from_numpy(ct)})
    torch.cuda.synchronize()
    B.check_status(B.tree_adjoint.last["ctl"])
    assert f.last_tree["generations"] == 3 and int(f.last_tree["mismatch"]) == 0
    specs, outs = ["i32", "f32", "key"], {"Q": ((16,), "f32"), "C": ((16,), "i32")}
    gx = gx.cpu().numpy()
    c64 = ct.astype(np.float64)
    checked = 0
    for i in [0, 5, 17, 999, 1500, 1999]:
        q = lambda dx: _eval(spawn_walk, specs, outs, (g[i:i + 1], np.array([x[i] + dx], np.float32),
                                                       keys[i:i + 1]), [], 100)["sums"]["Q"]
        d1, d2 = (float(np.dot(c64, (q(h) - q(-h)) / (2 * h))) for h in (1e-3, 2e-3))
        if abs(d1 - d2) > 1e-4 * max(abs(d1), 1e-3):
            continue              # (a descendant's trip count steps inside the difference: not differentiable there)
        checked += 1
        assert abs(float(gx[i]) - d1) <= 1e-3 * max(abs(d1), 1e-3), (i, float(gx[i]), d1)
    assert checked >= 4


def test_traced_tree_adjoint_poisons(cuda):
    """never a silently partial gradient: max_steps that truncates items, a Queue that drops children, a record
    too small for the tree -- each gives NaN cotangents"""
    args = _decay_args(2000)
    cts = {"Q": torch.ones(8)}
    f = _decay(M=2)
    _, (gw, ga) = f.value_and_grad(*args, np.float32(1.1), wrt=(1, 3), cotangents=cts)
    torch.cuda.synchronize()
    assert torch.isnan(ga) and torch.isnan(gw).all()
    f = _decay(Q=64)
    r, (gw, ga) = f.value_and_grad(*args, np.float32(1.1), wrt=(1, 3), cotangents=cts)
    torch.cuda.synchronize()
    if int(r.stats["children_dropped"]) > 0:
        assert torch.isnan(ga) and torch.isnan(gw).all()
    f = _decay()
    L = f.lowered((*args, np.float32(1.1)))
    t = B.tree_record(L.rec_program(), list(args), [np.float32(1.1)], max_steps=10, record=100)
    assert t["incomplete"] and t["total"] == 4000
    res = B.tree_adjoint(L.tree_program((0,)), t, [torch.ones(8)], max_steps=10)
    torch.cuda.synchronize()
    assert bool(res["poisoned"]) and res["info"]["launches"] == 2


def test_traced_tree_adjoint_detects_a_perturbed_record(cuda):
    """the reference's negative control (_reverse_spawn.py:22-26, 69-73): a record whose child no longer holds what
    its parent's replay spawns is counted as a replay mismatch and poisons the gradient; the untouched record gives
    none"""
    args = _decay_args(500)
    f = _decay()
    L = f.lowered((*args, np.float32(1.1)))
    rec, adj = L.rec_program(), L.tree_program((0,))
    t = B.tree_record(rec, list(args), [np.float32(1.1)], max_steps=10)
    clean = B.tree_adjoint(adj, t, [torch.ones(8)], max_steps=10)
    torch.cuda.synchronize()
    assert int(clean["info"]["mismatch"]) == 0 and not bool(clean["poisoned"])
    words = t["results"]["record"]
    rs = rec.record_bytes // 4
    words[1 * rs + 1] += 1           # record slot 1's float leaf (w): one ulp away from what the parent spawned
    bad = B.tree_adjoint(adj, t, [torch.ones(8)], max_steps=10)
    torch.cuda.synchronize()
    assert int(bad["info"]["mismatch"]) >= 1 and bool(bad["poisoned"])
