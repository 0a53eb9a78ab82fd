"""GPU parity of the branching shower: the warp-aggregated spawn ring against the oracle's
depth-first traversal.  With a ring large enough to drop nothing: particle count, spawned children, per-root trip
counts and truncation flags, and every stat bitwise; the depth deposit within the float-tally tolerance.  With a
tiny ring: children are dropped and counted, every popped child still runs exactly once, and no wait times out."""
import numpy as np
import pytest
import torch

from tallymap_b200 import backend as B

pytestmark = pytest.mark.gpu
FT = 1e-5


def gpu_sh(inp, X0=1.0, M=100000, Q=None):
    out = B.run(B.SH_FWD, list(inp), [np.float32(X0)], consts=(M,), queue=Q)
    torch.cuda.synchronize()
    B.check_status(B.run.last["ctl"])
    dep, count, stats, k, tr = [o.cpu().numpy() for o in out]
    return dict(dep=dep, count=count, stats=stats, k=k, trunc=tr.astype(bool))


@pytest.mark.parametrize("n", [1, 777, 20000])
def test_sh_forward(cuda, orc, n):
    inp = orc.sh_inputs(n)
    ref = orc.sh_fwd(*inp)
    got = gpu_sh(inp)
    assert np.array_equal(got["count"], ref["count"])
    assert np.array_equal(got["stats"], ref["stats"]) and got["stats"][1] == 0
    assert np.array_equal(got["k"], ref["k"]) and np.array_equal(got["trunc"], ref["trunc"])
    assert np.abs(got["dep"].astype(np.float64) - ref["dep"]).max() <= FT * np.abs(ref["dep"]).max()


def test_sh_truncation(cuda, orc):
    inp = orc.sh_inputs(3000)
    ref = orc.sh_fwd(*inp, max_steps=1)
    got = gpu_sh(inp, M=1)
    assert ref["stats"][2] > 0 and ref["trunc"].any()
    assert np.array_equal(got["stats"], ref["stats"]) and np.array_equal(got["count"], ref["count"])
    assert np.array_equal(got["trunc"], ref["trunc"])


@pytest.mark.parametrize("Q", [64, 4096])
def test_sh_small_ring_drops(cuda, orc, Q):
    inp = orc.sh_inputs(5000)
    got = gpu_sh(inp, Q=Q)
    spawned, dropped = int(got["stats"][0]), int(got["stats"][1])
    assert dropped > 0
    assert int(got["count"][0]) == 5000 + spawned          # every root and every pushed child ran once


def test_sh_full_size(cuda, orc):
    """N = 1,048,576 primaries (~10^9 particles): counts repeatable; energy conserved into the deposit (up to the
    deposits dropped beyond depth 64, counted in stats[4])"""
    inp = orc.sh_inputs(1048576)
    a = gpu_sh(inp)
    b = gpu_sh(inp)
    assert np.array_equal(a["count"], b["count"]) and np.array_equal(a["stats"], b["stats"])
    assert np.array_equal(a["k"], b["k"])
    assert int(a["count"][0]) == 1048576 + int(a["stats"][0]) and a["stats"][1] == 0
    e0 = float(inp[0].astype(np.float64).sum())
    assert abs(float(a["dep"].astype(np.float64).sum()) - e0) <= 1e-3 * e0
