"""Benchmark configuration 4's item as a user writes it (tests/items_lang.py lorenz), through the traced lowering,
against the hand-lowered kernels (csrc/items_ode.cuh) and the oracle: the forward bitwise (trip counts, flags, every
final state), the gradient w.r.t. beta by the generated forward-mode program and by the generated replay within the
float tolerance of the hand-lowered ones."""
import numpy as np
import pytest
import torch

import tallymap_b200 as tm
from tallymap_b200 import backend as B

pytestmark = pytest.mark.gpu
BETA = np.float32(8.0 / 3.0)


def _f(n, M=50000):
    from items_lang import lorenz
    return tm.vmap(lorenz, outputs={"final": tm.Sum((n, 3)), "mean_z": tm.Sum(())}, in_axes=(0, 0, 0, 0, None),
                   max_steps=M)


@pytest.mark.parametrize("n", [1, 3000])
def test_traced_lorenz_forward_bitwise(cuda, orc, n):
    inp = orc.od_inputs(n, seed=7)
    r = _f(n)(*inp, BETA)
    torch.cuda.synchronize()
    ref = orc.od_fwd(*inp)
    assert np.array_equal(r.per_item.cpu().numpy(), ref["k"])
    assert np.array_equal(r.outputs["final"].cpu().numpy().view(np.uint32), ref["final"].view(np.uint32))
    assert abs(float(r.outputs["mean_z"]) - float(ref["mean"][0])) <= 1e-5 * abs(float(ref["mean"][0]))


def test_traced_lorenz_gradients(cuda, orc):
    """value_and_grad (the generated forward-mode launch) and grad (the generated replay) against the hand-lowered
    one-pass and replay gradients"""
    n = 4000
    inp = orc.od_inputs(n, seed=11)
    ctf = np.random.default_rng(2).normal(size=(n, 3)).astype(np.float32)
    f = _f(n)
    cts = {"final": torch.from_numpy(ctf), "mean_z": torch.tensor(0.5)}
    r, g1 = f.value_and_grad(*inp, BETA, wrt=4, cotangents=cts)
    g2 = f.grad(*inp, BETA, wrt=4, cotangents=cts)
    torch.cuda.synchronize()
    hv = B.run(B.OD_VG1, list(inp), [BETA, ctf, np.float32(0.5)], consts=(50000,))
    hg = B.run(B.OD_GRAD, list(inp), [BETA, ctf, np.float32(0.5)], consts=(50000,))
    torch.cuda.synchronize()
    gv, gg = float(hv[2][0]), float(hg[0][0])
    assert abs(float(g1) - gv) <= 1e-4 * abs(gv)
    assert abs(float(g2) - gg) <= 1e-4 * abs(gg)
    assert np.array_equal(r.outputs["final"].cpu().numpy().view(np.uint32), hv[0].cpu().numpy().view(np.uint32))
