"""GPU: the device's exact f32 sum (the accumulator of every gradient's cotangent tally) against the golden known
answers of tests/golden/exact_sum.npz (the restated integer reference of the reference's tests/edge.py:2037-2064),
through the C ABI: tm_exact_scatter bitwise, and tm_exact_combine (the multi-GPU combine of per-rank words)
bitwise against the single-pass sum."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SETS = ["uniform", "wide", "subnormal", "cancel", "oob", "overflow"]


def words_len(nb):
    return nb * 5 + (nb + 1) // 2


def scatter(tmlib, vals, bins, nb):
    dev = torch.device("cuda", 0)
    v = torch.from_numpy(np.ascontiguousarray(vals, np.float32)).to(dev)
    b = torch.from_numpy(np.ascontiguousarray(bins, np.int32)).to(dev)
    w = torch.empty(words_len(nb), dtype=torch.int64, device=dev)
    out = torch.empty(nb, dtype=torch.float32, device=dev)
    st = torch.zeros(5, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    P = ctypes.c_void_p
    tmlib.check(tmlib.lib().tm_exact_scatter(P(s), P(v.data_ptr()), P(b.data_ptr()), len(vals), nb, P(w.data_ptr()),
                                             P(out.data_ptr()), P(st.data_ptr())))
    torch.cuda.synchronize()
    return out.cpu().numpy(), st.cpu().numpy(), w


@pytest.mark.parametrize("name", SETS)
def test_exact_scatter_golden(cuda, tmlib, name):
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    vals, bins, nb, exp = d[name + "_vals"], d[name + "_bins"], int(d[name + "_nb"]), d[name + "_expect"]
    out, st, _ = scatter(tmlib, vals, bins, nb)
    assert np.array_equal(out, exp, equal_nan=True)
    ok = ~np.isnan(exp)
    assert np.array_equal(out[ok].view(np.uint32), exp[ok].view(np.uint32))
    assert st[3] == int(np.isnan(exp).sum())
    assert st[4] == int(((bins < 0) | (bins >= nb)).sum())


@pytest.mark.parametrize("name", ["uniform", "wide", "subnormal"])
def test_exact_combine_matches_single_pass(cuda, tmlib, name):
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    vals, bins, nb, exp = d[name + "_vals"], d[name + "_bins"], int(d[name + "_nb"]), d[name + "_expect"]
    parts = np.array_split(np.arange(len(vals)), 3)
    words = torch.cat([scatter(tmlib, vals[p], bins[p], nb)[2] for p in parts])
    dev = torch.device("cuda", 0)
    out = torch.empty(nb, dtype=torch.float32, device=dev)
    st = torch.zeros(5, dtype=torch.int32, device=dev)
    P = ctypes.c_void_p
    tmlib.check(tmlib.lib().tm_exact_combine(P(torch.cuda.current_stream().cuda_stream), P(words.data_ptr()), 3, nb,
                                             P(out.data_ptr()), P(st.data_ptr())))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))
