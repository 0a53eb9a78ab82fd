"""GPU test of tm_exact_scatter_noalloc, the exact scatter-add for callers that cannot allocate device memory (an
XLA custom-call handler living inside XLA's memory pool, or a caller that must not block on cudaMalloc's implicit
synchronisation).  It keeps its scratch words in a fixed array inside libtm_b200.so instead of asking for a buffer.

Through the C ABI it must give bitwise the output of tm_exact_scatter (the entry point that takes caller scratch; the
exact sum's tolerance is zero), on two calls in a row with different inputs (the shared fixed array must be cleared
between calls), and must reject more bins than its fixed scratch holds.  This file is collected last, so a run that
stops at the first failure has run everything else first; it also passes alone in a fresh process (the first call on
the device does the one-time address lookup)."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MAX_BINS = 65536


def run_both(tmlib, vals, bins, nb):
    dev = torch.device("cuda", 0)
    P = ctypes.c_void_p
    v = torch.from_numpy(np.ascontiguousarray(vals, np.float32)).to(dev)
    b = torch.from_numpy(np.ascontiguousarray(bins, np.int32)).to(dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    words = torch.empty(nb * 5 + (nb + 1) // 2, dtype=torch.int64, device=dev)
    ref = torch.empty(nb, dtype=torch.float32, device=dev)
    ref_st = torch.zeros(5, dtype=torch.int32, device=dev)
    tmlib.check(tmlib.lib().tm_exact_scatter(P(s), P(v.data_ptr()), P(b.data_ptr()), len(vals), nb,
                                             P(words.data_ptr()), P(ref.data_ptr()), P(ref_st.data_ptr())))
    out = torch.full((nb,), 7.0, dtype=torch.float32, device=dev)
    st = torch.zeros(5, dtype=torch.int32, device=dev)
    tmlib.check(tmlib.lib().tm_exact_scatter_noalloc(P(s), P(v.data_ptr()), P(b.data_ptr()), len(vals), nb,
                                                     P(out.data_ptr()), P(st.data_ptr())))
    torch.cuda.synchronize()
    return out.cpu().numpy(), st.cpu().numpy(), ref.cpu().numpy(), ref_st.cpu().numpy()


def test_noalloc_matches_scratch_entry_point_twice(cuda, tmlib):
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    rng = np.random.default_rng(12)
    calls = [
        (d["wide_vals"], d["wide_bins"], int(d["wide_nb"])),                        # every word of the accumulator
        (rng.uniform(-3, 3, 200000).astype(np.float32),                              # more bins, other values
         rng.integers(-2, MAX_BINS + 2, 200000).astype(np.int32), MAX_BINS),         # (out-of-range bins included)
    ]
    for vals, bins, nb in calls:
        out, st, ref, ref_st = run_both(tmlib, vals, bins, nb)
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(st, ref_st)
    # and the first call's bins against the golden known answers themselves (the integer reference, rounded once)
    out, st, _, _ = run_both(tmlib, d["wide_vals"], d["wide_bins"], int(d["wide_nb"]))
    assert np.array_equal(out.view(np.uint32), d["wide_expect"].view(np.uint32))


def test_noalloc_rejects_more_bins_than_its_scratch(tmlib):
    L = tmlib.lib()
    one = (ctypes.c_float * 1)(1.0)
    zero = (ctypes.c_int32 * 1)(0)
    rc = L.tm_exact_scatter_noalloc(None, one, zero, 1, MAX_BINS + 1, one, zero)
    assert rc == tmlib.TM_EINVAL
    assert b"exceed its fixed scratch" in L.tm_last_error()
