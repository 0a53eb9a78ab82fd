"""Multi-rank host logic on CPU ranks (gloo, world size 2), as the reference tests sharding without a cluster
(tests/sharding.py:14-15: forced host devices): the item slices, the packed all-reduce of Sum tallies and stats, the
cross-rank combine of exact-tally words (bitwise the single-rank exact sum, checked against the golden integer
reference), and failure detection: a rank that dies before the collective makes the other rank's collective fail
within the process group's timeout instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tallymap_b200 import parallel

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_covers_items():
    for n, w in ((10, 3), (4194304, 8), (5, 8), (0, 2)):
        spans = [parallel.shard(n, r, w) for r in range(w)]
        assert sum(c for _, c in spans) == n
        assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(w - 1))


def words_of(orc, vals, bins, nb):
    """the exact tally's scratch layout (5 words per bin, then packed u32 flags) from the oracle's words"""
    w = orc.exact_words(vals, bins, nb).reshape(-1)
    return np.concatenate([w, np.zeros((nb + 1) // 2, np.int64)])


def combine_host(gathered, nb):
    """the reference integer value of the combined words (sum over ranks of sum_j w_j 2^(63 j)), rounded as the
    exact tally reads it out (tests/edge.py:2045-2056, restated in tests/golden/make_golden.py)"""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import f32_round
    out = []
    for b in range(nb):
        tot = 0
        for r in range(gathered.shape[0]):
            for j in range(5):
                tot += int(gathered[r, b * 5 + j]) << (63 * j)
        out.append(f32_round(tot))
    return np.array(out, np.float32)


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if mode == "reduce":
            h = torch.full((256,), float(rank + 1))
            c = torch.tensor([rank + 10], dtype=torch.int32)
            st = torch.arange(5, dtype=torch.int32) * (rank + 1)
            parallel.all_reduce_sums([h, c, st])
            q.put((rank, h.tolist()[:2], int(c), st.tolist()))
        elif mode == "span":
            # tallies laid out back to back in one allocation (as backend.alloc_results places them): reduced in
            # place as one range, with no packing copy (torch.cat must not be called)
            blob = torch.zeros(1024 + 16 + 32, dtype=torch.uint8)
            h = blob[:1024].view(torch.float32)
            side = blob[1024:1032].view(torch.float32)
            st = blob[1040:1060].view(torch.int32)
            h.fill_(rank + 1.0)
            side.fill_(2.0 * (rank + 1))
            st.copy_(torch.arange(5, dtype=torch.int32) * (rank + 1))

            def no_cat(*a, **k):
                raise AssertionError("packing copy")
            real, parallel.torch.cat = parallel.torch.cat, no_cat
            try:
                parallel.all_reduce_sums([h, side, st])
            finally:
                parallel.torch.cat = real
            q.put((rank, h.tolist()[:2] + side.tolist(), 0, st.tolist()))
        elif mode == "exact":
            from oracle import oracle as orc
            d = np.load(os.path.join(GOLD, "exact_sum.npz"))
            vals, bins, nb = d["wide_vals"], d["wide_bins"], int(d["wide_nb"])
            part = np.array_split(np.arange(len(vals)), world)[rank]
            w = torch.from_numpy(words_of(orc, vals[part], bins[part], nb))
            g = parallel.gather_words(w)
            q.put((rank, combine_host(g.numpy(), nb).view(np.uint32).tolist()))
        elif mode == "wide":
            # scaled fixed-point words (lo, then carry and flag int32 pairs) whose totals need the carries: rank r's
            # bin 0 holds 2^63 - 1 + r wrapped (carry 1 on rank 1), bin 1 -2^62 per rank, bin 2 a flag on rank 1
            S = 3
            lo = torch.tensor([2 ** 63 - 1 if rank == 0 else -(2 ** 63), -(2 ** 62), 5], dtype=torch.int64)
            cf = torch.tensor([0 if rank == 0 else 1, 0, 0, 0, 0, rank], dtype=torch.int32)
            w = torch.cat([lo, cf.view(torch.int64)])
            out = torch.zeros(S, dtype=torch.float64)
            st = torch.zeros(5, dtype=torch.int32)
            parallel.combine_wide(w, out, 2.0 ** 4, st)
            out_i = torch.zeros(S, dtype=torch.int64)
            parallel.combine_wide(w, out_i, 1.0, st)
            q.put((rank, out.tolist(), out_i.tolist(), st.tolist()))
        elif mode == "fail":
            if rank == 1:
                raise SystemExit(3)                    # this rank dies before the collective
            try:
                dist.all_reduce(torch.ones(4))
                q.put((rank, "no error"))
            except Exception as e:                     # noqa: BLE001 -- the collective must fail, not hang
                q.put((rank, type(e).__name__))
    finally:
        if mode != "fail":
            dist.destroy_process_group()


def run2(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    for p in ps:
        if p.is_alive():
            p.kill()
            raise AssertionError(f"rank process hung in mode {mode}")
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda r: r[0]), [p.exitcode for p in ps]


def test_all_reduce_sums_two_ranks():
    res, codes = run2("reduce")
    assert codes == [0, 0] and len(res) == 2
    for _, h, c, st in res:
        assert h == [3.0, 3.0] and c == 21 and st == [0, 3, 6, 9, 12]


def test_all_reduce_in_place_over_adjacent_tallies():
    res, codes = run2("span")
    assert codes == [0, 0] and len(res) == 2
    for _, h, _, st in res:
        assert h == [3.0, 3.0, 6.0, 6.0] and st == [0, 3, 6, 9, 12]


def test_exact_words_combine_two_ranks():
    d = np.load(os.path.join(GOLD, "exact_sum.npz"))
    want = d["wide_expect"].view(np.uint32).tolist()
    res, codes = run2("exact")
    assert codes == [0, 0] and len(res) == 2
    assert res[0][1] == want and res[1][1] == want


def test_rank_failure_is_detected_not_hung():
    res, codes = run2("fail")
    assert codes[1] == 3
    assert res and res[0][0] == 0 and res[0][1] != "no error"


def test_wide_words_combine_two_ranks():
    """scaled fixed-point Sums across ranks: the exact integer total of the ranks' (low word, carry) pairs read out
    once -- bin 0's total (2^63 - 1) + (-2^63 + 2^64) = 2^64 - 1 needs rank 1's carry; a flag on either rank makes a
    float bin NaN; an int64 output of a total past 2^63 saturates and counts in stats[3]"""
    import math
    res, codes = run2("wide")
    assert codes == [0, 0] and len(res) == 2
    for _, f64, i64, st in res:
        assert f64[0] == float(2 ** 64 - 1) / 16.0 and f64[1] == -(2.0 ** 63) / 16.0 and math.isnan(f64[2])
        assert i64 == [2 ** 63 - 1, -(2 ** 63), 10] and st[3] == 1
