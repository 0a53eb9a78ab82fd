"""Items sharded over 2 GPUs (one NCCL rank per GPU) against one GPU, as the reference's sharding test
(tests/sharding.py:112-122): per-item results of each shard bitwise, the exact gradient bitwise (its words are
all_gathered and combined with carries), float tallies within 1e-4 (the reference's tolerance for a sharded run).
The NCCL tests are skipped with fewer than 2 GPUs; the gloo test runs two ranks on one GPU."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rw_inputs(n):
    from tallymap_b200 import prng
    kx, ks = prng.split(prng.PRNGKey(1), 2)
    return prng.uniform(kx, n), prng.split(ks, n)


def _rank(rank, world, port, n, q):
    import torch.distributed as dist
    from tallymap_b200 import backend as B
    from tallymap_b200 import parallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, k = rw_inputs(n)
        s0, c = parallel.shard(n, rank, world)
        f = B.run(B.RW_FWD, [x[s0:s0 + c], k[s0:s0 + c]], [np.float32(1.0)], consts=(20000,))
        parallel.all_reduce_sums(f[:3])
        g = B.run(B.RW_GRAD, [x[s0:s0 + c], k[s0:s0 + c]],
                  [np.float32(1.0), np.ones(256, np.float32), np.zeros(2, np.float32)], consts=(20000,))
        words = B.run.last["results"]["ct_drift.exact"]
        gall = torch.zeros(1, device=dev)
        st = torch.zeros(5, dtype=torch.int32, device=dev)
        parallel.combine_exact(words, 1, gall, st)
        torch.cuda.synchronize()
        q.put((rank, f[0].cpu().numpy(), f[1].cpu().numpy(), f[3].cpu().numpy(), gall.cpu().numpy()))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gpu_sharding_matches_one(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from tallymap_b200 import backend as B
    n = 200003
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, n, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps)
    x, k = rw_inputs(n)
    one = B.run(B.RW_FWD, [x, k], [np.float32(1.0)], consts=(20000,))
    g1 = B.run(B.RW_GRAD, [x, k], [np.float32(1.0), np.ones(256, np.float32), np.zeros(2, np.float32)],
               consts=(20000,))
    hist1, side1, k1 = one[0].cpu().numpy(), one[1].cpu().numpy(), one[3].cpu().numpy()
    assert np.array_equal(np.concatenate([res[0][3], res[1][3]]), k1)
    for r in res:
        assert np.abs(r[1].astype(np.float64) - hist1).max() <= 1e-4 * np.abs(hist1).max()
        assert np.array_equal(r[2], side1)
        assert r[4].view(np.uint32)[0] == g1[0].cpu().numpy().view(np.uint32)[0]


def _rank_vg(rank, world, port, n, q):
    """the fused value-and-grad launch on a shard, then the bench's collective step"""
    import torch.distributed as dist
    from tallymap_b200 import backend as B
    from tallymap_b200 import parallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, k = rw_inputs(n)
        s0, c = parallel.shard(n, rank, world)
        out = B.run(B.RW_VG, [x[s0:s0 + c], k[s0:s0 + c]],
                    [np.float32(1.0), np.ones(256, np.float32), np.zeros(2, np.float32)], consts=(20000,))
        words = B.run.last["results"]["ct_drift.exact"]
        parallel.all_reduce_sums(out[:2] + [out[3]])
        gall = torch.zeros(1, device=dev)
        parallel.combine_exact(words, 1, gall, out[3])
        torch.cuda.synchronize()
        q.put((rank, out[0].cpu().numpy(), out[4].cpu().numpy(), gall.cpu().numpy()))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gpu_fused_value_and_grad_matches_one(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from tallymap_b200 import backend as B
    n = 300007
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_rank_vg, args=(r, 2, port, n, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps)
    x, k = rw_inputs(n)
    one = B.run(B.RW_VG, [x, k], [np.float32(1.0), np.ones(256, np.float32), np.zeros(2, np.float32)],
                consts=(20000,))
    hist1, g1, k1 = one[0].cpu().numpy(), one[2].cpu().numpy(), one[4].cpu().numpy()
    assert np.array_equal(np.concatenate([res[0][2], res[1][2]]), k1)
    for r in res:
        assert np.abs(r[1].astype(np.float64) - hist1).max() <= 1e-4 * np.abs(hist1).max()
        assert r[3].view(np.uint32)[0] == g1.view(np.uint32)[0]


def _rank_one_gpu(rank, world, port, n, q):
    """a rank of the sharded one-pass step on cuda:0, the collectives over gloo (the bench's collective step)"""
    import torch.distributed as dist
    from tallymap_b200 import backend as B
    from tallymap_b200 import parallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x, k = rw_inputs(n)
        s0, c = parallel.shard(n, rank, world)
        out = B.run(B.RW_VG1, [x[s0:s0 + c], k[s0:s0 + c]],
                    [np.float32(1.0), np.ones(256, np.float32), np.zeros(2, np.float32)], consts=(20000,))
        res = B.run.last["results"]
        parallel.all_reduce_sums(out[:2] + [out[3]])
        gall = torch.zeros(1, device=dev)
        parallel.combine_exact(res["ct_drift.exact"], 1, gall, out[3])
        torch.cuda.synchronize()
        q.put((rank, out[0].cpu().numpy(), out[1].cpu().numpy(), out[4].cpu().numpy(), gall.cpu().numpy(),
               out[3].cpu().numpy()))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_sharded_one_pass_two_ranks_on_one_gpu(cuda):
    """the sharded path of the default step with one GPU: two ranks as two processes on cuda:0 (their kernels
    never wait on each other), each running the one-pass launch on its half of the items, then the collective step
    over gloo -- all_reduce of the tallies and stats in place, all_gather of the exact gradient words and their
    combine on the device.  Against one launch over all items: per-item trip counts bitwise, the exact gradient
    bitwise, the side counts exactly, the histogram within 1e-4 (the reference's sharded-run tolerance,
    tests/sharding.py:112-122)"""
    import torch.multiprocessing as mp
    from tallymap_b200 import backend as B
    n = 300007
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_rank_one_gpu, args=(r, 2, port, n, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps)
    x, k = rw_inputs(n)
    one = B.run(B.RW_VG1, [x, k], [np.float32(1.0), np.ones(256, np.float32), np.zeros(2, np.float32)],
                consts=(20000,))
    hist1, side1, g1, st1, k1 = (o.cpu().numpy() for o in one[:5])
    assert np.array_equal(np.concatenate([res[0][3], res[1][3]]), k1)
    for r in res:
        assert np.abs(r[1].astype(np.float64) - hist1).max() <= 1e-4 * np.abs(hist1).max()
        assert np.array_equal(r[2], side1)
        assert r[4].view(np.uint32)[0] == g1.view(np.uint32)[0]
        assert np.array_equal(r[5], st1)


def _rank_shower_one_gpu(rank, world, port, n, q):
    import torch.distributed as dist
    from oracle import oracle as orc
    from tallymap_b200 import backend as B
    from tallymap_b200 import parallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        E0, d0, keys = orc.sh_inputs(n)
        s0, c = parallel.shard(n, rank, world)
        pi = [E0[s0:s0 + c], d0[s0:s0 + c], keys[s0:s0 + c]]
        ct = np.linspace(-1.0, 1.0, 512).astype(np.float32)
        r = B.sh_value_and_grad(pi, np.float32(1.0), ct, order=B.energy_order(torch.from_numpy(pi[0]).cuda()))
        parallel.all_reduce_sums([r["dep"], r["count"], r["stats"]])
        torch.cuda.synchronize()
        q.put((rank, r["dep"].cpu().numpy(), r["count"].cpu().numpy(), r["stats"].cpu().numpy(),
               r["k"].cpu().numpy(), r["g_E"].cpu().numpy()))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_sharded_shower_two_ranks_on_one_gpu(cuda):
    """the shower's sharded one-pass step (children stay on their rank's GPU; only the forward tallies and stats
    are reduced) as two gloo ranks on cuda:0, against one launch over all roots: particle count and stats exactly,
    per-root trip counts and gradients bitwise (exact per-root sums), the deposit within 1e-4"""
    import torch.multiprocessing as mp
    from oracle import oracle as orc
    from tallymap_b200 import backend as B
    n = 20001
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_rank_shower_one_gpu, args=(r, 2, port, n, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps)
    E0, d0, keys = orc.sh_inputs(n)
    ct = np.linspace(-1.0, 1.0, 512).astype(np.float32)
    one = B.sh_value_and_grad([E0, d0, keys], np.float32(1.0), ct)
    torch.cuda.synchronize()
    dep1 = one["dep"].cpu().numpy()
    assert np.array_equal(np.concatenate([res[0][4], res[1][4]]), one["k"].cpu().numpy())
    assert np.array_equal(np.concatenate([res[0][5], res[1][5]]).view(np.uint32),
                          one["g_E"].cpu().numpy().view(np.uint32))
    for r in res:
        assert np.abs(r[1].astype(np.float64) - dep1).max() <= 1e-4 * np.abs(dep1).max()
        assert np.array_equal(r[2], one["count"].cpu().numpy()) and np.array_equal(r[3], one["stats"].cpu().numpy())
