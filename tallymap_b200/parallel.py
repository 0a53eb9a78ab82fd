"""Items sharded over GPUs, one process per GPU (torch.distributed, NCCL over NVLink/NVSwitch).

The reference's only multi-device rule (tallymap/_primitive.py:216-320, custom_partitioning): per-item operands are
split along the item axis, broadcast operands replicated, each device runs its own items, and the Sum tallies and
the stats are psum'd; per-item results stay sharded.  Here each rank launches the same program on its contiguous
slice [rank * n, (rank + 1) * n) of the global items, then ONE collective step combines the partial results:

  * plain Sum tallies (f32, i32) and stats: all_reduce(SUM), grouped into one flat buffer per dtype;
  * exact f32 tallies (the reverse-mode cotangents): their carry-save words cannot be summed word by word (an int64
    word can overflow), so every rank's words are all_gathered (40 bytes per bin) and combined with carries on the
    device (tm_exact_combine), then read out once: bitwise the single-GPU result.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib


def shard(n_total, rank, world):
    """(start, count) of a rank's contiguous item slice (the last rank takes the remainder)."""
    per = n_total // world
    start = rank * per
    return start, (n_total - start if rank == world - 1 else per)


def contiguous_span(group):
    """one flat view over tensors of one dtype that lie back to back in one storage (in the given order), or None.
    backend.alloc_results places a program's tallies so that those of one dtype following each other do."""
    if not all(t.is_contiguous() for t in group):
        return None
    es = group[0].element_size()
    base = group[0].untyped_storage().data_ptr()
    for a, b in zip(group, group[1:]):
        if b.untyped_storage().data_ptr() != base or a.data_ptr() + a.numel() * es != b.data_ptr():
            return None
    g0 = group[0]
    return g0.new_empty(0).set_(g0.untyped_storage(), g0.storage_offset(), (sum(t.numel() for t in group),), (1,))


def all_reduce_sums(tensors):
    """in place: all_reduce(SUM) of float32, int32, float64 and int64 tensors, one collective per dtype.  Tensors of a dtype that
    are one contiguous range (a single tensor, or tallies laid out back to back by backend.alloc_results) are
    reduced in place; otherwise they are packed into a flat buffer and copied back."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return tensors
    for dt in (torch.float32, torch.int32, torch.float64, torch.int64):
        group = [t for t in tensors if t.dtype == dt]
        if not group:
            continue
        flat = contiguous_span(group)
        if flat is not None:
            dist.all_reduce(flat, op=dist.ReduceOp.SUM)
            continue
        flat = torch.cat([t.reshape(-1) for t in group])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM)
        o = 0
        for t in group:
            n = t.numel()
            t.copy_(flat[o:o + n].view_as(t))
            o += n
    return tensors


def gather_words(words):
    """every rank's exact scratch words, stacked [world, n] (all_gather; 40 bytes per bin per rank)."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    if world == 1:
        return words.reshape(1, -1)
    if dist.get_backend() == "nccl":
        gathered = torch.empty((world, words.numel()), dtype=words.dtype, device=words.device)
        dist.all_gather_into_tensor(gathered, words.reshape(-1))
        return gathered
    parts = [torch.empty_like(words.reshape(-1)) for _ in range(world)]
    dist.all_gather(parts, words.reshape(-1).contiguous())
    return torch.stack(parts)


def combine_exact(words, n_bins, out, stats):
    """the cross-rank total of an exact tally: all_gather every rank's scratch words (int64, the layout of
    tm_exact_combine), then combine and read out on this device into `out` (f32[n_bins])."""
    gathered = gather_words(words)
    world = gathered.shape[0]
    st = torch.cuda.current_stream(words.device).cuda_stream
    _lib.check(_lib.lib().tm_exact_combine(ctypes.c_void_p(st), ctypes.c_void_p(gathered.data_ptr()), world, n_bins,
                                           ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stats.data_ptr())))
    return out


def combine_wide(words, out, scale, stats=None):
    """the cross-rank total of a scaled fixed-point Sum (Sum(fixed_point=True) of float64 / int32 / int64): every
    rank's words all_gathered (per bin an int64 low word, then the i32 carries and u32 flags: 16 bytes per bin), each
    bin's exact integer total -- lo + carry * 2^64 summed over the ranks -- formed in Python integers, and read out
    once into `out` as the single-GPU launch reads out its own: the correctly rounded double of the total (Python's
    int -> float) times 1 / scale, NaN for a flagged float bin, the conversion toward zero saturating for an integer
    one; a value out of the output's range counts in stats[3].  Bitwise the single-GPU result, whatever the number of
    ranks (the words of an order-independent integer sum)."""
    S = out.numel()
    g = gather_words(words).cpu()
    lo = g[:, :S].numpy()
    cf = g[:, S:].contiguous().view(torch.int32).numpy()
    carry, flag = cf[:, :S], cf[:, S:]
    inv = 1.0 / float(scale)
    vals, over = [], 0
    floating = out.dtype == torch.float64
    lim = 2 ** 63 if out.dtype == torch.int64 else 2 ** 31
    for b in range(S):
        tot = sum(int(lo[r, b]) + (int(carry[r, b]) << 64) for r in range(g.shape[0]))
        bad = bool(flag[:, b].any())
        v = float(tot) * inv
        if floating:
            big = not abs(v) <= 1.7976931348623157e308
            over += int(big and not bad)
            vals.append(float("nan") if bad or big else v)
        else:
            over += int(not -lim <= v < lim)
            vals.append(lim - 1 if v >= lim else -lim if v < -lim else int(v))
    out.copy_(torch.tensor(vals, dtype=out.dtype))
    if stats is not None and over:
        stats[3] += over
    return out
