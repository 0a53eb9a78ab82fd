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
    """in place: all_reduce(SUM) of float32 and int32 tensors, one collective per dtype.  Tensors of a dtype that
    are one contiguous range (a single tensor, or tallies laid out back to back by backend.alloc_results) are
    reduced in place; otherwise they are packed into a flat buffer and copied back."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return tensors
    for dt in (torch.float32, torch.int32):
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
