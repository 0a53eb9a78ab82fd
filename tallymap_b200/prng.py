"""jax.random's key arithmetic on the host, in numpy: PRNGKey, split, fold_in, random_bits and uniform on threefry
key data (uint32[..., 2]), bitwise what jax.random computes under its default partitionable threefry mode.

The item kernels draw with the same functions on the device (csrc/tm_device.cuh); this module makes the per-item
keys and inputs of a launch without JAX.  Published jax.random algorithm (jax >= 0.6.2, the reference's pin,
pyproject.toml:17-20), as the reference's kernel backend expands it (backends/kernel/op_table.py:1665-1756,
tallymap/_compat.py:119-152):
  PRNGKey(seed)      = (seed >> 32, seed & 0xFFFFFFFF)
  fold_in(key, m)    = threefry2x32(key, (0, m))
  split(key, n)[i]   = threefry2x32(key, (0, i))            (iota_2x32 counters)
  random_bits(key, 32, (n,))[i] = o0 ^ o1 of threefry2x32(key, (0, i))
  uniform(key, (n,), lo, hi)[i] = max(lo, (bitcast((bits >> 9) | 0x3f800000) - 1) * (hi - lo) + lo)
"""
import numpy as np

_ROT = ((13, 15, 26, 6), (17, 29, 16, 24))


def threefry2x32(k0, k1, c0, c1):
    """Threefry-2x32, 20 rounds, elementwise over broadcast uint32 arrays -> (o0, o1)."""
    k0, k1, c0, c1 = (np.asarray(a, np.uint32) for a in (k0, k1, c0, c1))
    ks = (k0, k1, k0 ^ k1 ^ np.uint32(0x1BD11BDA))
    with np.errstate(over="ignore"):
        x0 = (c0 + ks[0]).astype(np.uint32)
        x1 = (c1 + ks[1]).astype(np.uint32)
        for g in range(5):
            for r in _ROT[g & 1]:
                x0 = x0 + x1
                x1 = (x1 << np.uint32(r)) | (x1 >> np.uint32(32 - r))
                x1 = x1 ^ x0
            x0 = x0 + ks[(g + 1) % 3]
            x1 = x1 + ks[(g + 2) % 3] + np.uint32(g + 1)
    return x0, x1


def PRNGKey(seed):
    s = int(seed) & 0xFFFFFFFFFFFFFFFF
    return np.array([s >> 32, s & 0xFFFFFFFF], np.uint32)


def fold_in(key, m):
    key = np.asarray(key, np.uint32)
    o0, o1 = threefry2x32(key[..., 0], key[..., 1], np.uint32(0), np.asarray(m, np.uint32))
    return np.stack([o0, o1], axis=-1)


def split(key, n=2, start=0):
    """split(key, start + n)[start:] (the rows a shard of items needs)."""
    key = np.asarray(key, np.uint32)
    i = np.arange(start, start + n, dtype=np.uint64).astype(np.uint32)
    o0, o1 = threefry2x32(key[0], key[1], np.uint32(0), i)
    return np.stack([o0, o1], axis=-1)


def random_bits(key, n, start=0):
    key = np.asarray(key, np.uint32)
    i = np.arange(start, start + n, dtype=np.uint64).astype(np.uint32)
    o0, o1 = threefry2x32(key[0], key[1], np.uint32(0), i)
    return o0 ^ o1


def uniform(key, n, lo=0.0, hi=1.0, start=0):
    """uniform(key, (start + n,), f32, lo, hi)[start:]"""
    bits = random_bits(key, n, start)
    f = ((bits >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)
    lo32, hi32 = np.float32(lo), np.float32(hi)
    r = f * (hi32 - lo32) + lo32
    return np.maximum(lo32, r).astype(np.float32)
