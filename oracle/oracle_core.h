// TEST INFRASTRUCTURE ONLY -- the CPU oracle for the tallymap kernel-backend hot path.
//
// Nothing in the product (tallymap_b200/) includes, links or calls this file.  Only tests/, the smoke check in
// __graft_entry__.py and the cpu_baseline / reference arm of bench.py load it, as the checker.
//
// This header restates, for the host, the arithmetic of the reference's CPU kernel target:
//   * threefry2x32, 20 rounds            tallymap/backends/kernel/kernel.py:137-150 (the PRELUDE's sj_threefry2x32)
//   * jax.random semantics on key data   tallymap/_compat.py:119-152, backends/kernel/op_table.py:1665-1756; the
//                                         published jax.random algorithm (jax >= 0.6.2, partitionable threefry):
//                                         fold_in(key, m) = threefry(key, (0, m)); split(key, n)[i] = threefry(key,
//                                         (0, i)); random_bits 32 = o0 ^ o1 of threefry(key, iota counter);
//                                         uniform = mantissa fill to [1, 2) minus 1, scaled, clamped by max(min, .)
//   * float -> int conversion             backends/kernel/host.py:133-146 (sj_f2i: truncate, saturate, NaN -> 0)
//   * exact f32 sum (TSpec.exact)         backends/kernel/kernel.py:870-941 (DENSE: 5 carry-save int64 words of
//                                         weight 2^(63 j), units of 2^-149, correctly rounded readout)
//   * f32 atomic add on the host          backends/kernel/host.py:154-158 (an IEEE compare-and-swap loop)
// Everything is compiled with -ffp-contract=off (host.py:35): every f32 + - * / is one IEEE rounding, no FMA.
#pragma once
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>

namespace orc {

typedef int32_t i32;
typedef uint32_t u32;
typedef int64_t i64;
typedef uint64_t u64;

// ------------------------------------------------------------------------------------------------ threefry2x32
static inline u32 rotl(u32 x, int d) { return (x << d) | (x >> (32 - d)); }

// Threefry-2x32 with 20 rounds (rotation schedule 13 15 26 6 / 17 29 16 24, a key injection after every 4 rounds,
// k2 = k0 ^ k1 ^ 0x1BD11BDA): kernel.py:137-150.
static inline void threefry2x32(u32 k0, u32 k1, u32 c0, u32 c1, u32* o0, u32* o1) {
  static const int rot[2][4] = {{13, 15, 26, 6}, {17, 29, 16, 24}};
  const u32 ks[3] = {k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
  u32 x0 = c0 + ks[0], x1 = c1 + ks[1];
  for (int g = 0; g < 5; ++g) {
    for (int r = 0; r < 4; ++r) {
      x0 += x1;
      x1 = rotl(x1, rot[g & 1][r]);
      x1 ^= x0;
    }
    x0 += ks[(g + 1) % 3];
    x1 += ks[(g + 2) % 3] + (u32)(g + 1);
  }
  *o0 = x0;
  *o1 = x1;
}

struct Key { u32 a, b; };

// jax.random.fold_in(key, m): threefry2x32(key, threefry_seed(m)) with threefry_seed(m) = (0, m) for 32-bit m.
static inline Key fold_in(Key k, u32 m) {
  Key o;
  threefry2x32(k.a, k.b, 0u, m, &o.a, &o.b);
  return o;
}

// jax.random.split(key, n)[i] under partitionable threefry: threefry2x32(key, iota_2x32(i)) = (key, (0, i)).
static inline Key split_at(Key k, u32 i) { return fold_in(k, i); }

// random_bits(key, 32, shape)[i] (partitionable): o0 ^ o1 of threefry2x32(key, (0, i)).
static inline u32 random_bits32(Key k, u32 i) {
  u32 o0, o1;
  threefry2x32(k.a, k.b, 0u, i, &o0, &o1);
  return o0 ^ o1;
}

static inline float bits_f32(u32 b) { float f; std::memcpy(&f, &b, 4); return f; }
static inline u32 f32_bits(float f) { u32 b; std::memcpy(&b, &f, 4); return b; }

// the lax.max of the uniform's clamp (NaN-propagating; a signed-zero tie gives +0): kernel.py:78-81 (sj_fmax)
static inline float fmax_lax(float a, float b) {
  return (a > b || a != a) ? a : ((b > a || b != b) ? b : (a == 0.0f ? a + b : a));
}

// jax.random.uniform(key, shape, float32, minval, maxval)[i]: 23 mantissa bits from bits >> 9 under exponent 1,
// minus 1, times (maxval - minval), plus minval, clamped below by minval.
static inline float uniform_f32(Key k, u32 i, float lo, float hi) {
  const float f = bits_f32((random_bits32(k, i) >> 9) | 0x3f800000u) - 1.0f;
  const float span = hi - lo;
  return fmax_lax(lo, f * span + lo);
}

// ------------------------------------------------------------------------------------------------ conversions
// float -> i32 as CUDA's __float2int_rz and the host target's sj_f2i (host.py:133-146): toward zero, saturating,
// NaN -> 0.
static inline i32 f2i_rz(float x) {
  if (x != x) return 0;
  if (x <= -2147483648.0f) return std::numeric_limits<i32>::min();
  if (x >= 2147483648.0f) return std::numeric_limits<i32>::max();
  return (i32)x;
}

// ------------------------------------------------------------------------------------------------ f32 atomic add
// the host target's atomicAdd(float*): an IEEE compare-and-swap loop (host.py:154-158)
static inline void atomic_add_f32(float* a, float v) {
  std::atomic_ref<u32> u(*reinterpret_cast<u32*>(a));
  u32 o = u.load(std::memory_order_relaxed);
  while (!u.compare_exchange_weak(o, f32_bits(bits_f32(o) + v), std::memory_order_relaxed)) {
  }
}

// ------------------------------------------------------------------------------------------------ exact f32 sum
// A bin holds the exact sum of its f32 emits as an integer in units of 2^-149, in kExactWords signed int64 words
// of weight 2^(63 j) (kernel.py:870-941).  An add into word j that overflows int64 carries +-2 into word j + 1
// (the word's true value is off by 2^64 = 2 x 2^63); a carry out of the top word reports "lost" and the caller flags
// the bin NaN.
static const int kExactWords = 5;

// word j += q, rippling carries; `atomic` selects fetch_add (shared accumulators) or a plain add (thread-private).
template <bool Atomic>
static inline bool exact_add_word(i64* a, int j, i64 q) {
  for (; j < kExactWords; ++j) {
    i64 o;
    if (Atomic) {
      o = (i64)std::atomic_ref<u64>(*reinterpret_cast<u64*>(&a[j])).fetch_add((u64)q, std::memory_order_relaxed);
    } else {
      o = a[j];
      a[j] = (i64)((u64)o + (u64)q);
    }
    const i64 r = (i64)((u64)o + (u64)q);
    if (q > 0 && r < o) q = 2;
    else if (q < 0 && r > o) q = -2;
    else return false;
  }
  return true;
}

// add one f32 into a bin's words; true: flag the bin (non-finite emit, or a carry out of the top word)
template <bool Atomic>
static inline bool exact_emit(i64* a, float v) {
  const u32 b = f32_bits(v), e = (b >> 23) & 255u;
  if (e == 255u) return true;
  const u64 m = (u64)(b & 0x7fffffu) | (e ? 0x800000ull : 0ull);
  if (m == 0ull) return false;
  const u32 p = e ? e - 1u : 0u, j = p / 63u, s = p - 63u * j;
  const i64 lo = (i64)((m << s) & 0x7fffffffffffffffull);
  const i64 hi = s >= 40u ? (i64)(m >> (63u - s)) : 0;
  const bool neg = (b >> 31) != 0u;
  bool lost = false;
  if (lo) lost = exact_add_word<Atomic>(a, (int)j, neg ? -lo : lo);
  if (hi) lost = exact_add_word<Atomic>(a, (int)j + 1, neg ? -hi : hi) || lost;
  return lost;
}

// the correctly rounded (nearest, ties to even) f32 of sum_j a[j] 2^(63 j) x 2^-149.  *bad: it overflows f32.
static inline float exact_read(const i64* a, bool* bad) {
  // 384-bit two's complement accumulator, little-endian 64-bit limbs
  u64 d[6] = {0, 0, 0, 0, 0, 0};
  for (int j = 0; j < kExactWords; ++j) {
    const i64 w = a[j];
    const int sh = 63 * j, limb = sh >> 6, bit = sh & 63;
    const u64 ext = w < 0 ? ~0ull : 0ull;
    u64 add[6];
    for (int k = 0; k < 6; ++k) add[k] = (k < limb) ? 0ull : ext;
    add[limb] = (u64)w << bit;
    if (limb + 1 < 6) add[limb + 1] = bit ? (u64)(w >> (64 - bit)) : ext;
    u64 c = 0;
    for (int k = 0; k < 6; ++k) {
      const u64 t = d[k] + add[k];
      const u64 u = t + c;
      c = (t < add[k] ? 1ull : 0ull) + (u < t ? 1ull : 0ull);
      d[k] = u;
    }
  }
  const bool neg = (i64)d[5] < 0;
  if (neg) {
    u64 c = 1;
    for (int k = 0; k < 6; ++k) { d[k] = ~d[k] + c; c = (c && d[k] == 0ull) ? 1ull : 0ull; }
  }
  int t = 5;
  while (t >= 0 && d[t] == 0ull) --t;
  if (t < 0) return 0.0f;
  const int lz = __builtin_clzll(d[t]);
  const u64 below = t >= 1 ? d[t - 1] : 0ull;
  const u64 top = lz ? (d[t] << lz) | (below >> (64 - lz)) : d[t];
  bool sticky = lz ? (below << lz) != 0ull : below != 0ull;
  for (int j = 0; j < t - 1; ++j) sticky = sticky || d[j] != 0ull;
  u64 q = top >> 40;
  const u64 rem = top & 0xffffffffffull, half = 0x8000000000ull;
  if (rem > half || (rem == half && (sticky || (q & 1ull)))) ++q;
  const double mag = std::ldexp((double)q, 64 * t + 40 - lz - 149);
  const float o = (float)mag;
  if (!(std::fabs((double)o) <= 3.4028234663852886e38)) *bad = true;
  return neg ? -o : o;
}

}  // namespace orc
