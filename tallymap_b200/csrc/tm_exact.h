// The exact f32 sum of the tallymap B200 backend: its word format and arithmetic, the same source on the host and
// the device (the device's atomic forms are in tm_device.cuh).
//
// Format (the reference's TSpec.exact accumulator, tallymap/backends/kernel/kernel.py:870-941): every finite f32 is
// an integer number of units 2^-149; a bin holds the exact sum of its f32 addends as kWords signed 64-bit words w_j
// of weight 2^(63 j) units, value = sum_j w_j 2^(63 j).  The words overlap by one bit, so a word can take any
// addend of at most 63 bits without leaving its range, and an add that does wrap a word by 2^64 moved +-2^64 * 2^(63 j)
// = +-2 * 2^(63 (j + 1)): the carry is +-2 into the next word.  A carry out of the top word loses the value: the bin
// is flagged and reads as NaN.
//
// Readout (this file's own method): the words are first brought to a canonical form, five limbs in [0, 2^63) and a
// small signed top carry c (value = sum_j L_j 2^(63 j) + c 2^315): c < 0 means a negative total, whose magnitude is
// the two's complement of the limbs.  The magnitude's bit length n gives the f32 directly: for n <= 24 the f32's bit
// pattern IS the integer (subnormals are m 2^-149; the first binade above them, exponent field 1, is 2^23 + f), and
// above it the top 24 bits q, one round bit and a sticky bit give bits = (n - 24) 2^23 + q', q' rounded to nearest
// with ties to even (a rounding carry into 2^24 steps the exponent field by itself).  Bits at or above 0x7f800000
// overflow f32.  No floating point is used, so the host and device results are equal bit for bit.
#pragma once
#ifdef __CUDACC_RTC__
#include <cuda/std/cstdint>
#else
#include <cstdint>
#include <cstring>
#endif

#if defined(__CUDACC__)
#define TMX_HD __host__ __device__ __forceinline__
#else
#define TMX_HD inline
#endif

namespace tmx {

#ifdef __CUDACC_RTC__
typedef cuda::std::int64_t s64;
typedef cuda::std::uint64_t w64;
typedef cuda::std::uint32_t w32;
#else
typedef int64_t s64;
typedef uint64_t w64;
typedef uint32_t w32;
#endif

constexpr int kWords = 5;
constexpr w64 kLimb = 0x7fffffffffffffffull;   // 2^63 - 1: a canonical limb's mask

TMX_HD w32 bits_of(float v) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(v);
#else
  w32 u;
  std::memcpy(&u, &v, 4);
  return u;
#endif
}
TMX_HD float float_of(w32 u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  std::memcpy(&f, &u, 4);
  return f;
#endif
}
TMX_HD int lead_zeros(w64 x) {   // x != 0
#if defined(__CUDA_ARCH__)
  return __clzll((long long)x);
#else
  return __builtin_clzll(x);
#endif
}

// One f32 addend in the word format: +-(a0 + a1 2^63) 2^(63 j) units, i.e. signed parts s0 for word j and s1 for
// word j + 1.  v = +-m 2^p units with m < 2^24 (the significand with its hidden bit) and p = max(exponent field - 1,
// 0) <= 253; p = 63 j + r; m 2^r < 2^87 splits at bit 63 into a0 = (m 2^r) mod 2^63 and a1 = m >> (63 - r), written
// (m >> 1) >> (62 - r) so every shift count stays in [0, 62].  j + 1 <= 4 whenever a1 != 0 (p <= 253 gives r <= 1
// at j = 4).
struct Addend {
  int j;
  s64 s0, s1;
  bool nonfinite;   // +-inf or NaN: the bin is flagged
};

TMX_HD Addend addend(float v) {
  const w32 b = bits_of(v);
  const w32 field = (b >> 23) & 0xffu;
  Addend a{0, 0, 0, field == 0xffu};
  if (a.nonfinite) return a;
  const w64 m = (w64)(b & 0x7fffffu) + (field ? (1ull << 23) : 0ull);
  const w32 p = field ? field - 1u : 0u;
  const w32 j = p / 63u, r = p - 63u * j;
  const w64 a0 = (m << r) & kLimb, a1 = (m >> 1) >> (62u - r);
  const bool neg = (b >> 31) != 0u;
  a.j = (int)j;
  a.s0 = neg ? -(s64)a0 : (s64)a0;
  a.s1 = neg ? -(s64)a1 : (s64)a1;
  return a;
}

// w += q modulo 2^64 -> the carry for the next word: 0, or +-2 when the signed add wrapped (the sum's sign differs
// from both operands'; a positive wrap leaves a negative word and owes +2 above, a negative one the reverse)
TMX_HD s64 add_wrap(s64& w, s64 q) {
  const s64 r = (s64)((w64)w + (w64)q);
  const bool wrapped = ((w ^ r) & (q ^ r)) < 0;
  w = r;
  return wrapped ? (r < 0 ? 2 : -2) : 0;
}

// words (any array-like of kWords s64: word(j) an lvalue) += q at word j, carries rippled upward; true if a carry
// leaves the top word (the value is lost)
template <class Word>
TMX_HD bool add_at(Word&& word, int j, s64 q) {
  for (; q != 0; ++j) {
    if (j >= kWords) return true;
    q = add_wrap(word(j), q);
  }
  return false;
}

// the addend of v into the words; true when the bin must be flagged (non-finite v, or a carry lost)
template <class Word>
TMX_HD bool add_float(Word&& word, float v) {
  const Addend a = addend(v);
  if (a.nonfinite) return true;
  bool lost = false;
  if (a.s0) lost = add_at(word, a.j, a.s0);
  if (a.s1) lost = add_at(word, a.j + 1, a.s1) || lost;
  return lost;
}

// bits [pos, pos + width) of the 5-limb number L (width <= 25)
TMX_HD w64 limb_field(const w64* L, int pos, int width) {
  const int q = pos / 63, r = pos - 63 * q;
  w64 f = L[q] >> r;
  if (q + 1 < kWords) f |= L[q + 1] << (63 - r);   // (63 - r in [1, 63]; the limb's bit 63 is 0)
  return f & ((1ull << width) - 1ull);
}

// any bit of L below position pos
TMX_HD bool limb_any_below(const w64* L, int pos) {
  const int q = pos / 63, r = pos - 63 * q;
  if (L[q] & ((1ull << r) - 1ull)) return true;
  for (int k = 0; k < q; ++k)
    if (L[k]) return true;
  return false;
}

// the correctly rounded (nearest, ties to even) f32 of the words' value; *overflow: |value| rounds beyond f32
TMX_HD float read(const s64* w, bool* overflow) {
  // canonical limbs: x_j + c = hi 2^63 + lo + c with hi in {-1, 0}, lo in [0, 2^63); the running carry c stays in
  // [-2, 1]
  w64 L[kWords];
  s64 c = 0;
  for (int j = 0; j < kWords; ++j) {
    const w64 lo = (w64)w[j] & kLimb;
    s64 hi = w[j] < 0 ? -1 : 0;
    if (c >= 0) {
      const w64 s = lo + (w64)c;            // <= 2^63
      L[j] = s & kLimb;
      hi += (s64)(s >> 63);
    } else if (lo >= (w64)(-c)) {
      L[j] = lo - (w64)(-c);
    } else {
      L[j] = lo + (1ull << 63) - (w64)(-c);  // borrow 2^63 from above
      hi -= 1;
    }
    c = hi;
  }
  const bool neg = c < 0;
  if (c > 0 || c < -1) {   // |value| >= 2^315 units: far beyond f32
    *overflow = true;
    return float_of(neg ? 0xffc00000u : 0x7fc00000u);
  }
  if (neg) {               // magnitude = 2^315 - sum L_j 2^(63 j): complement the limbs, add one
    w64 inc = 1ull;
    for (int j = 0; j < kWords; ++j) {
      const w64 s = (kLimb - L[j]) + inc;
      L[j] = s & kLimb;
      inc = s >> 63;
    }
    if (inc) {             // the limbs were all zero: magnitude 2^315
      *overflow = true;
      return float_of(0xffc00000u);
    }
  }
  int t = kWords - 1;
  while (t >= 0 && L[t] == 0ull) --t;
  if (t < 0) return float_of(neg ? 0x80000000u : 0u);
  const int n = 63 * t + (64 - lead_zeros(L[t]));   // bit length of the magnitude
  w64 bits;
  if (n <= 24) {
    bits = L[0];
  } else {
    const int sh = n - 24;
    const w64 g = limb_field(L, sh - 1, 25);         // the 24 kept bits and the round bit below them
    w64 q = g >> 1;
    if ((g & 1ull) && ((q & 1ull) || (sh > 1 && limb_any_below(L, sh - 1)))) ++q;
    bits = ((w64)sh << 23) + q;
  }
  if (bits >= 0x7f800000ull) {
    *overflow = true;
    bits = 0x7f800000ull;
  }
  return float_of((neg ? 0x80000000u : 0u) | (w32)bits);
}

}  // namespace tmx
