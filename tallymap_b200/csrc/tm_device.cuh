// Device primitives of the tallymap B200 runtime: scalar types, the kernel parameter block, jax.random's
// threefry2x32 draws, float->int conversion, the subnormal-safe f32 atomic add and the exact f32 sum.
//
// Semantics follow the reference's generated PRELUDE (tallymap/backends/kernel/kernel.py:26-188) and the word format of
// its DENSE accumulator (kernel.py:870-941; the arithmetic on it is this build's own, tm_exact.h); the code is
// written for sm_100a.  All product kernels are compiled with
// --fmad=false, so every f32 + - * below is one IEEE rounding, as the reference's NVRTC flags (-fmad=false,
// backends/kernel/compile.py:27) and its host target (-ffp-contract=off) make it.
#pragma once
#ifdef __CUDACC_RTC__
#include <cuda/std/cstdint>
#else
#include <cstdint>
#endif
#include "tm_exact.h"

namespace tmb {

#ifdef __CUDACC_RTC__
typedef cuda::std::int32_t i32;
typedef cuda::std::uint32_t u32;
typedef cuda::std::int64_t i64;
typedef cuda::std::uint64_t u64;
#else
typedef int32_t i32;
typedef uint32_t u32;
typedef int64_t i64;
typedef uint64_t u64;
#endif

// Kernel parameter block: every buffer pointer of a launch, args first then results (the layout of the reference's
// SjParams, kernel.py:596 / shim.cc:36-40), passed by value.  TM_MAXP bounds the pointers a program may use.
#define TM_MAXP 64
struct Params {
  void* p[TM_MAXP];
};

// control words of a launch (one result buffer, u32[8], zeroed by the launcher):
//   [0..1] item claim counter (u64)   [2] blocks finished (the last one runs the epilogue)   [3] device error word
//   [4] spawn/queue words or unused ...
enum { kCtlClaim = 0, kCtlDone = 2, kCtlError = 3, kCtlWords = 8 };

// stats slots (tallymap/_api.py:192-195, kernel.py:594-597): written by number
enum { kStSpawned = 0, kStChildrenDropped = 1, kStChildrenTruncated = 2, kStFixedPointOverflow = 3, kStDroppedEmits = 4 };

// ------------------------------------------------------------------------------------------------ threefry2x32
// 20 rounds, rotations 13 15 26 6 / 17 29 16 24, key injection every 4 rounds, k2 = k0 ^ k1 ^ 0x1BD11BDA
// (kernel.py:137-150; bitwise jax.random's threefry2x32_p).  A rotate is one funnel shift.
__device__ __forceinline__ u32 rotl(u32 x, int d) { return __funnelshift_l(x, x, d); }

// A round is an add, a rotate and an xor: three instructions of the integer ALU pipe, which bounds threefry.  Each
// round's add is written as a multiply-add by 1 held in constant memory (a value the compiler cannot fold), so it
// issues on the multiply-add pipe instead, beside the ALU's rotate and xor: at full occupancy on a B200 that ran
// threefry2x32 at 445 G/s against 389 G/s with plain adds, the results bitwise the same (x * 1 + y == x + y mod 2^32).
static __constant__ u32 kTmOne = 1u;
__device__ __forceinline__ u32 add_mad(u32 a, u32 b) {
  u32 d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(b), "r"(kTmOne), "r"(a));
  return d;
}

__device__ __forceinline__ void threefry2x32(u32 k0, u32 k1, u32 c0, u32 c1, u32& o0, u32& o1) {
  const u32 k2 = k0 ^ k1 ^ 0x1BD11BDAu;
  u32 x0 = c0 + k0, x1 = c1 + k1;
#define TM_R(r) x0 = add_mad(x0, x1); x1 = rotl(x1, r); x1 ^= x0;
  TM_R(13) TM_R(15) TM_R(26) TM_R(6)  x0 += k1; x1 += k2 + 1u;
  TM_R(17) TM_R(29) TM_R(16) TM_R(24) x0 += k2; x1 += k0 + 2u;
  TM_R(13) TM_R(15) TM_R(26) TM_R(6)  x0 += k0; x1 += k1 + 3u;
  TM_R(17) TM_R(29) TM_R(16) TM_R(24) x0 += k1; x1 += k2 + 4u;
  TM_R(13) TM_R(15) TM_R(26) TM_R(6)  x0 += k2; x1 += k0 + 5u;
#undef TM_R
  o0 = x0;
  o1 = x1;
}

struct Key {
  u32 a, b;
};

// jax.random.fold_in(key, m) = threefry2x32(key, (0, m)) for a 32-bit m (threefry_seed(m) = (0, m))
__device__ __forceinline__ Key fold_in(Key k, u32 m) {
  Key o;
  threefry2x32(k.a, k.b, 0u, m, o.a, o.b);
  return o;
}

// random_bits(key, 32, shape)[i] under partitionable threefry: o0 ^ o1 of threefry2x32(key, (0, i))
__device__ __forceinline__ u32 random_bits32(Key k, u32 i) {
  u32 o0, o1;
  threefry2x32(k.a, k.b, 0u, i, o0, o1);
  return o0 ^ o1;
}

// the f32 in [0, 1) of jax.random.uniform's mantissa fill: bitcast((bits >> 9) | 0x3f800000) - 1
__device__ __forceinline__ float bits_to_unit(u32 bits) { return __uint_as_float((bits >> 9) | 0x3f800000u) - 1.0f; }

// jax.random.uniform(key, (), f32) with minval 0, maxval 1.  jax computes max(0, f * (1 - 0) + 0); for f in [0, 1)
// that is f itself, bitwise (f * 1 = f, f + 0 = f for f >= +0, max(0, f) = f), so the scale and clamp are omitted.
__device__ __forceinline__ float uniform01(Key k, u32 i = 0u) { return bits_to_unit(random_bits32(k, i)); }

// jax.random.uniform(key, shape, f32, lo, hi)[i]: max(lo, f * (hi - lo) + lo), each op one rounding
__device__ __forceinline__ float uniform(Key k, u32 i, float lo, float hi) {
  const float f = bits_to_unit(random_bits32(k, i));
  const float r = f * (hi - lo) + lo;
  return (lo > r || lo != lo) ? lo : ((r > lo || r != r) ? r : (lo == 0.0f ? lo + r : lo));
}

// ------------------------------------------------------------------------------------------------ conversions
// x.astype(int32): toward zero, saturating, NaN -> 0 (PTX cvt.rzi.s32.f32; the reference's __float2int_rz)
__device__ __forceinline__ i32 f2i(float x) { return __float2int_rz(x); }

// ------------------------------------------------------------------------------------------------ f32 sum atomics
// The hardware f32 atomic add flushes subnormal inputs and results to zero.  An add of |v| >= 2^-102 never meets a
// subnormal (the bin is below half an ulp of v, and v + bin is a multiple of 2^-126 or above it), so it keeps the
// one-instruction atomic; a smaller nonzero v goes through a compare-and-swap loop of the IEEE add; +-0 changes no
// bin (kernel.py:112-135, sj_fatom).
__device__ __forceinline__ void fatom(float* a, float v) {
  if (v == 0.0f) return;
  if (!(fabsf(v) < __int_as_float(0x0c800000))) {   // 2^-102
    atomicAdd(a, v);
    return;
  }
  u32* const u = reinterpret_cast<u32*>(a);
  u32 o = *reinterpret_cast<volatile u32*>(u), w;
  do {
    w = o;
    o = atomicCAS(u, w, __float_as_uint(__fadd_rn(__uint_as_float(w), v)));
  } while (o != w);
}

// ------------------------------------------------------------------------------------------------ exact f32 sum
// A bin keeps the exact sum of its f32 emits in kExactWords signed 64-bit words of weight 2^(63 j) units of 2^-149
// (the format and its host/device arithmetic: tm_exact.h).  Here: the device's atomic forms and thread-private words.
constexpr int kExactWords = tmx::kWords;

// the rare carry of an atomic add: c (+-2) into word j and upward, one atomic per word; true if it leaves the top
// word (kept out of line: it almost never runs, and inlined it would hold registers in every emitting loop)
__device__ __noinline__ bool exact_atomic_ripple(u64* a, int j, i64 c) {
  for (; c != 0; ++j) {
    if (j >= kExactWords) return true;
    i64 old = (i64)atomicAdd((unsigned long long*)&a[j], (unsigned long long)c);
    c = tmx::add_wrap(old, c);
  }
  return false;
}

// word j of the bin at a += q with one atomic; a wrap of that word (detected from the value the atomic returned)
// carries into the words above.  True if a carry left the top word.
__device__ __forceinline__ bool exact_add_word(u64* a, int j, i64 q) {
  i64 old = (i64)atomicAdd((unsigned long long*)&a[j], (unsigned long long)q);
  const i64 c = tmx::add_wrap(old, q);
  return c != 0 && exact_atomic_ripple(a, j + 1, c);
}

// one f32 into the bin at a with atomics; true when the bin must be flagged (non-finite v, or a carry lost)
__device__ __forceinline__ bool exact_emit_atomic(u64* a, float v) {
  const tmx::Addend d = tmx::addend(v);
  if (d.nonfinite) return true;
  bool lost = false;
  if (d.s0) lost = exact_add_word(a, d.j, d.s0);
  if (d.s1) lost = exact_add_word(a, d.j + 1, d.s1) || lost;
  return lost;
}

// Thread-private words (no atomics): word(b, j) gives word j of bin b as an i64 lvalue.  Integer addition is
// associative, so adding per-item values here first and the thread's words into a shared or global bin later reads
// out bitwise the same as adding every emit straight into the bin.
template <class Word>
__device__ __forceinline__ bool exact_priv_add(Word&& word, int b, int j, i64 q) {
  return tmx::add_at([&word, b](int jj) -> i64& { return word(b, jj); }, j, q);
}

// one f32 into bin b of a thread's private words; flag: the bins' flag bits.  True when the bin must be flagged.
template <class Word>
__device__ __forceinline__ bool exact_priv_emit(Word&& word, u32& flag, int b, float v) {
  const bool bad = tmx::add_float([&word, b](int jj) -> i64& { return word(b, jj); }, v);
  if (bad) flag |= 1u << b;
  return bad;
}

template <int NB>
struct ExactPriv {
  i64 w[NB][kExactWords];
  u32 flag;   // bit b: bin b saw a non-finite emit or lost a carry

  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int j = 0; j < kExactWords; ++j) w[b][j] = 0;
    flag = 0u;
  }
  __device__ __forceinline__ i64 word(int b, int j) const { return w[b][j]; }
  __device__ __forceinline__ bool add_word(int b, int j, i64 q) {
    return exact_priv_add([this](int bb, int jj) -> i64& { return w[bb][jj]; }, b, j, q);
  }
  // add one f32 into bin b; returns true when the bin must be flagged (non-finite, or carry lost)
  __device__ __forceinline__ bool emit(int b, float v) {
    return exact_priv_emit([this](int bb, int jj) -> i64& { return w[bb][jj]; }, flag, b, v);
  }
};

// add a thread's private words into exact bins held elsewhere (shared or global): true if a carry was lost
__device__ __forceinline__ bool exact_merge_bin(u64* dst, const i64* src) {
  bool lost = false;
#pragma unroll
  for (int j = 0; j < kExactWords; ++j)
    if (src[j]) lost = exact_add_word(dst, j, src[j]) || lost;
  return lost;
}

// the correctly rounded f32 of a bin's words (tmx::read); *bad: the total overflows f32
__device__ __noinline__ float exact_read(const u64* a, bool* bad) {
  i64 w[kExactWords];
#pragma unroll
  for (int j = 0; j < kExactWords; ++j) w[j] = (i64)a[j];
  return tmx::read(w, bad);
}

}  // namespace tmb
