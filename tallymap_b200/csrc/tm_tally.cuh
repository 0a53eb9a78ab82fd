// Tally helpers shared by the item programs.
#pragma once
#include "tm_runtime.cuh"

namespace tmb {

// An exact cotangent tally of NB bins: per-thread private words (ExactPrivS: the thread's own slots in shared
// memory), merged into the block's shared words when the thread runs out of items, then by one thread into the
// launch's global words; the last block reads them out (backends/kernel/kernel.py:625-628: a flagged or overflowing
// bin is NaN, counted in stats[3]).
// Shared layout: NB x 5 u64 words, then a u32 flag per bin (rounded up to 8 bytes), then the private region
// (kPrivOffset): word (b, j) of thread t at u64 index (b * 5 + j) * BLK + t, BLK the block's threads.  Global layout:
// the words, flags packed after them.
template <int NB, int BLK = TM_BLOCK>
struct ExactBins {
  static constexpr int kPrivOffset = NB * kExactWords * 8 + ((NB * 4 + 7) / 8) * 8;
  static constexpr int kSmemBytes = kPrivOffset + NB * kExactWords * 8 * BLK;
  template <class Priv>
  __device__ static void flush(Priv& pv, unsigned char* smem, u64* gw, i32* stats, int tid) {
    u64* const sw = reinterpret_cast<u64*>(smem);
    u32* const sf = reinterpret_cast<u32*>(smem + NB * kExactWords * 8);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      bool lost = false;
#pragma unroll
      for (int j = 0; j < kExactWords; ++j) {
        const i64 v = pv.word(b, j);
        if (v) lost = exact_add_word(sw + b * kExactWords, j, v) || lost;
      }
      if (lost) {
        atomicAdd(&stats[kStFixedPointOverflow], 1);
        pv.flag |= 1u << b;
      }
      if ((pv.flag >> b) & 1u) atomicOr(&sf[b], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      u32* const gf = reinterpret_cast<u32*>(gw + NB * kExactWords);
      for (int b = 0; b < NB; ++b) {
        i64 wv[kExactWords];
        for (int j = 0; j < kExactWords; ++j) wv[j] = (i64)sw[b * kExactWords + j];
        const bool lost = exact_merge_bin(gw + b * kExactWords, wv);
        if (lost) atomicAdd(&stats[kStFixedPointOverflow], 1);
        if (lost || sf[b]) atomicOr(&gf[b], 1u);
      }
    }
  }
  __device__ static void readout(const u64* gw, float* out, i32* stats) {
    const u32* const gf = reinterpret_cast<const u32*>(gw + NB * kExactWords);
    for (int b = 0; b < NB; ++b) {
      bool bad = false;
      const float o = exact_read(gw + b * kExactWords, &bad);
      if (bad && !gf[b]) atomicAdd(&stats[kStFixedPointOverflow], 1);
      out[b] = (gf[b] || bad) ? __int_as_float(0x7fc00000) : o;
    }
  }
};

// A thread-private exact accumulator of NB bins whose words live in the thread's slots of ExactBins<NB, BLK>'s
// private region in shared memory (bind: the region's address), touched once per item.  Held in registers, its 5
// words per bin would stay live across the whole step loop and push the step's own values out to local memory.
template <int NB, int BLK = TM_BLOCK>
struct ExactPrivS {
  i64* w;       // this thread's word (0, 0)
  u32 flag;     // bit b: bin b saw a non-finite emit or lost a carry
  __device__ __forceinline__ void bind(unsigned char* region) {
    w = reinterpret_cast<i64*>(region) + threadIdx.x;
    flag = 0u;
  }
  __device__ __forceinline__ i64& at(int b, int j) const { return w[(b * kExactWords + j) * BLK]; }
  __device__ __forceinline__ i64 word(int b, int j) const { return at(b, j); }
  __device__ __forceinline__ bool emit(int b, float v) {
    return exact_priv_emit([this](int bb, int jj) -> i64& { return at(bb, jj); }, flag, b, v);
  }
};

// ------------------------------------------------------------------------------------------------ fixed-point Sums
// A Sum(fixed_point=True) of f32 (tallymap/_api.py:55-84; kernel.py:870-941): every emit is added exactly into its
// bin's carry-save words (atomics, on shared or global words), so the bin is the correctly rounded f32 of the exact
// sum whatever the order of the emits.  A non-finite emit or a carry out of the top word flags the bin (NaN at
// readout), counted in stats[3]; an index outside [0, S) is dropped and counted in stats[4].
// (exact_emit_atomic: tm_device.cuh)
template <int S>
struct ExactSum {
  // words: S x 5 u64, then S u32 flags (shared or global); bytes of that layout
  static constexpr int kBytes = S * kExactWords * 8 + S * 4;
  __device__ __forceinline__ static void emit(u64* words, i32* stats, i32 b, float v) {
    if ((u32)b >= (u32)S) {
      atomicAdd(&stats[kStDroppedEmits], 1);
      return;
    }
    if (exact_emit_atomic(words + (i64)b * kExactWords, v)) {
      atomicOr(reinterpret_cast<u32*>(words + (i64)S * kExactWords) + b, 1u);
      atomicAdd(&stats[kStFixedPointOverflow], 1);
    }
  }
  // a block's shared words into the launch's global words (global flags packed after the words, as ExactBins)
  __device__ static void flush(const u64* sw, u64* gw, i32* stats, int tid, int nth) {
    const u32* const sf = reinterpret_cast<const u32*>(sw + (i64)S * kExactWords);
    u32* const gf = reinterpret_cast<u32*>(gw + (i64)S * kExactWords);
    for (int b = tid; b < S; b += nth) {
      i64 wv[kExactWords];
      bool any = false;
      for (int j = 0; j < kExactWords; ++j) {
        wv[j] = (i64)sw[b * kExactWords + j];
        any = any || wv[j] != 0;
      }
      const bool lost = any && exact_merge_bin(gw + (i64)b * kExactWords, wv);
      if (lost) atomicAdd(&stats[kStFixedPointOverflow], 1);
      if (lost || sf[b]) atomicOr(&gf[b], 1u);
    }
  }
  // global words -> the f32 output (the last block, all its threads)
  __device__ static void readout(const u64* gw, float* out, i32* stats, int tid, int nth) {
    const u32* const gf = reinterpret_cast<const u32*>(gw + (i64)S * kExactWords);
    for (int b = tid; b < S; b += nth) {
      bool bad = false;
      const float o = exact_read(gw + (i64)b * kExactWords, &bad);
      if (bad && !gf[b]) atomicAdd(&stats[kStFixedPointOverflow], 1);
      out[b] = (gf[b] || bad) ? __int_as_float(0x7fc00000) : o;
    }
  }
};

// An f32 sum tally in global memory, accumulated in an f64 shadow and warp-aggregated.  The lanes of a warp that add
// into the same bin in this call (found with __match_any_sync) sum their values in f64 in ascending lane order, and
// the lowest lane issues one f64 atomic add; the epilogue rounds every bin once to f32 (f64_to_f32).
// Why: a hot bin (every photon's first deposit lands in the source voxel, all of the same value) takes one atomic
// per warp instead of one per lane (fewer serialised adds on the hot L2 line), and an f32 accumulator that receives
// thousands of equal addends rounds them the same way every time: measured 6e-5 relative on the source voxel for
// 5,000 photons, the reference's f32 atomics 1.9e-5.  In f64 the total is exact to ~1e-16 whatever the order, so the
// rounded f32 bin is the correctly rounded sum in all but the rarest ties.  v == 0 adds nothing and joins no group.
// Every lane that reaches the call must make it (a warp-collective over the active lanes).
__device__ __forceinline__ void datom_warp(double* base, i32 idx, float v) {
  const unsigned active = __activemask();
  const int lane = threadIdx.x & 31;
  const bool live = v != 0.0f;
  const unsigned peers = __match_any_sync(active, live ? idx : -1 - lane);
  if (!live) return;
  if (peers == (1u << lane)) {
    atomicAdd(&base[idx], (double)v);
    return;
  }
  double sum = 0.0;
  unsigned rest = peers;
  while (rest) {
    const int src = __ffs(rest) - 1;
    rest &= rest - 1u;
    sum = sum + (double)__shfl_sync(peers, v, src);
  }
  if (lane == __ffs(peers) - 1) atomicAdd(&base[idx], sum);
}

// datom_warp with a shared-memory window: when widx >= 0 (a function of idx: every lane of a group has the same) the
// group's sum goes to the block's f32 window bin widx instead of the global f64 bin idx.  The window holds the hot
// bins (a photon's first deposits land next to the source), so most adds are shared-memory atomics; the block adds
// its window into the f64 bins once, at its flush.  Per block a window bin sums a few thousand values in f32
// (relative error ~1e-6), and the f64 total over the blocks rounds once.
__device__ __forceinline__ void datom_warp_window(double* base, float* win, i32 idx, i32 widx, float v) {
  const unsigned active = __activemask();
  const int lane = threadIdx.x & 31;
  const bool live = v != 0.0f;
  const unsigned peers = __match_any_sync(active, live ? idx : -1 - lane);
  if (!live) return;
  double sum = (double)v;
  if (peers != (1u << lane)) {
    sum = 0.0;
    unsigned rest = peers;
    while (rest) {
      const int src = __ffs(rest) - 1;
      rest &= rest - 1u;
      sum = sum + (double)__shfl_sync(peers, v, src);
    }
    if (lane != __ffs(peers) - 1) return;
  }
  if (widx >= 0) atomicAdd(&win[widx], (float)sum);
  else atomicAdd(&base[idx], sum);
}

// datom_warp_window for an f32 tally accumulated in place: a group's values (the lanes of the warp adding into one
// bin in this call) are summed in f64 in ascending lane order and rounded once, then added with one f32 atomic into
// the block's window bin widx (widx >= 0: a shared-memory f32 window of hot bins, added into the tally once per
// block) or into the global bin idx (fatom: one red.global.add.f32, a compare-and-swap add below 2^-102).  The f64
// group sum keeps a hot bin's per-warp addends from rounding the same way thousands of times; the global bins get one
// f32 add per warp group, the source voxel's window one per block.  Every lane that reaches the call must make it.
__device__ __forceinline__ void fatom_warp_window(float* base, float* win, i32 idx, i32 widx, float v) {
  const unsigned active = __activemask();
  const int lane = threadIdx.x & 31;
  const bool live = v != 0.0f;
  const unsigned peers = __match_any_sync(active, live ? idx : -1 - lane);
  if (!live) return;
  float sum = v;
  if (peers != (1u << lane)) {
    double d = 0.0;
    unsigned rest = peers;
    while (rest) {
      const int src = __ffs(rest) - 1;
      rest &= rest - 1u;
      d = d + (double)__shfl_sync(peers, v, src);
    }
    if (lane != __ffs(peers) - 1) return;
    sum = __double2float_rn(d);
  }
  if (widx >= 0) atomicAdd(&win[widx], sum);
  else fatom(&base[idx], sum);
}

// the epilogue of an f64-accumulated tally: out[i] = f32(acc[i]) (round to nearest), block-wide
__device__ __forceinline__ void f64_to_f32(const double* acc, float* out, int n, int tid, int nth) {
  for (int i = tid; i < n; i += nth) out[i] = __double2float_rn(acc[i]);
}

// a privatised f32 sum tally of S bins at `off` bytes into shared memory: emit (drop + count when out of range) and
// flush of the nonzero bins with global atomics (kernel.py:681-688)
template <int S>
struct SumPriv {
  __device__ static void emit(float* sh, i32* stats, i32 b, float v) {
    if ((u32)b >= (u32)S) atomicAdd(&stats[kStDroppedEmits], 1);
    else fatom(&sh[b], v);
  }
  __device__ static void flush(const float* sh, float* g, int tid, int nth) {
    for (int b = tid; b < S; b += nth) {
      const float v = sh[b];
      if (v != 0.0f) fatom(&g[b], v);
    }
  }
};

// A scaled fixed-point sum (a Sum(fixed_point=True) of another dtype than float32; tallymap/_api.py:55-84): a bin
// is an int64 word `lo` that wraps, a signed count `carry` of its wraps (+1 when an add of q > 0 left it below its old
// value, -1 when one of q < 0 left it above), and a flag.  Whatever order the adds run in, the bin's total is exactly
// lo + carry * 2^64.  Layout of the scratch: lo[S], then carry i32[S], then flag u32[S].
struct WideSum {
  // add round(x) (x = v * scale); |x| >= 9.2e18 is not representable: dropped, counted and the bin flagged
  __device__ __forceinline__ static void emit(unsigned long long* lo, i32* carry, u32* flag, i32* stats, i32 b,
                                              double x) {
    if (!(fabs(x) < 9.2e18)) {
      atomicAdd(&stats[kStFixedPointOverflow], 1);
      flag[b] = 1u;
      return;
    }
    const long long q = __double2ll_rn(x);
    if (q == 0) return;
    const long long before = (long long)atomicAdd(&lo[b], (unsigned long long)q);
    const long long after = (long long)((unsigned long long)before + (unsigned long long)q);
    if (q > 0 && after < before) atomicAdd(&carry[b], 1);
    if (q < 0 && after > before) atomicAdd(&carry[b], -1);
  }
  // the 128-bit integer lo + carry * 2^64 rounded once to double: its magnitude split into high and low 64-bit
  // halves, the top 64 significant bits converted by the hardware's round-to-nearest-even with every bit below them
  // folded into the lowest one (a sticky bit: it decides a tie the way the full value does), then scaled by 2^shift
  __device__ static double total(unsigned long long lo, i32 carry) {
    if (carry == 0) return (double)(long long)lo;
    unsigned long long hi = (unsigned long long)((long long)carry + ((long long)lo < 0 ? -1ll : 0ll));
    unsigned long long low = lo;
    const bool neg = (long long)hi < 0;
    if (neg) {                                         // the magnitude: two's complement negation of hi:low
      low = ~low + 1ull;
      hi = ~hi + (low == 0ull ? 1ull : 0ull);
    }
    if (hi == 0ull) return neg ? -(double)low : (double)low;
    const int bits = 64 - __clzll((long long)hi);      // significant bits of hi: the magnitude has 64 + bits
    const unsigned long long top = bits == 64 ? hi : ((hi << (64 - bits)) | (low >> bits));
    const unsigned long long below = bits == 64 ? low : (low << (64 - bits));
    const double m = ldexp((double)(top | (below != 0ull ? 1ull : 0ull)), bits);
    return neg ? -m : m;
  }
  // readout into the output (once per launch, after every emit): total / scale in the output's type; a flagged
  // bin is NaN in a float output; a value outside the output's range counts in fixed_point_overflow (a float bin
  // NaN, an integer bin saturated by the conversion)
  template <class O>
  __device__ static void readout(const unsigned long long* lo, const i32* carry, const u32* flag, O* out, i64 S,
                                 double inv_scale, i32* stats, int tid, int nth) {
    for (i64 i = tid; i < S; i += nth) {
      const double v = total(lo[i], carry[i]) * inv_scale;
      if (sizeof(O) == 8 && (O)0.5 != (O)0) {          // double
        const bool big = !(fabs(v) <= 1.7976931348623157e308);
        if (big && !flag[i]) atomicAdd(&stats[kStFixedPointOverflow], 1);
        out[i] = (flag[i] || big) ? (O)__longlong_as_double(0x7ff8000000000000ll) : (O)v;
      } else {
        const double lim = sizeof(O) == 8 ? 9223372036854775808.0 : 2147483648.0;
        if (!(v >= -lim && v < lim)) atomicAdd(&stats[kStFixedPointOverflow], 1);
        out[i] = (O)v;
      }
    }
  }
};

}  // namespace tmb
