// Tally helpers shared by the item programs.
#pragma once
#include "tm_runtime.cuh"

namespace tmb {

// An exact cotangent tally of NB bins: per-thread register words (ExactPriv), merged into the block's shared words
// when the thread runs out of items, then by one thread into the launch's global words; the last block reads them
// out (backends/kernel/kernel.py:625-628: a flagged or overflowing bin is NaN, counted in stats[3]).
// Shared layout: NB x 5 u64 words, then a u32 flag per bin.  Global layout: the same, flags packed after the words.
template <int NB>
struct ExactBins {
  static constexpr int kSmemBytes = NB * kExactWords * 8 + ((NB * 4 + 7) / 8) * 8;
  __device__ static void flush(ExactPriv<NB>& pv, unsigned char* smem, u64* gw, i32* stats, int tid) {
    u64* const sw = reinterpret_cast<u64*>(smem);
    u32* const sf = reinterpret_cast<u32*>(smem + NB * kExactWords * 8);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (exact_merge_bin(sw + b * kExactWords, pv.w[b])) {
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

}  // namespace tmb
