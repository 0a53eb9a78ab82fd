// Auxiliary kernels of the tallymap B200 backend:
//   exact_combine_kernel   the cross-GPU step of an exact (TSpec.exact) tally: every rank's carry-save words for a
//                          bin, gathered, are added with their carries and read out once, correctly rounded
//   exact_scatter_kernel   an exact f32 scatter-add of (value, bin) pairs (the exact Sum accumulator on its own)
//   tree_hist_kernel, tree_scan_kernel, tree_scatter_kernel
//                          the generation lists of a recorded spawn tree (the launch order of the tree adjoint)
//   probe_threefry_kernel  the calibration probe of the roofline: threefry2x32 evaluations per second at full
//                          occupancy with no memory traffic (the issue-rate peak of the walkers' dominant op mix)
//   probe_fp32_kernel      the FP32 instruction rate (independent multiply and add chains)
#pragma once
#include "tm_device.cuh"
#include "tm_math.h"

namespace tmb {

// words: [n_src][n_bins * 5 words, then per-bin u32 flags packed into (n_bins + 1) / 2 u64]: the exact scratch
// buffers of n_src launches (ranks) laid end to end.  One thread per bin: the bin's words from every source are
// added with their carries in registers, then read out.  out[b]: the correctly rounded f32, NaN if any source
// flagged the bin, a carry left the top word, or the total overflows f32 (each counted in stats[3]).
__global__ void exact_combine_kernel(const u64* words, int n_src, int n_bins, float* out, i32* stats) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_bins) return;
  const long long stride = (long long)n_bins * kExactWords + (n_bins + 1) / 2;
  ExactPriv<1> acc;
  acc.zero();
  bool flagged = false, lost = false;
  for (int r = 0; r < n_src; ++r) {
    const u64* w = words + r * stride;
    for (int j = 0; j < kExactWords; ++j) {
      const i64 q = (i64)w[(long long)b * kExactWords + j];
      if (q) lost = acc.add_word(0, j, q) || lost;
    }
    const u32* fl = reinterpret_cast<const u32*>(w + (long long)n_bins * kExactWords);
    flagged = flagged || fl[b] != 0u;
  }
  if (lost) atomicAdd(&stats[kStFixedPointOverflow], 1);
  u64 tw[kExactWords];
  for (int j = 0; j < kExactWords; ++j) tw[j] = (u64)acc.w[0][j];
  bool bad = false;
  const float o = exact_read(tw, &bad);
  if (bad && !flagged && !lost) atomicAdd(&stats[kStFixedPointOverflow], 1);
  out[b] = (flagged || lost || bad) ? __int_as_float(0x7fc00000) : o;
}

// exact scatter-add: bins[i] in [0, n_bins) receives vals[i] exactly (out of range: dropped, counted in stats[4]);
// words / flags in the exact scratch layout above (zeroed by the caller).
__global__ void exact_scatter_kernel(const float* vals, const i32* bins, long long n, int n_bins, u64* words,
                                     i32* stats) {
  u32* const flags = reinterpret_cast<u32*>(words + (long long)n_bins * kExactWords);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const i32 b = bins[i];
    if ((u32)b >= (u32)n_bins) { atomicAdd(&stats[kStDroppedEmits], 1); continue; }
    const bool bad = exact_emit_atomic(words + (long long)b * kExactWords, vals[i]);
    if (bad) { atomicAdd(&stats[kStFixedPointOverflow], 1); atomicOr(&flags[b], 1u); }
  }
}

// readout of exact words (layout above) into f32
__global__ void exact_readout_kernel(const u64* words, int n_bins, float* out, i32* stats) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_bins) return;
  const u32* fl = reinterpret_cast<const u32*>(words + (long long)n_bins * kExactWords);
  bool bad = false;
  const float o = exact_read(words + (long long)b * kExactWords, &bad);
  if (bad && !fl[b]) atomicAdd(&stats[kStFixedPointOverflow], 1);
  out[b] = (fl[b] || bad) ? __int_as_float(0x7fc00000) : o;
}

// the backend's f32 math on the device, elementwise (fn 0 log, 1 exp, 2 sin, 3 cos, 4 pow(x, y))
// ---- generation lists of a recorded spawn tree.  The reference orders each generation of the record with XLA
// scatters and a while loop (tallymap/_reverse_spawn.py:255-283) and launches the adjoint one generation at a time.
// Record r's generation is an integer of gen_bytes bytes (2: u16, 4: i32) at byte gen_off + r * stride; generations
// >= n_gen (or < 0) are counted in counts[n_gen] and listed nowhere (the host poisons the gradient: the reference's
// 'generation_overflow').  Within a generation the list order is arbitrary: each adjoint item writes only its own
// slot, and broadcast cotangents are exact tallies.
__device__ __forceinline__ int tree_gen_of(const unsigned char* rec, long long r, int stride, int gen_off,
                                           int gen_bytes, int n_gen) {
  const unsigned char* p = rec + r * stride + gen_off;
  const int g = gen_bytes == 2 ? (int)*reinterpret_cast<const unsigned short*>(p) : *reinterpret_cast<const int*>(p);
  return (g >= 0 && g < n_gen) ? g : n_gen;
}

// add 1 for this lane to counter[g] in shared memory, lanes of a warp with the same g sharing one atomic; -> the
// counter's value before this lane's add
__device__ __forceinline__ u32 shared_add_one(u32* counter, int g) {
  const int lane = threadIdx.x & 31;
  const unsigned peers = __match_any_sync(__activemask(), g);
  const int leader = __ffs(peers) - 1;
  u32 base = 0u;
  if (lane == leader) base = atomicAdd(&counter[g], (u32)__popc(peers));
  base = __shfl_sync(peers, base, leader);
  return base + __popc(peers & ((1u << lane) - 1u));
}

// counts[g] += the records of generation g (shared-memory histogram of n_gen + 1 bins per block)
__global__ void tree_hist_kernel(const unsigned char* rec, long long n, int stride, int gen_off, int gen_bytes,
                                 int n_gen, unsigned long long* counts) {
  extern __shared__ u32 hist[];
  for (int i = threadIdx.x; i <= n_gen; i += blockDim.x) hist[i] = 0u;
  __syncthreads();
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (long long)gridDim.x * blockDim.x)
    shared_add_one(hist, tree_gen_of(rec, r, stride, gen_off, gen_bytes, n_gen));
  __syncthreads();
  for (int i = threadIdx.x; i <= n_gen; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[i], (unsigned long long)hist[i]);
}

// cursor[g] = the exclusive prefix sum of counts (one thread: n_gen is a few thousand at most)
__global__ void tree_scan_kernel(const unsigned long long* counts, int n_gen, unsigned long long* cursor) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  unsigned long long a = 0ull;
  for (int g = 0; g <= n_gen; ++g) {
    cursor[g] = a;
    a += counts[g];
  }
}

// lists[...] = r for every record r of generation g < n_gen, grouped by generation.  A block takes a contiguous chunk
// of the records: it counts the chunk's generations in shared memory, reserves its range of each generation's list
// with one global atomic per generation, then places its records with shared-memory counters (one global atomic per
// generation per block instead of one per warp and generation)
__global__ void tree_scatter_kernel(const unsigned char* rec, long long n, int stride, int gen_off, int gen_bytes,
                                    int n_gen, unsigned long long* cursor, i32* lists) {
  extern __shared__ u32 sh[];
  u32* const cnt = sh;                       // [n_gen + 1]
  unsigned long long* const base = reinterpret_cast<unsigned long long*>(sh + ((n_gen + 2) & ~1));
  const long long chunk = (n + gridDim.x - 1) / gridDim.x;
  const long long lo = (long long)blockIdx.x * chunk, hi = lo + chunk < n ? lo + chunk : n;
  for (int i = threadIdx.x; i <= n_gen; i += blockDim.x) cnt[i] = 0u;
  __syncthreads();
  for (long long r = lo + threadIdx.x; r < hi; r += blockDim.x)
    shared_add_one(cnt, tree_gen_of(rec, r, stride, gen_off, gen_bytes, n_gen));
  __syncthreads();
  for (int i = threadIdx.x; i < n_gen; i += blockDim.x) {
    base[i] = cnt[i] ? atomicAdd(&cursor[i], (unsigned long long)cnt[i]) : 0ull;
    cnt[i] = 0u;
  }
  __syncthreads();
  for (long long r = lo + threadIdx.x; r < hi; r += blockDim.x) {
    const int g = tree_gen_of(rec, r, stride, gen_off, gen_bytes, n_gen);
    if (g < n_gen) lists[base[g] + shared_add_one(cnt, g)] = (i32)r;
  }
}

__global__ void math_eval_kernel(int fn, const float* x, const float* y, float* out, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    out[i] = tmm::eval(fn, x[i], y ? y[i] : 0.0f);
  }
}

// The FP32 instruction rate: per iteration 8 independent chains of one f32 multiply and one f32 add (separate
// instructions: the library is built with --fmad=false, as every kernel here), 16 FP32 instructions per thread.
__global__ void __launch_bounds__(128) probe_fp32_kernel(u32 iters, u32* out) {
  const u32 t = blockIdx.x * blockDim.x + threadIdx.x;
  float a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = 1.0f + 1e-7f * (float)(t + j);
  const float m = 0.999999f, d = 1e-7f;
  for (u32 i = 0; i < iters; ++i) {
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = __fadd_rn(__fmul_rn(a[j], m), d);
  }
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += a[j];
  out[t] = __float_as_uint(s);
}

// iters independent threefry2x32 evaluations per thread, folded into one word per thread (so none is dead code)
__global__ void __launch_bounds__(128) probe_threefry_kernel(u32 iters, u32* out) {
  const u32 t = blockIdx.x * blockDim.x + threadIdx.x;
  u32 acc = 0u;
  for (u32 i = 0; i < iters; ++i) {
    u32 o0, o1;
    threefry2x32(t, 0x9e3779b9u, 0u, i, o0, o1);
    acc ^= o0 ^ o1;
  }
  out[t] = acc;
}

}  // namespace tmb
