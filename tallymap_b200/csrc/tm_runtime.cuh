// The persistent-thread runtime of the tallymap B200 backend: the forward kernel and the reverse-mode replay kernel,
// templated on an ITEM (a lowered item program).  Hand-written for sm_100a.
//
// What the reference does (tallymap/backends/kernel/kernel.py:727-838): every thread claims items through a
// warp-aggregated atomic counter and runs one item at a time to completion; under its default 'item' schedule a
// warp then costs its LONGEST item.  Here the unit of work is one loop STEP: each lane holds one item's loop state in
// registers, evaluates one step per iteration, and a lane whose item has ended claims the next item at once (the
// reference's opt-in 'step' schedule, kernel.py:225-295, made the only schedule).  The warp stays converged on the
// step body, which is the whole cost, whatever the spread of trip counts.
//
// ITEM interface (static members; State lives in registers):
//   kSmemBytes                         bytes of privatised tallies in shared memory (zeroed by the runtime)
//   Ctx                                per-thread view of the launch: buffer pointers, broadcast scalars
//   setup(Ctx&, const Params&, unsigned char* smem)
//   stage(const Params&, unsigned char* smem)   copy small read-only tables into shared memory (block-wide)
//   State start(const Ctx&, i64 item)  the code before the item's top-level loop
//   bool cond(const Ctx&, const State&)   the loop predicate, max_steps cap included
//   void step(const Ctx&, State&)      one loop step, tallies emitted through Ctx
//   void finish(const Ctx&, const State&, i64 item)   the code after the loop: emits, per-item results
//   void flush(const Ctx&, const unsigned char* smem, int tid, int nth)   privatised tallies -> global (block-wide)
//   void epilogue(const Ctx&, int tid, int nth)   once per launch, by the last block to finish (readouts)
// For the replay kernel additionally:
//   Adj                                the per-item cotangent accumulators (active carries, broadcast cotangents)
//   void adj_start(const Ctx&, Adj&)
//   void micro(const Ctx&, const State& at, State& next, Adj&, bool vjp)   next = step(at); if vjp, also apply the
//                                      step's VJP at `at` (the forward part is shared by every lane of the warp)
//   void post_vjp(const Ctx&, const State& final, Adj&)   cotangents of the loop outputs from the code after it
//   void adj_finish(const Ctx&, const State& init, const State& final, Adj&, i64 item)   pre-loop VJP, cotangent
//                                      emits, per-item results (the replay's truncation flag)
//   void adj_flush(const Ctx&, unsigned char* smem, int tid, int nth)  (private accumulators -> shared -> global)
#pragma once
#include "tm_device.cuh"

namespace tmb {

#ifndef TM_BLOCK
#define TM_BLOCK 128
#endif

// Warp-aggregated claim (kernel.py:732-739): the lanes that need an item this iteration take one contiguous run of
// the counter between them, one atomic per warp.  -> this lane's item index (>= n_items: nothing left).
__device__ __forceinline__ u64 claim_item(u64* ctr) {
  const unsigned m = __activemask();
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  const unsigned rank = __popc(m & ((1u << lane) - 1u));
  unsigned long long base = 0ull;
  if (lane == leader) base = atomicAdd((unsigned long long*)ctr, (unsigned long long)__popc(m));
  base = __shfl_sync(m, base, leader);
  return (u64)base + rank;
}

// zero the block's privatised tallies
__device__ __forceinline__ void smem_zero(unsigned char* smem, int bytes) {
  for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x) reinterpret_cast<u32*>(smem)[i] = 0u;
}

// After the block has flushed: count it finished; the last block of the grid (all others' flushes visible)
// runs the epilogue.
template <class I>
__device__ __forceinline__ void finish_block(const typename I::Ctx& cx, u32* ctl) {
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&ctl[kCtlDone], 1u) == gridDim.x - 1) ? 1 : 0;
  __syncthreads();
  if (last) {
    __threadfence();
    I::epilogue(cx, threadIdx.x, blockDim.x);
  }
}

// ------------------------------------------------------------------------------------------------ forward kernel
template <class I>
__global__ void __launch_bounds__(TM_BLOCK) forward_kernel(const Params P, const i64 n_items) {
  extern __shared__ __align__(16) unsigned char smem[];
  typename I::Ctx cx;
  I::setup(cx, P, smem);
  smem_zero(smem, I::kSmemBytes);
  __syncthreads();
  I::stage(P, smem);
  __syncthreads();
  u32* const ctl = static_cast<u32*>(P.p[I::kCtl]);
  u64* const ctr = reinterpret_cast<u64*>(ctl + kCtlClaim);
  typename I::State x;
  i64 item = 0;
  bool active = false;
  for (;;) {
    if (!active) {
      const u64 t = claim_item(ctr);
      if (t >= (u64)n_items) break;
      item = (i64)t;
      x = I::start(cx, item);
      active = true;
    }
    if (I::cond(cx, x)) {
      I::step(cx, x);
    } else {
      I::finish(cx, x, item);
      active = false;
    }
  }
  __syncthreads();
  I::flush(cx, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cx, ctl);
}

// ------------------------------------------------------------------------------------------------ replay kernel
// The reverse-mode program of an item with one top-level loop: the checkpointed loop of tallymap/_reverse.py:324-444
// run as a per-lane state machine, one loop step (or one step VJP) per iteration.  Per item:
//   COUNT  the forward pass: the state before step k goes to head[min(k, C)] (slot C is a sink), K = trip count
//   CKPT   (K > C) replay from the initial state, keeping every m-th state, m = max(C, ceil(K / C))
//   per segment s = ns-1 .. 0, per sub-chunk u = nsub-1 .. 0 of at most C states:
//     FILL  advance from checkpoint s by u*C steps, then store the sub-chunk's states in the tape
//     SWEEP apply the step VJP at each stored state, newest first (the first sub-chunk reads the head)
// The step VJPs therefore run in the same order, on the same states, as the reference's nested loops, so the
// cotangents are bitwise the same; only the interleaving across lanes differs.  Lanes in different phases still
// share the forward step (ITEM::micro), so a warp issues one step body per iteration.
template <class I, int C>
__global__ void __launch_bounds__(TM_BLOCK) replay_kernel(const Params P, const i64 n_items) {
  extern __shared__ __align__(16) unsigned char smem[];
  typename I::Ctx cx;
  I::setup(cx, P, smem);
  smem_zero(smem, I::kSmemBytes);
  __syncthreads();
  I::stage(P, smem);
  __syncthreads();
  u32* const ctl = static_cast<u32*>(P.p[I::kCtl]);
  u64* const ctr = reinterpret_cast<u64*>(ctl + kCtlClaim);

  enum { IDLE, COUNT, CKPT, SEG, SUB, FILL, SWEEP, DONE };
  typename I::State head[C + 1], ck[C], tape[C];
  typename I::State x, init, fin, at;
  typename I::Adj adj;
  int phase = IDLE;
  i64 item = 0, k = 0, K = 0, m = 0, ns = 0, s = 0, L = 0, u = 0, LL = 0, j = 0, a = 0, i = 0;
  bool first = false;
  for (;;) {
    bool vjp = false, stop = false;
    for (;;) {   // bookkeeping until this lane has a step or a step VJP to evaluate
      if (phase == COUNT) {
        if (I::cond(cx, x)) {
          head[k < C ? k : C] = x;
          ++k;
          break;
        }
        K = k;
        fin = x;
        I::post_vjp(cx, fin, adj);
        m = K > (i64)C * C ? (K + C - 1) / C : C;
        ns = (K + m - 1) / m;
        if (K == 0) { phase = DONE; continue; }
        if (ns > 1) { x = init; j = 0; phase = CKPT; } else { s = 0; phase = SEG; }
        continue;
      }
      if (phase == CKPT) {
        if (j % m == 0) ck[j / m] = x;
        if (j == (ns - 1) * m) { s = ns - 1; phase = SEG; continue; }
        ++j;
        break;
      }
      if (phase == SEG) {
        L = min(m, K - s * m);
        u = (L + C - 1) / C - 1;
        phase = SUB;
        continue;
      }
      if (phase == SUB) {
        LL = min((i64)C, L - u * C);
        first = (s == 0 && u == 0);
        if (first) { i = LL - 1; phase = SWEEP; continue; }
        x = ck[s];
        a = 0;
        phase = FILL;
        continue;
      }
      if (phase == FILL) {
        if (a >= u * C) tape[a - u * C] = x;
        if (a == u * C + LL - 1) { i = LL - 1; phase = SWEEP; continue; }
        ++a;
        break;
      }
      if (phase == SWEEP) {
        if (i >= 0) {
          at = first ? head[i] : tape[i];
          --i;
          vjp = true;
          break;
        }
        if (u > 0) { --u; phase = SUB; continue; }
        if (s > 0) { --s; phase = SEG; continue; }
        phase = DONE;
        continue;
      }
      if (phase == DONE) {
        I::adj_finish(cx, init, fin, adj, item);
        phase = IDLE;
        continue;
      }
      // IDLE: claim the next item
      const u64 t = claim_item(ctr);
      if (t >= (u64)n_items) { stop = true; break; }
      item = (i64)t;
      init = I::start(cx, item);
      x = init;
      ck[0] = init;
      k = 0;
      I::adj_start(cx, adj);
      phase = COUNT;
    }
    if (stop) break;
    if (vjp) {
      typename I::State nx;
      I::micro(cx, at, nx, adj, true);
    } else {
      I::micro(cx, x, x, adj, false);
    }
  }
  __syncthreads();
  I::adj_flush(cx, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cx, ctl);
}

}  // namespace tmb
