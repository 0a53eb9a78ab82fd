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
//   Stored, store, restore, fwd, vjp   the compact stored state and the split step (see replay_kernel)
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
// the counter between them, one atomic per warp.  -> this lane's claim ticket (>= n_items: nothing left).
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

// The item a ticket runs: order[t] when the launch gives a claim order (a permutation of 0..N-1, e.g. longest
// items first from a primal call's trip counts), else t.  The order only moves work between threads and in time:
// per-item results are written at the item's own index and exact tallies are order-independent.
__device__ __forceinline__ i64 ticket_item(const i32* order, u64 t) { return order ? (i64)__ldg(&order[t]) : (i64)t; }

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
  const i32* const order = static_cast<const i32*>(P.p[I::kOrder]);
  typename I::State x;
  i64 item = 0;
  bool active = false, alive = true;
  // warp-uniform loop: a lane with no item left keeps iterating (idle) until its whole warp is done, so the step
  // body always runs reconverged, every stepping lane of the warp in one pass
  for (;;) {
    if (alive && !active) {
      const u64 t = claim_item(ctr);
      if (t >= (u64)n_items) {
        alive = false;
      } else {
        item = ticket_item(order, t);
        x = I::start(cx, item);
        active = true;
      }
    }
    if (!__any_sync(0xffffffffu, alive)) break;
    const bool stepping = alive && I::cond(cx, x);
    __syncwarp();
    if (stepping) {
      I::step(cx, x);
    } else if (alive) {
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
// run as a per-lane state machine, one loop step per iteration (or up to V step VJPs).  Per item:
//   COUNT  the forward pass: the state before step k goes to head[min(k, C)] (slot C is a sink), K = trip count
//   CKPT   (K > C) replay from the initial state, keeping every m-th state, m = max(C, ceil(K / C))
//   per segment s = ns-1 .. 0, per sub-chunk u = nsub-1 .. 0 of at most C states:
//     FILL  advance from checkpoint s by u*C steps, storing the sub-chunk's states in the tape
//     SWEEP apply the step VJP at each stored state, newest first (the first sub-chunk reads the head)
// The step VJPs run in the same order, on the same states, as the reference's nested loops, whatever C is, so the
// cotangents are bitwise the reference's; only the work and the memory depend on C.
//
// B200 layout: the head, checkpoint and tape buffers (3C + 1 compact states per resident thread) live in a global
// scratch buffer, contiguous per thread, so a lane's consecutive stores and loads fill and drain whole sectors; C is
// a launch constant sized by the host from device memory: C >= max_steps when the heads of every resident thread fit
// (then the scratch is the head alone, C + 1 states per thread, and every item is counted and swept with no replay:
// one forward evaluation per step), else as large as the memory budget allows.  A lane in SWEEP applies up to V step VJPs per iteration (a VJP is a few instructions against a
// forward step's two threefry2x32), so lanes sweeping and lanes stepping share the warp's iterations.
//
// ITEM additions for this kernel: Stored (the compact state: the carries a step reads that are not the step index),
// store(State) -> Stored, restore(Ctx, Stored, i64 step) -> State, fwd(Ctx, State&) (one step, no emits),
// vjp(Ctx, const State& at, Adj&) (the step VJP at the state before the step); kReplay (the scratch buffer) and the
// launch constants kConstM (max_steps), kConstC (C) and kConstThreads (threads the scratch holds).
template <class I, int V>
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
  const i32* const consts = static_cast<const i32*>(P.p[I::kConsts]);
  const i32* const order = static_cast<const i32*>(P.p[I::kOrder]);
  const i32 C = __ldg(&consts[I::kConstC]);
  const i64 cap = __ldg(&consts[I::kConstThreads]);
  const i64 gtid = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  typedef typename I::Stored S;
  typedef typename I::State X;
  // a thread beyond the scratch the host sized (a launch on a device with more resident threads than planned for)
  // takes no items: the others claim them; the error word records it (bit 1)
  const bool have = gtid < cap && C >= 1;
  if (!have) atomicOr(&ctl[kCtlError], 2u);
  // C >= max_steps: every item fits the head (K <= C, one segment, no checkpoints or tape), so a thread's scratch is
  // the head alone
  const bool head_only = C >= __ldg(&consts[I::kConstM]);
  const i64 stride = head_only ? (i64)C + 1 : 3 * (i64)C + 1;
  S* const head = static_cast<S*>(P.p[I::kReplay]) + (have ? gtid : 0) * stride;
  S* const ck = head + C + 1;
  S* const tape = ck + C;

  enum { IDLE, COUNT, CKPT, SEG, SUB, FILL, SWEEP, DONE };
  X x, init, fin;
  typename I::Adj adj;
  int phase = have ? IDLE : -1;   // -1: no work left for this lane
  // step counts are bounded by max_steps < 2^31 (the cap is an i32 launch constant), so 32-bit bookkeeping
  i64 item = 0;
  i32 k = 0, K = 0, m = 0, ns = 0, s = 0, L = 0, u = 0, LL = 0, j = 0, a = 0, i = 0, base = 0;
  bool first = false;
  // warp-uniform loop: a lane with no work left keeps iterating (idle) until its whole warp is done; after the
  // (divergent) bookkeeping the warp reconverges, so every lane that steps runs the step body in one pass
  for (;;) {
    bool vjp = false, stop = phase < 0;
    while (!stop) {   // bookkeeping until this lane has a step or step VJPs to evaluate
      if (phase == COUNT) {
        if (I::cond(cx, x)) {
          head[k < C ? k : C] = I::store(x);
          ++k;
          break;
        }
        K = k;
        fin = x;
        I::post_vjp(cx, fin, adj);
        m = (i64)K > (i64)C * C ? (K + C - 1) / C : C;
        ns = (K + m - 1) / m;
        if (K == 0) { phase = DONE; continue; }
        if (ns > 1) { x = init; j = 0; phase = CKPT; } else { s = 0; phase = SEG; }
        continue;
      }
      if (phase == SWEEP) {
        if (i >= 0) { vjp = true; break; }
        if (u > 0) { --u; phase = SUB; continue; }
        if (s > 0) { --s; phase = SEG; continue; }
        phase = DONE;
        continue;
      }
      if (phase == FILL) {
        if (a >= u * C) tape[a - u * C] = I::store(x);
        if (a == u * C + LL - 1) { i = LL - 1; phase = SWEEP; continue; }
        ++a;
        break;
      }
      if (phase == CKPT) {
        if (j % m == 0) ck[j / m] = I::store(x);
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
        LL = min(C, L - u * C);
        first = (s == 0 && u == 0);
        base = s * m + u * C;
        if (first) { i = LL - 1; phase = SWEEP; continue; }
        x = I::restore(cx, ck[s], s * m);
        a = 0;
        phase = FILL;
        continue;
      }
      if (phase == DONE) {
        I::adj_finish(cx, init, fin, adj, item);
        phase = IDLE;
        continue;
      }
      if (phase == IDLE) {
        const u64 t = claim_item(ctr);
        if (t >= (u64)n_items) { phase = -1; stop = true; break; }
        item = ticket_item(order, t);
        init = I::start(cx, item);
        x = init;
        if (!head_only) ck[0] = I::store(init);   // (read when a one-segment item refills: C < K)
        k = 0;
        I::adj_start(cx, adj);
        phase = COUNT;
        continue;
      }
      phase = -1;   // no scratch for this thread
      stop = true;
    }
    if (!__any_sync(0xffffffffu, phase >= 0)) break;
    __syncwarp();
    if (!stop && !vjp) I::fwd(cx, x);
    __syncwarp();
    if (vjp) {
      // up to V stored states, newest first: the loads issue together, then the VJPs run in order
      const S* const src = first ? head : tape;
      S st[V];
#pragma unroll
      for (int v = 0; v < V; ++v) st[v] = src[i - v >= 0 ? i - v : 0];
#pragma unroll
      for (int v = 0; v < V; ++v)
        if (i - v >= 0) I::vjp(cx, I::restore(cx, st[v], base + i - v), adj);
      i -= V;
    }
  }
  __syncthreads();
  I::adj_flush(cx, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cx, ctl);
}

}  // namespace tmb
