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
#ifdef __CUDACC_RTC__
#include <cuda/std/type_traits>
namespace tmstd = cuda::std;
#else
#include <type_traits>
namespace tmstd = std;
#endif

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

// ------------------------------------------------------------------------------------------------ optional hooks
// Two optional parts of the ITEM interface, detected at compile time:
//
// Draws (kUnroll > 1; typedef Draw; Draw draw(const Ctx&, const State&, int j); void apply(const Ctx&, State&,
// const Draw&)): the random draws of the step kc + j depend only on the item's key and the step index, not on the
// state (counter-based RNG: fold_in(key, kc) and its uniforms), so one iteration draws for up to kUnroll steps as
// independent threefry chains and then applies the steps one after another while the loop predicate holds
// (step == apply(draw(0))).  The chains interleave, so a warp that runs alone (the end of a launch, where a few long
// items remain) is no longer bound by the latency of one dependent threefry chain.  The draws of the steps past the
// item's end are wasted: at most kUnroll - 1 steps' draws per item.
//
// Parking (typedef Parked; Parked park(const Ctx&, const State&, i64 item); State unpark(Ctx&, const Parked&,
// i64& item)): everything an item in flight needs besides the launch's context, so it can move to another thread of
// the block.  Once the item counter runs dry, lanes whose items ended stay idle while their warp still steps the
// others; with parking, the block instead gathers its items in flight every kEpoch iterations and deals them to its
// first warps, so its stepping warps stay full and the others stop issuing.
// The block size of an ITEM's forward kernel: kBlock threads (with kMinBlocks resident blocks per SM, the launch
// bounds' register cap) when it defines them, else TM_BLOCK (and no minimum: 0 leaves the register allocation to
// ptxas, as launch bounds without one).  Larger blocks give the end-of-launch compaction below
// more warps to gather items from.
template <class T, class = void>
struct block_of : tmstd::integral_constant<int, TM_BLOCK> {};
template <class T>
struct block_of<T, tmstd::void_t<decltype(T::kBlock)>> : tmstd::integral_constant<int, T::kBlock> {};
template <class T, class = void>
struct min_blocks_of : tmstd::integral_constant<int, 0> {};
template <class T>
struct min_blocks_of<T, tmstd::void_t<decltype(T::kMinBlocks)>> : tmstd::integral_constant<int, T::kMinBlocks> {};

template <class T, class = void>
struct draws_trait : tmstd::false_type {};
template <class T>
struct draws_trait<T, tmstd::void_t<decltype(T::kUnroll)>> : tmstd::integral_constant<bool, (T::kUnroll > 1)> {};
template <class T, class = void>
struct park_trait : tmstd::false_type {};
template <class T>
struct park_trait<T, tmstd::void_t<typename T::Parked>> : tmstd::true_type {};

// one iteration's work for a lane whose loop predicate holds: one step, or up to kUnroll steps of pre-drawn
// randomness (each after the first only while the predicate still holds)
template <class I>
__device__ __forceinline__ void run_step(const typename I::Ctx& cx, typename I::State& x) {
  if constexpr (draws_trait<I>::value) {
    typename I::Draw d[I::kUnroll];
#pragma unroll
    for (int j = 0; j < I::kUnroll; ++j) d[j] = I::draw(cx, x, j);
    I::apply(cx, x, d[0]);
#pragma unroll
    for (int j = 1; j < I::kUnroll; ++j) {
      if (!I::cond(cx, x)) break;
      I::apply(cx, x, d[j]);
    }
  } else {
    I::step(cx, x);
  }
}

// The end of a launch for an ITEM with parking: every block runs its items in flight to their end in epochs of
// kEpoch iterations, gathering them into a shared-memory pool before each epoch and dealing them to threads
// 0, 1, ..., so the first ceil(L / 32) warps step full and the rest wait at the barrier (issuing nothing).
// Items keep their per-item results and their emits (privatised tallies are the block's; a thread's private exact
// words take whatever items it finishes), so moving an item changes no result.
constexpr int kEpoch = 16;
template <class I>
__device__ __forceinline__ void forward_tail(typename I::Ctx& cx, typename I::State& x, i64& item, bool live) {
  __shared__ typename I::Parked pool[block_of<I>::value];
  __shared__ int pool_n;
  for (;;) {
    __syncthreads();                               // (the previous epoch's reads of the pool are done)
    if (threadIdx.x == 0) pool_n = 0;
    __syncthreads();
    if (live) pool[atomicAdd(&pool_n, 1)] = I::park(cx, x, item);
    __syncthreads();
    const int n = pool_n;
    if (n == 0) break;
    live = (int)threadIdx.x < n;
    if (live) x = I::unpark(cx, pool[threadIdx.x], item);
    if (!__any_sync(0xffffffffu, live)) continue;
    for (int e = 0; e < kEpoch; ++e) {
      const bool stepping = live && I::cond(cx, x);
      __syncwarp();
      if (stepping) {
        run_step<I>(cx, x);
      } else if (live) {
        I::finish(cx, x, item);
        live = false;
      }
      if (!__any_sync(0xffffffffu, live)) break;
    }
  }
}

// ------------------------------------------------------------------------------------------------ forward kernel
// (each kernel is a __device__ body plus a __global__ wrapper, so that a program compiled at run time can wrap the
// same body in an `extern "C"` entry point: see tallymap_b200/lower.py)
template <class I>
__device__ __forceinline__ void forward_body(const Params& P, const i64 n_items) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr bool kPark = park_trait<I>::value;
  __shared__ int pool_dry;        // (parking) a claim of this block found the item counter run dry
  typename I::Ctx cx;
  I::setup(cx, P, smem);
  smem_zero(smem, I::kSmemBytes);
  if (kPark && threadIdx.x == 0) pool_dry = 0;
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
        if (kPark) *static_cast<volatile int*>(&pool_dry) = 1;
      } else {
        item = ticket_item(order, t);
        x = I::start(cx, item);
        active = true;
      }
    }
    if (!__any_sync(0xffffffffu, alive)) break;
    // (parking: once the counter has run dry, the block's warps go on to the end-of-launch epochs together)
    if (kPark && __any_sync(0xffffffffu, *static_cast<volatile int*>(&pool_dry) != 0)) break;
    // while every lane's item steps, steps run back to back without the claim and finish checks, until one ends
    // (parking: the run also stops when the counter runs dry, so no warp of the block keeps the others waiting)
    if (__all_sync(0xffffffffu, active && I::cond(cx, x))) {
      do {
        run_step<I>(cx, x);
      } while (__all_sync(0xffffffffu, I::cond(cx, x) && !(kPark && *static_cast<volatile int*>(&pool_dry))));
    }
    const bool stepping = alive && I::cond(cx, x);
    __syncwarp();
    if (stepping) {
      run_step<I>(cx, x);
    } else if (alive) {
      I::finish(cx, x, item);
      active = false;
    }
  }
  if constexpr (kPark) forward_tail<I>(cx, x, item, active);
  __syncthreads();
  I::flush(cx, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cx, ctl);
}

// (two entry points: launch bounds with a minimum of resident blocks only for an ITEM that asks for one -- a
// minimum of 0 does not always leave ptxas's register allocation as no minimum does)
template <class I>
__global__ void __launch_bounds__(block_of<I>::value) forward_kernel(const Params P, const i64 n_items) {
  forward_body<I>(P, n_items);
}
template <class I>
__global__ void __launch_bounds__(block_of<I>::value, min_blocks_of<I>::value)
    forward_kernel_occ(const Params P, const i64 n_items) {
  forward_body<I>(P, n_items);
}

// An ITEM with `static constexpr bool kFused = true` is a value-and-gradient program (FusedVG below): its replay's
// count pass is the forward pass itself, emitting the forward tallies (fwd_emit) and writing the forward's per-item
// results (fwd_finish), so one launch yields the outputs and their gradient for cotangents given up front.
template <class T, class = void>
struct fused_trait : tmstd::false_type {};
template <class T>
struct fused_trait<T, tmstd::void_t<decltype(T::kFused)>> : tmstd::integral_constant<bool, T::kFused> {};

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
__device__ __forceinline__ void replay_body(const Params& P, const i64 n_items) {
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
  S pre;          // (V == 1) the next stored state of the sweep, loaded while the current VJP runs
  typename I::Adj adj;
  int phase = have ? IDLE : -1;   // -1: no work left for this lane
  // step counts are bounded by max_steps < 2^31 (the cap is an i32 launch constant), so 32-bit bookkeeping
  i64 item = 0;
  i32 k = 0, K = 0, m = 0, ns = 0, s = 0, L = 0, u = 0, LL = 0, j = 0, a = 0, i = 0, base = 0;
  bool first = false;
  // warp-uniform loop: a lane with no work left keeps iterating (idle) until its whole warp is done; after the
  // (divergent) bookkeeping the warp reconverges, so every lane that steps runs the step body in one pass
  constexpr bool kFused = fused_trait<I>::value;
  for (;;) {
    bool vjp = false, stop = phase < 0, counting = false;
    while (!stop) {   // bookkeeping until this lane has a step or step VJPs to evaluate
      if (phase == COUNT) {
        if (I::cond(cx, x)) {
          head[k < C ? k : C] = I::store(x);
          ++k;
          counting = true;
          break;
        }
        K = k;
        fin = x;
        if constexpr (kFused) I::fwd_finish(cx, fin, item);
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
        if (a == u * C + LL - 1) {
          i = LL - 1;
          if constexpr (V == 1) pre = tape[i];
          phase = SWEEP;
          continue;
        }
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
        if (first) {
          i = LL - 1;
          if constexpr (V == 1) pre = head[i];
          phase = SWEEP;
          continue;
        }
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
    if (!stop && !vjp) {
      if constexpr (kFused) {
        I::fwd_emit(cx, x, counting);   // the count pass emits the forward tallies; checkpoint and refill passes do not
      } else {
        I::fwd(cx, x);
      }
    }
    __syncwarp();
    if (vjp) {
      const S* const src = first ? head : tape;
      if constexpr (V == 1) {
        // one VJP per iteration, software-pipelined: the state for this VJP was loaded in the previous iteration
        // (or when the sweep began), and the next one's load issues before this VJP's arithmetic, so its latency
        // hides behind it
        const S cur = pre;
        if (i > 0) pre = src[i - 1];
        I::vjp(cx, I::restore(cx, cur, base + i), adj);
        i -= 1;
      } else {
        // up to V stored states, newest first: the loads issue together, then the VJPs run in order
        S st[V];
#pragma unroll
        for (int v = 0; v < V; ++v) st[v] = src[i - v >= 0 ? i - v : 0];
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (i - v >= 0) I::vjp(cx, I::restore(cx, st[v], base + i - v), adj);
        i -= V;
      }
    }
  }
  __syncthreads();
  I::adj_flush(cx, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cx, ctl);
}

template <class I, int V>
__global__ void __launch_bounds__(TM_BLOCK) replay_kernel(const Params P, const i64 n_items) {
  replay_body<I, V>(P, n_items);
}
template <class I, int V>
__global__ void __launch_bounds__(TM_BLOCK, min_blocks_of<I>::value) replay_kernel_occ(const Params P,
                                                                                       const i64 n_items) {
  replay_body<I, V>(P, n_items);
}

// ------------------------------------------------------------------------------------------------ pipelined value and grad
// vg_kernel<I, V>: a fused value-and-grad program (I::kFused) when every item fits the scratch (C >= max_steps).
// In the replay kernel a lane counts an item, then sweeps it, so at any iteration some lanes of a warp count and
// others sweep and the warp pays for both paths.  Here each lane keeps a ring tape of T = C + 1 stored states
// (T a power of two >= max_steps + 2): it counts items back to back into the tape -- one forward step with emits per
// iteration, each item followed by its final state -- while it sweeps the oldest counted item, newest state first,
// one step VJP per iteration (up to V when it has nothing left to count).  So the forward step and one VJP run for
// nearly every lane every iteration.  A lane whose tape or queue of counted items is full waits (sweeping) before
// it counts on.  The step VJPs of an item run in the replay's order on the same states: the gradient is bitwise the
// replay's.  ITEM additions: restore() of an item's final state at step K.
template <class I, int V>
__device__ __forceinline__ void vg_body(const Params& P, const i64 n_items) {
  static_assert(fused_trait<I>::value, "vg_kernel runs fused value-and-grad programs");
  constexpr int kQ = 8;             // counted items awaiting their sweep, per lane
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
  const u32 T = (u32)C + 1u, mask = T - 1u;
  // the host launches this kernel only with T a power of two >= max_steps + 2; a thread beyond the planned scratch,
  // or a launch that breaks that rule, takes no items and sets the error word (bit 1)
  const bool have = gtid < cap && C >= 1 && (T & mask) == 0u && (i64)T >= (i64)__ldg(&consts[I::kConstM]) + 2;
  if (!have) atomicOr(&ctl[kCtlError], 2u);
  S* const tape = static_cast<S*>(P.p[I::kReplay]) + (have ? gtid : 0) * (i64)T;
  typename I::Ctx cs = cx;          // the sweeping item's context (its per-item fields, the thread's accumulators)
  X x, sinit, sfin;
  typename I::Adj adj;
  i64 item = 0, sitem = 0;
  i32 k = 0, si = -1, sK = 0;
  u32 wpos = 0u, rlo = 0u, cstart = 0u, sstart = 0u;   // tape positions (mod 2^32; the tape index is pos & mask)
  i64 q_item[kQ];
  i32 q_k[kQ];
  u32 q_start[kQ];
  u32 qh = 0u, qt = 0u;
  bool counting = false, sweeping = false, alive = have;
  for (;;) {
    bool c_ok = counting && I::cond(cx, x);
    if (counting && !c_ok && qt - qh < (u32)kQ && wpos - rlo < T) {
      // the count pass ended: the forward's post-loop code; the final state follows the item's states on the tape
      I::fwd_finish(cx, x, item);
      tape[wpos & mask] = I::store(x);
      ++wpos;
      q_item[qt % kQ] = item;
      q_k[qt % kQ] = k;
      q_start[qt % kQ] = cstart;
      ++qt;
      counting = false;
    }
    if (alive && !counting) {
      const u64 t = claim_item(ctr);
      if (t >= (u64)n_items) {
        alive = false;
      } else {
        item = ticket_item(order, t);
        x = I::start(cx, item);
        k = 0;
        cstart = wpos;
        counting = true;
        c_ok = I::cond(cx, x);
      }
    }
    if (!sweeping && qh != qt) {
      sitem = q_item[qh % kQ];
      sK = q_k[qh % kQ];
      sstart = q_start[qh % kQ];
      ++qh;
      sinit = I::start(cs, sitem);     // (re-derives the item's per-item context; the accumulators stay)
      sfin = I::restore(cs, tape[(sstart + (u32)sK) & mask], sK);
      I::adj_start(cs, adj);
      I::post_vjp(cs, sfin, adj);
      si = sK - 1;
      sweeping = true;
    }
    if (!__any_sync(0xffffffffu, counting || sweeping || alive)) break;
    // a step needs its slot and one more for the item's final state
    const bool step_now = c_ok && (wpos - rlo + 2u <= T);
    __syncwarp();
    if (step_now) {
      tape[wpos & mask] = I::store(x);
      ++wpos;
      ++k;
      I::fwd_emit(cx, x, true);
    }
    __syncwarp();
    if (sweeping) {
      const int nv = counting ? 1 : V;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (v < nv && si >= 0) {
          I::vjp(cs, I::restore(cs, tape[(sstart + (u32)si) & mask], si), adj);
          --si;
        }
      }
      if (si < 0) {
        I::adj_finish(cs, sinit, sfin, adj, sitem);
        rlo = sstart + (u32)sK + 1u;
        sweeping = false;
      }
    }
  }
  __syncthreads();
  I::handoff(cs, cx);   // one context for the flush: the counting context's, with the sweeping one's accumulators
  I::adj_flush(cs, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cs, ctl);
}

template <class I, int V>
__global__ void __launch_bounds__(TM_BLOCK) vg_kernel(const Params P, const i64 n_items) {
  vg_body<I, V>(P, n_items);
}

// ------------------------------------------------------------------------------------------------ value and grad
// FusedVG<F, G, Map>: forward item F and its adjoint G as one replay program.  The launch's buffers are G's, with F's
// result buffers that G lacks (its tallies and per-item results) inserted where the host's layout puts them; Map
// gives, for each of F's and G's buffer indices, the fused index (Map::f(i), Map::g(i); shared buffers -- inputs,
// constants, claim order, control words, stats, the truncation flags -- map to one index) and Map::kNF, kNG, kNBuf
// the buffer counts.  G's constants start with max_steps, as F's.  Shared memory: G's block, then F's (16-byte
// aligned).
template <class F, class G, class Map>
struct FusedVG {
  static constexpr bool kFused = true;
  static constexpr int kGSmem = (G::kSmemBytes + 15) / 16 * 16;
  static constexpr int kSmemBytes = kGSmem + F::kSmemBytes;
  enum { kConsts = Map::g(G::kConsts), kOrder = Map::g(G::kOrder), kCtl = Map::g(G::kCtl),
         kReplay = Map::g(G::kReplay), kNBuf = Map::kNBuf };
  enum { kConstM = G::kConstM, kConstC = G::kConstC, kConstThreads = G::kConstThreads };
  typedef typename G::State State;
  typedef typename G::Adj Adj;
  typedef typename G::Stored Stored;
  struct Ctx {
    typename G::Ctx g;
    typename F::Ctx f;
  };
  __device__ __forceinline__ static Params remap_g(const Params& P) {
    Params Q;
#pragma unroll
    for (int i = 0; i < Map::kNG; ++i) Q.p[i] = P.p[Map::g(i)];
    return Q;
  }
  __device__ __forceinline__ static Params remap_f(const Params& P) {
    Params Q;
#pragma unroll
    for (int i = 0; i < Map::kNF; ++i) Q.p[i] = P.p[Map::f(i)];
    return Q;
  }
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    G::setup(c.g, remap_g(P), smem);
    F::setup(c.f, remap_f(P), smem + kGSmem);
  }
  __device__ static void stage(const Params& P, unsigned char* smem) {
    G::stage(remap_g(P), smem);
    F::stage(remap_f(P), smem + kGSmem);
  }
  __device__ static State start(Ctx& c, i64 item) {
    F::start(c.f, item);
    return G::start(c.g, item);
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return G::cond(c.g, s); }
  __device__ __forceinline__ static void fwd_emit(const Ctx& c, State& s, bool emit) {
    if (emit) F::step(c.f, s);
    else G::fwd(c.g, s);
  }
  __device__ __forceinline__ static void fwd(const Ctx& c, State& s) { G::fwd(c.g, s); }
  __device__ static void fwd_finish(const Ctx& c, const State& fin, i64 item) { F::finish(c.f, fin, item); }
  __device__ __forceinline__ static void handoff(Ctx& sweep, const Ctx& count) {
    const auto pv = sweep.g.pv;      // the thread's exact cotangent words stay with the sweeping context
    sweep = count;
    sweep.g.pv = pv;
  }
  __device__ static void adj_start(const Ctx& c, Adj& a) { G::adj_start(c.g, a); }
  __device__ __forceinline__ static Stored store(const State& s) { return G::store(s); }
  __device__ __forceinline__ static State restore(const Ctx& c, Stored v, i64 step) { return G::restore(c.g, v, step); }
  __device__ __forceinline__ static void vjp(const Ctx& c, const State& at, Adj& a) { G::vjp(c.g, at, a); }
  __device__ static void post_vjp(const Ctx& c, const State& fin, Adj& a) { G::post_vjp(c.g, fin, a); }
  __device__ static void adj_finish(const Ctx& c, const State& init, const State& fin, Adj& a, i64 item) {
    G::adj_finish(c.g, init, fin, a, item);
  }
  __device__ static void adj_flush(const Ctx& c, unsigned char* smem, int tid, int nth) {
    G::adj_flush(c.g, smem, tid, nth);
    F::flush(c.f, smem + kGSmem, tid, nth);
  }
  __device__ static void epilogue(const Ctx& c, int tid, int nth) {
    G::epilogue(c.g, tid, nth);
    F::epilogue(c.f, tid, nth);
  }
};

// An item whose loop carries do not depend on the differentiated operands (no active carry: the walkers, whose
// operand enters only the emitted values) has a separable adjoint: the VJP of step k needs the state the step starts
// from and the output cotangents, never a later state or a carry cotangent.  OnePassVG<F, G, Map> sums those step
// VJPs while the forward runs, for forward_body: no replay, no stored states, one pass over each item.  The
// gradient is the reverse program's up to the f32 summation order of each item's cotangent (oldest step first here,
// newest first in the replay: _reverse.py:324-444), within the float tolerance, not bitwise; the per-item sums go
// into the same exact tally.  F and G as for FusedVG (G's replay scratch, if it has one, is not used: Map::g of
// G::kReplay may be any index); F::State and G::State are one type; G::adj_finish gets the final state for the
// initial one (the walkers' pre-loop code has no VJP).
template <class F, class G>
struct OnePassCtx {
  typename G::Ctx g;
  typename F::Ctx f;
};
template <class F, class G>
struct OnePassState {
  typename G::State s;
  typename G::Adj a;
};
// (the forward's optional draws and parking, carried over to the one-pass program when the forward has them: the
// step VJP is applied before each pre-drawn step, and a parked item keeps its running cotangents)
template <class F, class G, bool = draws_trait<F>::value>
struct OnePassDraws {};
template <class F, class G>
struct OnePassDraws<F, G, true> {
  static constexpr int kUnroll = F::kUnroll;
  typedef typename F::Draw Draw;
  __device__ __forceinline__ static Draw draw(const OnePassCtx<F, G>& c, const OnePassState<F, G>& st, int j) {
    return F::draw(c.f, st.s, j);
  }
  __device__ __forceinline__ static void apply(const OnePassCtx<F, G>& c, OnePassState<F, G>& st, const Draw& d) {
    G::vjp(c.g, st.s, st.a);
    F::apply(c.f, st.s, d);
  }
};
template <class F, class G, bool = park_trait<F>::value>
struct OnePassPark {};
template <class F, class G>
struct OnePassPark<F, G, true> {
  struct Parked {
    typename F::Parked f;
    typename G::Adj a;
  };
  __device__ __forceinline__ static Parked park(const OnePassCtx<F, G>& c, const OnePassState<F, G>& st, i64 item) {
    return Parked{F::park(c.f, st.s, item), st.a};
  }
  __device__ __forceinline__ static OnePassState<F, G> unpark(OnePassCtx<F, G>& c, const Parked& p, i64& item) {
    OnePassState<F, G> st;
    st.s = F::unpark(c.f, p.f, item);
    G::start(c.g, item);            // (the adjoint's per-item context, from the item's inputs)
    st.a = p.a;
    return st;
  }
};

template <class F, class G, class Map>
struct OnePassVG : OnePassDraws<F, G>, OnePassPark<F, G> {
  static constexpr int kBlock = block_of<G>::value, kMinBlocks = min_blocks_of<G>::value;
  static constexpr int kGSmem = (G::kSmemBytes + 15) / 16 * 16;
  static constexpr int kSmemBytes = kGSmem + F::kSmemBytes;
  enum { kConsts = Map::g(G::kConsts), kOrder = Map::g(G::kOrder), kCtl = Map::g(G::kCtl), kNBuf = Map::kNBuf };
  typedef OnePassState<F, G> State;
  typedef OnePassCtx<F, G> Ctx;
  __device__ __forceinline__ static Params remap_g(const Params& P) {
    Params Q;
#pragma unroll
    for (int i = 0; i < Map::kNG; ++i) Q.p[i] = P.p[Map::g(i)];
    return Q;
  }
  __device__ __forceinline__ static Params remap_f(const Params& P) {
    Params Q;
#pragma unroll
    for (int i = 0; i < Map::kNF; ++i) Q.p[i] = P.p[Map::f(i)];
    return Q;
  }
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    G::setup(c.g, remap_g(P), smem);
    F::setup(c.f, remap_f(P), smem + kGSmem);
  }
  __device__ static void stage(const Params& P, unsigned char* smem) {
    G::stage(remap_g(P), smem);
    F::stage(remap_f(P), smem + kGSmem);
  }
  __device__ static State start(Ctx& c, i64 item) {
    State st;
    st.s = F::start(c.f, item);
    G::start(c.g, item);
    G::adj_start(c.g, st.a);
    return st;
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& st) { return F::cond(c.f, st.s); }
  __device__ __forceinline__ static void step(const Ctx& c, State& st) {
    G::vjp(c.g, st.s, st.a);           // the step's VJP at the state it starts from
    F::step(c.f, st.s);
  }
  // (copies: the loop's state never has its address taken by a call the compiler may not inline, so it stays in
  // registers for the whole loop)
  __device__ __forceinline__ static void finish(const Ctx& c, const State& st, i64 item) {
    const typename G::State s = st.s;
    typename G::Adj a = st.a;
    F::finish(c.f, s, item);
    G::post_vjp(c.g, s, a);
    G::adj_finish(c.g, s, s, a, item);
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    G::adj_flush(c.g, const_cast<unsigned char*>(smem), tid, nth);
    F::flush(c.f, smem + kGSmem, tid, nth);
  }
  __device__ static void epilogue(const Ctx& c, int tid, int nth) {
    G::epilogue(c.g, tid, nth);
    F::epilogue(c.f, tid, nth);
  }
};

}  // namespace tmb
