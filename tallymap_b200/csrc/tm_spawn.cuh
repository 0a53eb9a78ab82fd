// The spawn queue of the tallymap B200 runtime and the persistent kernel that runs items that spawn children.
//
// The reference (backends/kernel/kernel.py:778-811, 1007-1044) runs a bounded MPMC ticket ring: per child, an
// occupancy reservation, a ticket, a spin on the slot's sequence number, the leaves, a fence, the publication and a
// pending count -- five atomics on five control words per child, and each consumer pops one child at a time.  With
// 10^8..10^9 particles per call those per-child atomics on a handful of addresses serialise.  Here every queue
// operation is warp-aggregated: the lanes of a warp that push in one iteration reserve their slots with ONE atomic on
// the occupancy word and ONE on the tail, and the lanes that need work pop with one atomic on the pending count and
// one on the head.  Slot states are lap-encoded sequence words, so zeroed memory is an empty ring (no prep kernel):
// for ticket t, slot t % Q, lap L = t / Q, the slot is free for L when seq == 2L, published when 2L + 1, and freed to
// 2L + 2 by its consumer.  Control words sit on separate 128-byte lines (the reference's QCTL_STRIDE, kernel.py:307).
//
// Work sharing: a lane keeps the children it spawns on a private stack (its newest entries in shared memory, older
// ones in local memory) and runs them depth-first, with no atomics, unless lanes are hungry: a lane that finds no
// work counts itself in the hungry word until it gets some, and a lane that spawns shares its children through the
// ring while the ring holds fewer pending children than there are hungry lanes (looked at every 16 iterations while
// not sharing, every iteration while sharing).  So the ring carries only the children other lanes are waiting for.  A breadth-first FIFO over 10^6 roots
// would need a ring as wide as the whole forest's frontier (the reference sizes its Queue to the pending children);
// depth-first lanes share only what hungry lanes wait for, so the ring never overflows and a count is deterministic.
// in a different order than the reference's ring runs them, which changes no tally bit beyond float summation order.
//
// Termination: a lane is counted in flight from its claim (root) or global pop (child) until it has finished its item
// and emptied its private stack, after its shared children are published; a lane with nothing to run leaves when no
// lane is in flight and nothing is pending.  A
// reservation increments in-flight before it decrements pending, so no work is ever invisible to both counts, and
// it is attempted only while pending is positive (a pending count pushed below zero by a reservation in progress is
// not work; polling lanes that reacted to it would keep the counts from ever settling).
//
// Every wait is bounded (kSpinLimit polls): a wait that gives up sets the device error word (bit 0), drops the
// child (counted in stats[1]) or abandons the ticket, and the host raises after the launch (tm_check_status).
#pragma once
#include "tm_runtime.cuh"

namespace tmb {

constexpr int kQStride = 32;      // u32 words between control words (128 B)
enum { kQTail = 0, kQHead = 1, kQPending = 2, kQOcc = 3, kQFlight = 4, kQHungry = 5, kQWords = 6 };
constexpr u32 kSpinLimit = 1u << 22;   // polls of a slot sequence word (~0.3 s with the back-off)
constexpr u64 kIdleLimitNs = 20000000000ull;   // 20 s without progress: give up (the error word says so)
constexpr int kPrivate = 48;       // a lane's private stack of children (a shower's tree is < 80 generations deep)
constexpr int kStackShared = 8;    // its newest entries live in the thread's column of shared memory

// A lane's private children: a stack whose newest entries (up to kStackShared) are in shared memory (word w of entry
// e of thread t at u32 [(e * W + w) * TM_BLOCK + t]: conflict-free whatever entry each lane touches); when they are
// all taken, they move to local memory together.  In local memory alone, the lanes' different stack depths put
// every lane's word in its own sector, and the stacks of a full SM overflow L1 into L2 and DRAM.
template <class I>
struct SpawnSmem {
  static constexpr int kCW = (int)(sizeof(typename I::Child) / 4);
  static constexpr int kItemBytes = (I::kSmemBytes + 15) / 16 * 16;
  static constexpr int kBytes = kItemBytes + kStackShared * kCW * 4 * TM_BLOCK;
};

__device__ __forceinline__ u32* qword(u32* q, int w) { return q + w * kQStride; }
__device__ __forceinline__ u32 ld_volatile(const u32* p) { return *reinterpret_cast<const volatile u32*>(p); }
// a slot's sequence word: published / freed with release stores, polled with acquire loads, so the leaves written
// before a release are visible to the reader after its acquire (no full fences on the ring's data path)
__device__ __forceinline__ u32 ld_acquire(const u32* p) {
  u32 v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(u32* p, u32 v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ u64 globaltimer() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// wait (bounded) until seq[slot] == want (an acquire: what was written before its publication is visible); false if
// the wait gave up
__device__ __forceinline__ bool wait_seq(const u32* seq, u32 slot, u32 want) {
  for (u32 i = 0; i < kSpinLimit; ++i) {
    if (ld_acquire(&seq[slot]) == want) return true;
    __nanosleep(64);
  }
  return false;
}

// ITEM interface for spawn_kernel, in addition to forward_kernel's:
//   Child                      the leaves of a child (the mapped per-item inputs)
//   kQueue, kSeq, kQctl        buffer indices of the ring (Child[Q]), its sequence words (u32[Q]) and control words
//   kConstQ                    index of Q in the launch constants
//   start_child(Ctx&, const Child&) -> State       a popped child's pre-loop code
//   step(const Ctx&, State&, Child& o0, Child& o1, int& n_out)   one step; up to 2 children to spawn (kept
//                              privately, o0 runs first: an item that puts its smaller subtree in o0 keeps the
//                              private stack at most log2 of the subtree deep)
//   finish(const Ctx&, const State&, i64 item, bool child)   post-loop code; per-item results for roots only
// or, with kPostSpawn = true (children spawned after the loop, tallymap/_tally.py spawn in the post-loop code):
//   finish(const Ctx&, const State&, i64 item, bool child, Child& o0, Child& o1, int& n_out)
template <class T, class = void>
struct post_spawn_trait : tmstd::false_type {};
template <class T>
struct post_spawn_trait<T, tmstd::void_t<decltype(T::kPostSpawn)>> : tmstd::integral_constant<bool, T::kPostSpawn> {};

template <class I>
__device__ __forceinline__ void spawn_body(const Params& P, const i64 n_items) {
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
  typedef typename I::Child Child;
  Child* const ring = static_cast<Child*>(P.p[I::kQueue]);
  u32* const seq = static_cast<u32*>(P.p[I::kSeq]);
  u32* const q = static_cast<u32*>(P.p[I::kQctl]);
  i32* const stats = static_cast<i32*>(P.p[I::kStats]);
  const u32 Q = (u32)__ldg(static_cast<const i32*>(P.p[I::kConsts]) + I::kConstQ);
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;

  typename I::State x;
  i64 item = 0;
  bool active = false, alive = true, child = false, roots_left = true, hungry = false;
  u64 idle_since = 0;
  u32 spawned = 0;                  // this thread's spawned children, added to stats[0] once at the end
  static_assert(sizeof(Child) % 4 == 0, "a child is whole 4-byte words");
  constexpr int kCW = SpawnSmem<I>::kCW;
  union ChildWords {
    Child c;
    u32 w[kCW];
  };
  u32* const sstk = reinterpret_cast<u32*>(smem + SpawnSmem<I>::kItemBytes) + threadIdx.x;
  int sn = 0;                       // entries in shared memory (the newest)
  u32 iter = 0u;
  bool share_c = false;             // the sharing decision, refreshed every 16 iterations
  Child stk[kPrivate];              // older entries, moved here kStackShared at a time when the shared part is full
  int nl = 0;
  auto sput = [&](int e, const Child& ch) {
    ChildWords u;
    u.c = ch;
#pragma unroll
    for (int j = 0; j < kCW; ++j) sstk[(e * kCW + j) * TM_BLOCK] = u.w[j];
  };
  auto sget = [&](int e) {
    ChildWords u;
#pragma unroll
    for (int j = 0; j < kCW; ++j) u.w[j] = sstk[(e * kCW + j) * TM_BLOCK];
    return u.c;
  };
  auto has_room = [&]() { return sn < kStackShared || nl + kStackShared <= kPrivate; };
  auto push = [&](const Child& ch) {          // (has_room() holds)
    if (sn == kStackShared) {
      for (int e = 0; e < kStackShared; ++e) stk[nl + e] = sget(e);
      nl += kStackShared;
      sn = 0;
    }
    sput(sn++, ch);
  };
  auto pop = [&]() { return sn > 0 ? sget(--sn) : stk[--nl]; };   // (a private child exists)
  for (;;) {
    // ---- lanes without an item: their own children first, then the ring's, then roots
    bool needy = alive && !active;
    if (needy && (sn > 0 || nl > 0)) {
      x = I::start_child(cx, pop());
      child = true;
      active = true;
      needy = false;
    }
    const unsigned m = __ballot_sync(0xffffffffu, needy);
    if (m) {
      const int leader = __ffs(m) - 1;
      const u32 n = __popc(m);
      u32 avail = 0, head = 0;
      // reserve only while pending is positive: a negative value is another warp's reservation in progress (it
      // gives back what it cannot take), and reacting to it would keep both counts perturbed for ever
      if (lane == leader && (i32)ld_volatile(qword(q, kQPending)) > 0) {
        atomicAdd(qword(q, kQFlight), n);                       // in flight before pending drops
        const i32 p = (i32)atomicSub(qword(q, kQPending), n);
        avail = p <= 0 ? 0u : (p >= (i32)n ? n : (u32)p);
        if (avail < n) {
          atomicAdd(qword(q, kQPending), n - avail);
          atomicSub(qword(q, kQFlight), n - avail);
        }
        if (avail) head = atomicAdd(qword(q, kQHead), avail);
      }
      avail = __shfl_sync(0xffffffffu, avail, leader);
      head = __shfl_sync(0xffffffffu, head, leader);
      const u32 rank = __popc(m & lt);
      bool got = false;
      if (needy && rank < avail) {
        const u32 t = head + rank, slot = t % Q, lap = t / Q;
        if (wait_seq(seq, slot, 2u * lap + 1u)) {
          const Child ch = ring[slot];
          st_release(&seq[slot], 2u * lap + 2u);      // (the read above completes before the slot is free)
          atomicSub(qword(q, kQOcc), 1u);
          x = I::start_child(cx, ch);
          child = true;
          got = true;
        } else {
          atomicOr(&ctl[kCtlError], 1u);                        // a published child never showed: abandon it
          atomicSub(qword(q, kQFlight), 1u);
        }
      }
      // the rest claim roots (warp-aggregated) while any are left
      const bool want_root = needy && !got;
      const unsigned mr = __ballot_sync(0xffffffffu, want_root && roots_left);
      if (mr) {
        const int lr = __ffs(mr) - 1;
        unsigned long long base = 0ull;
        if (lane == lr) {
          base = atomicAdd((unsigned long long*)ctr, (unsigned long long)__popc(mr));
          const u64 b = base, e = base + __popc(mr);
          const u32 nroot = e <= (u64)n_items ? __popc(mr) : (b >= (u64)n_items ? 0u : (u32)((u64)n_items - b));
          if (nroot) atomicAdd(qword(q, kQFlight), nroot);
        }
        base = __shfl_sync(0xffffffffu, base, lr);
        if (want_root && roots_left) {
          const u64 t = (u64)base + __popc(mr & lt);
          if (t < (u64)n_items) {
            item = ticket_item(order, t);
            x = I::start(cx, item);
            child = false;
            got = true;
          } else {
            roots_left = false;
          }
        }
      }
      if (got) {
        active = true;
        idle_since = 0;
        if (hungry) {
          atomicSub(qword(q, kQHungry), 1u);
          hungry = false;
        }
      } else if (needy) {
        // nothing to run: count as hungry; leave once nothing is in flight or pending (bounded by the idle limit)
        if (!hungry) {
          atomicAdd(qword(q, kQHungry), 1u);
          hungry = true;
        }
        const u32 fl = ld_volatile(qword(q, kQFlight));
        const i32 pe = (i32)ld_volatile(qword(q, kQPending));
        if (!roots_left && fl == 0u && pe <= 0) {
          alive = false;
          atomicSub(qword(q, kQHungry), 1u);
          hungry = false;
        } else {
          const u64 now = globaltimer();
          if (idle_since == 0) idle_since = now;
          if (now - idle_since > kIdleLimitNs) {
            atomicOr(&ctl[kCtlError], 1u);
            alive = false;
            atomicSub(qword(q, kQHungry), 1u);
            hungry = false;
          }
          __nanosleep(256);
        }
      }
    }
    if (!__any_sync(0xffffffffu, alive)) break;

    // ---- one step for every lane that has an item
    Child o0, o1;
    int n_out = 0;
    bool done = false;
    if (active) {
      if (I::cond(cx, x)) {
        I::step(cx, x, o0, o1, n_out);
        // an item this step finished is finished in this iteration, not one later: a shower particle takes ~1.2
        // steps, so the later finish cost nearly half of every lane's iterations (an item that spawns after its
        // loop keeps the later finish: its children need the step's child slots)
        if constexpr (!post_spawn_trait<I>::value) {
          if (!I::cond(cx, x)) done = true;
        }
      } else {
        done = true;
        if constexpr (post_spawn_trait<I>::value) I::finish(cx, x, item, child, o0, o1, n_out);
      }
    }
    // ---- spawned children: onto the private stack unless lanes are hungry for them (or the stack is full), else
    // into the ring, warp-aggregated
    // whether to share: while not sharing, re-read every 16 iterations (warp-uniform, one load per warp), not at
    // every spawn -- a load of the two control words at every spawn put an L2 round trip on the path of nearly every
    // iteration; while sharing (the launch's tail), every iteration, so that sharing stops as soon as the ring holds
    // what the hungry lanes wait for.  The decision is a policy: it changes no count and no termination.
    if (share_c || (++iter & 15u) == 0u)
      share_c = (i32)ld_volatile(qword(q, kQPending)) < (i32)ld_volatile(qword(q, kQHungry));
    // o0 runs first: a lane whose item ended with this step continues with o0 itself (no round trip through the
    // stack) and keeps o1 on its private stack; otherwise o1 then o0 go on the stack, so o0 is on top.  With the
    // item putting its smaller subtree in o0, every entry on a lane's stack is the larger sibling of a node whose
    // subtree at least halved on the way down, so a stack holds at most log2 of its root's subtree.
    bool cont = false;
    int first = 0;                   // the ring's first child: o0 (0) or o1 (1)
    if (n_out > 0) {
      spawned += (u32)n_out;
      const bool share = share_c;
      bool r0 = false, r1 = false;   // o0 / o1 go to the ring
      if (n_out > 1) {
        if (!share && has_room()) push(o1);
        else r1 = true;
      }
      if constexpr (!post_spawn_trait<I>::value) cont = done && !share;
      if (!cont) {
        if (!share && has_room()) push(o0);
        else r0 = true;
      }
      first = r0 ? 0 : 1;
      n_out = (int)r0 + (int)r1;     // the children left for the ring
    }
    const unsigned mp = __ballot_sync(0xffffffffu, n_out > 0);
    if (mp) {
      // exclusive scan of n_out over the warp
      u32 off = 0, tot = 0;
      for (int l = 0; l < 32; ++l) {
        const u32 v = __shfl_sync(0xffffffffu, (u32)n_out, l);
        if (l < lane) off += v;
        tot += v;
      }
      const int leader = __ffs(mp) - 1;
      u32 allowed = 0, base = 0;
      if (lane == leader) {
        const u32 o = atomicAdd(qword(q, kQOcc), tot);
        allowed = o >= Q ? 0u : (Q - o >= tot ? tot : Q - o);
        if (allowed < tot) {
          atomicSub(qword(q, kQOcc), tot - allowed);
          atomicAdd(&stats[kStChildrenDropped], (i32)(tot - allowed));
        }
        if (allowed) base = atomicAdd(qword(q, kQTail), allowed);
        if (allowed < tot) atomicSub(&stats[kStSpawned], (i32)(tot - allowed));
      }
      allowed = __shfl_sync(0xffffffffu, allowed, leader);
      base = __shfl_sync(0xffffffffu, base, leader);
      u32 published = 0;
      for (int j = 0; j < n_out; ++j) {
        if (off + j >= allowed) break;
        const u32 t = base + off + j, slot = t % Q, lap = t / Q;
        if (wait_seq(seq, slot, 2u * lap)) {
          ring[slot] = (j == 0 && first == 0) ? o0 : o1;
          st_release(&seq[slot], 2u * lap + 1u);      // (the leaves above are visible to whoever acquires this)
          ++published;
        } else {
          // the slot never freed: publish nothing there (its ticket is lost: a consumer waiting on it times out)
          atomicOr(&ctl[kCtlError], 1u);
          atomicAdd(&stats[kStChildrenDropped], 1);
          atomicSub(&stats[kStSpawned], 1);
        }
      }
      // pending counts only published children, after the whole warp has published
      u32 warp_pub = published;
      for (int d = 16; d > 0; d >>= 1) warp_pub += __shfl_xor_sync(0xffffffffu, warp_pub, d);
      if (lane == leader && warp_pub) atomicAdd(qword(q, kQPending), warp_pub);
    }
    if (done) {
      if constexpr (!post_spawn_trait<I>::value) I::finish(cx, x, item, child);
      if (cont) {                                // (still in flight: the lane runs its own child o0 next)
        x = I::start_child(cx, o0);
        child = true;
      } else {
        active = false;
        if (sn == 0 && nl == 0) {                // busy -> idle: leave the in-flight count
          __threadfence();
          atomicSub(qword(q, kQFlight), 1u);
        }
      }
    }
  }
  if (spawned) atomicAdd(&stats[kStSpawned], (i32)spawned);
  __syncthreads();
  I::flush(cx, smem, threadIdx.x, blockDim.x);
  finish_block<I>(cx, ctl);
}

template <class I>
// (at least 6 blocks per SM: ptxas then keeps the loop's values in up to 80 registers instead of spilling them at
// the 64-72 it picks unbounded; the shower's step 105 -> 95 ms, 5 blocks gave the same)
__global__ void __launch_bounds__(TM_BLOCK, 6) spawn_kernel(const Params P, const i64 n_items) {
  spawn_body<I>(P, n_items);
}

}  // namespace tmb
