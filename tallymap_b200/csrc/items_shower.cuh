// Item program of the branching-shower configuration (benchmark configuration 5), lowered for the spawn runtime
// (tm_spawn.cuh).  The item, as a tallymap user writes it (one particle; children are spawned with the same inputs):
//
//   def particle(t, E, depth, key, X0):                    # per item: E, depth, key; broadcast: X0
//     def body(c):
//       k, E, depth, alive, t = c
//       kk = fold_in(key, k)
//       u = uniform(kk, (3,))                               # travel, split decision, energy fraction
//       depth = depth + X0 * -log(1 - u[0])                 # exponential path of mean X0 (never log 0)
//       low = E < 0.5
//       t = t.add("dep", where(low, (depth * 8).astype(int32), 0), where(low, E, 0.0))   # deposit all, stop
//       split = ~low & (u[1] < 0.7)
//       z = 0.1 + 0.8 * u[2]
//       t = t.spawn((E * z, depth, fold_in(kk, 0)), when=split)
//       t = t.spawn((E * (1 - z), depth, fold_in(kk, 1)), when=split)
//       return k + 1, E, depth, ~low & ~split, t
//     k, E, depth, alive, t = while_loop(lambda c: c[3], body, (0, E, depth, True, t))
//     t = t.add("count", 0, 1)
//     return t, k
//
// with max_steps = 100,000 per particle (retrace(cap): children count into stats[2] when they truncate) and a
// Queue of capacity Q.  A split particle ends, replaced by its two children; an unsplit one steps again.
//
// Buffers:
//   sh_fwd   E0 f32[N], depth0 f32[N], keys u32[N,2], X0 f32, consts i32[2] (max_steps, Q), order |
//            dep f32[512], count i32[1], seq u32[Q], qctl u32[6*32], ctl, stats | k i32[N], trunc u8[N],
//            ring (E, depth, key)[Q]
#pragma once
#include "tm_math.h"
#include "tm_spawn.cuh"
#include "tm_tally.cuh"

namespace tmb {

// A child in the forward and one-pass launches carries its parent's step key kk and its index j (0 or 1) instead of
// its own key fold_in(kk, j), which it derives at its first step (child_key): the two fold_ins of a split ran in a
// branch that 41 % of the lanes take, and the warp issued it nearly every step; the one fold_in of a child's first step
// runs in a branch that 83 % of the lanes take (a shower particle takes ~1.2 steps).  j travels in the sign bit of the
// child's energy, which is always positive (a particle splits only with E >= 0.5, into fractions z and 1 - z of at
// least 0.1): the Child keeps its size, and so the shared-memory stacks theirs.  The keys, and so every result,
// are the same bits.
__device__ __forceinline__ float child_energy(float E, u32 j) { return j ? -E : E; }

struct ShowerChild {
  float E, depth;     // (E: the energy, its sign bit the child's index j)
  u32 ka, kb;         // the parent's step key
};

struct ShowerState {
  i32 kc, k;
  float E, depth;
  Key key;
  bool alive;
  i32 kj;             // -1: key is the particle's key; 0 / 1: key is its parent's step key and j this (child_key)
};

// a child's key at its first step: fold_in(parent step key, j)
template <class St>
__device__ __forceinline__ void child_key(St& s) {
  if (s.kj >= 0) {
    s.key = fold_in(s.key, (u32)s.kj);
    s.kj = -1;
  }
}

// The loop body above, shared by the forward, the recording forward and the adjoint's replay: travel, the deposit
// when low (emitted through `emit` unless null), the split decision.  -> the split flag, the energy fraction z of
// child 0 and the step key (the children's keys are fold_in(kk, 0) and fold_in(kk, 1)).
struct ShowerStepOut {
  bool split, low;
  float z, L;
  Key kk;
};
template <class St>
__device__ __forceinline__ ShowerStepOut shower_advance(float X0, St& s) {
  const Key kk = fold_in(s.key, (u32)s.k);
  const float u0 = uniform01(kk, 0u), u1 = uniform01(kk, 1u), u2 = uniform01(kk, 2u);
  const float L = -tmm::logf(1.0f - u0);
  s.depth = s.depth + X0 * L;
  const bool low = s.E < 0.5f;
  const bool split = !low && u1 < 0.7f;
  s.alive = !low && !split;
  s.kc += 1;
  s.k += 1;
  return ShowerStepOut{split, low, 0.1f + 0.8f * u2, L, kk};
}

struct SHFwd {
  enum { kE0, kDepth0, kKeys, kX0, kConsts, kOrder, kDep, kCount, kSeq, kQctl, kCtl, kStats, kK, kTrunc, kQueue,
         kNBuf };
  enum { kConstM, kConstQ };
  static constexpr int kNB = 512;
  static constexpr int kSmemBytes = kNB * 4 + 16;
  typedef ShowerChild Child;
  typedef ShowerState State;
  struct Ctx {
    const float *E0, *d0;
    const uint2* keys;
    float X0;
    i32 M;
    float* sh;
    i32* shc;
    float* dep;
    i32* count;
    i32* stats;
    i32* kout;
    uint8_t* trunc;
    mutable i32 n;     // particles this thread finished
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.E0 = static_cast<const float*>(P.p[kE0]);
    c.d0 = static_cast<const float*>(P.p[kDepth0]);
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.X0 = __ldg(static_cast<const float*>(P.p[kX0]));
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]) + kConstM);
    c.sh = reinterpret_cast<float*>(smem);
    c.shc = reinterpret_cast<i32*>(smem + kNB * 4);
    c.dep = static_cast<float*>(P.p[kDep]);
    c.count = static_cast<i32*>(P.p[kCount]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.n = 0;
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    return State{0, 0, __ldg(&c.E0[item]), __ldg(&c.d0[item]), Key{kk.x, kk.y}, true, -1};
  }
  __device__ static State start_child(Ctx&, const Child& ch) {
    return State{0, 0, fabsf(ch.E), ch.depth, Key{ch.ka, ch.kb}, true, (i32)(__float_as_uint(ch.E) >> 31)};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ __forceinline__ static void step(const Ctx& c, State& s, Child& o0, Child& o1, int& n_out) {
    child_key(s);
    const ShowerStepOut o = shower_advance(c.X0, s);
    if (o.low) SumPriv<kNB>::emit(c.sh, c.stats, f2i(s.depth * 8.0f), s.E);
    if (o.split) {
      const Child a{child_energy(s.E * o.z, 0u), s.depth, o.kk.a, o.kk.b};
      const Child b{child_energy(s.E * (1.0f - o.z), 1u), s.depth, o.kk.a, o.kk.b};
      const bool swap = o.z > 0.5f;          // the lower-energy child (the smaller subtree) runs first
      o0 = swap ? b : a;
      o1 = swap ? a : b;
      n_out = 2;
    }
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child) {
    c.n += 1;                                              // count: Sum((1,)) int32, per thread, then per block
    const bool tr = s.kc >= c.M && s.alive;
    if (child) {
      if (tr) atomicAdd(&c.stats[kStChildrenTruncated], 1);
    } else {
      c.kout[item] = s.k;
      c.trunc[item] = tr ? 1 : 0;
    }
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    SumPriv<kNB>::flush(reinterpret_cast<const float*>(smem), c.dep, tid, nth);
    if (c.n) atomicAdd(c.shc, c.n);
    __syncthreads();
    if (tid == 0) {
      const i32 v = *reinterpret_cast<const i32*>(smem + kNB * 4);
      if (v) atomicAdd(c.count, v);
    }
  }
  __device__ static void epilogue(const Ctx&, int, int) {}
};

// ------------------------------------------------------------------------------------ one pass: forward mode
// The shower's value and gradient in one spawn launch.  Only E reaches an emitted value (the deposit E when low);
// depth and X0 reach the outputs only through the integer bin index, so their cotangents are zero (the tree adjoint
// computes the same +0).  E is linear along a particle's ancestry (a child has E * z or E * (1 - z), z independent
// of E), so each particle carries the tangent tE of its E w.r.t. its root's E0 (a root 1; children tE * z and
// tE * (1 - z)) and its root's index; a deposit at bin b adds ct_dep[b] * tE (one f32 product) to its root's
// gradient.  A thread keeps the exact words of its current root in its shared-memory slots (ExactPrivS) and merges
// them into the root's global exact words (atomics) when it starts a particle of another root and at the end, so
// each root's gradient is the correctly rounded exact sum of its contributions: the same whatever thread ran which
// particle.  The same gradient as the tree adjoint, summed differently: within the float tolerance, not bitwise.
//   sh_vg_onepass  E0, depth0, keys, X0, ct_dep f32[512], consts (max_steps, Q, N), order | dep f32[512], count i32[1],
//                  g_E f32[N] (read out from the words by the host's exact combine), steps u64[1] (every
//                  particle's steps: the work count of the launch), g_E exact words
//                  u64[5N + (N + 1) / 2], seq, qctl, ctl, stats | k i32[N], trunc u8[N], ring (E, depth, key, tE,
//                  root)[Q]
struct ShowerVGChild {
  float E, depth;     // (E: the energy, its sign bit the child's index j)
  u32 ka, kb;         // the parent's step key
  float tE;
  i32 root;
};

struct ShowerVGState {
  i32 kc, k;
  float E, depth;
  Key key;
  bool alive;
  i32 kj;             // as ShowerState's
  float tE;
  i32 root;
};

struct SHVG1 {
  enum { kE0, kDepth0, kKeys, kX0, kCtDep, kConsts, kOrder, kDep, kCount, kGOut, kSteps, kGE, kSeq, kQctl, kCtl, kStats,
         kK, kTrunc, kQueue, kNBuf };
  enum { kConstM, kConstQ, kConstN };
  static constexpr int kNB = 512;
  static constexpr int kXOff = kNB * 4 + 16;                       // after the dep bins and the count word
  static constexpr int kCtOff = kXOff + ExactBins<1>::kSmemBytes;  // ct_dep staged
  static constexpr int kSmemBytes = kCtOff + kNB * 4;
  typedef ShowerVGChild Child;
  typedef ShowerVGState State;
  struct Ctx {
    const float *E0, *d0;
    const uint2* keys;
    float X0;
    i32 M, N;
    float* sh;
    i32* shc;
    const float* ct;
    float* dep;
    i32* count;
    u64* gE;
    i32* stats;
    i32* kout;
    uint8_t* trunc;
    unsigned long long* steps;
    mutable i32 n;            // particles this thread finished
    mutable u32 ns;           // steps this thread ran
    mutable i32 cur;          // the root whose words this thread's slots hold (-1: none)
    mutable ExactPrivS<1> pv;
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.E0 = static_cast<const float*>(P.p[kE0]);
    c.d0 = static_cast<const float*>(P.p[kDepth0]);
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.X0 = __ldg(static_cast<const float*>(P.p[kX0]));
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]) + kConstM);
    c.N = __ldg(static_cast<const i32*>(P.p[kConsts]) + kConstN);
    c.sh = reinterpret_cast<float*>(smem);
    c.shc = reinterpret_cast<i32*>(smem + kNB * 4);
    c.ct = reinterpret_cast<const float*>(smem + kCtOff);
    c.dep = static_cast<float*>(P.p[kDep]);
    c.count = static_cast<i32*>(P.p[kCount]);
    c.gE = static_cast<u64*>(P.p[kGE]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.steps = static_cast<unsigned long long*>(P.p[kSteps]);
    c.n = 0;
    c.ns = 0u;
    c.cur = -1;
    c.pv.bind(smem + kXOff + ExactBins<1>::kPrivOffset);
  }
  __device__ static void stage(const Params& P, unsigned char* smem) {
    const float* ct = static_cast<const float*>(P.p[kCtDep]);
    float* d = reinterpret_cast<float*>(smem + kCtOff);
    for (int b = threadIdx.x; b < kNB; b += blockDim.x) d[b] = __ldg(&ct[b]);
  }
  // this thread's words of root c.cur into the root's global words (then zeroed); a lost carry or a flagged word
  // flags the root (NaN at readout)
  __device__ static void merge(const Ctx& c) {
    if (c.cur < 0) return;
    u64* const w = c.gE + (i64)c.cur * kExactWords;
    bool lost = false;
#pragma unroll
    for (int j = 0; j < kExactWords; ++j) {
      const i64 v = c.pv.word(0, j);
      if (v) lost = exact_add_word(w, j, v) || lost;
      c.pv.at(0, j) = 0;
    }
    if (lost) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
    if (lost || (c.pv.flag & 1u)) {
      // flag words after the N roots' words: u32 per root (the exact scratch layout)
      atomicOr(reinterpret_cast<u32*>(c.gE + (i64)c.N * kExactWords) + c.cur, 1u);
    }
    c.pv.flag = 0u;
  }
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    return State{0, 0, __ldg(&c.E0[item]), __ldg(&c.d0[item]), Key{kk.x, kk.y}, true, -1, 1.0f, (i32)item};
  }
  __device__ static State start_child(Ctx&, const Child& ch) {
    return State{0, 0, fabsf(ch.E), ch.depth, Key{ch.ka, ch.kb}, true, (i32)(__float_as_uint(ch.E) >> 31), ch.tE,
                 ch.root};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ __forceinline__ static void step(const Ctx& c, State& s, Child& o0, Child& o1, int& n_out) {
    child_key(s);
    const ShowerStepOut o = shower_advance(c.X0, s);
    c.ns += 1u;
    if (o.low) {
      const i32 b = f2i(s.depth * 8.0f);
      SumPriv<kNB>::emit(c.sh, c.stats, b, s.E);
      if ((u32)b < (u32)kNB) {
        if (s.root != c.cur) {
          merge(c);
          c.cur = s.root;
        }
        if (c.pv.emit(0, c.ct[b] * s.tE)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
      }
    }
    if (o.split) {
      const Child a{child_energy(s.E * o.z, 0u), s.depth, o.kk.a, o.kk.b, s.tE * o.z, s.root};
      const Child b{child_energy(s.E * (1.0f - o.z), 1u), s.depth, o.kk.a, o.kk.b, s.tE * (1.0f - o.z), s.root};
      const bool swap = o.z > 0.5f;          // the lower-energy child (the smaller subtree) runs first
      o0 = swap ? b : a;
      o1 = swap ? a : b;
      n_out = 2;
    }
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child) {
    c.n += 1;
    const bool tr = s.kc >= c.M && s.alive;
    if (child) {
      if (tr) atomicAdd(&c.stats[kStChildrenTruncated], 1);
    } else {
      c.kout[item] = s.k;
      c.trunc[item] = tr ? 1 : 0;
    }
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    merge(c);
    if (c.ns) atomicAdd(c.steps, (unsigned long long)c.ns);
    SumPriv<kNB>::flush(reinterpret_cast<const float*>(smem), c.dep, tid, nth);
    if (c.n) atomicAdd(c.shc, c.n);
    __syncthreads();
    if (tid == 0) {
      const i32 v = *reinterpret_cast<const i32*>(smem + kNB * 4);
      if (v) atomicAdd(c.count, v);
    }
  }
  __device__ static void epilogue(const Ctx&, int, int) {}
};

// ------------------------------------------------------------------------------------ reverse mode: the tree adjoint
// The reference differentiates through spawn with a recording primal and one adjoint launch per generation
// (tallymap/_reverse_spawn.py:1-45): the record holds every child's initial state, parent, ordinal and generation;
// the adjoint of generation g replays each of its items and injects, at the spawn step, the cotangents of the
// children's initial states computed by generation g + 1's launch.
//
// Record of a child (one 32-byte sector per slot; slots from a warp-aggregated counter, never reused):
//   E, depth, key   its initial state (the leaves the ring carries)
//   prev            the slot of its parent's previous child (-1: none), so a parent's children form a chain
//                   from its newest child backwards: the order in which the parent's adjoint consumes them
//   last            its own newest child (-1: none), written when it finishes
//   gen             its generation (a root's children are generation 1)
// A root's newest child goes to the per-item result `last`.  With the chains, the adjoint reaches a parent's children
// without the reference's (parent, ordinal) sort of every generation (_reverse_spawn.py:255-283); the generation
// lists only decide launch order.  A slot past the record's capacity R is not written; the host then poisons the
// gradient (the reference's 'drop_risk', _reverse_spawn.py:30-33).
struct __align__(16) ShowerRecord {
  float E, depth;
  u32 ka, kb;
  i32 prev, last, gen, pad;
};

struct ShowerRecChild {
  float E, depth;
  u32 ka, kb;
  i32 slot, gen;
};

struct ShowerRecState {
  i32 kc, k;
  float E, depth;
  Key key;
  bool alive;
  i32 me, gen, last;   // me: own record slot (a child) or -1 (a root)
};

// the recording forward (rec_primal, _reverse_spawn.py:85-109): the forward's outputs, plus the record.
//   sh_rec   E0 f32[N], depth0 f32[N], keys u32[N,2], X0 f32, consts i32[3] (max_steps, Q, R), order |
//            dep f32[512], count i32[1], seq u32[Q], qctl u32[6*32], ctl, stats, tree u64[4] (0: children
//            recorded or not) | k i32[N], trunc u8[N], last i32[N], ring ShowerRecChild[Q], record ShowerRecord[R],
//            gen u16[R] (each record's generation, compact)
struct SHRec {
  enum { kE0, kDepth0, kKeys, kX0, kConsts, kOrder, kDep, kCount, kSeq, kQctl, kCtl, kStats, kTree, kK, kTrunc,
         kLast, kQueue, kRecord, kGen, kNBuf };
  enum { kConstM, kConstQ, kConstR };
  static constexpr int kNB = 512;
  static constexpr int kSmemBytes = kNB * 4 + 16;
  typedef ShowerRecChild Child;
  typedef ShowerRecState State;
  struct Ctx {
    const float *E0, *d0;
    const uint2* keys;
    float X0;
    i32 M;
    u64 R;
    float* sh;
    i32* shc;
    float* dep;
    i32* count;
    i32* stats;
    u64* tree;
    i32* kout;
    uint8_t* trunc;
    i32* lastout;
    ShowerRecord* rec;
    unsigned short* gen;   // each child's generation again, compact (the generation lists read these)
    mutable i32 n;     // particles this thread finished
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    const i32* consts = static_cast<const i32*>(P.p[kConsts]);
    c.E0 = static_cast<const float*>(P.p[kE0]);
    c.d0 = static_cast<const float*>(P.p[kDepth0]);
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.X0 = __ldg(static_cast<const float*>(P.p[kX0]));
    c.M = __ldg(consts + kConstM);
    c.R = (u64)(u32)__ldg(consts + kConstR);
    c.sh = reinterpret_cast<float*>(smem);
    c.shc = reinterpret_cast<i32*>(smem + kNB * 4);
    c.dep = static_cast<float*>(P.p[kDep]);
    c.count = static_cast<i32*>(P.p[kCount]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.tree = static_cast<u64*>(P.p[kTree]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.lastout = static_cast<i32*>(P.p[kLast]);
    c.rec = static_cast<ShowerRecord*>(P.p[kRecord]);
    c.gen = static_cast<unsigned short*>(P.p[kGen]);
    c.n = 0;
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    return State{0, 0, __ldg(&c.E0[item]), __ldg(&c.d0[item]), Key{kk.x, kk.y}, true, -1, 0, -1};
  }
  __device__ static State start_child(Ctx&, const Child& ch) {
    return State{0, 0, ch.E, ch.depth, Key{ch.ka, ch.kb}, true, ch.slot, ch.gen, -1};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ __forceinline__ static void step(const Ctx& c, State& s, Child& o0, Child& o1, int& n_out) {
    const ShowerStepOut o = shower_advance(c.X0, s);
    if (o.low) SumPriv<kNB>::emit(c.sh, c.stats, f2i(s.depth * 8.0f), s.E);
    // record slots for the children of this iteration's splitting lanes: one atomic per warp
    const unsigned m = __activemask();
    const unsigned ms = __ballot_sync(m, o.split);
    if (o.split) {
      const int lane = threadIdx.x & 31;
      const int leader = __ffs(ms) - 1;
      unsigned long long base = 0ull;
      if (lane == leader) base = atomicAdd(reinterpret_cast<unsigned long long*>(c.tree), 2ull * __popc(ms));
      base = __shfl_sync(ms, base, leader) + 2ull * __popc(ms & ((1u << lane) - 1u));
      const Key c0 = fold_in(o.kk, 0u), c1 = fold_in(o.kk, 1u);
      const float e0 = s.E * o.z, e1 = s.E * (1.0f - o.z);
      const i32 r0 = (u64)base < c.R ? (i32)base : -1;
      const i32 r1 = (u64)base + 1 < c.R ? (i32)(base + 1) : -1;
      const unsigned short g16 = (unsigned short)(s.gen + 1 < 65535 ? s.gen + 1 : 65535);
      if (r0 >= 0) {
        c.rec[r0] = ShowerRecord{e0, s.depth, c0.a, c0.b, s.last, -1, s.gen + 1, 0};
        c.gen[r0] = g16;
      }
      if (r1 >= 0) {
        c.rec[r1] = ShowerRecord{e1, s.depth, c1.a, c1.b, r0, -1, s.gen + 1, 0};
        c.gen[r1] = g16;
      }
      s.last = r1;
      o0 = Child{e0, s.depth, c0.a, c0.b, r0, s.gen + 1};
      o1 = Child{e1, s.depth, c1.a, c1.b, r1, s.gen + 1};
      n_out = 2;
    }
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child) {
    c.n += 1;
    const bool tr = s.kc >= c.M && s.alive;
    if (child) {
      if (tr) atomicAdd(&c.stats[kStChildrenTruncated], 1);
      if (s.me >= 0) c.rec[s.me].last = s.last;
    } else {
      c.kout[item] = s.k;
      c.trunc[item] = tr ? 1 : 0;
      c.lastout[item] = s.last;
    }
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    SumPriv<kNB>::flush(reinterpret_cast<const float*>(smem), c.dep, tid, nth);
    if (c.n) atomicAdd(c.shc, c.n);
    __syncthreads();
    if (tid == 0) {
      const i32 v = *reinterpret_cast<const i32*>(smem + kNB * 4);
      if (v) atomicAdd(c.count, v);
    }
  }
  __device__ static void epilogue(const Ctx&, int, int) {}
};

// The adjoint of one generation (or of the roots): replay_kernel over the generation's record slots (the claim order
// is the generation's list) or over the root items.  Per particle, newest step first: the children's cotangents
// (dx of the newest child first, following the chain), the deposit's cotangent ct_dep[bin] into E, then the travel
// depth' = depth + X0 * L: ct_X0 += ct_depth' * L.  The particle's initial-state cotangent goes to dx[slot] (a child)
// or to the per-item results g_E, g_depth (a root); ct_X0 is an exact tally.  Replay consistency
// (_reverse_spawn.py:22-26): a child slot must exist where the replay spawns and hold exactly the state the replay
// spawns, and the chain must end with the particle's last spawn; otherwise tree[0] counts a mismatch and the host
// poisons the gradient.
//   sh_grad  E0 f32[N], depth0 f32[N], keys u32[N,2], X0 f32, ct_dep f32[512], record ShowerRecord[R], last i32[N],
//            consts i32[5] (max_steps, C, threads, roots, R), order (the generation's slots) |
//            ctl, g_X0 f32[1], exact words, stats, tree u32[4] | g_E f32[N], g_depth f32[N], dx float2[R], replay
struct SHGrad {
  enum { kE0, kDepth0, kKeys, kX0, kCtDep, kRecord, kRootLast, kConsts, kOrder, kCtl, kGX0, kExact, kStats, kTree,
         kGE, kGDepth, kDx, kReplay, kNBuf };
  enum { kConstM, kConstC, kConstThreads, kConstRoots, kConstR };
  static constexpr int kNB = 512;
  static constexpr int kSmemBytes = ExactBins<1>::kSmemBytes + kNB * 4;
  typedef ShowerState State;
  struct Ctx {
    const float *E0, *d0;
    const uint2* keys;
    float X0;
    i32 M;
    bool roots;
    i32 R;
    const float* ct;
    const ShowerRecord* rec;
    const i32* root_last;
    float2* dx;
    float *gE, *gD;
    u64* gw;
    float* g;
    i32* stats;
    u32* tree;
    Key key;           // the current item's key, energy and newest child
    float E;
    i32 last;
    mutable ExactPrivS<1> pv;
  };
  struct Adj {
    float ctE, ctd, ctX;
    i32 cur;           // the next child to consume (newest first)
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    const i32* consts = static_cast<const i32*>(P.p[kConsts]);
    c.E0 = static_cast<const float*>(P.p[kE0]);
    c.d0 = static_cast<const float*>(P.p[kDepth0]);
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.X0 = __ldg(static_cast<const float*>(P.p[kX0]));
    c.M = __ldg(consts + kConstM);
    c.roots = __ldg(consts + kConstRoots) != 0;
    c.R = __ldg(consts + kConstR);
    c.ct = reinterpret_cast<const float*>(smem + ExactBins<1>::kSmemBytes);
    c.rec = static_cast<const ShowerRecord*>(P.p[kRecord]);
    c.root_last = static_cast<const i32*>(P.p[kRootLast]);
    c.dx = static_cast<float2*>(P.p[kDx]);
    c.gE = static_cast<float*>(P.p[kGE]);
    c.gD = static_cast<float*>(P.p[kGDepth]);
    c.gw = static_cast<u64*>(P.p[kExact]);
    c.g = static_cast<float*>(P.p[kGX0]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.tree = static_cast<u32*>(P.p[kTree]);
    c.pv.bind(smem + ExactBins<1>::kPrivOffset);
  }
  __device__ static void stage(const Params& P, unsigned char* smem) {
    const float* ct = static_cast<const float*>(P.p[kCtDep]);
    float* d = reinterpret_cast<float*>(smem + ExactBins<1>::kSmemBytes);
    for (int b = threadIdx.x; b < kNB; b += blockDim.x) d[b] = __ldg(&ct[b]);
  }
  __device__ static State start(Ctx& c, i64 item) {
    float E, d;
    if (c.roots) {
      const uint2 kk = __ldg(&c.keys[item]);
      c.key = Key{kk.x, kk.y};
      E = __ldg(&c.E0[item]);
      d = __ldg(&c.d0[item]);
      c.last = __ldg(&c.root_last[item]);
    } else {
      const ShowerRecord r = c.rec[item];
      c.key = Key{r.ka, r.kb};
      E = r.E;
      d = r.depth;
      c.last = r.last;
    }
    c.E = E;
    return State{0, 0, E, d, c.key, true, -1};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ static void adj_start(const Ctx& c, Adj& a) { a = Adj{0.0f, 0.0f, 0.0f, c.last}; }
  typedef float Stored;   // a stored state is alive with the item's E and key: only depth varies
  __device__ __forceinline__ static Stored store(const State& s) { return s.depth; }
  __device__ __forceinline__ static State restore(const Ctx& c, Stored d, i64 step) {
    return State{(i32)step, (i32)step, c.E, d, c.key, true, -1};
  }
  __device__ __forceinline__ static void fwd(const Ctx& c, State& s) { shower_advance(c.X0, s); }
  // one recorded child for the spawn being transposed: its initial-state cotangent, after checking that the record
  // holds what the replay spawns; advances the chain
  __device__ __forceinline__ static float2 child_ct(const Ctx& c, Adj& a, float E, float depth, Key k) {
    const i32 r = a.cur;
    if (r < 0 || r >= c.R) {
      atomicAdd(&c.tree[0], 1u);
      return make_float2(0.0f, 0.0f);
    }
    const ShowerRecord rc = c.rec[r];
    if (__float_as_uint(rc.E) != __float_as_uint(E) || __float_as_uint(rc.depth) != __float_as_uint(depth) ||
        rc.ka != k.a || rc.kb != k.b)
      atomicAdd(&c.tree[0], 1u);
    a.cur = rc.prev;
    return c.dx[r];
  }
  __device__ __forceinline__ static void vjp(const Ctx& c, const State& at, Adj& a) {
    State s = at;
    const ShowerStepOut o = shower_advance(c.X0, s);
    if (o.split) {
      const float f1 = 1.0f - o.z;
      const float2 d1 = child_ct(c, a, at.E * f1, s.depth, fold_in(o.kk, 1u));
      a.ctE = a.ctE + d1.x * f1;
      a.ctd = a.ctd + d1.y;
      const float2 d0 = child_ct(c, a, at.E * o.z, s.depth, fold_in(o.kk, 0u));
      a.ctE = a.ctE + d0.x * o.z;
      a.ctd = a.ctd + d0.y;
    }
    if (o.low) {
      const i32 b = f2i(s.depth * 8.0f);
      if ((u32)b < (u32)kNB) a.ctE = a.ctE + c.ct[b];
    }
    a.ctX = a.ctX + a.ctd * o.L;
  }
  __device__ static void post_vjp(const Ctx&, const State&, Adj&) {}
  __device__ static void adj_finish(const Ctx& c, const State&, const State& fin, Adj& a, i64 item) {
    if (a.cur != -1) atomicAdd(&c.tree[0], 1u);           // recorded children the replay did not spawn
    if (fin.kc >= c.M && fin.alive) atomicAdd(&c.tree[1], 1u);
    if (c.roots) {
      c.gE[item] = a.ctE;
      c.gD[item] = a.ctd;
    } else {
      c.dx[item] = make_float2(a.ctE, a.ctd);
    }
    if (c.pv.emit(0, a.ctX)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
  }
  __device__ static void adj_flush(const Ctx& c, unsigned char* smem, int tid, int) {
    ExactBins<1>::flush(c.pv, smem, c.gw, c.stats, tid);
  }
  __device__ static void epilogue(const Ctx& c, int tid, int) {
    if (tid == 0) ExactBins<1>::readout(c.gw, c.g, c.stats);
  }
};

}  // namespace tmb
