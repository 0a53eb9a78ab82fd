// Item program of the branching-shower configuration, lowered for the spawn runtime
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
//            dep f32[512], count i32[1], seq u32[Q], qctl u32[5*32], ctl, stats | k i32[N], trunc u8[N],
//            ring (E, depth, key)[Q]
#pragma once
#include "tm_math.h"
#include "tm_spawn.cuh"
#include "tm_tally.cuh"

namespace tmb {

struct ShowerChild {
  float E, depth;
  u32 ka, kb;
};

struct ShowerState {
  i32 kc, k;
  float E, depth;
  Key key;
  bool alive;
};

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
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    return State{0, 0, __ldg(&c.E0[item]), __ldg(&c.d0[item]), Key{kk.x, kk.y}, true};
  }
  __device__ static State start_child(Ctx&, const Child& ch) {
    return State{0, 0, ch.E, ch.depth, Key{ch.ka, ch.kb}, true};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ __forceinline__ static void step(const Ctx& c, State& s, Child* out, int* n_out) {
    const Key kk = fold_in(s.key, (u32)s.k);
    const float u0 = uniform01(kk, 0u), u1 = uniform01(kk, 1u), u2 = uniform01(kk, 2u);
    s.depth = s.depth + c.X0 * (-tmm::logf(1.0f - u0));
    const bool low = s.E < 0.5f;
    SumPriv<kNB>::emit(c.sh, c.stats, low ? f2i(s.depth * 8.0f) : 0, low ? s.E : 0.0f);
    const bool split = !low && u1 < 0.7f;
    if (split) {
      const float z = 0.1f + 0.8f * u2;
      const Key c0 = fold_in(kk, 0u), c1 = fold_in(kk, 1u);
      out[0] = Child{s.E * z, s.depth, c0.a, c0.b};
      out[1] = Child{s.E * (1.0f - z), s.depth, c1.a, c1.b};
      *n_out = 2;
    }
    s.alive = !low && !split;
    s.kc += 1;
    s.k += 1;
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item, bool child) {
    atomicAdd(c.shc, 1);                                   // count: Sum((1,)) int32, privatised
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
    if (tid == 0) {
      const i32 v = *reinterpret_cast<const i32*>(smem + kNB * 4);
      if (v) atomicAdd(c.count, v);
    }
  }
  __device__ static void epilogue(const Ctx&, int, int) {}
};

}  // namespace tmb
