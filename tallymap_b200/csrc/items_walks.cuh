// Item programs of the two walker configurations, lowered for the runtime (tm_runtime.cuh): forward and replay
// adjoint.  Each is the jaxpr of a tallymap item after retrace(cap=max_steps) (tallymap/_rewrite.py:517-528: a
// counter kc joins the loop, which runs while kc < M && pred; truncated iff kc >= M && pred(out)), with emits as
// _emit_rule (backends/kernel/kernel.py:984-1003: an index outside [0, S) is dropped and counted in stats[4]).  The
// adjoints are vjp_prog's (tallymap/_reverse.py:1079-1180): one step VJP per state, the broadcast operand's
// cotangent summed in f32 newest step first and emitted once per item into an exact tally.
//
// Buffer layouts (Params indices; args, then results; the first results up to and including stats are zeroed by the
// launcher, the layout of backends/kernel/kernel.py:570-591):
// [per-item inputs] [broadcast inputs, output cotangents] [hoisted constants: i32 max_steps] [item order] | results:
//   q1_fwd   x0 f32[N], keys u32[N,2], theta f32, consts, order | hist f32[16], ctl u32[8], stats i32[5] | k i32[N],
//            trunc u8[N]
//   q1_grad  x0, keys, theta, ct_hist f32[16], consts, order | g_theta f32[1], exact u64[6], ctl, stats | trunc u8[N],
//            replay scratch
//   rw_fwd   x0, keys, drift f32, consts, order | hist f32[256], side f32[2], ctl, stats | k i32[N], trunc u8[N]
//   rw_grad  x0, keys, drift, ct_hist f32[256], ct_side f32[2], consts, order | g_drift f32[1], exact u64[6], ctl,
//            stats | trunc u8[N], replay scratch
// order: an optional i32[N] permutation, the order in which items are claimed (null: 0..N-1); it changes which
// thread runs an item when, never a result.  exact: the cotangent tally's 5 carry-save words, then a flag word.  An
// adjoint's consts are i32[3]: max_steps, the checkpoint count C, the threads its replay scratch holds; the scratch is
// (3C + 1) stored states per thread and is not zeroed.  A walker's stored state is x alone: both loop counters equal
// the step index.
#pragma once
#include "tm_tally.cuh"

namespace tmb {

// kc: the retrace counter (the loop's steps so far, capped by max_steps); the item's own step counter k equals it
// (both start at 0 and gain 1 per step), so one register holds both
struct WalkState {
  i32 kc, k;
  float x;
};

// ================================================================================================= Q1 quickstart
//   body: u = uniform(fold_in(key, k)); t.add("hist", int32(x * 16), theta * (1 - x)); k + 1, x * (0.5 + 0.5 u)
//   pred: x > 0.05
struct Q1Common {
  static constexpr int kNB = 16;
  __device__ __forceinline__ static bool pred(float x) { return x > 0.05f; }
};

struct Q1Fwd : Q1Common {
  enum { kX0, kKeys, kTheta, kConsts, kOrder, kHist, kCtl, kStats, kK, kTrunc, kNBuf };
  static constexpr int kSmemBytes = kNB * 4;
  struct Ctx {
    const float* x0;
    const uint2* keys;
    float theta;
    i32 M;
    float* sh;
    float* hist;
    i32* stats;
    i32* kout;
    uint8_t* trunc;
    Key key;
  };
  typedef WalkState State;
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.x0 = static_cast<const float*>(P.p[kX0]);
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.theta = __ldg(static_cast<const float*>(P.p[kTheta]));
    c.sh = reinterpret_cast<float*>(smem);
    c.hist = static_cast<float*>(P.p[kHist]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
  }
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{0, 0, __ldg(&c.x0[item])};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && pred(s.x); }
  __device__ __forceinline__ static void step(const Ctx& c, State& s) {
    const float u = uniform01(fold_in(c.key, (u32)s.kc));
    SumPriv<kNB>::emit(c.sh, c.stats, f2i(s.x * 16.0f), c.theta * (1.0f - s.x));
    s.kc += 1;
    s.x = s.x * (0.5f + 0.5f * u);
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item) {
    c.kout[item] = s.kc;
    c.trunc[item] = (s.kc >= c.M && pred(s.x)) ? 1 : 0;
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    SumPriv<kNB>::flush(reinterpret_cast<const float*>(smem), c.hist, tid, nth);
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static void epilogue(const Ctx&, int, int) {}
};

// grad of <ct_hist, hist> w.r.t. theta: the step VJP adds ct_hist[bin] * (1 - x) (0 for a dropped emit,
// _tally.py:72-82); x does not depend on theta, so it is not an active carry.
struct Q1Grad : Q1Common {
  enum { kX0, kKeys, kTheta, kCt, kConsts, kOrder, kG, kExact, kCtl, kStats, kTrunc, kReplay, kNBuf };
  enum { kConstM, kConstC, kConstThreads };
  static constexpr int kSmemBytes = ExactBins<1>::kSmemBytes + kNB * 4;
  struct Ctx {
    const float* x0;
    const uint2* keys;
    i32 M;
    const float* ct;     // staged in shared memory
    u64* gw;
    float* g;
    i32* stats;
    uint8_t* trunc;
    Key key;
    mutable ExactPrivS<1> pv;
  };
  typedef WalkState State;
  struct Adj {
    float ctb;
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.x0 = static_cast<const float*>(P.p[kX0]);
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.gw = static_cast<u64*>(P.p[kExact]);
    c.g = static_cast<float*>(P.p[kG]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.ct = reinterpret_cast<const float*>(smem + ExactBins<1>::kSmemBytes);
    c.pv.bind(smem + ExactBins<1>::kPrivOffset);
  }
  __device__ static void stage(const Params& P, unsigned char* smem) {
    const float* ct = static_cast<const float*>(P.p[kCt]);
    float* d = reinterpret_cast<float*>(smem + ExactBins<1>::kSmemBytes);
    for (int b = threadIdx.x; b < kNB; b += blockDim.x) d[b] = __ldg(&ct[b]);
  }
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{0, 0, __ldg(&c.x0[item])};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && pred(s.x); }
  __device__ static void adj_start(const Ctx&, Adj& a) { a.ctb = 0.0f; }
  typedef float Stored;
  __device__ __forceinline__ static Stored store(const State& s) { return s.x; }
  __device__ __forceinline__ static State restore(const Ctx&, Stored x, i64 step) {
    return State{(i32)step, (i32)step, x};
  }
  __device__ __forceinline__ static void fwd(const Ctx& c, State& s) {
    const float u = uniform01(fold_in(c.key, (u32)s.kc));
    s.kc += 1;
    s.x = s.x * (0.5f + 0.5f * u);
  }
  __device__ __forceinline__ static void vjp(const Ctx& c, const State& at, Adj& a) {
    const i32 b = f2i(at.x * 16.0f);
    const float cv = ((u32)b < (u32)kNB) ? c.ct[b] : 0.0f;
    a.ctb = a.ctb + cv * (1.0f - at.x);
  }
  __device__ static void post_vjp(const Ctx&, const State&, Adj&) {}
  __device__ static void adj_finish(const Ctx& c, const State&, const State& fin, Adj& a, i64 item) {
    c.trunc[item] = (fin.kc >= c.M && pred(fin.x)) ? 1 : 0;
    if (c.pv.emit(0, a.ctb)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
  }
  __device__ static void adj_flush(const Ctx& c, unsigned char* smem, int tid, int) {
    ExactBins<1>::flush(c.pv, smem, c.gw, c.stats, tid);
  }
  __device__ static void epilogue(const Ctx& c, int tid, int) {
    if (tid == 0) ExactBins<1>::readout(c.gw, c.g, c.stats);
  }
};

// ================================================================================================= RW 1-D walk
//   body: u = uniform(fold_in(key, k)); t.add("hist", int32(x * 256), drift * x); k + 1, x + 0.02 * (2u - 1)
//   pred: 0 <= x <= 1;  after the loop: t.add("side", int32(x > 1), 1.0)
struct RWCommon {
  static constexpr int kNB = 256;
  __device__ __forceinline__ static bool pred(float x) { return x >= 0.0f && x <= 1.0f; }
  __device__ __forceinline__ static float move(float x, float u) { return x + 0.02f * (2.0f * u - 1.0f); }
};

// BLK: the block's threads.  Each 128 threads of a block add into their own privatised histogram (kSub of them),
// so a bin's f32 partial sum takes as many additions before the flush whatever the block size (its rounding error
// stays that of a 128-thread block's).
template <int BLK>
struct RWFwdT : RWCommon {
  enum { kX0, kKeys, kDrift, kConsts, kOrder, kHist, kSide, kCtl, kStats, kK, kTrunc, kNBuf };
  static constexpr int kSub = BLK / 128 > 1 ? BLK / 128 : 1;
  static constexpr int kSmemBytes = kSub * (kNB + 2) * 4;
  struct Ctx {
    const float* x0;
    const uint2* keys;
    float drift;
    i32 M;
    float* sh;
    float* hist;
    float* side;
    i32* stats;
    i32* kout;
    uint8_t* trunc;
    Key key;
  };
  typedef WalkState State;
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.x0 = static_cast<const float*>(P.p[kX0]);
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.drift = __ldg(static_cast<const float*>(P.p[kDrift]));
    c.sh = reinterpret_cast<float*>(smem) + (threadIdx.x / 128) * (kNB + 2);
    c.hist = static_cast<float*>(P.p[kHist]);
    c.side = static_cast<float*>(P.p[kSide]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
  }
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{0, 0, __ldg(&c.x0[item])};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && pred(s.x); }
  // the step's uniform depends on the key and the step index only: draw(j) is step kc + j's, drawn ahead
  // (tm_runtime.cuh, run_step), apply the step given its uniform; step = apply(draw(0))
  static constexpr int kUnroll = 4;
  typedef float Draw;
  __device__ __forceinline__ static Draw draw(const Ctx& c, const State& s, int j) {
    return uniform01(fold_in(c.key, (u32)(s.kc + j)));
  }
  __device__ __forceinline__ static void apply(const Ctx& c, State& s, Draw u) {
    SumPriv<kNB>::emit(c.sh, c.stats, f2i(s.x * 256.0f), c.drift * s.x);
    s.kc += 1;
    s.x = move(s.x, u);
  }
  __device__ __forceinline__ static void step(const Ctx& c, State& s) { apply(c, s, draw(c, s, 0)); }
  // an item in flight, movable to another thread of the block: its position, step count, key and index
  struct Parked {
    float x;
    i32 kc;
    u32 ka, kb;
    i32 item;     // (an item index is below 2^31, the reference's limit on N)
  };
  __device__ __forceinline__ static Parked park(const Ctx& c, const State& s, i64 item) {
    return Parked{s.x, s.kc, c.key.a, c.key.b, (i32)item};
  }
  __device__ __forceinline__ static State unpark(Ctx& c, const Parked& p, i64& item) {
    c.key = Key{p.ka, p.kb};
    item = p.item;
    return State{p.kc, p.kc, p.x};
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item) {
    SumPriv<2>::emit(c.sh + kNB, c.stats, s.x > 1.0f ? 1 : 0, 1.0f);
    c.kout[item] = s.kc;
    c.trunc[item] = (s.kc >= c.M && pred(s.x)) ? 1 : 0;
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    for (int q = 0; q < kSub; ++q) {
      const float* sh = reinterpret_cast<const float*>(smem) + q * (kNB + 2);
      SumPriv<kNB>::flush(sh, c.hist, tid, nth);
      SumPriv<2>::flush(sh + kNB, c.side, tid, nth);
    }
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static void epilogue(const Ctx&, int, int) {}
};
typedef RWFwdT<TM_BLOCK> RWFwd;

// grad of <ct_hist, hist> + <ct_side, side> w.r.t. drift: the step VJP adds ct_hist[bin] * x; the side tally does
// not depend on drift.  BLK: the block's threads (the layout of the threads' private exact words).
template <int BLK>
struct RWGradT : RWCommon {
  enum { kX0, kKeys, kDrift, kCtHist, kCtSide, kConsts, kOrder, kG, kExact, kCtl, kStats, kTrunc, kReplay, kNBuf };
  enum { kConstM, kConstC, kConstThreads };
  static constexpr int kBlock = BLK, kMinBlocks = BLK > 256 ? 2048 / BLK : 0;
  typedef ExactBins<1, BLK> Bins;
  static constexpr int kSmemBytes = Bins::kSmemBytes + kNB * 4;
    struct Ctx {
    const float* x0;
    const uint2* keys;
    i32 M;
    const float* ct;
    u64* gw;
    float* g;
    i32* stats;
    uint8_t* trunc;
    Key key;
    mutable ExactPrivS<1, BLK> pv;
  };
  typedef WalkState State;
  struct Adj {
    float ctb;
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.x0 = static_cast<const float*>(P.p[kX0]);
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.gw = static_cast<u64*>(P.p[kExact]);
    c.g = static_cast<float*>(P.p[kG]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.ct = reinterpret_cast<const float*>(smem + Bins::kSmemBytes);
    c.pv.bind(smem + Bins::kPrivOffset);
  }
  __device__ static void stage(const Params& P, unsigned char* smem) {
    const float* ct = static_cast<const float*>(P.p[kCtHist]);
    float* d = reinterpret_cast<float*>(smem + Bins::kSmemBytes);
    for (int b = threadIdx.x; b < kNB; b += blockDim.x) d[b] = __ldg(&ct[b]);
  }
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{0, 0, __ldg(&c.x0[item])};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && pred(s.x); }
  __device__ static void adj_start(const Ctx&, Adj& a) { a.ctb = 0.0f; }
  typedef float Stored;
  __device__ __forceinline__ static Stored store(const State& s) { return s.x; }
  __device__ __forceinline__ static State restore(const Ctx&, Stored x, i64 step) {
    return State{(i32)step, (i32)step, x};
  }
  __device__ __forceinline__ static void fwd(const Ctx& c, State& s) {
    const float u = uniform01(fold_in(c.key, (u32)s.kc));
    s.kc += 1;
    s.x = move(s.x, u);
  }
  __device__ __forceinline__ static void vjp(const Ctx& c, const State& at, Adj& a) {
    const i32 b = f2i(at.x * 256.0f);
    const float cv = ((u32)b < (u32)kNB) ? c.ct[b] : 0.0f;
    a.ctb = a.ctb + cv * at.x;
  }
  __device__ static void post_vjp(const Ctx&, const State&, Adj&) {}
  __device__ static void adj_finish(const Ctx& c, const State&, const State& fin, Adj& a, i64 item) {
    c.trunc[item] = (fin.kc >= c.M && pred(fin.x)) ? 1 : 0;
    if (c.pv.emit(0, a.ctb)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
  }
  __device__ static void adj_flush(const Ctx& c, unsigned char* smem, int tid, int) {
    Bins::flush(c.pv, smem, c.gw, c.stats, tid);
  }
  __device__ static void epilogue(const Ctx& c, int tid, int) {
    if (tid == 0) Bins::readout(c.gw, c.g, c.stats);
  }
};
typedef RWGradT<TM_BLOCK> RWGrad;

// ================================================================================================= value and grad
// The fused programs (FusedVG, tm_runtime.cuh): the forward's outputs and the gradient of <ct, outputs> in one launch.
//   q1_vg    x0, keys, theta, ct_hist, consts, order | hist f32[16], g_theta f32[1], exact u64[6], ctl, stats |
//            k i32[N], trunc u8[N], replay scratch
//   rw_vg    x0, keys, drift, ct_hist, ct_side, consts, order | hist f32[256], side f32[2], g_drift f32[1],
//            exact u64[6], ctl, stats | k i32[N], trunc u8[N], replay scratch
struct Q1VGMap {
  enum { kNF = Q1Fwd::kNBuf, kNG = Q1Grad::kNBuf, kNBuf = 14 };
  __host__ __device__ static constexpr int f(int i) {
    constexpr int m[kNF] = {0, 1, 2, 4, 5, 6, 9, 10, 11, 12};
    return m[i];
  }
  __host__ __device__ static constexpr int g(int i) {
    constexpr int m[kNG] = {0, 1, 2, 3, 4, 5, 7, 8, 9, 10, 12, 13};
    return m[i];
  }
};
typedef FusedVG<Q1Fwd, Q1Grad, Q1VGMap> Q1VG;

struct RWVGMap {
  enum { kNF = RWFwd::kNBuf, kNG = RWGrad::kNBuf, kNBuf = 16 };
  __host__ __device__ static constexpr int f(int i) {
    constexpr int m[kNF] = {0, 1, 2, 5, 6, 7, 8, 11, 12, 13, 14};
    return m[i];
  }
  __host__ __device__ static constexpr int g(int i) {
    constexpr int m[kNG] = {0, 1, 2, 3, 4, 5, 6, 9, 10, 11, 12, 14, 15};
    return m[i];
  }
};
typedef FusedVG<RWFwd, RWGrad, RWVGMap> RWVG;

// The one-pass value-and-grad programs (OnePassVG, tm_runtime.cuh): the walkers have no active carry, so each step's
// VJP is summed as the forward runs.  The fused layouts above without the replay scratch; consts = max_steps only.
//   q1_vg_onepass   x0, keys, theta, ct_hist, consts, order | hist, g_theta, exact, ctl, stats | k, trunc
//   rw_vg_onepass   x0, keys, drift, ct_hist, ct_side, consts, order | hist, side, g_drift, exact, ctl, stats | k,
//                   trunc
struct Q1VG1Map {
  enum { kNF = Q1Fwd::kNBuf, kNG = Q1Grad::kNBuf, kNBuf = 13 };
  __host__ __device__ static constexpr int f(int i) { return Q1VGMap::f(i); }
  __host__ __device__ static constexpr int g(int i) { return i == Q1Grad::kReplay ? 0 : Q1VGMap::g(i); }
};
typedef OnePassVG<Q1Fwd, Q1Grad, Q1VG1Map> Q1VG1;

struct RWVG1Map {
  enum { kNF = RWFwd::kNBuf, kNG = RWGrad::kNBuf, kNBuf = 15 };
  __host__ __device__ static constexpr int f(int i) { return RWVGMap::f(i); }
  __host__ __device__ static constexpr int g(int i) { return i == RWGrad::kReplay ? 0 : RWVGMap::g(i); }
};
// (1024-thread blocks, two per SM: the end-of-launch compaction gathers the items in flight of 32 warps)
typedef OnePassVG<RWFwdT<1024>, RWGradT<1024>, RWVG1Map> RWVG1;

}  // namespace tmb
