// Item program of the photon-slab configuration (benchmark configuration 3), lowered for the runtime: forward and replay
// adjoint w.r.t. (mu_a, mu_s).  The item, as a tallymap user writes it (g, the box and the roulette constants are
// Python floats, so 1 - g*g etc. are formed in double and rounded once to f32):
//
//   def photon(t, key, mu_a, mu_s):                       # per item: key; broadcast: mu_a, mu_s
//     mu_t = mu_a + mu_s; albedo = mu_s / mu_t; frac = mu_a / mu_t
//     def body(c):
//       k, p, d, w, alive, t = c
//       u = uniform(fold_in(key, k), (4,))                # path, HG cos(theta), phi, roulette
//       s = -log(1 - u[0]) / mu_t                         # (1 - u: a step of 0 for u = 0, never infinite)
//       p = p + s * d
//       inside = all(0 <= p) & all(p < 64)
//       i = clip(p.astype(int32), 0, 63)
//       t = t.add("dep", (i[0], i[1], i[2]), where(inside, w * frac, 0.0))
//       w = w * albedo
//       tmp = (1 - g*g) / (1 - g + 2*g*u[1]);  cos_t = clip((1 + g*g - tmp**2) / (2*g), -1, 1)
//       sin_t = sqrt(1 - cos_t**2);  phi = 2*pi*u[2]
//       d = rotate(d, cos_t, sin_t, cos(phi), sin(phi))   # the standard scattering frame, |d_z| > 0.99999 special
//       low = w < 1e-3;  survive = u[3] < 0.1
//       w = where(low, where(survive, w * 10, 0.0), w)
//       return k + 1, p, d, w, inside & ~(low & ~survive), t
//     k, p, d, w, alive, t = while_loop(lambda c: c[4], body, (0, (32, 32, 0), (0, 0, 1), 1.0, True, t))
//     return t, k
//
// with max_steps = 100,000 (retrace(cap): a counter kc, truncated iff kc >= M && alive).  The transcendentals are
// tm_math.h's (bitwise equal on host and device).
//
// Reverse mode (vjp_prog, tallymap/_reverse.py:1079-1180) of <ct_dep, dep> w.r.t. mu_a and mu_s.  The only ACTIVE
// carry is w (positions depend on mu_t but reach the outputs only through integer voxel indices and comparisons, so
// their cotangents are identically zero; their terms add +-0, which no f32 sum and no exact tally can see).  Per step,
// newest first, from ct_w2 (the cotangent of w after the step):
//   ct_w1 = low ? (survive ? ct_w2 * 10 : 0) : ct_w2
//   ct_albedo += ct_w1 * w;       ct_w = ct_w1 * albedo
//   cv = inside ? ct_dep[i] : 0;  ct_frac += cv * w;   ct_w = ct_w + cv * frac
// and, once per item, the pre-loop code's VJP (div's transpose: numerator ct / y, denominator (-ct * x) * (1 / y^2)):
//   r = 1 / (mu_t * mu_t);  ct_mu_t = ((-ct_frac) * mu_a) * r + ((-ct_albedo) * mu_s) * r
//   ct_mu_a = ct_frac / mu_t + ct_mu_t;   ct_mu_s = ct_albedo / mu_t + ct_mu_t
// emitted into a 2-bin exact tally.
//
// Buffers:
//   ph_fwd   keys u32[N,2], mu_a f32, mu_s f32, consts i32[1], order | dep f32[64^3], ctl, stats | k i32[N],
//            trunc u8[N]   (the deposits go into dep with warp-aggregated f32 atomics, each group's sum formed in
//            f64 and rounded once; the 16^3 voxels around the source first per block into a shared f32 window)
//   ph_grad  keys, mu_a, mu_s, ct_dep f32[64^3], consts i32[3], order | g f32[2], exact u64[11], ctl, stats |
//            trunc u8[N], replay scratch (stored state: p, d, w; the counters are the step index, alive is true)
#pragma once
#include "tm_math.h"
#include "tm_tally.cuh"

namespace tmb {

struct PhotonState {
  i32 kc, k;
  float px, py, pz, dx, dy, dz, w;
  bool alive;
};

struct PhotonCommon {
  static constexpr int kBox = 64;
  static constexpr int kS = kBox * kBox * kBox;
  // one step's draws, position update, deposit decision and scattering; the adjoint re-runs the parts it needs
  struct Draws {
    float u0, u1, u2, u3;
  };
  __device__ __forceinline__ static Draws draws(Key key, i32 k) {
    const Key nk = fold_in(key, (u32)k);
    return Draws{uniform01(nk, 0u), uniform01(nk, 1u), uniform01(nk, 2u), uniform01(nk, 3u)};
  }
  __device__ __forceinline__ static float path(float u0, float mu_t) { return (-tmm::logf(1.0f - u0)) / mu_t; }
  __device__ __forceinline__ static bool in_box(float x) { return x >= 0.0f && x < 64.0f; }
  __device__ __forceinline__ static i32 voxel(float x) { return min(max(f2i(x), 0), kBox - 1); }
  __device__ __forceinline__ static void scatter(PhotonState& s, float u1, float u2) {
    const float tmp = 0.19f / (0.1f + 1.8f * u1);
    float cos_t = (1.81f - tmp * tmp) / 1.8f;
    cos_t = fminf(fmaxf(cos_t, -1.0f), 1.0f);
    const float sin_t = sqrtf(1.0f - cos_t * cos_t);
    float sp, cp;
    tmm::sincosf(6.2831855f * u2, &sp, &cp);
    const float dx = s.dx, dy = s.dy, dz = s.dz;
    if (fabsf(dz) > 0.99999f) {
      s.dx = sin_t * cp;
      s.dy = sin_t * sp;
      s.dz = cos_t * (dz > 0.0f ? 1.0f : -1.0f);
    } else {
      const float t = sqrtf(1.0f - dz * dz);
      s.dx = (sin_t * ((dx * dz) * cp - dy * sp)) / t + dx * cos_t;
      s.dy = (sin_t * ((dy * dz) * cp + dx * sp)) / t + dy * cos_t;
      s.dz = ((-sin_t) * cp) * t + dz * cos_t;
    }
  }
};

struct PHFwd : PhotonCommon {
  enum { kKeys, kMuA, kMuS, kConsts, kOrder, kDep, kCtl, kStats, kK, kTrunc, kNBuf };
  // the shared-memory window of hot voxels: x, y in [32 - kW/2, 32 + kW/2), z in [0, kW) (the source is (32, 32, 0))
  static constexpr int kW = 16, kW0 = 32 - kW / 2;
  static constexpr int kSmemBytes = kW * kW * kW * 4;
  struct Ctx {
    const uint2* keys;
    float mu_t, albedo, frac;
    i32 M;
    float* dep;
    i32* stats;
    i32* kout;
    uint8_t* trunc;
    Key key;
    float* win;
  };
  typedef PhotonState State;
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.win = reinterpret_cast<float*>(smem);
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    const float mu_a = __ldg(static_cast<const float*>(P.p[kMuA]));
    const float mu_s = __ldg(static_cast<const float*>(P.p[kMuS]));
    c.mu_t = mu_a + mu_s;
    c.albedo = mu_s / c.mu_t;
    c.frac = mu_a / c.mu_t;
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.dep = static_cast<float*>(P.p[kDep]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{0, 0, 32.0f, 32.0f, 0.0f, 0.0f, 0.0f, 1.0f, 1.0f, true};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ __forceinline__ static void step(const Ctx& c, State& s) {
    const Draws u = draws(c.key, s.k);
    const float sl = path(u.u0, c.mu_t);
    s.px = s.px + sl * s.dx;
    s.py = s.py + sl * s.dy;
    s.pz = s.pz + sl * s.dz;
    const bool inside = in_box(s.px) && in_box(s.py) && in_box(s.pz);
    const i32 ix = voxel(s.px), iy = voxel(s.py), iz = voxel(s.pz);
    const i32 flat = (ix * kBox + iy) * kBox + iz;
    const bool in_win = (u32)(ix - kW0) < (u32)kW && (u32)(iy - kW0) < (u32)kW && iz < kW;
    const i32 widx = in_win ? ((ix - kW0) * kW + (iy - kW0)) * kW + iz : -1;
    fatom_warp_window(c.dep, c.win, flat, widx, inside ? s.w * c.frac : 0.0f);
    const float w1 = s.w * c.albedo;
    scatter(s, u.u1, u.u2);
    const bool low = w1 < 0.001f, survive = u.u3 < 0.1f;
    s.w = low ? (survive ? w1 * 10.0f : 0.0f) : w1;
    s.alive = inside && !(low && !survive);
    s.kc += 1;
    s.k += 1;
  }
  __device__ static void finish(const Ctx& c, const State& s, i64 item) {
    c.kout[item] = s.k;
    c.trunc[item] = (s.kc >= c.M && s.alive) ? 1 : 0;
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    const float* win = reinterpret_cast<const float*>(smem);
    for (int b = tid; b < kW * kW * kW; b += nth) {
      const float v = win[b];
      if (v == 0.0f) continue;
      const int ix = kW0 + b / (kW * kW), iy = kW0 + (b / kW) % kW, iz = b % kW;
      fatom(&c.dep[(ix * kBox + iy) * kBox + iz], v);
    }
  }
  __device__ static void epilogue(const Ctx&, int, int) {}
};

struct PHGrad : PhotonCommon {
  static constexpr int kMinBlocks = 5;   // (96 registers without the spill ptxas picks unbounded)
  enum { kKeys, kMuA, kMuS, kCtDep, kConsts, kOrder, kG, kExact, kCtl, kStats, kTrunc, kReplay, kNBuf };
  enum { kConstM, kConstC, kConstThreads };
  static constexpr int kSmemBytes = ExactBins<2>::kSmemBytes;
  struct Ctx {
    const uint2* keys;
    float mu_a, mu_s, mu_t, albedo, frac;
    i32 M;
    const float* ct;
    u64* gw;
    float* g;
    i32* stats;
    uint8_t* trunc;
    Key key;
    mutable ExactPrivS<2> pv;
  };
  typedef PhotonState State;
  struct Adj {
    float ct_w, ct_frac, ct_albedo;
  };
  // (padded to 32 bytes and 16-byte aligned: a state moves as two 128-bit accesses)
  struct __align__(16) Stored {
    float px, py, pz, dx, dy, dz, w, pad;
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.mu_a = __ldg(static_cast<const float*>(P.p[kMuA]));
    c.mu_s = __ldg(static_cast<const float*>(P.p[kMuS]));
    c.mu_t = c.mu_a + c.mu_s;
    c.albedo = c.mu_s / c.mu_t;
    c.frac = c.mu_a / c.mu_t;
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.ct = static_cast<const float*>(P.p[kCtDep]);
    c.gw = static_cast<u64*>(P.p[kExact]);
    c.g = static_cast<float*>(P.p[kG]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.pv.bind(smem + ExactBins<2>::kPrivOffset);
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{0, 0, 32.0f, 32.0f, 0.0f, 0.0f, 0.0f, 1.0f, 1.0f, true};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& s) { return s.kc < c.M && s.alive; }
  __device__ __forceinline__ static Stored store(const State& s) {
    return Stored{s.px, s.py, s.pz, s.dx, s.dy, s.dz, s.w};
  }
  __device__ __forceinline__ static State restore(const Ctx&, const Stored& v, i64 step) {
    return State{(i32)step, (i32)step, v.px, v.py, v.pz, v.dx, v.dy, v.dz, v.w, true};
  }
  __device__ static void adj_start(const Ctx&, Adj& a) { a.ct_w = a.ct_frac = a.ct_albedo = 0.0f; }
  __device__ __forceinline__ static void fwd(const Ctx& c, State& s) {
    const Draws u = draws(c.key, s.k);
    const float sl = path(u.u0, c.mu_t);
    s.px = s.px + sl * s.dx;
    s.py = s.py + sl * s.dy;
    s.pz = s.pz + sl * s.dz;
    const bool inside = in_box(s.px) && in_box(s.py) && in_box(s.pz);
    const float w1 = s.w * c.albedo;
    scatter(s, u.u1, u.u2);
    const bool low = w1 < 0.001f, survive = u.u3 < 0.1f;
    s.w = low ? (survive ? w1 * 10.0f : 0.0f) : w1;
    s.alive = inside && !(low && !survive);
    s.kc += 1;
    s.k += 1;
  }
  __device__ __forceinline__ static void vjp(const Ctx& c, const State& at, Adj& a) {
    const Key nk = fold_in(c.key, (u32)at.k);
    const float u0 = uniform01(nk, 0u), u3 = uniform01(nk, 3u);
    const float sl = path(u0, c.mu_t);
    const float px = at.px + sl * at.dx, py = at.py + sl * at.dy, pz = at.pz + sl * at.dz;
    const bool inside = in_box(px) && in_box(py) && in_box(pz);
    const float w = at.w, w1 = w * c.albedo;
    const bool low = w1 < 0.001f, survive = u3 < 0.1f;
    const float ct_w1 = low ? (survive ? a.ct_w * 10.0f : 0.0f) : a.ct_w;
    a.ct_albedo = a.ct_albedo + ct_w1 * w;
    float ct_w = ct_w1 * c.albedo;
    const i32 flat = (voxel(px) * kBox + voxel(py)) * kBox + voxel(pz);
    const float cv = inside ? __ldg(&c.ct[flat]) : 0.0f;
    a.ct_frac = a.ct_frac + cv * w;
    a.ct_w = ct_w + cv * c.frac;
  }
  __device__ static void post_vjp(const Ctx&, const State&, Adj& a) { a.ct_w = 0.0f; }
  __device__ static void adj_finish(const Ctx& c, const State&, const State& fin, Adj& a, i64 item) {
    c.trunc[item] = (fin.kc >= c.M && fin.alive) ? 1 : 0;
    const float r = 1.0f / (c.mu_t * c.mu_t);
    const float ct_mu_t = ((-a.ct_frac) * c.mu_a) * r + ((-a.ct_albedo) * c.mu_s) * r;
    const float g_a = a.ct_frac / c.mu_t + ct_mu_t;
    const float g_s = a.ct_albedo / c.mu_t + ct_mu_t;
    if (c.pv.emit(0, g_a)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
    if (c.pv.emit(1, g_s)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
  }
  __device__ static void adj_flush(const Ctx& c, unsigned char* smem, int tid, int) {
    ExactBins<2>::flush(c.pv, smem, c.gw, c.stats, tid);
  }
  __device__ static void epilogue(const Ctx& c, int tid, int) {
    if (tid == 0) ExactBins<2>::readout(c.gw, c.g, c.stats);
  }
};

// ================================================================================================= one pass
// Value and gradient in one forward pass, by forward mode: the only active carry is w, and its tangent with respect
// to albedo travels with the state (tw: w1 = w * albedo gives tw1 = tw * albedo + w; the roulette scales both by the
// same 10 or 0).  Each deposit w * frac adds cv * w to the cotangent of frac and (cv * frac) * tw to that of albedo
// (cv = ct_dep at the voxel, 0 outside); at the item's end the pre-loop code's VJP maps (frac, albedo) to (mu_a,
// mu_s) as in PHGrad::adj_finish.  The same gradient as the replay adjoint, summed in another order (forward, not
// newest first): within the float tolerance, not bitwise.  No replay scratch: the forward's cost plus a load of
// ct_dep and four multiply-adds per step.
//   ph_vg_onepass  keys, mu_a, mu_s, ct_dep f32[64^3], consts i32[1], order | dep f32[64^3], g f32[2],
//                  exact u64[11], ctl, stats | k i32[N], trunc u8[N]
struct PHVG1 : PhotonCommon {
  enum { kKeys, kMuA, kMuS, kCtDep, kConsts, kOrder, kDep, kG, kExact, kCtl, kStats, kK, kTrunc, kNBuf };
  static constexpr int kW = PHFwd::kW, kW0 = PHFwd::kW0;
  static constexpr int kXBytes = (ExactBins<2>::kSmemBytes + 15) / 16 * 16;
  static constexpr int kSmemBytes = kXBytes + PHFwd::kSmemBytes;
  struct Ctx {
    const uint2* keys;
    float mu_a, mu_s, mu_t, albedo, frac;
    i32 M;
    const float* ct;
    float* dep;
    u64* gw;
    float* g;
    i32* stats;
    i32* kout;
    uint8_t* trunc;
    Key key;
    float* win;
    mutable ExactPrivS<2> pv;
  };
  struct State {
    PhotonState s;
    float tw, cf, ca;     // d w / d albedo; the item's cotangents of frac and albedo so far
  };
  __device__ static void setup(Ctx& c, const Params& P, unsigned char* smem) {
    c.win = reinterpret_cast<float*>(smem + kXBytes);
    c.keys = static_cast<const uint2*>(P.p[kKeys]);
    c.mu_a = __ldg(static_cast<const float*>(P.p[kMuA]));
    c.mu_s = __ldg(static_cast<const float*>(P.p[kMuS]));
    c.mu_t = c.mu_a + c.mu_s;
    c.albedo = c.mu_s / c.mu_t;
    c.frac = c.mu_a / c.mu_t;
    c.M = __ldg(static_cast<const i32*>(P.p[kConsts]));
    c.ct = static_cast<const float*>(P.p[kCtDep]);
    c.dep = static_cast<float*>(P.p[kDep]);
    c.gw = static_cast<u64*>(P.p[kExact]);
    c.g = static_cast<float*>(P.p[kG]);
    c.stats = static_cast<i32*>(P.p[kStats]);
    c.kout = static_cast<i32*>(P.p[kK]);
    c.trunc = static_cast<uint8_t*>(P.p[kTrunc]);
    c.pv.bind(smem + ExactBins<2>::kPrivOffset);
  }
  __device__ static void stage(const Params&, unsigned char*) {}
  __device__ static State start(Ctx& c, i64 item) {
    const uint2 kk = __ldg(&c.keys[item]);
    c.key = Key{kk.x, kk.y};
    return State{PhotonState{0, 0, 32.0f, 32.0f, 0.0f, 0.0f, 0.0f, 1.0f, 1.0f, true}, 0.0f, 0.0f, 0.0f};
  }
  __device__ __forceinline__ static bool cond(const Ctx& c, const State& st) { return st.s.kc < c.M && st.s.alive; }
  __device__ __forceinline__ static void step(const Ctx& c, State& st) {
    PhotonState& s = st.s;
    const Draws u = draws(c.key, s.k);
    const float sl = path(u.u0, c.mu_t);
    s.px = s.px + sl * s.dx;
    s.py = s.py + sl * s.dy;
    s.pz = s.pz + sl * s.dz;
    const bool inside = in_box(s.px) && in_box(s.py) && in_box(s.pz);
    const i32 ix = voxel(s.px), iy = voxel(s.py), iz = voxel(s.pz);
    const i32 flat = (ix * kBox + iy) * kBox + iz;
    const bool in_win = (u32)(ix - kW0) < (u32)kW && (u32)(iy - kW0) < (u32)kW && iz < kW;
    const i32 widx = in_win ? ((ix - kW0) * kW + (iy - kW0)) * kW + iz : -1;
    fatom_warp_window(c.dep, c.win, flat, widx, inside ? s.w * c.frac : 0.0f);
    const float cv = inside ? __ldg(&c.ct[flat]) : 0.0f;
    st.cf = st.cf + cv * s.w;
    st.ca = st.ca + (cv * c.frac) * st.tw;
    const float w1 = s.w * c.albedo, tw1 = st.tw * c.albedo + s.w;
    scatter(s, u.u1, u.u2);
    const bool low = w1 < 0.001f, survive = u.u3 < 0.1f;
    s.w = low ? (survive ? w1 * 10.0f : 0.0f) : w1;
    st.tw = low ? (survive ? tw1 * 10.0f : 0.0f) : tw1;
    s.alive = inside && !(low && !survive);
    s.kc += 1;
    s.k += 1;
  }
  __device__ static void finish(const Ctx& c, const State& st, i64 item) {
    c.kout[item] = st.s.k;
    c.trunc[item] = (st.s.kc >= c.M && st.s.alive) ? 1 : 0;
    const float r = 1.0f / (c.mu_t * c.mu_t);
    const float ct_mu_t = ((-st.cf) * c.mu_a) * r + ((-st.ca) * c.mu_s) * r;
    if (c.pv.emit(0, st.cf / c.mu_t + ct_mu_t)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
    if (c.pv.emit(1, st.ca / c.mu_t + ct_mu_t)) atomicAdd(&c.stats[kStFixedPointOverflow], 1);
  }
  __device__ static void flush(const Ctx& c, const unsigned char* smem, int tid, int nth) {
    ExactBins<2>::flush(c.pv, const_cast<unsigned char*>(smem), c.gw, c.stats, tid);
    const float* win = reinterpret_cast<const float*>(smem + kXBytes);
    for (int b = tid; b < kW * kW * kW; b += nth) {
      const float v = win[b];
      if (v == 0.0f) continue;
      const int ix = kW0 + b / (kW * kW), iy = kW0 + (b / kW) % kW, iz = b % kW;
      fatom(&c.dep[(ix * kBox + iy) * kBox + iz], v);
    }
  }
  __device__ static void epilogue(const Ctx& c, int tid, int) {
    if (tid == 0) ExactBins<2>::readout(c.gw, c.g, c.stats);
  }
};

}  // namespace tmb

namespace tmb {

// Roofline probe of this item (tm_probe_issue kind 4): `iters` photon steps per thread on register state -- the
// draws, the path, the voxel indices and deposit value (summed into a register instead of the tally's atomics), the
// Henyey-Greenstein scattering and the roulette -- a photon that ends being restarted at the source with the next
// key, so every iteration is a full step; no claims, no memory traffic besides one word per thread.  Its rate at
// full occupancy is the issue-rate speed of light of the photon step's own instruction mix.
__global__ void __launch_bounds__(TM_BLOCK) probe_photon_kernel(u32 iters, u32* out) {
  const u32 t = blockIdx.x * blockDim.x + threadIdx.x;
  const float mu_t = 10.1f, frac = 0.1f / 10.1f, albedo = 10.0f / 10.1f;
  Key key{t, 0x9e3779b9u};
  PhotonState s{0, 0, 32.0f, 32.0f, 0.0f, 0.0f, 0.0f, 1.0f, 1.0f, true};
  float acc = 0.0f;
  for (u32 i = 0; i < iters; ++i) {
    const PhotonCommon::Draws u = PhotonCommon::draws(key, s.k);
    const float sl = PhotonCommon::path(u.u0, mu_t);
    s.px = s.px + sl * s.dx;
    s.py = s.py + sl * s.dy;
    s.pz = s.pz + sl * s.dz;
    const bool inside = PhotonCommon::in_box(s.px) && PhotonCommon::in_box(s.py) && PhotonCommon::in_box(s.pz);
    const i32 flat = (PhotonCommon::voxel(s.px) * 64 + PhotonCommon::voxel(s.py)) * 64 + PhotonCommon::voxel(s.pz);
    acc = acc + (inside ? s.w * frac : 0.0f) + (float)(flat & 1);
    const float w1 = s.w * albedo;
    PhotonCommon::scatter(s, u.u1, u.u2);
    const bool low = w1 < 0.001f, survive = u.u3 < 0.1f;
    s.w = low ? (survive ? w1 * 10.0f : 0.0f) : w1;
    s.alive = inside && !(low && !survive);
    s.k += 1;
    if (!s.alive) {
      key.b += 1u;
      s = PhotonState{0, 0, 32.0f, 32.0f, 0.0f, 0.0f, 0.0f, 1.0f, 1.0f, true};
    }
  }
  out[t] = __float_as_uint(acc) ^ (u32)s.k;
}

}  // namespace tmb
