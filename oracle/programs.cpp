// TEST INFRASTRUCTURE ONLY -- CPU restatements of the benchmark item programs, forward and reverse, in the
// reference's CPU kernel-target execution model (oracle_run.h) and arithmetic (oracle_core.h): single-rounding f32
// arithmetic with no FMA (compiled -ffp-contract=off, backends/kernel/host.py:35), emits as _emit_rule
// (backends/kernel/kernel.py:984-1003: an index outside [0, S) is dropped and counted in stats[4]), the max_steps
// cap as retrace(cap) (tallymap/_rewrite.py:517-528: loop while k < M && pred; truncated iff k >= M && pred(out)),
// and reverse mode as vjp_prog (_reverse.py:1079-1180): the checkpointed loop, VJPs of one step newest first, the
// broadcast operand's cotangent accumulated in f32 across the sweep (ctb + db, _reverse.py:387) and emitted once per
// item into an exact tally (_reverse.py:1172-1176).
//
// The item functions are the benchmark configurations written as tallymap items (jax-style pseudo code in each
// struct's comment).  Exposed through a plain C ABI for ctypes (oracle/oracle.py).
#include <cstdio>
#include <type_traits>
#include <vector>

#include "../tallymap_b200/csrc/tm_math.h"
#include "oracle_run.h"

using namespace orc;

namespace {

// The flush of a privatised sum tally.  The reference's host target keeps f32 partials and adds them with an IEEE
// compare-and-swap loop (Acc = float: the timed CPU baseline).  The checker mode (Acc = double) keeps partials and
// the shared output in f64 and rounds once at the end, so a parity tolerance measures the kernel's own summation
// error, not the checker's.
template <class Acc>
static inline void add_out(Acc* o, Acc v) {
  std::atomic_ref<Acc>(*o).fetch_add(v, std::memory_order_relaxed);
}

// ================================================================================================= Q1: quickstart
// examples/quickstart.py:19-30 with max_steps=100:
//   def walker(t, x, key, theta):
//     def body(c):
//       k, x, t = c
//       u = uniform(fold_in(key, k))
//       t = t.add("hist", (x * 16).astype(int32), theta * (1.0 - x))
//       return k + 1, x * (0.5 + 0.5 * u), t
//     k, x, t = while_loop(lambda c: c[1] > 0.05, body, (0, x, t))
//     return t, k
struct Q1State { i32 kc, k; float x; };

struct Q1Base {
  const float* x0;
  const u32* keys;
  float theta;
  i32 M;
  Key key(i64 i) const { return Key{keys[2 * i], keys[2 * i + 1]}; }
  bool pred(float x) const { return x > 0.05f; }
};

template <class Acc>
struct Q1Fwd : Q1Base {
  Acc* hist;           // [16]
  i32* k_out;          // [N]
  uint8_t* trunc;      // [N]
  i32* stats;          // [5]
  struct Priv { Acc h[16] = {}; };
  void item(i64 i, Priv& p) const {
    const Key kk = key(i);
    float x = x0[i];
    i32 k = 0, kc = 0;
    while (kc < M && pred(x)) {
      ++kc;
      const float u = uniform_f32(fold_in(kk, (u32)k), 0u, 0.0f, 1.0f);
      const i32 b = f2i_rz(x * 16.0f);
      const float v = theta * (1.0f - x);
      if ((u32)b >= 16u) stat_add(stats, 4, 1); else p.h[b] += v;
      k = k + 1;
      x = x * (0.5f + 0.5f * u);
    }
    trunc[i] = (kc >= M && pred(x)) ? 1 : 0;
    k_out[i] = k;
  }
  void flush(Priv& p) const {
    for (int b = 0; b < 16; ++b) if (p.h[b] != 0) add_out(&hist[b], p.h[b]);
  }
};

// grad of <ct_hist, hist> w.r.t. theta.  The step VJP: the emit's transpose gathers ct at the emitted index (0 when
// out of range, _tally.py:72-82); mul's transpose gives ct_val * (1 - x); x does not depend on theta (not active).
struct Q1Grad : Q1Base {
  const float* ct;     // [16] cotangent of hist
  int C;
  float* g_theta;      // [1] readout
  uint8_t* trunc;      // [N]: the replay's own truncation flags
  i32* stats;
  ExactBins* gbins;
  struct Adj { float ctb; };
  struct Priv { ExactBins b{1}; };
  bool cond(const Q1State& s) const { return s.kc < M && pred(s.x); }
  Key kk;              // (per-item: set in item(); a copy of the struct per item)
  Q1State step(const Q1State& s) const {
    const float u = uniform_f32(fold_in(kk, (u32)s.k), 0u, 0.0f, 1.0f);
    return Q1State{s.kc + 1, s.k + 1, s.x * (0.5f + 0.5f * u)};
  }
  void vjp_step(const Q1State& s, Adj& a) const {
    const i32 b = f2i_rz(s.x * 16.0f);
    const float cv = ((u32)b < 16u) ? ct[b] : 0.0f;
    const float db = cv * (1.0f - s.x);
    a.ctb = a.ctb + db;
  }
  void item(i64 i, Priv& p) const {
    Q1Grad me = *this;
    me.kk = key(i);
    Adj a{0.0f};
    Q1State fin;
    checkpointed_while(me, Q1State{0, 0, x0[i]}, C, a, &fin, [](const Q1State&, Adj&) {});
    trunc[i] = (fin.kc >= M && pred(fin.x)) ? 1 : 0;
    exact_emit_priv(p.b, 0, a.ctb, stats);
  }
  void flush(Priv& p) const { exact_flush(p.b, *gbins, 1, stats); }
};

// ================================================================================================= RW: 1-D walk
//   def walk(t, x, key, drift):
//     def body(c):
//       k, x, t = c
//       u = uniform(fold_in(key, k))
//       t = t.add("hist", (x * 256).astype(int32), drift * x)
//       return k + 1, x + 0.02 * (2 * u - 1), t
//     k, x, t = while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
//     t = t.add("side", (x > 1).astype(int32), 1.0)
//     return t, k
// max_steps = 20,000.
struct RWState { i32 kc, k; float x; };

struct RWBase {
  const float* x0;
  const u32* keys;
  float drift;
  i32 M;
  Key key(i64 i) const { return Key{keys[2 * i], keys[2 * i + 1]}; }
  static bool pred(float x) { return x >= 0.0f && x <= 1.0f; }
  static float move(float x, float u) { return x + 0.02f * (2.0f * u - 1.0f); }
};

template <class Acc>
struct RWFwd : RWBase {
  Acc* hist;           // [256]
  Acc* side;           // [2]
  i32* k_out;
  uint8_t* trunc;
  i32* stats;
  struct Priv { Acc h[256] = {}; Acc s[2] = {}; };
  void item(i64 i, Priv& p) const {
    const Key kk = key(i);
    float x = x0[i];
    i32 k = 0, kc = 0;
    while (kc < M && pred(x)) {
      ++kc;
      const float u = uniform_f32(fold_in(kk, (u32)k), 0u, 0.0f, 1.0f);
      const i32 b = f2i_rz(x * 256.0f);
      const float v = drift * x;
      if ((u32)b >= 256u) stat_add(stats, 4, 1); else p.h[b] += v;
      k = k + 1;
      x = move(x, u);
    }
    p.s[x > 1.0f ? 1 : 0] += (Acc)1.0f;
    trunc[i] = (kc >= M && pred(x)) ? 1 : 0;
    k_out[i] = k;
  }
  void flush(Priv& p) const {
    for (int b = 0; b < 256; ++b) if (p.h[b] != 0) add_out(&hist[b], p.h[b]);
    for (int b = 0; b < 2; ++b) if (p.s[b] != 0) add_out(&side[b], p.s[b]);
  }
};

// grad of <ct_hist, hist> + <ct_side, side> w.r.t. drift: side does not depend on drift; the step VJP is
// ct_hist[bin] * x (0 for a dropped emit).
struct RWGrad : RWBase {
  const float* ct;     // [256]
  int C;
  uint8_t* trunc;
  i32* stats;
  ExactBins* gbins;
  Key kk;
  struct Adj { float ctb; };
  struct Priv { ExactBins b{1}; };
  bool cond(const RWState& s) const { return s.kc < M && pred(s.x); }
  RWState step(const RWState& s) const {
    const float u = uniform_f32(fold_in(kk, (u32)s.k), 0u, 0.0f, 1.0f);
    return RWState{s.kc + 1, s.k + 1, move(s.x, u)};
  }
  void vjp_step(const RWState& s, Adj& a) const {
    const i32 b = f2i_rz(s.x * 256.0f);
    const float cv = ((u32)b < 256u) ? ct[b] : 0.0f;
    a.ctb = a.ctb + cv * s.x;
  }
  void item(i64 i, Priv& p) const {
    RWGrad me = *this;
    me.kk = key(i);
    Adj a{0.0f};
    RWState fin;
    checkpointed_while(me, RWState{0, 0, x0[i]}, C, a, &fin, [](const RWState&, Adj&) {});
    trunc[i] = (fin.kc >= M && pred(fin.x)) ? 1 : 0;
    exact_emit_priv(p.b, 0, a.ctb, stats);
  }
  void flush(Priv& p) const { exact_flush(p.b, *gbins, 1, stats); }
};

// ================================================================================================= PH: photon slab
// The item of benchmark configuration 3 (its jax-style source is in tallymap_b200/csrc/items_photon.cuh, restated here):
// per step u = uniform(fold_in(key, k), (4,)); s = -log(1 - u0) / mu_t; p += s d; deposit w * mu_a / mu_t at the
// clipped voxel when p is inside the 64^3 box; w *= albedo; Henyey-Greenstein (g = 0.9) scattering by (cos_t, phi =
// 2 pi u2); roulette below 1e-3 with survival u3 < 0.1 (w * 10); the loop runs while the photon is inside and alive.
// Math: SharedMath = the backend's tm_math.h (bitwise with the device: trip counts comparable exactly);
// LibmMath = the C library, as the reference's host target (host.py:9-11): comparable statistically.
struct SharedMath {
  static float log(float x) { return tmm::logf(x); }
  static void sincos(float x, float* s, float* c) { tmm::sincosf(x, s, c); }
};
struct LibmMath {
  static float log(float x) { return std::log(x); }
  static void sincos(float x, float* s, float* c) { *s = std::sin(x); *c = std::cos(x); }
};

struct PhState { i32 kc, k; float px, py, pz, dx, dy, dz, w; bool alive; };

template <class MathT>
struct PhBase {
  const u32* keys;
  float mu_a, mu_s, mu_t, albedo, frac;
  i32 M;
  void init(float a, float s) { mu_a = a; mu_s = s; mu_t = a + s; albedo = s / mu_t; frac = a / mu_t; }
  Key key(i64 i) const { return Key{keys[2 * i], keys[2 * i + 1]}; }
  static PhState start() { return PhState{0, 0, 32.0f, 32.0f, 0.0f, 0.0f, 0.0f, 1.0f, 1.0f, true}; }
  static bool in_box(float x) { return x >= 0.0f && x < 64.0f; }
  static i32 voxel(float x) { return std::min(std::max(f2i_rz(x), 0), 63); }
  float path(float u0) const { return (-MathT::log(1.0f - u0)) / mu_t; }
  static void scatter(PhState& s, float u1, float u2) {
    const float tmp = 0.19f / (0.1f + 1.8f * u1);
    float cos_t = (1.81f - tmp * tmp) / 1.8f;
    cos_t = std::fmin(std::fmax(cos_t, -1.0f), 1.0f);
    const float sin_t = std::sqrt(1.0f - cos_t * cos_t);
    float sp, cp;
    MathT::sincos(6.2831855f * u2, &sp, &cp);
    const float dx = s.dx, dy = s.dy, dz = s.dz;
    if (std::fabs(dz) > 0.99999f) {
      s.dx = sin_t * cp;
      s.dy = sin_t * sp;
      s.dz = cos_t * (dz > 0.0f ? 1.0f : -1.0f);
    } else {
      const float t = std::sqrt(1.0f - dz * dz);
      s.dx = (sin_t * ((dx * dz) * cp - dy * sp)) / t + dx * cos_t;
      s.dy = (sin_t * ((dy * dz) * cp + dx * sp)) / t + dy * cos_t;
      s.dz = ((-sin_t) * cp) * t + dz * cos_t;
    }
  }
  // one step; deposit (flat index, value) reported through dflat / dval (value 0: nothing added)
  void step(Key kk, PhState& s, i32* dflat, float* dval) const {
    const Key nk = fold_in(kk, (u32)s.k);
    const float u0 = uniform_f32(nk, 0u, 0.0f, 1.0f), u1 = uniform_f32(nk, 1u, 0.0f, 1.0f);
    const float u2 = uniform_f32(nk, 2u, 0.0f, 1.0f), u3 = uniform_f32(nk, 3u, 0.0f, 1.0f);
    const float sl = path(u0);
    s.px = s.px + sl * s.dx;
    s.py = s.py + sl * s.dy;
    s.pz = s.pz + sl * s.dz;
    const bool inside = in_box(s.px) && in_box(s.py) && in_box(s.pz);
    *dflat = (voxel(s.px) * 64 + voxel(s.py)) * 64 + voxel(s.pz);
    *dval = inside ? s.w * frac : 0.0f;
    const float w1 = s.w * albedo;
    scatter(s, u1, u2);
    const bool low = w1 < 0.001f, survive = u3 < 0.1f;
    s.w = low ? (survive ? w1 * 10.0f : 0.0f) : w1;
    s.alive = inside && !(low && !survive);
    s.kc += 1;
    s.k += 1;
  }
};

// Acc = float: the reference host target (a 1 MiB tally is not privatised, kernel.py:313-324: every deposit is an
// atomic add into the shared grid).  Acc = double: the checker, with a private f64 grid per thread, flushed once.
template <class MathT, class Acc>
struct PhFwd : PhBase<MathT> {
  Acc* dep;            // [64^3]
  i32* k_out;
  uint8_t* trunc;
  i32* stats;
  struct Priv { std::vector<double> d; Priv() : d(std::is_same<Acc, double>::value ? 64 * 64 * 64 : 0, 0.0) {} };
  void item(i64 i, Priv& p) const {
    const Key kk = this->key(i);
    PhState s = this->start();
    while (s.kc < this->M && s.alive) {
      i32 f;
      float v;
      this->step(kk, s, &f, &v);
      if (v == 0.0f) continue;
      if (std::is_same<Acc, double>::value) p.d[f] += (double)v;
      else add_out(&dep[f], (Acc)v);
    }
    trunc[i] = (s.kc >= this->M && s.alive) ? 1 : 0;
    k_out[i] = s.k;
  }
  void flush(Priv& p) const {
    for (size_t f = 0; f < p.d.size(); ++f)
      if (p.d[f] != 0.0) add_out(&dep[f], (Acc)p.d[f]);
  }
};

// reverse mode: see items_photon.cuh for the step VJP and the pre-loop VJP restated here
template <class MathT>
struct PhGrad : PhBase<MathT> {
  const float* ct;     // [64^3]
  int C;
  uint8_t* trunc;
  i32* stats;
  ExactBins* gbins;
  Key kk;
  struct Adj { float ct_w, ct_frac, ct_albedo; };
  struct Priv { ExactBins b{2}; };
  bool cond(const PhState& s) const { return s.kc < this->M && s.alive; }
  PhState step(const PhState& s) const {
    PhState n = s;
    i32 f;
    float v;
    PhBase<MathT>::step(kk, n, &f, &v);
    return n;
  }
  void vjp_step(const PhState& at, Adj& a) const {
    const Key nk = fold_in(kk, (u32)at.k);
    const float u0 = uniform_f32(nk, 0u, 0.0f, 1.0f), u3 = uniform_f32(nk, 3u, 0.0f, 1.0f);
    const float sl = this->path(u0);
    const float px = at.px + sl * at.dx, py = at.py + sl * at.dy, pz = at.pz + sl * at.dz;
    const bool inside = this->in_box(px) && this->in_box(py) && this->in_box(pz);
    const float w = at.w, w1 = w * this->albedo;
    const bool low = w1 < 0.001f, survive = u3 < 0.1f;
    const float ct_w1 = low ? (survive ? a.ct_w * 10.0f : 0.0f) : a.ct_w;
    a.ct_albedo = a.ct_albedo + ct_w1 * w;
    const float ct_w = ct_w1 * this->albedo;
    const i32 flat = (this->voxel(px) * 64 + this->voxel(py)) * 64 + this->voxel(pz);
    const float cv = inside ? ct[flat] : 0.0f;
    a.ct_frac = a.ct_frac + cv * w;
    a.ct_w = ct_w + cv * this->frac;
  }
  // C = -1: forward mode, the order of the backend's one-pass program (the tangent tw of w w.r.t. albedo carried
  // with the state; each deposit adds cv * w to ct_frac and (cv * frac) * tw to ct_albedo): the checker of that
  // program, not the reference's order
  void forward_mode(PhState& s, Adj& a) const {
    float tw = 0.0f;
    while (cond(s)) {
      const Key nk = fold_in(kk, (u32)s.k);
      const float u0 = uniform_f32(nk, 0u, 0.0f, 1.0f), u3 = uniform_f32(nk, 3u, 0.0f, 1.0f);
      const float sl = this->path(u0);
      const float px = s.px + sl * s.dx, py = s.py + sl * s.dy, pz = s.pz + sl * s.dz;
      const bool inside = this->in_box(px) && this->in_box(py) && this->in_box(pz);
      const i32 flat = (this->voxel(px) * 64 + this->voxel(py)) * 64 + this->voxel(pz);
      const float cv = inside ? ct[flat] : 0.0f;
      a.ct_frac = a.ct_frac + cv * s.w;
      a.ct_albedo = a.ct_albedo + (cv * this->frac) * tw;
      const float w1 = s.w * this->albedo, tw1 = tw * this->albedo + s.w;
      const bool low = w1 < 0.001f, survive = u3 < 0.1f;
      tw = low ? (survive ? tw1 * 10.0f : 0.0f) : tw1;
      s = step(s);
    }
  }
  void item(i64 i, Priv& p) const {
    PhGrad me = *this;
    me.kk = this->key(i);
    Adj a{0.0f, 0.0f, 0.0f};
    PhState fin;
    if (C < 0) {
      fin = this->start();
      me.forward_mode(fin, a);
    } else {
      checkpointed_while(me, this->start(), C, a, &fin, [](const PhState&, Adj& ad) { ad.ct_w = 0.0f; });
    }
    trunc[i] = (fin.kc >= this->M && fin.alive) ? 1 : 0;
    const float r = 1.0f / (this->mu_t * this->mu_t);
    const float ct_mu_t = ((-a.ct_frac) * this->mu_a) * r + ((-a.ct_albedo) * this->mu_s) * r;
    exact_emit_priv(p.b, 0, a.ct_frac / this->mu_t + ct_mu_t, stats);
    exact_emit_priv(p.b, 1, a.ct_albedo / this->mu_t + ct_mu_t, stats);
  }
  void flush(Priv& p) const { exact_flush(p.b, *gbins, 2, stats); }
};

template <class MathT>
static void ph_fwd_run(i64 n, const u32* keys, float mu_a, float mu_s, i32 M, int nthreads, float* dep, i32* k_out,
                       uint8_t* trunc, i32* stats, int f64acc) {
  if (f64acc) {
    std::vector<double> d(64 * 64 * 64, 0.0);
    PhFwd<MathT, double> p;
    p.keys = keys; p.init(mu_a, mu_s); p.M = M;
    p.dep = d.data(); p.k_out = k_out; p.trunc = trunc; p.stats = stats;
    team_run(p, n, nthreads);
    for (size_t b = 0; b < d.size(); ++b) dep[b] = (float)d[b];
    return;
  }
  PhFwd<MathT, float> p;
  p.keys = keys; p.init(mu_a, mu_s); p.M = M;
  p.dep = dep; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
  team_run(p, n, nthreads);
}

template <class MathT>
static void ph_grad_run(i64 n, const u32* keys, float mu_a, float mu_s, const float* ct, i32 M, int C, int nthreads,
                        float* g, uint8_t* trunc, i32* stats) {
  ExactBins gb(2);
  PhGrad<MathT> p;
  p.keys = keys; p.init(mu_a, mu_s); p.M = M; p.ct = ct; p.C = C;
  p.trunc = trunc; p.stats = stats; p.gbins = &gb;
  team_run(p, n, nthreads);
  exact_readout(gb, 2, g, stats);
}

// ================================================================================================= OD: Lorenz RK45
// The item of benchmark configuration 4 (jax-style source in tallymap_b200/csrc/items_ode.cuh, restated here): Dormand-
// Prince 5(4) with FSAL on the Lorenz field, RMS error norm with atol 1e-9 / rtol 1e-6, step factor
// clip(0.9 err^-0.2, 0.2, 10) (stop_gradient'ed), t in [0, 10], h0 = 1e-3; the final state is emitted at
// (item_id, slot) and y_z / 2^20 into a scalar.  Reverse mode restates the hand-derived VJP in the same order.
static inline float fr(double p, double q) { return (float)(p / q); }
struct DPT {
  // a[i][j]: stage i+2's coefficient of k_{j+1}; b: 5th-order weights of k1..k6; e: error weights of k1..k7
  float a[5][5], b[6], e[7];
  DPT() {
    const double A[5][5][2] = {{{1, 5}}, {{3, 40}, {9, 40}}, {{44, 45}, {-56, 15}, {32, 9}},
                               {{19372, 6561}, {-25360, 2187}, {64448, 6561}, {-212, 729}},
                               {{9017, 3168}, {-355, 33}, {46732, 5247}, {49, 176}, {-5103, 18656}}};
    for (int i = 0; i < 5; ++i)
      for (int j = 0; j <= i; ++j) a[i][j] = fr(A[i][j][0], A[i][j][1]);
    const double B[6][2] = {{35, 384}, {0, 1}, {500, 1113}, {125, 192}, {-2187, 6784}, {11, 84}};
    for (int j = 0; j < 6; ++j) b[j] = fr(B[j][0], B[j][1]);
    const double E[7][2] = {{71, 57600}, {0, 1}, {-71, 16695}, {71, 1920}, {-17253, 339200}, {22, 525}, {-1, 40}};
    for (int j = 0; j < 7; ++j) e[j] = fr(E[j][0], E[j][1]);
  }
};
static const DPT kDP;

struct OdState { i32 kc, k; float tt, h; float y[3], k1[3]; };

struct OdBase {
  const float *sigma, *rho, *y0;
  const i32* id;
  float beta;
  i32 M;
  i64 nbins;
  static void f(float sg, float rh, float bt, const float* y, float* o) {
    o[0] = sg * (y[1] - y[0]);
    o[1] = y[0] * (rh - y[2]) - y[1];
    o[2] = y[0] * y[1] - bt * y[2];
  }
  // stages: K[0] = k1 (given), K[1..5] = k2..k6, K[6] = k7; Z[1..5] = the stage points, Y5 = the 5th-order state
  struct St { float K[7][3], Z[6][3], Y5[3]; };
  static void stages(float sg, float rh, float bt, const float* y, const float* k1, float hh, St& s) {
    for (int c = 0; c < 3; ++c) s.K[0][c] = k1[c];
    for (int i = 1; i <= 5; ++i) {          // stage i+1: z = y + hh * (a_i0 k1 + ... )
      for (int c = 0; c < 3; ++c) {
        float d = kDP.a[i - 1][0] * s.K[0][c];
        for (int j = 1; j < i; ++j) d = d + kDP.a[i - 1][j] * s.K[j][c];
        s.Z[i][c] = y[c] + hh * d;
      }
      f(sg, rh, bt, s.Z[i], s.K[i]);
    }
    for (int c = 0; c < 3; ++c) {
      float d = kDP.b[0] * s.K[0][c];
      for (int j = 2; j < 6; ++j) d = d + kDP.b[j] * s.K[j][c];
      s.Y5[c] = y[c] + hh * d;
    }
    f(sg, rh, bt, s.Y5, s.K[6]);
  }
  static bool control(const float* y, const St& s, float hh, float* fac) {
    float q[3];
    for (int c = 0; c < 3; ++c) {
      float d = kDP.e[0] * s.K[0][c];
      for (int j = 2; j < 7; ++j) d = d + kDP.e[j] * s.K[j][c];
      const float ev = hh * d;
      const float sc = 1e-9f + 1e-6f * std::fmax(std::fabs(y[c]), std::fabs(s.Y5[c]));
      q[c] = ev / sc;
    }
    const float err = std::sqrt((q[0] * q[0] + q[1] * q[1] + q[2] * q[2]) / 3.0f);
    const float f0 = 0.9f * tmm::powf(err, -0.2f);
    *fac = std::fmin(std::fmax(f0, 0.2f), 10.0f);
    return err <= 1.0f;
  }
  static void advance(float sg, float rh, float bt, OdState& st) {
    const float hh = std::fmin(st.h, 10.0f - st.tt);
    St s;
    stages(sg, rh, bt, st.y, st.k1, hh, s);
    float fac;
    if (control(st.y, s, hh, &fac)) {
      st.tt = st.tt + hh;
      for (int c = 0; c < 3; ++c) { st.y[c] = s.Y5[c]; st.k1[c] = s.K[6][c]; }
    }
    st.h = hh * fac;
    st.kc += 1;
    st.k += 1;
  }
  OdState start(i64 i) const {
    OdState s;
    s.kc = s.k = 0;
    s.tt = 0.0f;
    s.h = 1e-3f;
    for (int c = 0; c < 3; ++c) s.y[c] = y0[3 * i + c];
    f(sigma[i], rho[i], beta, s.y, s.k1);
    return s;
  }
  bool cond(const OdState& s) const { return s.kc < M && s.tt < 10.0f; }
};

template <class Acc>
struct OdFwd : OdBase {
  float* fin;
  Acc* mean;
  i32* k_out;
  uint8_t* trunc;
  i32* stats;
  struct Priv { Acc m = 0; };
  void item(i64 i, Priv& p) const {
    OdState s = start(i);
    while (cond(s)) advance(sigma[i], rho[i], beta, s);
    const i32 iid = id[i];
    for (int c = 0; c < 3; ++c) {
      if (iid < 0 || (i64)iid * 3 + c >= nbins) stat_add(stats, 4, 1);
      else add_out(&fin[(i64)iid * 3 + c], s.y[c]);
    }
    p.m += (Acc)(s.y[2] * (1.0f / 1048576.0f));
    trunc[i] = (s.kc >= M && s.tt < 10.0f) ? 1 : 0;
    k_out[i] = s.k;
  }
  void flush(Priv& p) const { if (p.m != 0) add_out(mean, p.m); }
};

struct OdGrad : OdBase {
  const float *ctf, *ctm;
  int C;
  uint8_t* trunc;
  i32* stats;
  ExactBins* gbins;
  float sg, rh;        // the current item's parameters
  struct Adj { float cy[3], ck1[3], cb; };
  struct Priv { ExactBins b{1}; };
  OdState step(const OdState& s) const { OdState n = s; advance(sg, rh, beta, n); return n; }
  // f's VJP at y for cotangent g: adds into cy (order as items_ode.cuh) and returns the beta term
  float f_vjp_add(const float* y, const float* g, float* cz) const {
    cz[0] = (-sg) * g[0] + (rh - y[2]) * g[1] + y[1] * g[2];
    cz[1] = sg * g[0] - g[1] + y[0] * g[2];
    cz[2] = (-(y[0] * g[1])) - beta * g[2];
    return -(y[2] * g[2]);
  }
  void vjp_step(const OdState& at, Adj& a) const {
    const float hh = std::fmin(at.h, 10.0f - at.tt);
    St s;
    stages(sg, rh, beta, at.y, at.k1, hh, s);
    float fac;
    if (!control(at.y, s, hh, &fac)) return;
    float cz[3], ck[7][3] = {};
    float dsum = f_vjp_add(s.Y5, a.ck1, cz);            // k7 = f(y5)
    float cy[3], s5[3];
    for (int c = 0; c < 3; ++c) { cy[c] = a.cy[c] + cz[c]; s5[c] = hh * cy[c]; }
    const int bj[5] = {0, 2, 3, 4, 5};
    for (int t = 0; t < 5; ++t)
      for (int c = 0; c < 3; ++c) ck[bj[t]][c] = kDP.b[bj[t]] * s5[c];
    for (int i = 5; i >= 1; --i) {                      // stages k6 .. k2
      dsum = dsum + f_vjp_add(s.Z[i], ck[i], cz);
      float sz[3];
      for (int c = 0; c < 3; ++c) { cy[c] = cy[c] + cz[c]; sz[c] = hh * cz[c]; }
      for (int j = 0; j < i; ++j)
        for (int c = 0; c < 3; ++c) ck[j][c] = ck[j][c] + kDP.a[i - 1][j] * sz[c];
    }
    for (int c = 0; c < 3; ++c) { a.cy[c] = cy[c]; a.ck1[c] = ck[0][c]; }
    a.cb = a.cb + dsum;
  }
  void item(i64 i, Priv& p) const {
    OdGrad me = *this;
    me.sg = sigma[i];
    me.rh = rho[i];
    const i32 iid = id[i];
    Adj a{};
    OdState fin;
    checkpointed_while(me, start(i), C, a, &fin, [&](const OdState&, Adj& ad) {
      float g[3];
      for (int c = 0; c < 3; ++c) {
        const bool in = iid >= 0 && (i64)iid * 3 + c < nbins;
        g[c] = in ? ctf[(i64)iid * 3 + c] : 0.0f;
      }
      ad.cy[0] = g[0]; ad.cy[1] = g[1]; ad.cy[2] = g[2] + ctm[0] * (1.0f / 1048576.0f);
      ad.ck1[0] = ad.ck1[1] = ad.ck1[2] = 0.0f;
    });
    trunc[i] = (fin.kc >= M && fin.tt < 10.0f) ? 1 : 0;
    float y0v[3] = {y0[3 * i], y0[3 * i + 1], y0[3 * i + 2]}, cz[3];
    const float db = me.f_vjp_add(y0v, a.ck1, cz);     // the pre-loop k1 = f(y0)
    exact_emit_priv(p.b, 0, a.cb + db, stats);
  }
  void flush(Priv& p) const { exact_flush(p.b, *gbins, 1, stats); }
};

// Forward mode w.r.t. beta, the checker of the backend's one-pass Lorenz program (items_ode.cuh ODVG1, its order, not
// the reference's): each item carries the tangents dy, dk1 of y and k1 (dy = 0 and dk1 = f_jvp(y0, 0) before the
// loop); a step's stage tangents are dz = dy + hh * (sum a_j dk_j) in the primal's order and dk = f_jvp(z, dz), beta's
// tangent 1, hh and the step control without tangents (the step factor is stop_gradient'ed); an accepted step takes
// dy5 and dk7.  An item adds ((ct_f0 dy_x + ct_f1 dy_y) + ct_f2 dy_z) + ct_mean (dy_z / 2^20) to an exact bin.
struct OdVG1 : OdBase {
  const float *ctf, *ctm;
  i32* k_out;
  uint8_t* trunc;
  i32* stats;
  ExactBins* gbins;
  struct Priv { ExactBins b{1}; };
  static void f_jvp(float sg, float rh, float bt, const float* y, const float* dy, float* o) {
    o[0] = sg * (dy[1] - dy[0]);
    o[1] = (dy[0] * (rh - y[2]) + y[0] * (-dy[2])) - dy[1];
    o[2] = (dy[0] * y[1] + y[0] * dy[1]) - (y[2] + bt * dy[2]);
  }
  void item(i64 i, Priv& p) const {
    const float sg = sigma[i], rh = rho[i];
    OdState s = start(i);
    float dy[3] = {0.0f, 0.0f, 0.0f}, dk1[3];
    f_jvp(sg, rh, beta, s.y, dy, dk1);
    while (cond(s)) {
      const float hh = std::fmin(s.h, 10.0f - s.tt);
      St st;
      stages(sg, rh, beta, s.y, s.k1, hh, st);
      float dK[6][3], dz[3], dy5[3], dk7[3];
      for (int c = 0; c < 3; ++c) dK[0][c] = dk1[c];
      for (int q = 1; q <= 5; ++q) {
        for (int c = 0; c < 3; ++c) {
          float d = kDP.a[q - 1][0] * dK[0][c];
          for (int j = 1; j < q; ++j) d = d + kDP.a[q - 1][j] * dK[j][c];
          dz[c] = dy[c] + hh * d;
        }
        f_jvp(sg, rh, beta, st.Z[q], dz, dK[q]);
      }
      for (int c = 0; c < 3; ++c) {
        float d = kDP.b[0] * dK[0][c];
        for (int j = 2; j < 6; ++j) d = d + kDP.b[j] * dK[j][c];
        dy5[c] = dy[c] + hh * d;
      }
      f_jvp(sg, rh, beta, st.Y5, dy5, dk7);
      float fac;
      if (control(s.y, st, hh, &fac)) {
        s.tt = s.tt + hh;
        for (int c = 0; c < 3; ++c) {
          s.y[c] = st.Y5[c];
          s.k1[c] = st.K[6][c];
          dy[c] = dy5[c];
          dk1[c] = dk7[c];
        }
      }
      s.h = hh * fac;
      s.kc += 1;
      s.k += 1;
    }
    const i32 iid = id[i];
    float gi = 0.0f;
    for (int c = 0; c < 3; ++c) {
      if (iid < 0 || (i64)iid * 3 + c >= nbins) continue;
      const float t = ctf[(i64)iid * 3 + c] * dy[c];
      gi = c == 0 ? t : gi + t;
    }
    gi = gi + ctm[0] * (dy[2] * (1.0f / 1048576.0f));
    exact_emit_priv(p.b, 0, gi, stats);
    trunc[i] = (s.kc >= M && s.tt < 10.0f) ? 1 : 0;
    k_out[i] = s.k;
  }
  void flush(Priv& p) const { exact_flush(p.b, *gbins, 1, stats); }
};

// ================================================================================================= SH: shower
// The item of benchmark configuration 5 (jax-style source in tallymap_b200/csrc/items_shower.cuh, restated here).  The
// reference runs spawned children through a shared ticket ring on its OpenMP team (kernel.py:778-811, 1007-1044);
// every child is an independent item, so when the ring drops nothing the tallies are the same sums whatever order
// the children run in.  The oracle therefore runs each root's whole tree depth-first on one thread (a private stack
// of pending children), which is that schedule with an unbounded ring: the spawned count is every child.
struct ShChild { float E, depth; Key key; };

template <class Acc>
struct ShFwd {
  const float *E0, *d0;
  const u32* keys;
  float X0;
  i32 M;
  Acc* dep;            // [512]
  i32* count;
  i32* k_out;
  uint8_t* trunc;
  i32* stats;
  struct Priv { Acc h[512] = {}; i64 n = 0, spawned = 0, ctrunc = 0; std::vector<ShChild> stack; };
  // run one particle; pushes its children; returns (k, truncated)
  void particle(ShChild p, Priv& pv, i32* k_ret, bool* tr_ret) const {
    i32 kc = 0, k = 0;
    bool alive = true;
    float E = p.E, depth = p.depth;
    while (kc < M && alive) {
      const Key kk = fold_in(p.key, (u32)k);
      const float u0 = uniform_f32(kk, 0u, 0.0f, 1.0f), u1 = uniform_f32(kk, 1u, 0.0f, 1.0f);
      const float u2 = uniform_f32(kk, 2u, 0.0f, 1.0f);
      depth = depth + X0 * (-tmm::logf(1.0f - u0));
      const bool low = E < 0.5f;
      if (low) {
        const i32 b = f2i_rz(depth * 8.0f);
        if ((u32)b >= 512u) stat_add(stats, 4, 1); else pv.h[b] += (Acc)E;
      }
      const bool split = !low && u1 < 0.7f;
      if (split) {
        const float z = 0.1f + 0.8f * u2;
        pv.stack.push_back(ShChild{E * (1.0f - z), depth, fold_in(kk, 1u)});   // popped second
        pv.stack.push_back(ShChild{E * z, depth, fold_in(kk, 0u)});
        pv.spawned += 2;
      }
      alive = !low && !split;
      kc += 1;
      k += 1;
    }
    pv.n += 1;
    *k_ret = k;
    *tr_ret = kc >= M && alive;
  }
  void item(i64 i, Priv& pv) const {
    i32 k;
    bool tr;
    particle(ShChild{E0[i], d0[i], Key{keys[2 * i], keys[2 * i + 1]}}, pv, &k, &tr);
    k_out[i] = k;
    trunc[i] = tr ? 1 : 0;
    while (!pv.stack.empty()) {
      const ShChild c = pv.stack.back();
      pv.stack.pop_back();
      i32 kk;
      bool t2;
      particle(c, pv, &kk, &t2);
      if (t2) pv.ctrunc += 1;
    }
  }
  void flush(Priv& pv) const {
    for (int b = 0; b < 512; ++b) if (pv.h[b] != 0) add_out(&dep[b], pv.h[b]);
    stat_add(count, 0, (i32)pv.n);
    stat_add(stats, 0, (i32)pv.spawned);
    stat_add(stats, 2, (i32)pv.ctrunc);
  }
};

// SH reverse mode: the tree adjoint (tallymap/_reverse_spawn.py:1-45; tree_vjp 233-336).  The reference records
// every child (rec_primal, 85-109) and runs one adjoint launch per generation, deepest first, so that a parent's
// replay finds its children's initial-state cotangents ready; here a post-order traversal of each root's tree gives
// the same order per particle: a particle's children are differentiated before its own steps are transposed.  Per
// particle the step VJPs run newest first; at the spawn step the children's cotangents enter newest child first
// (dx1 then dx0), then the deposit's cotangent, then the travel depth' = depth + X0 * L (ct_X0 += ct_depth' * L).
// Each particle's ct_X0 is one exact emit.  Truncated particles are counted (the gradient is poisoned by the caller).
struct ShGrad {
  const float *E0, *d0;
  const u32* keys;
  float X0;
  i32 M;
  const float* ct;     // [512] cotangent of dep
  float *gE, *gD;      // [N] cotangents of the roots' E and depth
  i32* stats;
  ExactBins* gbins;
  struct Priv { ExactBins b{1}; i64 trunc = 0, nodes = 0; std::vector<float> buf; };
  struct StepOut { bool split, low; float z, L, d1; Key kk; };
  StepOut advance(Key key, i32 k, float E, float depth) const {
    const Key kk = fold_in(key, (u32)k);
    const float u0 = uniform_f32(kk, 0u, 0.0f, 1.0f), u1 = uniform_f32(kk, 1u, 0.0f, 1.0f);
    const float u2 = uniform_f32(kk, 2u, 0.0f, 1.0f);
    const float L = -tmm::logf(1.0f - u0);
    const float d1 = depth + X0 * L;
    const bool low = E < 0.5f;
    return StepOut{!low && u1 < 0.7f, low, 0.1f + 0.8f * u2, L, d1, kk};
  }
  // the adjoint of one particle (and, first, of its subtree): -> the cotangents of its initial E and depth
  void particle(float E, float depth, Key key, Priv& p, float* dE, float* dD) const {
    p.nodes += 1;
    std::vector<float> ds;           // depth before each step
    i32 kc = 0;
    bool alive = true, split = false;
    float d = depth;
    StepOut last{};
    while (kc < M && alive) {
      ds.push_back(d);
      last = advance(key, kc, E, d);
      d = last.d1;
      split = last.split;
      alive = !last.low && !last.split;
      kc += 1;
    }
    if (kc >= M && alive) p.trunc += 1;
    float dE1 = 0.0f, dD1 = 0.0f, dE0 = 0.0f, dD0 = 0.0f;
    if (split) {
      particle(E * (1.0f - last.z), d, fold_in(last.kk, 1u), p, &dE1, &dD1);
      particle(E * last.z, d, fold_in(last.kk, 0u), p, &dE0, &dD0);
    }
    float ctE = 0.0f, ctd = 0.0f, ctX = 0.0f;
    for (i32 k = kc - 1; k >= 0; --k) {
      const StepOut o = advance(key, k, E, ds[k]);
      if (o.split) {
        const float f1 = 1.0f - o.z;
        ctE = ctE + dE1 * f1;
        ctd = ctd + dD1;
        ctE = ctE + dE0 * o.z;
        ctd = ctd + dD0;
      }
      if (o.low) {
        const i32 b = f2i_rz(o.d1 * 8.0f);
        if ((u32)b < 512u) ctE = ctE + ct[b];
      }
      ctX = ctX + ctd * o.L;
    }
    exact_emit_priv(p.b, 0, ctX, stats);
    *dE = ctE;
    *dD = ctd;
  }
  void item(i64 i, Priv& p) const {
    particle(E0[i], d0[i], Key{keys[2 * i], keys[2 * i + 1]}, p, &gE[i], &gD[i]);
  }
  void flush(Priv& p) const {
    exact_flush(p.b, *gbins, 1, stats);
    stat_add(stats, 2, (i32)p.trunc);
  }
};

}  // namespace

// ================================================================================================= C ABI
extern "C" {

int or_num_threads(void) { return omp_get_max_threads(); }

void or_threefry2x32(u32 k0, u32 k1, u32 c0, u32 c1, u32* out) { threefry2x32(k0, k1, c0, c1, &out[0], &out[1]); }

// split(key, n) -> out[n][2]
void or_split(u32 k0, u32 k1, i64 n, u32* out) {
  for (i64 i = 0; i < n; ++i) {
    const Key k = split_at(Key{k0, k1}, (u32)i);
    out[2 * i] = k.a;
    out[2 * i + 1] = k.b;
  }
}

// uniform(key, (n,), f32, lo, hi) -> out[n]
void or_uniform(u32 k0, u32 k1, i64 n, float lo, float hi, float* out) {
  for (i64 i = 0; i < n; ++i) out[i] = uniform_f32(Key{k0, k1}, (u32)i, lo, hi);
}

// the exact sum of vals into bins (out-of-range bins dropped), read out as the kernel's exact tally
void or_exact_sum(const float* vals, const i32* bins, i64 n, int nb, float* out, i32* stats) {
  ExactBins g(nb);
  for (i64 i = 0; i < n; ++i) {
    if ((u32)bins[i] >= (u32)nb) continue;
    if (exact_emit<false>(&g.w[(size_t)bins[i] * kExactWords], vals[i])) { stats[3] += 1; g.flag[bins[i]] = 1; }
  }
  exact_readout(g, nb, out, stats);
}

// the raw words of an exact sum (test of the word layout): words[nb][5]
void or_exact_words(const float* vals, const i32* bins, i64 n, int nb, i64* words) {
  ExactBins g(nb);
  for (i64 i = 0; i < n; ++i)
    if ((u32)bins[i] < (u32)nb) exact_emit<false>(&g.w[(size_t)bins[i] * kExactWords], vals[i]);
  for (size_t j = 0; j < g.w.size(); ++j) words[j] = g.w[j];
}

float or_exact_read(const i64* words, int* bad) {
  bool b = false;
  const float o = exact_read(words, &b);
  *bad = b ? 1 : 0;
  return o;
}

// f64acc: 0 = the reference's f32 partials (timed baseline), 1 = f64 partials rounded once (checker)
int or_q1_fwd(i64 n, const float* x0, const u32* keys, float theta, i32 max_steps, int nthreads, float* hist,
              i32* k_out, uint8_t* trunc, i32* stats, int f64acc) {
  if (f64acc) {
    std::vector<double> h(16, 0.0);
    Q1Fwd<double> p;
    p.x0 = x0; p.keys = keys; p.theta = theta; p.M = max_steps;
    p.hist = h.data(); p.k_out = k_out; p.trunc = trunc; p.stats = stats;
    team_run(p, n, nthreads);
    for (int b = 0; b < 16; ++b) hist[b] = (float)h[b];
    return 0;
  }
  Q1Fwd<float> p;
  p.x0 = x0; p.keys = keys; p.theta = theta; p.M = max_steps;
  p.hist = hist; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
  team_run(p, n, nthreads);
  return 0;
}

int or_q1_grad(i64 n, const float* x0, const u32* keys, float theta, const float* ct, i32 max_steps, int C,
               int nthreads, float* g_theta, uint8_t* trunc, i32* stats) {
  ExactBins g(1);
  Q1Grad p;
  p.x0 = x0; p.keys = keys; p.theta = theta; p.M = max_steps; p.ct = ct; p.C = C;
  p.trunc = trunc; p.stats = stats; p.gbins = &g;
  team_run(p, n, nthreads);
  exact_readout(g, 1, g_theta, stats);
  return 0;
}

int or_rw_fwd(i64 n, const float* x0, const u32* keys, float drift, i32 max_steps, int nthreads, float* hist,
              float* side, i32* k_out, uint8_t* trunc, i32* stats, int f64acc) {
  if (f64acc) {
    std::vector<double> h(256, 0.0), sd(2, 0.0);
    RWFwd<double> p;
    p.x0 = x0; p.keys = keys; p.drift = drift; p.M = max_steps;
    p.hist = h.data(); p.side = sd.data(); p.k_out = k_out; p.trunc = trunc; p.stats = stats;
    team_run(p, n, nthreads);
    for (int b = 0; b < 256; ++b) hist[b] = (float)h[b];
    for (int b = 0; b < 2; ++b) side[b] = (float)sd[b];
    return 0;
  }
  RWFwd<float> p;
  p.x0 = x0; p.keys = keys; p.drift = drift; p.M = max_steps;
  p.hist = hist; p.side = side; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
  team_run(p, n, nthreads);
  return 0;
}

int or_rw_grad(i64 n, const float* x0, const u32* keys, float drift, const float* ct, i32 max_steps, int C,
               int nthreads, float* g_drift, uint8_t* trunc, i32* stats) {
  ExactBins g(1);
  RWGrad p;
  p.x0 = x0; p.keys = keys; p.drift = drift; p.M = max_steps; p.ct = ct; p.C = C;
  p.trunc = trunc; p.stats = stats; p.gbins = &g;
  team_run(p, n, nthreads);
  exact_readout(g, 1, g_drift, stats);
  return 0;
}

// libm: 0 = the backend's shared math (bitwise with the device), 1 = the C library (the reference host target)
int or_ph_fwd(i64 n, const u32* keys, float mu_a, float mu_s, i32 max_steps, int nthreads, float* dep, i32* k_out,
              uint8_t* trunc, i32* stats, int f64acc, int libm) {
  if (libm) ph_fwd_run<LibmMath>(n, keys, mu_a, mu_s, max_steps, nthreads, dep, k_out, trunc, stats, f64acc);
  else ph_fwd_run<SharedMath>(n, keys, mu_a, mu_s, max_steps, nthreads, dep, k_out, trunc, stats, f64acc);
  return 0;
}

int or_ph_grad(i64 n, const u32* keys, float mu_a, float mu_s, const float* ct, i32 max_steps, int C, int nthreads,
               float* g, uint8_t* trunc, i32* stats, int libm) {
  if (libm) ph_grad_run<LibmMath>(n, keys, mu_a, mu_s, ct, max_steps, C, nthreads, g, trunc, stats);
  else ph_grad_run<SharedMath>(n, keys, mu_a, mu_s, ct, max_steps, C, nthreads, g, trunc, stats);
  return 0;
}

// the shared math on the host, elementwise (fn 0 log, 1 exp, 2 sin, 3 cos, 4 pow(x, y))
void or_math(int fn, const float* x, const float* y, float* out, i64 n) {
  for (i64 i = 0; i < n; ++i) out[i] = tmm::eval(fn, x[i], y ? y[i] : 0.0f);
}

int or_od_fwd(i64 n, const float* sigma, const float* rho, const float* y0, const i32* id, float beta, i32 max_steps,
              int nthreads, float* fin, float* mean, i32* k_out, uint8_t* trunc, i32* stats, int f64acc) {
  if (f64acc) {
    double m = 0.0;
    OdFwd<double> p;
    p.sigma = sigma; p.rho = rho; p.y0 = y0; p.id = id; p.beta = beta; p.M = max_steps; p.nbins = 3 * n;
    p.fin = fin; p.mean = &m; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
    team_run(p, n, nthreads);
    *mean = (float)m;
    return 0;
  }
  OdFwd<float> p;
  p.sigma = sigma; p.rho = rho; p.y0 = y0; p.id = id; p.beta = beta; p.M = max_steps; p.nbins = 3 * n;
  p.fin = fin; p.mean = mean; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
  team_run(p, n, nthreads);
  return 0;
}

int or_od_grad(i64 n, const float* sigma, const float* rho, const float* y0, const i32* id, float beta,
               const float* ctf, const float* ctm, i32 max_steps, int C, int nthreads, float* g, uint8_t* trunc,
               i32* stats) {
  ExactBins gb(1);
  OdGrad p;
  p.sigma = sigma; p.rho = rho; p.y0 = y0; p.id = id; p.beta = beta; p.M = max_steps; p.nbins = 3 * n;
  p.ctf = ctf; p.ctm = ctm; p.C = C; p.trunc = trunc; p.stats = stats; p.gbins = &gb;
  team_run(p, n, nthreads);
  exact_readout(gb, 1, g, stats);
  return 0;
}

int or_od_vg1(i64 n, const float* sigma, const float* rho, const float* y0, const i32* id, float beta,
              const float* ctf, const float* ctm, i32 max_steps, int nthreads, float* g, i32* k_out, uint8_t* trunc,
              i32* stats) {
  ExactBins gb(1);
  OdVG1 p;
  p.sigma = sigma; p.rho = rho; p.y0 = y0; p.id = id; p.beta = beta; p.M = max_steps; p.nbins = 3 * n;
  p.ctf = ctf; p.ctm = ctm; p.k_out = k_out; p.trunc = trunc; p.stats = stats; p.gbins = &gb;
  team_run(p, n, nthreads);
  exact_readout(gb, 1, g, stats);
  return 0;
}

// Forward mode through spawn, the checker of the backend's one-pass shower program (not the reference's order):
// each particle carries the tangent tE of its energy w.r.t. its root's E0 (a root 1; children tE * z and
// tE * (1 - z), as their energies E * z and E * (1 - z)); a deposit of E at bin b adds ct[b] * tE (one f32
// product) to its root's exact sum.  Depth and X0 reach the outputs only through the integer bin index, so their
// cotangents are zero.
struct ShVG1 {
  const float *E0, *d0;
  const u32* keys;
  float X0;
  i32 M;
  const float* ct;
  float* gE;
  i32* stats;
  struct P { float E, depth, tE; Key key; };
  struct Priv { std::vector<P> stack; };
  void item(i64 i, Priv& pv) const {
    ExactBins acc(1);
    pv.stack.push_back(P{E0[i], d0[i], 1.0f, Key{keys[2 * i], keys[2 * i + 1]}});
    while (!pv.stack.empty()) {
      const P p = pv.stack.back();
      pv.stack.pop_back();
      i32 kc = 0, k = 0;
      bool alive = true;
      const float E = p.E;
      float depth = p.depth;
      while (kc < M && alive) {
        const Key kk = fold_in(p.key, (u32)k);
        const float u0 = uniform_f32(kk, 0u, 0.0f, 1.0f), u1 = uniform_f32(kk, 1u, 0.0f, 1.0f);
        const float u2 = uniform_f32(kk, 2u, 0.0f, 1.0f);
        depth = depth + X0 * (-tmm::logf(1.0f - u0));
        const bool low = E < 0.5f;
        if (low) {
          const i32 b = f2i_rz(depth * 8.0f);
          if ((u32)b < 512u) exact_emit_priv(acc, 0, ct[b] * p.tE, stats);
        }
        const bool split = !low && u1 < 0.7f;
        if (split) {
          const float z = 0.1f + 0.8f * u2;
          pv.stack.push_back(P{E * (1.0f - z), depth, p.tE * (1.0f - z), fold_in(kk, 1u)});
          pv.stack.push_back(P{E * z, depth, p.tE * z, fold_in(kk, 0u)});
        }
        alive = !low && !split;
        kc += 1;
        k += 1;
      }
    }
    exact_readout(acc, 1, &gE[i], stats);
  }
  void flush(Priv&) const {}
};

// the tree adjoint: g_X0 (exact), g_E[n], g_depth[n]; stats[2] counts truncated particles of the whole forest
int or_sh_grad(i64 n, const float* E0, const float* d0, const u32* keys, float X0, const float* ct_dep, i32 max_steps,
               int nthreads, float* g_X0, float* g_E, float* g_depth, i32* stats) {
  ExactBins gb(1);
  ShGrad p;
  p.E0 = E0; p.d0 = d0; p.keys = keys; p.X0 = X0; p.M = max_steps; p.ct = ct_dep;
  p.gE = g_E; p.gD = g_depth; p.stats = stats; p.gbins = &gb;
  team_run(p, n, nthreads);
  exact_readout(gb, 1, g_X0, stats);
  return 0;
}

// the one-pass (forward mode) gradient of <ct_dep, dep> w.r.t. each root's E0: g_E[n]
int or_sh_vg1(i64 n, const float* E0, const float* d0, const u32* keys, float X0, const float* ct_dep, i32 max_steps,
              int nthreads, float* g_E, i32* stats) {
  ShVG1 p;
  p.E0 = E0; p.d0 = d0; p.keys = keys; p.X0 = X0; p.M = max_steps; p.ct = ct_dep; p.gE = g_E; p.stats = stats;
  team_run(p, n, nthreads);
  return 0;
}

int or_sh_fwd(i64 n, const float* E0, const float* d0, const u32* keys, float X0, i32 max_steps, int nthreads,
              float* dep, i32* count, i32* k_out, uint8_t* trunc, i32* stats, int f64acc) {
  if (f64acc) {
    std::vector<double> d(512, 0.0);
    ShFwd<double> p;
    p.E0 = E0; p.d0 = d0; p.keys = keys; p.X0 = X0; p.M = max_steps;
    p.dep = d.data(); p.count = count; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
    team_run(p, n, nthreads);
    for (int b = 0; b < 512; ++b) dep[b] = (float)d[b];
    return 0;
  }
  ShFwd<float> p;
  p.E0 = E0; p.d0 = d0; p.keys = keys; p.X0 = X0; p.M = max_steps;
  p.dep = dep; p.count = count; p.k_out = k_out; p.trunc = trunc; p.stats = stats;
  team_run(p, n, nthreads);
  return 0;
}

}  // extern "C"
