// TEST INFRASTRUCTURE ONLY -- the oracle's execution model (see oracle_core.h for who may use it).
//
// Restates the reference's CPU kernel target:
//   * the persistent claim loop of sj_main (backends/kernel/kernel.py:812-838) on an OpenMP team, each host thread
//     one CUDA thread of a one-thread block (backends/kernel/host.py:1-16, host_shim.cc:83-138): items are claimed
//     one at a time from a shared counter; privatised tallies are per-thread arrays flushed atomically at the end
//     (kernel.py:681-688 with host.py's per-thread stand-in for __shared__);
//   * the reverse-mode CHECKPOINTED LOOP (tallymap/_reverse.py:324-444): a forward count pass that stores a head of
//     C + 1 states, a checkpoint pass at stride m = max(C, ceil(K / C)), and per segment (last first) per sub-chunk
//     of C states (last first): advance, fill a C-slot tape (the first sub-chunk reads the head), and apply one step
//     VJP per state, newest first.
#pragma once
#include <omp.h>

#include <algorithm>
#include <atomic>
#include <vector>

#include "oracle_core.h"

namespace orc {

// Run prog.item(i, priv) for every i in [0, n) on `nthreads` host threads that claim one item at a time.  Each
// thread owns a P::Priv (privatised accumulators), flushed with prog.flush(priv) when the thread runs out of items.
template <class P>
void team_run(const P& prog, i64 n, int nthreads) {
  if (nthreads <= 0) nthreads = omp_get_max_threads();
  std::atomic<i64> ctr{0};
#pragma omp parallel num_threads(nthreads)
  {
    typename P::Priv priv;
    for (;;) {
      const i64 t = ctr.fetch_add(1, std::memory_order_relaxed);
      if (t >= n) break;
      prog.item(t, priv);
    }
    prog.flush(priv);
  }
}

// The checkpointed loop's adjoint for one item (_reverse.py:343-440).  P provides: State, cond(State),
// step(State) -> State, vjp_step(State, Adj&) (one body step's VJP at the state before it).  post(final, adj) seeds
// the cotangents of the loop's outputs before the sweep (called between the count pass and the sweep).
// Returns K, the number of steps the forward ran; *final receives the loop's output state.
template <class P, class S, class A, class Post>
i64 checkpointed_while(const P& prog, const S& init, int C, A& adj, S* final, Post&& post) {
  if (C < 0) {
    // C = -1: the one-pass order of an item with no active carry (each step's VJP applied before the step, oldest
    // first; post last): the checker of the backend's one-pass value-and-grad programs, not the reference's order
    S c = init;
    i64 K = 0;
    while (prog.cond(c)) {
      prog.vjp_step(c, adj);
      c = prog.step(c);
      ++K;
    }
    *final = c;
    post(c, adj);
    return K;
  }
  // the head, checkpoint and tape buffers are per host thread and reused across items (only their first slots up
  // to what an item writes are read), so a large C -- which makes the replay linear in K, bitwise the same
  // cotangents as any other C -- costs no per-item allocation
  thread_local std::vector<S> head, ck, tape;
  if (head.size() < (size_t)C + 1) {
    head.resize(C + 1);
    ck.resize(C);
    tape.resize(C);
  }
  S c = init;
  i64 K = 0;
  while (prog.cond(c)) {                       // count pass: head slot min(k, C) (slot C: scratch sink)
    head[std::min<i64>(K, C)] = c;
    c = prog.step(c);
    ++K;
  }
  *final = c;
  post(c, adj);
  const i64 m = std::max<i64>(C, (K + C - 1) / C);  // checkpoint stride
  const i64 ns = (K + m - 1) / m;                   // segments (<= C)
  S x = init;
  ck[0] = init;
  for (i64 s = 1; s < ns; ++s) {                   // checkpoint pass (empty when K <= C)
    for (i64 j = 0; j < m; ++j) x = prog.step(x);
    ck[s] = x;
  }
  for (i64 sr = 0; sr < ns; ++sr) {
    const i64 s = ns - 1 - sr;
    const i64 L = std::min<i64>(m, K - s * m);
    const i64 nsub = (L + C - 1) / C;
    for (i64 ur = 0; ur < nsub; ++ur) {
      const i64 u = nsub - 1 - ur;
      const i64 LL = std::min<i64>(C, L - u * C);
      const bool first = (s == 0 && u == 0);         // states 0..LL-1: the head's slots
      S c2 = ck[s];
      for (i64 a = 0; a < u * C; ++a) c2 = prog.step(c2);
      tape[0] = c2;
      const i64 lim = first ? 1 : LL;
      for (i64 v = 1; v < lim; ++v) {
        c2 = prog.step(c2);
        tape[v] = c2;
      }
      for (i64 vr = 0; vr < LL; ++vr) {
        const i64 i = LL - 1 - vr;
        prog.vjp_step(first ? head[i] : tape[i], adj);
      }
    }
  }
  return K;
}

// the cotangent tally of a broadcast operand: exact f32 sum (TSpec.exact, _reverse.py:1172-1176), one bin per element
struct ExactBins {
  std::vector<i64> w;       // kExactWords per bin
  std::vector<u32> flag;    // per bin: non-finite emit or carry lost
  explicit ExactBins(int nb = 0) : w((size_t)nb * kExactWords, 0), flag(nb, 0) {}
};

// readout of an exact tally (kernel.py:625-628): NaN for a flagged bin, else the correctly rounded sum.
// Counts into stats[3] a bin that overflows f32 without a flag.
static inline void exact_readout(const ExactBins& g, int nb, float* out, i32* stats) {
  for (int b = 0; b < nb; ++b) {
    bool bad = false;
    const float o = exact_read(&g.w[(size_t)b * kExactWords], &bad);
    if (bad && !g.flag[b]) stats[3] += 1;
    out[b] = (g.flag[b] || bad) ? std::numeric_limits<float>::quiet_NaN() : o;
  }
}

static inline void stat_add(i32* stats, int slot, i32 v) {
  std::atomic_ref<i32>(stats[slot]).fetch_add(v, std::memory_order_relaxed);
}

// flush a thread's private exact words into the shared bins: each word added with its carries (kernel.py:644-647)
static inline void exact_flush(const ExactBins& priv, ExactBins& g, int nb, i32* stats) {
  for (int b = 0; b < nb; ++b) {
    bool lost = false;
    for (int j = 0; j < kExactWords; ++j) {
      const i64 q = priv.w[(size_t)b * kExactWords + j];
      if (q) lost = exact_add_word<true>(&g.w[(size_t)b * kExactWords], j, q) || lost;
    }
    if (lost || priv.flag[b]) {
      if (lost) stat_add(stats, 3, 1);
      std::atomic_ref<u32>(g.flag[b]).fetch_or(1u, std::memory_order_relaxed);
    }
  }
}

// one exact emit into a thread's private bins (kernel.py sj_emit of an exact tally: flag + count on a lost carry)
static inline void exact_emit_priv(ExactBins& p, int bin, float v, i32* stats) {
  if (exact_emit<false>(&p.w[(size_t)bin * kExactWords], v)) {
    stat_add(stats, 3, 1);
    p.flag[bin] = 1u;
  }
}

}  // namespace orc
