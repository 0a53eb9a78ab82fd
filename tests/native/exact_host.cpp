// Host build of the backend's exact f32 sum (tallymap_b200/csrc/tm_exact.h, the same source the kernels include),
// exported for tests/test_exact_host.py: the word arithmetic and the readout checked on the CPU against the golden
// known answers and against Python's integer rounding of arbitrary word states.
#include <cstdint>

#include "../../tallymap_b200/csrc/tm_exact.h"

extern "C" {

// words: n_bins x 5 int64, flags: n_bins u32 (both zeroed by the caller); out-of-range bins are skipped
void tmx_scatter(const float* vals, const int32_t* bins, long long n, int n_bins, int64_t* words, uint32_t* flags) {
  for (long long i = 0; i < n; ++i) {
    const int32_t b = bins[i];
    if (b < 0 || b >= n_bins) continue;
    int64_t* w = words + (long long)b * tmx::kWords;
    if (tmx::add_float([w](int j) -> int64_t& { return w[j]; }, vals[i])) flags[b] = 1u;
  }
}

// the f32 of each bin's words; ovf[b] = 1 when the value overflows f32
void tmx_read(const int64_t* words, int n_bins, float* out, int32_t* ovf) {
  for (int b = 0; b < n_bins; ++b) {
    bool o = false;
    out[b] = tmx::read(words + (long long)b * tmx::kWords, &o);
    ovf[b] = o ? 1 : 0;
  }
}

// the addend decomposition of one f32: (j, s0, s1, nonfinite)
void tmx_addend(float v, int32_t* j, int64_t* s0, int64_t* s1, int32_t* nonfinite) {
  const tmx::Addend a = tmx::addend(v);
  *j = a.j;
  *s0 = a.s0;
  *s1 = a.s1;
  *nonfinite = a.nonfinite ? 1 : 0;
}

}
