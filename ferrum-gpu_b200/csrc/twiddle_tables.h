// Host-side construction of the twiddle tables (shared by the runtime and the
// CPU emulator in the test suite).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <vector>

#include "plan.h"

namespace ferrum {

// exp(-2 pi i e / M) in double precision, rounded once to float.
inline float2 root_of_unity(int64_t e, int64_t m) {
  const double a = -2.0 * M_PI * ((double)e / (double)m);
  return make_float2((float)cos(a), (float)sin(a));
}

// Stage tables of a length-2^log_n plan with 2^lp values per thread
// (default plan_log_p(log_n)), concatenated in stage order (layout
// documented in plan.h).
inline void append_stage_tables(std::vector<float2>& out, int log_n, int lp = -1) {
  if (lp < 0) lp = plan_log_p(log_n);
  const int stages = plan_num_stages(log_n, lp);
  for (int s = 1; s < stages; ++s) {
    const int lr = plan_log_radix(log_n, lp, s);
    const int64_t r_count = (int64_t)1 << lr;
    const int64_t ns = (int64_t)1 << plan_log_ns(lp, s);
    for (int64_t r = 1; r < r_count; ++r)
      for (int64_t k = 0; k < ns; ++k) out.push_back(root_of_unity(r * k, ns * r_count));
  }
}

// Two-level twiddle tables of modulus M = 2^log_m (used by the pass kernels'
// fused twiddle multiply): LO[e] = W_M^e for e < min(M, 2^kFourStepLoBits),
// HI[h] = W_M^(h * 2^kFourStepLoBits) for h < max(1, M / 2^kFourStepLoBits),
// so W_M^e = HI[e >> kFourStepLoBits] * LO[e mod 2^kFourStepLoBits].
inline void append_four_step_tables(std::vector<float2>& lo, std::vector<float2>& hi, int log_m) {
  const int64_t m = (int64_t)1 << log_m;
  const int64_t lo_n = m < ((int64_t)1 << kFourStepLoBits) ? m : ((int64_t)1 << kFourStepLoBits);
  const int64_t hi_n = m >> kFourStepLoBits ? (m >> kFourStepLoBits) : 1;
  for (int64_t e = 0; e < lo_n; ++e) lo.push_back(root_of_unity(e, m));
  for (int64_t h = 0; h < hi_n; ++h) hi.push_back(root_of_unity(h << kFourStepLoBits, m));
}

}  // namespace ferrum
