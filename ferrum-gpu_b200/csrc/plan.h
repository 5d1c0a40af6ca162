// Radix plans shared by the host runtime and the device kernels.
//
// A length-N = 2^LOGN transform runs inside one thread group as a Stockham
// auto-sort FFT: every thread owns P = 2^LOGP complex values, the group has
// T = N/P threads, and the stages use radix P except an optional final
// stage of radix 2^(LOGN mod LOGP). Stage s has NS(s) = P^s (the product of
// the radices before it) and, for s >= 1, reads the twiddles
//   W_{NS*R}^{r*k},  r in [1, R), k in [0, NS)
// from a table laid out [(r-1)*NS + k]; the stage tables are concatenated in
// stage order. The reference builds its radix-2/4/8/16 tables in
// crates/ferrum-gpu-fft/src/twiddles.rs:10-104; these tables hold the same
// roots of unity, computed in double precision and rounded once to float.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define FERRUM_HD __host__ __device__
#else
#define FERRUM_HD
#endif

namespace ferrum {

// Lengths from 2^kLogP32From up give each thread 32 values (radix-32 stages):
// fewer stages, exchanges and threads per transform where one transform
// fills an SM.
constexpr int kLogP32From = 13;

// Elements owned by one thread: N below 16, 32 from 2^kLogP32From, else 16.
FERRUM_HD constexpr int plan_log_p(int log_n) {
  return log_n < 4 ? log_n : (log_n >= kLogP32From ? 5 : 4);
}

FERRUM_HD constexpr int plan_num_stages(int log_n, int log_p) {
  return log_n / log_p + ((log_n % log_p) ? 1 : 0);
}

FERRUM_HD constexpr int plan_log_radix(int log_n, int log_p, int s) {
  return (s < log_n / log_p) ? log_p : (log_n % log_p);
}

// log2 of NS for stage s: every stage before s has radix P.
FERRUM_HD constexpr int plan_log_ns(int log_p, int s) { return s * log_p; }

// Complex entries in stage s's twiddle table (0 for stage 0).
FERRUM_HD constexpr int64_t plan_stage_tw_count(int log_n, int log_p, int s) {
  return s == 0 ? 0
                : (int64_t)((1 << plan_log_radix(log_n, log_p, s)) - 1) *
                      ((int64_t)1 << plan_log_ns(log_p, s));
}

FERRUM_HD constexpr int64_t plan_stage_tw_offset(int log_n, int log_p, int s) {
  return s <= 1 ? 0
                : plan_stage_tw_offset(log_n, log_p, s - 1) +
                      plan_stage_tw_count(log_n, log_p, s - 1);
}

FERRUM_HD constexpr int64_t plan_tw_count(int log_n, int log_p) {
  return plan_stage_tw_offset(log_n, log_p, plan_num_stages(log_n, log_p) - 1) +
         plan_stage_tw_count(log_n, log_p, plan_num_stages(log_n, log_p) - 1);
}

// Lengths whose plan takes 16 values per thread but for which the device also
// holds stage tables with 32 (tile kernels that run them with 32 values per
// thread: fewer exchanges, measured faster at these lengths).
FERRUM_HD constexpr bool tile_p32_table(int log_n) { return log_n >= 9 && log_n <= 12; }

// Largest single-pass length (one HBM read + one HBM write per element).
constexpr int kMaxSinglePassLogN = 14;
// Largest 1D length (multi-pass; the pass splits are in passes.h).
constexpr int kMaxLogN = 26;
// Split of the four-step twiddle exponent: W_N^e = HI[e >> 12] * LO[e & 4095].
constexpr int kFourStepLoBits = 12;

}  // namespace ferrum
