// Launch helpers shared by the launcher translation units (launch_*.cu):
// per-CTA shapes of the pass kernels, the once-per-device shared-memory
// opt-in and the stale-error handling around launches. The launchers are
// split over several files so that the template instantiations compile in
// parallel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "plan.h"

namespace ferrum {
namespace launch_detail {

constexpr int kRowsThreads = 256;   // batched rows: 256 threads per CTA up to N = 4096
// Sizes that use fft_rows_pf_kernel (prefetch into the exchange buffer): the
// sizes with 32 values per thread, where one or two CTAs fill an SM and the
// load phase is otherwise exposed (per 2 GiB: N = 16384 0.99 -> 0.85 ms,
// N = 8192 0.79 -> 0.73 ms); with 16 values per thread (N <= 4096, four or
// more CTAs per SM) it measured slower.
constexpr bool rows_pf_enabled(int log_n) { return log_n == 13 || log_n == 14; }
constexpr int kColsThreads = 512;   // strided passes: up to 16 columns / rows per CTA

constexpr int rows_fpb(int log_n) {
  return (plan_log_p(log_n) == log_n || (1 << (log_n - plan_log_p(log_n))) <= kRowsThreads)
             ? kRowsThreads / (1 << (log_n - plan_log_p(log_n)))
             : 1;
}
constexpr int cols_fpb(int log_n, int threads = kColsThreads) {
  // clamp(threads / T, 1, 16)
  return (threads >> (log_n - plan_log_p(log_n))) < 1
             ? 1
             : ((threads >> (log_n - plan_log_p(log_n))) > 16
                    ? 16
                    : (threads >> (log_n - plan_log_p(log_n))));
}
// The SFU-twiddle column passes of the multi-pass 1D transform are latency-
// bound (their block barriers keep a CTA's warps in step); 256-thread CTAs,
// more of them per SM and out of step, measured 2-3 % faster at 2^18 and 2^19
// and level elsewhere, although N1 = 1024 then reads 32-byte row segments.
constexpr int kSfuColsThreads = 256;

// Raise the dynamic shared-memory limit once per (kernel, device). `done` is
// a per-instantiation flag word owned by the caller (one bit per device).
template <class K>
cudaError_t ensure_smem(K kernel, size_t bytes, std::atomic<uint64_t>& done) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Every launch below is followed by cudaGetLastError(), which reports the
// last error of any runtime call in the process. Consuming an earlier,
// unrelated error (a failed lookup or allocation by the caller) first keeps it
// from being reported as a failure of this launch; sticky errors persist
// and are still reported.
inline void clear_stale_error() { (void)cudaGetLastError(); }

}  // namespace launch_detail
}  // namespace ferrum

// Switch cases over the compiled transform lengths.
#define FERRUM_CASE_2_14(X) \
  X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)
#define FERRUM_CASE_4_14(X) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)
