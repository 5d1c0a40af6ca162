// Launchers of the contiguous-row kernels (fft_rows_kernel, fft_rows_pf_kernel).
#include <atomic>

#include "fft_kernels.cuh"
#include "fft_launch.h"
#include "launch_common.cuh"
#include "fft_rows_tma.cuh"
#include "passes.h"

namespace ferrum {
namespace {

using namespace launch_detail;

template <int LOGN, bool CI, bool CO>
cudaError_t rows_impl(const float2* in, float2* out, const float2* tw, int64_t nfft, float scale,
                      int log_block, int64_t block_rows, cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = rows_fpb(LOGN);
  using C = RowsCfg<LOGN, LOGP, FPB, CI, CO>;
  auto k = fft_rows_kernel<LOGN, LOGP, FPB, CI, CO>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  const int64_t blocks = ceil_div(nfft, FPB);
  clear_stale_error();
  k<<<(unsigned)blocks, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, nfft, scale, log_block,
                                                        block_rows);
  return cudaGetLastError();
}

// Persistent rows kernel prefetching into its own exchange buffer
// (fft_rows_tma.cuh, fft_rows_pf_kernel).
template <int LOGN, bool CI, bool CO>
cudaError_t rows_pf_impl(const float2* in, float2* out, const float2* tw, int64_t nfft,
                         float scale, int* err, cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = rows_fpb(LOGN);
  using C = RowsPfCfg<LOGN, LOGP, FPB, CI, CO>;
  auto k = fft_rows_pf_kernel<LOGN, LOGP, FPB, CI, CO>;
  static std::atomic<uint64_t> smem_done{0};
  static std::atomic<int> grid_cache[64];
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  int resident = grid_cache[dev & 63].load(std::memory_order_relaxed);
  if (resident == 0) {
    int per_sm = 0, sms = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, C::THREADS, C::SMEM_BYTES)) !=
        cudaSuccess)
      return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return e;
    resident = (per_sm < 1 ? 1 : per_sm) * sms;
    grid_cache[dev & 63].store(resident, std::memory_order_relaxed);
  }
  const int64_t tiles = ceil_div(nfft, FPB);
  const int64_t grid = tiles < resident ? tiles : resident;
  clear_stale_error();
  k<<<(unsigned)grid, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, nfft, scale, err);
  return cudaGetLastError();
}

template <int LOGN>
cudaError_t rows_dispatch(bool ci, bool co, const float2* in, float2* out, const float2* tw,
                          int64_t nfft, float scale, int lb, int64_t br, int* err, cudaStream_t s) {
  if constexpr (rows_pf_enabled(LOGN)) {
    if (err != nullptr && lb >= LOGN && ((uintptr_t)in & 15u) == 0) {
      if (ci && co) return rows_pf_impl<LOGN, true, true>(in, out, tw, nfft, scale, err, s);
      if (ci) return rows_pf_impl<LOGN, true, false>(in, out, tw, nfft, scale, err, s);
      if (co) return rows_pf_impl<LOGN, false, true>(in, out, tw, nfft, scale, err, s);
      return rows_pf_impl<LOGN, false, false>(in, out, tw, nfft, scale, err, s);
    }
  }
  if (ci && co) return rows_impl<LOGN, true, true>(in, out, tw, nfft, scale, lb, br, s);
  if (ci) return rows_impl<LOGN, true, false>(in, out, tw, nfft, scale, lb, br, s);
  if (co) return rows_impl<LOGN, false, true>(in, out, tw, nfft, scale, lb, br, s);
  return rows_impl<LOGN, false, false>(in, out, tw, nfft, scale, lb, br, s);
}

}  // namespace

cudaError_t launch_rows(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                        const float2* tw, int64_t nfft, float scale, cudaStream_t stream,
                        int log_block, int* err_flag, int64_t block_rows) {
  if (log_block < 0 || log_block > log_n) log_block = log_n;
  if (block_rows <= 0) block_rows = nfft;
  switch (log_n) {
#define X(L) \
  case L:    \
    return rows_dispatch<L>(conj_in, conj_out, in, out, tw, nfft, scale, log_block, block_rows, \
                            err_flag, stream);
    FERRUM_CASE_2_14(X)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace ferrum
