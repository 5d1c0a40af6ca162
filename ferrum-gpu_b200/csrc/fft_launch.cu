// Template dispatch from runtime (log_n, direction flags) to the pass kernels.
#include <atomic>

#include "dist_kernels.cuh"
#include "fft_kernels.cuh"
#include "fft_launch.h"
#include "fft_rows_tma.cuh"
#include "layout_kernels.cuh"
#include "passes.h"

namespace ferrum {
namespace {

constexpr int kRowsThreads = 256;   // batched rows: 256 threads per CTA up to N = 4096
// The persistent TMA-prefetch rows kernel (fft_rows_tma.cuh) measured slower
// than fft_rows_kernel on B200 for every N in 32..4096 at 2 GiB (4.87 vs 5.36
// TB/s at N = 4096): the staging copy adds a shared-memory write and read per
// element and costs one resident CTA per SM, and the kernel is bound by the
// L1/shared pipe and issue rate rather than by DRAM latency. It stays off.
constexpr bool kRowsTmaEnabled = false;
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

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Every launch below is followed by cudaGetLastError(), which reports the
// last error of any runtime call in the process. Consuming an earlier,
// unrelated error (a failed lookup or allocation by the caller) first keeps it
// from being reported as a failure of this launch; sticky errors persist
// and are still reported.
inline void clear_stale_error() { (void)cudaGetLastError(); }

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

// Persistent TMA-prefetch variant (fft_rows_tma.cuh): one CTA per resident
// slot, every CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...
template <int LOGN, bool CI, bool CO>
cudaError_t rows_tma_impl(const float2* in, float2* out, const float2* tw, int64_t nfft,
                          float scale, int* err, cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = rows_fpb(LOGN);
  using C = RowsTmaCfg<LOGN, LOGP, FPB, CI, CO>;
  auto k = fft_rows_tma_kernel<LOGN, LOGP, FPB, CI, CO>;
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

template <int LOGN, bool CI, bool CO, int TW>
cudaError_t pass_impl(const float2* in, float2* out, const float2* tw, const PassArgs& a,
                      cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = cols_fpb(LOGN, TW == 2 ? kSfuColsThreads : kColsThreads);
  using C = PassCfg<LOGN, LOGP, FPB, CI, CO, TW>;
  auto k = fft_pass_kernel<LOGN, LOGP, FPB, CI, CO, TW>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  const int64_t blocks = ceil_div(a.nfft, FPB);
  clear_stale_error();
  k<<<(unsigned)blocks, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, a);
  return cudaGetLastError();
}

template <int L1, int L2, int W, int THREADS, int MINB, bool CI, bool CO>
cudaError_t cols_l2_impl(const float2* in, float2* out, float2* ws, const float2* tw1,
                         const float2* tw2, const ColsL2Args& a, int64_t slots, cudaStream_t s) {
  using C = ColsL2Cfg<L1, L2, W, THREADS>;
  auto k = fft_cols_l2_kernel<L1, L2, W, THREADS, MINB, CI, CO>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  const int64_t grid = a.tiles < slots ? a.tiles : slots;
  if (grid < 1) return cudaSuccess;
  clear_stale_error();
  k<<<(unsigned)grid, THREADS, C::SMEM_BYTES, s>>>(in, out, ws, tw1, tw2, a);
  return cudaGetLastError();
}

template <int L1, int L2, int W, int THREADS, int MINB>
cudaError_t cols_l2_dispatch(bool ci, bool co, const float2* in, float2* out, float2* ws,
                             const float2* tw1, const float2* tw2, const ColsL2Args& a,
                             int64_t slots, cudaStream_t s) {
  if (ci && co)
    return cols_l2_impl<L1, L2, W, THREADS, MINB, true, true>(in, out, ws, tw1, tw2, a, slots, s);
  if (ci)
    return cols_l2_impl<L1, L2, W, THREADS, MINB, true, false>(in, out, ws, tw1, tw2, a, slots, s);
  if (co)
    return cols_l2_impl<L1, L2, W, THREADS, MINB, false, true>(in, out, ws, tw1, tw2, a, slots, s);
  return cols_l2_impl<L1, L2, W, THREADS, MINB, false, false>(in, out, ws, tw1, tw2, a, slots, s);
}

template <int LOGN, bool CO>
cudaError_t rows_t_impl(const float2* in, float2* out, const float2* tw, const RowsTArgs& a,
                        cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = cols_fpb(LOGN);
  using C = RowsTCfg<LOGN, LOGP, FPB, CO>;
  auto k = fft_rows_t_kernel<LOGN, LOGP, FPB, CO>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  const int64_t blocks = ceil_div(a.nfft, FPB);
  clear_stale_error();
  k<<<(unsigned)blocks, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, a);
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
  if constexpr (kRowsTmaEnabled && LOGN >= 4 && LOGN <= 12) {
    // TMA bulk copies need a 16-byte aligned source; blocked stores keep the
    // plain kernel.
    if (err != nullptr && lb >= LOGN && ((uintptr_t)in & 15u) == 0) {
      if (ci && co) return rows_tma_impl<LOGN, true, true>(in, out, tw, nfft, scale, err, s);
      if (ci) return rows_tma_impl<LOGN, true, false>(in, out, tw, nfft, scale, err, s);
      if (co) return rows_tma_impl<LOGN, false, true>(in, out, tw, nfft, scale, err, s);
      return rows_tma_impl<LOGN, false, false>(in, out, tw, nfft, scale, err, s);
    }
  }
  if (ci && co) return rows_impl<LOGN, true, true>(in, out, tw, nfft, scale, lb, br, s);
  if (ci) return rows_impl<LOGN, true, false>(in, out, tw, nfft, scale, lb, br, s);
  if (co) return rows_impl<LOGN, false, true>(in, out, tw, nfft, scale, lb, br, s);
  return rows_impl<LOGN, false, false>(in, out, tw, nfft, scale, lb, br, s);
}

// Instantiates exactly the combinations pass_flags_supported() allows.
template <int LOGN>
cudaError_t pass_dispatch(bool ci, bool co, bool tw, const float2* in, float2* out,
                          const float2* stw, const PassArgs& a, cudaStream_t s) {
  if (!pass_flags_supported(ci, co, tw)) return cudaErrorInvalidValue;
  if (tw && a.tw_sfu) {
    if constexpr (pass_sfu_supported(LOGN)) {
      if (ci) return pass_impl<LOGN, true, false, 2>(in, out, stw, a, s);
      return pass_impl<LOGN, false, false, 2>(in, out, stw, a, s);
    }
    return cudaErrorInvalidValue;
  }
  if (tw) {
    if (ci) return pass_impl<LOGN, true, false, 1>(in, out, stw, a, s);
    return pass_impl<LOGN, false, false, 1>(in, out, stw, a, s);
  }
  if (ci) return pass_impl<LOGN, true, false, 0>(in, out, stw, a, s);
  if (co) return pass_impl<LOGN, false, true, 0>(in, out, stw, a, s);
  return pass_impl<LOGN, false, false, 0>(in, out, stw, a, s);
}

template <int LOGN>
cudaError_t rows_t_dispatch(bool co, const float2* in, float2* out, const float2* tw,
                            const RowsTArgs& a, cudaStream_t s) {
  if (co) return rows_t_impl<LOGN, true>(in, out, tw, a, s);
  return rows_t_impl<LOGN, false>(in, out, tw, a, s);
}


template <int LOGN, bool CI>
cudaError_t rows_scatter_impl(const float2* in, const PeerPtrs& dst, const float2* tw,
                              int64_t nfft, int log_b, cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = rows_fpb(LOGN);
  using C = RowsCfg<LOGN, LOGP, FPB, CI, false>;
  auto k = fft_rows_scatter_kernel<LOGN, LOGP, FPB, CI>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  clear_stale_error();
  k<<<(unsigned)ceil_div(nfft, FPB), C::THREADS, C::SMEM_BYTES, s>>>(in, dst, tw, nfft, log_b);
  return cudaGetLastError();
}

template <int LOGN, bool CO>
cudaError_t rows_gather_impl(const PeerPtrs& src, float2* out, const float2* tw, int64_t nfft,
                             float scale, int log_b, cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = rows_fpb(LOGN);
  using C = RowsCfg<LOGN, LOGP, FPB, false, CO>;
  auto k = fft_rows_gather_kernel<LOGN, LOGP, FPB, CO>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  clear_stale_error();
  k<<<(unsigned)ceil_div(nfft, FPB), C::THREADS, C::SMEM_BYTES, s>>>(src, out, tw, nfft, scale,
                                                                     log_b);
  return cudaGetLastError();
}

template <int LOGN, bool CI, bool CO>
cudaError_t rows_split_impl(const float* in_re, const float* in_im, float* out_re, float* out_im,
                            const float2* tw, int64_t nfft, float scale, cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = rows_fpb(LOGN);
  using C = RowsCfg<LOGN, LOGP, FPB, CI, CO>;
  auto k = fft_rows_split_kernel<LOGN, LOGP, FPB, CI, CO>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  clear_stale_error();
  k<<<(unsigned)ceil_div(nfft, FPB), C::THREADS, C::SMEM_BYTES, s>>>(in_re, in_im, out_re, out_im,
                                                                     tw, nfft, scale);
  return cudaGetLastError();
}

unsigned elementwise_grid(int64_t n) {
  int64_t g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return (unsigned)(g < 1 ? 1 : g);
}

// out[r * out_ld + p*bw + c] = in[p*in_bs + r*bw + c] for p < nblocks, r < rows,
// c < bw; one thread moves two complex values.
__global__ void __launch_bounds__(256) block_gather_kernel(const float4* __restrict__ in,
                                                           float4* __restrict__ out,
                                                           int64_t nblocks, int64_t rows,
                                                           int64_t bw2, int64_t in_bs2,
                                                           int64_t out_ld2) {
  const int64_t total2 = nblocks * rows * bw2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total2; i += stride) {
    const int64_t c = i % bw2;
    const int64_t r = (i / bw2) % rows;
    const int64_t p = i / (bw2 * rows);
    out[r * out_ld2 + p * bw2 + c] = __ldcs(in + p * in_bs2 + r * bw2 + c);
  }
}

}  // namespace

cudaError_t launch_block_gather(const float2* in, float2* out, int64_t nblocks, int64_t rows,
                                int64_t bw, int64_t in_block_stride, int64_t out_ld,
                                cudaStream_t stream) {
  if (bw % 2 != 0 || in_block_stride % 2 != 0 || out_ld % 2 != 0 || ((uintptr_t)in & 15) ||
      ((uintptr_t)out & 15))
    return cudaErrorInvalidValue;
  const int64_t total2 = nblocks * rows * bw / 2;
  int64_t grid = (total2 + 255) / 256;
  if (grid > 148 * 32) grid = 148 * 32;
  if (grid < 1) grid = 1;
  clear_stale_error();
  block_gather_kernel<<<(unsigned)grid, 256, 0, stream>>>((const float4*)in, (float4*)out, nblocks,
                                                          rows, bw / 2, in_block_stride / 2,
                                                          out_ld / 2);
  return cudaGetLastError();
}

#define FERRUM_CASE_4_14(X) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)

cudaError_t launch_rows_scatter(int log_n, bool conj_in, const float2* in, const PeerPtrs& dst,
                                const float2* tw, int64_t nfft, int log_b, cudaStream_t stream) {
  if (log_b < 1 || log_b > log_n) return cudaErrorInvalidValue;
  switch (log_n) {
#define X(L)                                                                        \
  case L:                                                                           \
    return conj_in ? rows_scatter_impl<L, true>(in, dst, tw, nfft, log_b, stream)   \
                   : rows_scatter_impl<L, false>(in, dst, tw, nfft, log_b, stream);
    FERRUM_CASE_4_14(X)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rows_gather(int log_n, bool conj_out, const PeerPtrs& src, float2* out,
                               const float2* tw, int64_t nfft, float scale, int log_b,
                               cudaStream_t stream) {
  if (log_b < 1 || log_b > log_n) return cudaErrorInvalidValue;
  switch (log_n) {
#define X(L)                                                                                  \
  case L:                                                                                     \
    return conj_out ? rows_gather_impl<L, true>(src, out, tw, nfft, scale, log_b, stream)     \
                    : rows_gather_impl<L, false>(src, out, tw, nfft, scale, log_b, stream);
    FERRUM_CASE_4_14(X)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_peer_block_gather(const PeerPtrs& src, float2* out, int nranks, int64_t rows,
                                     int64_t b, int64_t out_ld, cudaStream_t stream) {
  if (nranks < 1 || nranks > kMaxPeers || b % 2 != 0 || out_ld % 2 != 0 || ((uintptr_t)out & 15))
    return cudaErrorInvalidValue;
  for (int q = 0; q < nranks; ++q)
    if ((uintptr_t)src.p[q] & 15) return cudaErrorInvalidValue;
  const int64_t total2 = (int64_t)nranks * rows * b / 2;
  int64_t grid = (total2 + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  if (grid < 1) grid = 1;
  clear_stale_error();
  peer_block_gather_kernel<<<(unsigned)grid, 256, 0, stream>>>(src, (float4*)out, nranks, rows,
                                                               b / 2, out_ld / 2);
  return cudaGetLastError();
}

cudaError_t launch_dist_barrier(const PeerFlags& flags, int rank, int nranks, uint32_t epoch,
                                uint64_t timeout_ns, int* err, cudaStream_t stream) {
  if (nranks < 1 || nranks > kMaxPeers || rank < 0 || rank >= nranks || err == nullptr)
    return cudaErrorInvalidValue;
  clear_stale_error();
  dist_barrier_kernel<<<1, 32, 0, stream>>>(flags, rank, nranks, epoch, timeout_ns, err);
  return cudaGetLastError();
}

cudaError_t launch_cmul_interleaved(const float2* a, const float2* b, float2* out, int64_t n,
                                    cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  clear_stale_error();
  cmul_interleaved_kernel<<<elementwise_grid(n), 256, 0, stream>>>(a, b, out, n);
  return cudaGetLastError();
}

cudaError_t launch_cmul_split(const float* a_re, const float* a_im, const float* b_re,
                              const float* b_im, float* o_re, float* o_im, int64_t n,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  clear_stale_error();
  cmul_split_kernel<<<elementwise_grid(n), 256, 0, stream>>>(a_re, a_im, b_re, b_im, o_re, o_im, n);
  return cudaGetLastError();
}

cudaError_t launch_deinterleave(const float2* in, float* re, float* im, int64_t n,
                                cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  clear_stale_error();
  deinterleave_kernel<<<elementwise_grid(n), 256, 0, stream>>>(in, re, im, n);
  return cudaGetLastError();
}

cudaError_t launch_interleave(const float* re, const float* im, float2* out, int64_t n,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  clear_stale_error();
  interleave_kernel<<<elementwise_grid(n), 256, 0, stream>>>(re, im, out, n);
  return cudaGetLastError();
}

#define FERRUM_CASE_2_14(X) \
  X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)

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

cudaError_t launch_rows_split(int log_n, bool conj_in, bool conj_out, const float* in_re,
                              const float* in_im, float* out_re, float* out_im, const float2* tw,
                              int64_t nfft, float scale, cudaStream_t stream) {
  switch (log_n) {
#define X(L)                                                                                  \
  case L:                                                                                     \
    if (conj_in && conj_out)                                                                  \
      return rows_split_impl<L, true, true>(in_re, in_im, out_re, out_im, tw, nfft, scale, stream); \
    if (conj_in)                                                                              \
      return rows_split_impl<L, true, false>(in_re, in_im, out_re, out_im, tw, nfft, scale, stream); \
    if (conj_out)                                                                             \
      return rows_split_impl<L, false, true>(in_re, in_im, out_re, out_im, tw, nfft, scale, stream); \
    return rows_split_impl<L, false, false>(in_re, in_im, out_re, out_im, tw, nfft, scale, stream);
    FERRUM_CASE_2_14(X)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pass(int log_n, bool conj_in, bool conj_out, bool tw, const float2* in,
                        float2* out, const float2* stage_tw, const PassArgs& args,
                        cudaStream_t stream) {
  switch (log_n) {
#define X(L) \
  case L:    \
    return pass_dispatch<L>(conj_in, conj_out, tw, in, out, stage_tw, args, stream);
    FERRUM_CASE_2_14(X)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_cols_l2(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                           float2* ws, const float2* tw1, const float2* tw2, const ColsL2Args& a,
                           cudaStream_t stream) {
  if (ws == nullptr || cols_l2_width(log_n) == 0) return cudaErrorInvalidValue;
  const int64_t slots = cols_l2_slots(log_n);
  switch (log_n) {
#define FERRUM_COLS_L2(L)                                                                  \
  case L:                                                                                  \
    return cols_l2_dispatch<L - L / 2, L / 2, cols_l2_width(L), cols_l2_threads(L),        \
                            cols_l2_ctas_per_sm(L)>(conj_in, conj_out, in, out, ws, tw1, tw2, a, \
                                                    slots, stream);
    FERRUM_COLS_L2(12)
#undef FERRUM_COLS_L2
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rows_t(int log_n, bool conj_out, const float2* in, float2* out,
                          const float2* tw, const RowsTArgs& args, cudaStream_t stream) {
  switch (log_n) {
#define X(L) \
  case L:    \
    return rows_t_dispatch<L>(conj_out, in, out, tw, args, stream);
    X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace ferrum
