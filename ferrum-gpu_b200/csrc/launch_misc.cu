// Launchers of the fused column kernel, the transposed-row kernel, the
// distributed-transform kernels and the split-layout / elementwise kernels.
#include <atomic>

#include "dist_kernels.cuh"
#include "fft_kernels.cuh"
#include "fft_launch.h"
#include "launch_common.cuh"
#include "layout_kernels.cuh"
#include "passes.h"

namespace ferrum {
namespace {

using namespace launch_detail;

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

template <int LOGN, bool CI, bool CO>
cudaError_t rows_t_impl(const float2* in, float2* out, const float2* tw, const RowsTArgs& a,
                        cudaStream_t s) {
  constexpr int LOGP = plan_log_p(LOGN);
  constexpr int FPB = cols_fpb(LOGN);
  using C = RowsTCfg<LOGN, LOGP, FPB, CI, CO>;
  auto k = fft_rows_t_kernel<LOGN, LOGP, FPB, CI, CO>;
  static std::atomic<uint64_t> smem_done{0};
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  const int64_t blocks = ceil_div(a.nfft, FPB);
  clear_stale_error();
  k<<<(unsigned)blocks, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, a);
  return cudaGetLastError();
}

// A pass never both conjugates its input and its output.
template <int LOGN>
cudaError_t rows_t_dispatch(bool ci, bool co, const float2* in, float2* out, const float2* tw,
                            const RowsTArgs& a, cudaStream_t s) {
  if (ci && co) return cudaErrorInvalidValue;
  if (ci) return rows_t_impl<LOGN, true, false>(in, out, tw, a, s);
  if (co) return rows_t_impl<LOGN, false, true>(in, out, tw, a, s);
  return rows_t_impl<LOGN, false, false>(in, out, tw, a, s);
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

cudaError_t launch_rows_t(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                          const float2* tw, const RowsTArgs& args, cudaStream_t stream) {
  switch (log_n) {
#define X(L) \
  case L:    \
    return rows_t_dispatch<L>(conj_in, conj_out, in, out, tw, args, stream);
    X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)
#undef X
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace ferrum
