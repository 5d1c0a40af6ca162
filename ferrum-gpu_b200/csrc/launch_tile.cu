// Launchers of the persistent tile kernels (fft_tile_kernels.cuh) and the
// host-side tensor maps they read.
//
// Each launcher checks the layout conditions its kernel relies on (unit
// column strides, whole tiles, 16-byte aligned buffers and row pitches, TMA
// coordinates that fit in 32 bits) and returns cudaErrorNotSupported when
// one fails, so that the caller runs the plain kernel of the same pass
// instead. A tensor map is encoded on the host at every launch (a few
// microseconds) from the buffer pointers of that launch.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "fft_launch.h"
#include "fft_tile_kernels.cuh"
#include "launch_common.cuh"
#include "passes.h"

namespace ferrum {
namespace {

using namespace launch_detail;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      (void)cudaGetLastError();
  });
  return fn;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// 2D map of 8-byte elements over [base, base + rows*ld), rows of `ld`
// elements, box {box_x, box_y}.
cudaError_t encode_map(CUtensorMap* map, const void* base, int64_t ld, int64_t rows, int box_x,
                       int box_y) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (fn == nullptr) return cudaErrorNotSupported;
  if (!aligned16(base) || (ld * 8) % 16 != 0 || rows < 1 || rows >= ((int64_t)1 << 31) ||
      ld >= ((int64_t)1 << 31))
    return cudaErrorNotSupported;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 8};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_INT64, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorNotSupported;
}

// Rows of a 2D view with pitch `ld` that cover every element a strided pass
// touches: offsets o*so + j*sj + c + e*ld.
int64_t view_rows(const PassArgs& a, int log_n, int64_t so, int64_t sj, int64_t ld) {
  const int64_t ncols = (int64_t)1 << a.log_w, nj = (int64_t)1 << a.log_j;
  const int64_t no = a.nfft >> (a.log_w + a.log_j);
  const int64_t last = (no - 1) * so + (nj - 1) * sj + (ncols - 1) + (((int64_t)1 << log_n) - 1) * ld;
  return last / ld + 1;
}

// Column tiles need unit column strides, whole tiles, and tile origins on
// whole rows of the view (so the TMA x coordinate is the column).
bool cols_layout_ok(const PassArgs& a, int w, bool out_side) {
  if (a.in_c != 1 || a.out_c != 1 || (((int64_t)1 << a.log_w) % w) != 0) return false;
  if (a.in_o % a.in_e != 0 || a.in_j % a.in_e != 0) return false;
  if (out_side && (a.out_o % a.out_e != 0 || a.out_j % a.out_e != 0)) return false;
  return true;
}

template <class K>
cudaError_t resident_grid(K kernel, int threads, size_t smem, int64_t ntiles, int& grid) {
  int dev = 0, per_sm = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int64_t g = (int64_t)(per_sm < 1 ? 1 : per_sm) * sms;
  grid = (int)(ntiles < g ? ntiles : g);
  return cudaSuccess;
}

template <int L, int LP, int W, bool CI, int TW>
cudaError_t cols_prefetch_impl(const float2* in, float2* out, const float2* tw, const PassArgs& a,
                               cudaStream_t s) {
  using C = ColsTileCfg<L, LP, W>;
  auto k = fft_cols_tile_kernel<L, LP, W, CI, false, TW, kPfTensor>;
  static std::atomic<uint64_t> smem_done{0};
  if (!cols_layout_ok(a, W, false)) return cudaErrorNotSupported;
  CUtensorMap map;
  cudaError_t e = encode_map(&map, in, a.in_e, view_rows(a, L, a.in_o, a.in_j, a.in_e), W,
                             tile_box_rows(L));
  if (e != cudaSuccess) return e;
  if ((e = ensure_smem(k, C::SMEM_BYTES, smem_done)) != cudaSuccess) return e;
  const int64_t ntiles = a.nfft / W;
  int grid = 0;
  if ((e = resident_grid(k, C::THREADS, C::SMEM_BYTES, ntiles, grid)) != cudaSuccess) return e;
  clear_stale_error();
  k<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, a, ntiles, map);
  return cudaGetLastError();
}

template <int L, int W, bool CI, int TW>
cudaError_t cols_tma_impl(const float2* in, float2* out, const float2* tw, const PassArgs& a,
                          int* err, cudaStream_t s) {
  constexpr int LP = plan_log_p(L);
  using C = TmaTileCfg<L, LP, W>;
  auto k = fft_cols_tma_kernel<L, LP, W, CI, false, TW>;
  static std::atomic<uint64_t> smem_done{0};
  if (err == nullptr || !cols_layout_ok(a, W, true)) return cudaErrorNotSupported;
  CUtensorMap in_map, out_map;
  cudaError_t e = encode_map(&in_map, in, a.in_e, view_rows(a, L, a.in_o, a.in_j, a.in_e), W,
                             C::BOX_ROWS);
  if (e == cudaSuccess)
    e = encode_map(&out_map, out, a.out_e, view_rows(a, L, a.out_o, a.out_j, a.out_e), W,
                   C::BOX_ROWS);
  if (e != cudaSuccess) return e;
  if ((e = ensure_smem(k, C::SMEM_BYTES, smem_done)) != cudaSuccess) return e;
  const int64_t ntiles = a.nfft / W;
  int grid = 0;
  if ((e = resident_grid(k, C::THREADS, C::SMEM_BYTES, ntiles, grid)) != cudaSuccess) return e;
  clear_stale_error();
  k<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(tw, a, ntiles, in_map, out_map, err);
  return cudaGetLastError();
}

// Rows-transposed tiles: whole tiles, 16-byte aligned row starts.
bool rows_t_layout_ok(const float2* in, const RowsTArgs& a, int w) {
  return (((int64_t)1 << a.log_w) % w) == 0 && aligned16(in) && a.in_c % 2 == 0 &&
         a.in_o % 2 == 0 && a.in_j % 2 == 0;
}

template <int L, int LP, int W, bool CI, bool CO>
cudaError_t rows_t_prefetch_impl(const float2* in, float2* out, const float2* tw,
                                 const RowsTArgs& a, cudaStream_t s) {
  using C = RowsTTileCfg<L, LP, W>;
  auto k = fft_rows_t_tile_kernel<L, LP, W, CI, CO, kPfThreads>;
  static std::atomic<uint64_t> smem_done{0};
  if (!rows_t_layout_ok(in, a, W)) return cudaErrorNotSupported;
  cudaError_t e = ensure_smem(k, C::SMEM_BYTES, smem_done);
  if (e != cudaSuccess) return e;
  const int64_t ntiles = a.nfft / W;
  int grid = 0;
  if ((e = resident_grid(k, C::THREADS, C::SMEM_BYTES, ntiles, grid)) != cudaSuccess) return e;
  clear_stale_error();
  k<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(in, out, tw, a, ntiles);
  return cudaGetLastError();
}

template <int L, int W, bool CI, bool CO>
cudaError_t rows_t_tma_impl(const float2* in, float2* out, const float2* tw, const RowsTArgs& a,
                            cudaStream_t s) {
  constexpr int LP = plan_log_p(L);
  using C = TmaTileCfg<L, LP, W>;
  auto k = fft_rows_t_tma_kernel<L, LP, W, CI, CO>;
  static std::atomic<uint64_t> smem_done{0};
  if (!rows_t_layout_ok(in, a, W) || a.out_o % a.out_e != 0 || a.out_j % a.out_e != 0)
    return cudaErrorNotSupported;
  // Output element (o, j, c, k) at o*out_o + j*out_j + c + k*out_e.
  const int64_t nc = (int64_t)1 << a.log_w, nj = (int64_t)1 << a.log_j;
  const int64_t no = a.nfft >> (a.log_w + a.log_j);
  const int64_t last = (no - 1) * a.out_o + (nj - 1) * a.out_j + (nc - 1) +
                       (((int64_t)1 << L) - 1) * a.out_e;
  CUtensorMap map;
  cudaError_t e = encode_map(&map, out, a.out_e, last / a.out_e + 1, W, C::BOX_ROWS);
  if (e != cudaSuccess) return e;
  if ((e = ensure_smem(k, C::SMEM_BYTES, smem_done)) != cudaSuccess) return e;
  const int64_t ntiles = a.nfft / W;
  int grid = 0;
  if ((e = resident_grid(k, C::THREADS, C::SMEM_BYTES, ntiles, grid)) != cudaSuccess) return e;
  clear_stale_error();
  k<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(in, tw, a, ntiles, map);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pass_tile(TileMode mode, int w, int log_p, int log_n, bool conj_in,
                             bool conj_out, bool tw, const float2* in, float2* out,
                             const float2* stage_tw, const PassArgs& a, int* err,
                             cudaStream_t stream) {
  // Compiled: the column passes of the 2^19..2^23 plans (SFU twiddle, no
  // conjugated output).
  if (conj_out || !tw || !a.tw_sfu || stage_tw == nullptr) return cudaErrorNotSupported;
  if (mode == TileMode::Prefetch && w == 16 && log_p == 5) {
    if (log_n == 9)
      return conj_in ? cols_prefetch_impl<9, 5, 16, true, 2>(in, out, stage_tw, a, stream)
                     : cols_prefetch_impl<9, 5, 16, false, 2>(in, out, stage_tw, a, stream);
    if (log_n == 10)
      return conj_in ? cols_prefetch_impl<10, 5, 16, true, 2>(in, out, stage_tw, a, stream)
                     : cols_prefetch_impl<10, 5, 16, false, 2>(in, out, stage_tw, a, stream);
  }
  if (mode == TileMode::Tma && w == 4 && log_n == 11 && log_p == 4)
    return conj_in ? cols_tma_impl<11, 4, true, 2>(in, out, stage_tw, a, err, stream)
                   : cols_tma_impl<11, 4, false, 2>(in, out, stage_tw, a, err, stream);
  return cudaErrorNotSupported;
}

template <int L, int LP, int W>
cudaError_t rows_t_prefetch_dispatch(bool ci, bool co, const float2* in, float2* out,
                                     const float2* tw, const RowsTArgs& a, cudaStream_t s) {
  if (ci) return rows_t_prefetch_impl<L, LP, W, true, false>(in, out, tw, a, s);
  if (co) return rows_t_prefetch_impl<L, LP, W, false, true>(in, out, tw, a, s);
  return rows_t_prefetch_impl<L, LP, W, false, false>(in, out, tw, a, s);
}

template <int L, int W>
cudaError_t rows_t_tma_dispatch(bool ci, bool co, const float2* in, float2* out, const float2* tw,
                                const RowsTArgs& a, cudaStream_t s) {
  if (ci) return rows_t_tma_impl<L, W, true, false>(in, out, tw, a, s);
  if (co) return rows_t_tma_impl<L, W, false, true>(in, out, tw, a, s);
  return rows_t_tma_impl<L, W, false, false>(in, out, tw, a, s);
}

cudaError_t launch_rows_t_tile(TileMode mode, int w, int log_p, int log_n, bool conj_in,
                               bool conj_out, const float2* in, float2* out, const float2* tw,
                               const RowsTArgs& a, cudaStream_t stream) {
  // Compiled: the last passes of the 2^19..2^23 plans and both passes of the
  // 2D plans for N = 1024..4096; no pass conjugates both ways.
  if ((conj_in && conj_out) || tw == nullptr) return cudaErrorNotSupported;
  if (mode == TileMode::Prefetch && w == 8) {
    if (log_n == 10 && log_p == 5)
      return rows_t_prefetch_dispatch<10, 5, 8>(conj_in, conj_out, in, out, tw, a, stream);
    if (log_n == 11 && log_p == 4)
      return rows_t_prefetch_dispatch<11, 4, 8>(conj_in, conj_out, in, out, tw, a, stream);
  }
  if (mode == TileMode::Tma && w == 4 && log_n == 12 && log_p == 4)
    return rows_t_tma_dispatch<12, 4>(conj_in, conj_out, in, out, tw, a, stream);
  return cudaErrorNotSupported;
}

}  // namespace ferrum
