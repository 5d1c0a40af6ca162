// Launchers of the strided pass kernel (fft_pass_kernel).
#include <atomic>

#include "fft_kernels.cuh"
#include "fft_launch.h"
#include "launch_common.cuh"
#include "passes.h"

namespace ferrum {
namespace {

using namespace launch_detail;

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

}  // namespace

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

}  // namespace ferrum
