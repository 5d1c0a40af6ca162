// Allocation-free 1D entry point: ferrum_fft_1d_c2c_pow2_noalloc.
//
// Lengths above 2^14 run the multi-pass transform (two passes up to 2^23,
// three from 2^24), whose passes keep an N*batch intermediate in scratch
// memory; with at most 2^22 values here, only the two-pass plans (2^15..2^22)
// reach the scratch. ferrum_fft_1d_c2c_pow2 takes that scratch
// from a stream-ordered pool and ferrum_fft_1d_c2c_pow2_ws from the caller;
// this entry point instead uses one file-scope __device__ array, so the call
// itself never allocates device memory. It exists for callers that cannot
// allocate at call time: applications whose device memory is owned by their
// own allocator (a caching allocator or a pool reserved at start-up, where a
// library allocation would fail or eat into a budget), and latency-critical
// loops where an allocation may block in the driver and stall other streams.
//
// The scratch holds kNoAllocScratchElems complex64 values (32 MiB), so
// N * batch must not exceed 2^22 for lengths above 2^14; larger requests are
// rejected with FERRUM_ERR_INVALID_ARG. Every GPU that loads this module keeps
// the 32 MiB until the process exits. Lengths up to 2^14 need no scratch and
// run the same single-pass kernel as ferrum_fft_1d_c2c_pow2.
//
// The array is shared by every call on a device and keeps the last call's
// contents. Nothing in it needs to start at zero: every pass reads only
// scratch elements that an earlier pass of the same call wrote. Calls whose kernels overlap on the
// GPU (different streams, no ordering between them) race on the array.
//
// The host-side name of a __device__ array is not a device address, so the
// first call on each device looks the address up with cudaGetSymbolAddress
// while that device is current, and caches it; a failed lookup is not
// cached, so a later call tries again. That set-up happens inside the first
// call, so the first call on a device should come before any stream capture.
// cudaDeviceReset destroys the module's device copy: a process that resets a
// device must not call this entry point on it again.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "runtime.h"

namespace ferrum {
namespace {

constexpr size_t kNoAllocScratchElems = size_t(1) << 22;
constexpr size_t kNoAllocScratchBytes = kNoAllocScratchElems * sizeof(float2);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float2 g_noalloc_scratch[kNoAllocScratchElems];

std::mutex g_scratch_mu;
float2* g_scratch_address[kMaxDevices] = {};  // guarded by g_scratch_mu; NULL until looked up

// Device address of the scratch on `ordinal`, which must be the current device.
ferrum_status scratch_address(int ordinal, float2** out) {
  if (ordinal < 0 || ordinal >= kMaxDevices)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2_noalloc: device ordinal " +
                                                 std::to_string(ordinal) + " out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_address[ordinal] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                        "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch_address[ordinal] = static_cast<float2*>(p);
  }
  *out = g_scratch_address[ordinal];
  return FERRUM_OK;
}

}  // namespace
}  // namespace ferrum

using namespace ferrum;

extern "C" ferrum_status ferrum_fft_1d_c2c_pow2_noalloc(ferrum_device* dev, const void* in_dev,
                                                        void* out_dev, int log_n, size_t batch,
                                                        int direction, int normalize,
                                                        void* stream) {
  clear_error();
  if (dev == nullptr || dev->tables == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "device handle is NULL or destroyed");
  if (log_n < 2 || log_n > kMaxLogN)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2_noalloc: log_n must be in [2, 26], got " +
                                                 std::to_string(log_n));
  if (ferrum_status s = check_elements(log_n, batch, "fft_1d_c2c_pow2_noalloc")) return s;
  if (direction != 1 && direction != -1)
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "fft_1d_c2c_pow2_noalloc: direction must be +1 (forward) or -1 (inverse), got " +
                         std::to_string(direction));
  if (in_dev == nullptr || out_dev == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2_noalloc: in/out is NULL");
  if (((uintptr_t)in_dev & 7u) || ((uintptr_t)out_dev & 7u))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2_noalloc: in/out must be 8-byte aligned");
  const size_t need = workspace_1d_bytes(log_n, (int64_t)batch);
  if (need > kNoAllocScratchBytes)
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "fft_1d_c2c_pow2_noalloc: N * batch = " + std::to_string(need / sizeof(float2)) +
                         " complex values exceed the static scratch of " +
                         std::to_string(kNoAllocScratchElems) + " (" +
                         std::to_string(kNoAllocScratchBytes) +
                         " bytes); use ferrum_fft_1d_c2c_pow2 or _ws for larger transforms");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  float2* ws = nullptr;
  if (need > 0) {
    if (ferrum_status s = scratch_address(dev->ordinal, &ws)) return s;
  }
  return enqueue_1d(dev, (const float2*)in_dev, (float2*)out_dev, log_n, (int64_t)batch, direction,
                    normalize != 0, ws, (cudaStream_t)stream);
}
