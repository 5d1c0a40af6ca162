// Host-pointer entry points: copy in, transform, copy out.
//
// The reference's call path (crates/ferrum-gpu-py/src/lib.rs:86-250) copies
// the whole input with one synchronous H2D, launches one kernel, copies the
// whole output back and then conjugates/scales on the host. Here the batch is
// cut into chunks of whole transforms that rotate over three streams, so the
// H2D of one chunk, the kernels of another and the D2H of a third overlap;
// conjugation and scaling are fused into the kernels. Pageable host memory is
// staged through pinned buffers with multi-threaded memcpy; pinned (or
// device) memory is copied directly.
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <thread>
#include <vector>

#include "runtime.h"

namespace ferrum {
namespace {

constexpr size_t kChunkTarget = 64ull << 20;  // bytes of transform data per chunk

void parallel_memcpy(void* dst, const void* src, size_t bytes) {
  const size_t kMinPerThread = 8ull << 20;
  unsigned hw = std::thread::hardware_concurrency();
  size_t threads = std::min<size_t>(hw ? hw : 1, 8);
  threads = std::min(threads, std::max<size_t>(1, bytes / kMinPerThread));
  if (threads <= 1) {
    memcpy(dst, src, bytes);
    return;
  }
  std::vector<std::thread> pool;
  const size_t per = (bytes + threads - 1) / threads;
  for (size_t t = 0; t < threads; ++t) {
    const size_t off = t * per;
    if (off >= bytes) break;
    const size_t len = std::min(per, bytes - off);
    pool.emplace_back([=] { memcpy((char*)dst + off, (const char*)src + off, len); });
  }
  for (auto& th : pool) th.join();
}

bool is_pinned_or_device(const void* p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeHost || attr.type == cudaMemoryTypeDevice ||
         attr.type == cudaMemoryTypeManaged;
}

ferrum_status ensure_host_resources(ferrum_device* dev, size_t chunk_bytes, size_t ws_bytes,
                                    bool need_pinned) {
  cudaError_t e;
  for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
    if (!dev->host_streams[i]) {
      e = cudaStreamCreateWithFlags(&dev->host_streams[i], cudaStreamNonBlocking);
      if (e != cudaSuccess) return cuda_error(e, "cudaStreamCreate");
    }
  }
  if (chunk_bytes > dev->host_chunk_bytes) {
    for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
      if (dev->host_dbuf[i]) cudaFree(dev->host_dbuf[i]);
      if (dev->host_pin_in[i]) cudaFreeHost(dev->host_pin_in[i]);
      if (dev->host_pin_out[i]) cudaFreeHost(dev->host_pin_out[i]);
      dev->host_dbuf[i] = dev->host_pin_in[i] = dev->host_pin_out[i] = nullptr;
    }
    dev->host_chunk_bytes = 0;
    for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
      e = cudaMalloc(&dev->host_dbuf[i], chunk_bytes);
      if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(host-path chunk)");
    }
    dev->host_chunk_bytes = chunk_bytes;
  }
  if (need_pinned && dev->host_pin_in[0] == nullptr) {
    for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
      e = cudaMallocHost(&dev->host_pin_in[i], dev->host_chunk_bytes);
      if (e != cudaSuccess) return cuda_error(e, "cudaMallocHost(staging)");
      e = cudaMallocHost(&dev->host_pin_out[i], dev->host_chunk_bytes);
      if (e != cudaSuccess) return cuda_error(e, "cudaMallocHost(staging)");
    }
  }
  if (ws_bytes > dev->host_ws_bytes) {
    for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
      if (dev->host_ws[i]) cudaFree(dev->host_ws[i]);
      dev->host_ws[i] = nullptr;
    }
    dev->host_ws_bytes = 0;
    for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
      e = cudaMalloc(&dev->host_ws[i], ws_bytes);
      if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(host-path workspace)");
    }
    dev->host_ws_bytes = ws_bytes;
  }
  return FERRUM_OK;
}

ferrum_status run_host(ferrum_device* dev, const void* in_host, void* out_host, int log_n,
                       size_t batch, int direction, int normalize, int kind) {
  const int64_t n = (int64_t)1 << log_n;
  const size_t unit_elems = kind == 1 ? (size_t)n : (size_t)n * (size_t)n;
  const size_t unit_bytes = unit_elems * sizeof(float2);
  const size_t units_per_chunk = std::max<size_t>(1, kChunkTarget / unit_bytes);
  const size_t chunk_units = std::min(units_per_chunk, batch);
  const size_t chunk_bytes = chunk_units * unit_bytes;
  const size_t ws_bytes = kind == 1 ? workspace_1d_bytes(log_n, (int64_t)chunk_units)
                                    : workspace_2d_bytes(log_n, (int64_t)chunk_units);
  const bool direct_in = is_pinned_or_device(in_host);
  const bool direct_out = is_pinned_or_device(out_host);

  std::lock_guard<std::mutex> lock(dev->host_mu);
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  if (ferrum_status s = ensure_host_resources(dev, chunk_bytes, ws_bytes, !(direct_in && direct_out)))
    return s;

  const int S = ferrum_device::kHostStreams;
  const size_t nchunks = (batch + chunk_units - 1) / chunk_units;
  std::vector<size_t> pending_off(S, 0), pending_bytes(S, 0);
  std::vector<bool> pending(S, false);
  auto finish = [&](int s) -> ferrum_status {
    if (!pending[s]) return FERRUM_OK;
    cudaError_t e = cudaStreamSynchronize(dev->host_streams[s]);
    if (e != cudaSuccess) return cuda_error(e, "host-path stream");
    if (!direct_out)
      parallel_memcpy((char*)out_host + pending_off[s], dev->host_pin_out[s], pending_bytes[s]);
    pending[s] = false;
    return FERRUM_OK;
  };
  ferrum_status status = FERRUM_OK;
  for (size_t c = 0; c < nchunks && status == FERRUM_OK; ++c) {
    const int s = (int)(c % S);
    status = finish(s);
    if (status != FERRUM_OK) break;
    const size_t units = std::min(chunk_units, batch - c * chunk_units);
    const size_t bytes = units * unit_bytes;
    const size_t off = c * chunk_units * unit_bytes;
    const void* src = (const char*)in_host + off;
    cudaStream_t st = dev->host_streams[s];
    if (!direct_in) {
      parallel_memcpy(dev->host_pin_in[s], src, bytes);
      src = dev->host_pin_in[s];
    }
    cudaError_t e = cudaMemcpyAsync(dev->host_dbuf[s], src, bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) {
      status = cuda_error(e, "H2D copy");
      break;
    }
    float2* buf = (float2*)dev->host_dbuf[s];
    if (kind == 1)
      status = enqueue_1d(dev, buf, buf, log_n, (int64_t)units, direction, normalize != 0,
                          (float2*)dev->host_ws[s], st);
    else
      status = enqueue_2d(dev, buf, buf, log_n, (int64_t)units, direction, normalize != 0,
                          (float2*)dev->host_ws[s], st);
    if (status != FERRUM_OK) break;
    void* dst = direct_out ? (char*)out_host + off : dev->host_pin_out[s];
    e = cudaMemcpyAsync(dst, dev->host_dbuf[s], bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) {
      status = cuda_error(e, "D2H copy");
      break;
    }
    pending[s] = true;
    pending_off[s] = off;
    pending_bytes[s] = bytes;
  }
  for (int s = 0; s < S; ++s) {
    ferrum_status fs = finish(s);
    if (status == FERRUM_OK) status = fs;
  }
  if (status == FERRUM_OK) status = check_device_flag(dev);
  return status;
}

}  // namespace
}  // namespace ferrum

using namespace ferrum;

extern "C" {

ferrum_status ferrum_fft_1d_c2c_pow2_host(ferrum_device* dev, const void* in_host,
                                          void* out_host, int log_n, size_t batch,
                                          int direction, int normalize) {
  clear_error();
  if (dev == nullptr || dev->tables == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "device handle is NULL or destroyed");
  if (log_n < 2 || log_n > kMaxLogN)
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "fft_1d_c2c_pow2: log_n must be in [2, 26], got " + std::to_string(log_n));
  if (ferrum_status s = check_elements(log_n, batch, "fft_1d_c2c_pow2")) return s;
  if (direction != 1 && direction != -1)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2: direction must be +1 or -1");
  if (in_host == nullptr || out_host == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2: in/out is NULL");
  return run_host(dev, in_host, out_host, log_n, batch, direction, normalize, 1);
}

ferrum_status ferrum_fft_2d_c2c_pow2_host(ferrum_device* dev, const void* in_host,
                                          void* out_host, int log_n, size_t batch,
                                          int direction, int normalize) {
  clear_error();
  if (dev == nullptr || dev->tables == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "device handle is NULL or destroyed");
  if (log_n < 2 || log_n > kMaxSinglePassLogN)
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "fft_2d_c2c_pow2: log_n must be in [2, 14], got " + std::to_string(log_n));
  if (ferrum_status s = check_elements(2 * log_n, batch, "fft_2d_c2c_pow2")) return s;
  if (direction != 1 && direction != -1)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2: direction must be +1 or -1");
  if (in_host == nullptr || out_host == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2: in/out is NULL");
  return run_host(dev, in_host, out_host, log_n, batch, direction, normalize, 2);
}

}  // extern "C"
