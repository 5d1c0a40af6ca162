// Internal runtime shared by the C ABI (capi.cu) and the distributed path
// (dist.cu). Not part of the public interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "../../include/ferrum_fft.h"
#include "plan.h"

struct ferrum_device {
  int ordinal = -1;
  // All twiddle tables in one device allocation.
  float2* tables = nullptr;
  size_t table_entries = 0;
  int64_t stage_off[ferrum::kMaxSinglePassLogN + 1] = {};  // per log_n, -1 if absent
  // Stage tables with 32 values per thread for the lengths whose plan uses
  // 16 (the tile kernels that run them with 32; ferrum::kTileP32Lengths).
  int64_t stage32_off[ferrum::kMaxSinglePassLogN + 1] = {};
  int64_t tw4_lo_off[ferrum::kMaxLogN + 1] = {};
  int64_t tw4_hi_off[ferrum::kMaxLogN + 1] = {};
  cudaMemPool_t pool = nullptr;  // stream-ordered workspace pool
  int* err_flag = nullptr;       // device word set by kernels whose bounded waits expire

  // Host-pointer path resources (grown on demand, guarded by host_mu).
  std::mutex host_mu;
  static constexpr int kHostStreams = 3;
  cudaStream_t host_streams[kHostStreams] = {};
  void* host_dbuf[kHostStreams] = {};
  void* host_ws[kHostStreams] = {};
  void* host_pin_in[kHostStreams] = {};
  void* host_pin_out[kHostStreams] = {};
  size_t host_chunk_bytes = 0;
  size_t host_ws_bytes = 0;
};

namespace ferrum {

// Thread-local error message for ferrum_last_error().
ferrum_status set_error(ferrum_status code, const std::string& msg);
ferrum_status cuda_error(cudaError_t e, const char* what);
void clear_error();

// Makes `ordinal` current and restores the previous device on scope exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(int ordinal);
  ~DeviceGuard();
  cudaError_t status() const { return status_; }

 private:
  int prev_ = -1;
  cudaError_t status_ = cudaSuccess;
};

const float2* stage_table(const ferrum_device* dev, int log_n);
// Stage table of length 2^log_n with 2^log_p values per thread (log_p 4 or
// 5; NULL where the device holds none).
const float2* stage_table_p(const ferrum_device* dev, int log_n, int log_p);
const float2* tw4_lo_table(const ferrum_device* dev, int log_n);
const float2* tw4_hi_table(const ferrum_device* dev, int log_n);

// Enqueue a batched 1D transform on device memory. `ws` must hold
// workspace_1d_bytes(log_n, batch) bytes (ignored for single-pass sizes).
ferrum_status enqueue_1d(ferrum_device* dev, const float2* in, float2* out, int log_n,
                         int64_t batch, int direction, bool normalize, float2* ws,
                         cudaStream_t stream);
// `ws` must hold workspace_2d_bytes(log_n, batch) bytes (may be NULL when 0).
ferrum_status enqueue_2d(ferrum_device* dev, const float2* in, float2* out, int log_n,
                         int64_t batch, int direction, bool normalize, float2* ws,
                         cudaStream_t stream);
size_t workspace_1d_bytes(int log_n, int64_t batch);
size_t workspace_2d_bytes(int log_n, int64_t batch);
struct PassPlan;
// Enqueue every pass of `plan`; buffer roles In/Out/Ws map to in/out/ws.
ferrum_status run_plan(ferrum_device* dev, const PassPlan& plan, const float2* in, float2* out,
                       float2* ws, cudaStream_t stream);
// Reads and clears the device error flag; FERRUM_ERR_TIMEOUT if it was set.
ferrum_status check_device_flag(ferrum_device* dev);

// Largest number of complex values one call may cover: 2^36 (512 GiB, more
// than a B200 holds). Below it every byte count, element index and grid size
// the plans form stays far from overflow.
constexpr int kMaxLogElems = 36;
// FERRUM_ERR_INVALID_ARG unless batch * 2^elem_log <= 2^kMaxLogElems
// (elem_log = log_n for 1D, 2 * log_n for 2D); checked before any size is
// computed from the batch.
ferrum_status check_elements(int elem_log, size_t batch, const char* what);

}  // namespace ferrum
