// Runtime and C ABI of the B200 FFT path (include/ferrum_fft.h).
//
// The device handle replaces the reference's persistent `Device` (a CUDA
// context plus a loaded PTX module, crates/ferrum-gpu-py/src/lib.rs:389-417):
// here it owns every twiddle table, uploaded once, and a stream-ordered
// memory pool for four-step workspaces. The reference instead rebuilt and
// re-uploaded its twiddles, allocated input/output/twiddle buffers and
// conjugated on the host on every call (lib.rs:105-140, :237-247).
#include <cuda_runtime.h>

#include <initializer_list>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "fft_kernels.cuh"
#include "fft_launch.h"
#include "passes.h"
#include "runtime.h"
#include "twiddle_tables.h"

#define FERRUM_VERSION "0.3.0-b200"

namespace ferrum {

namespace {
thread_local std::string g_last_error;
}

ferrum_status set_error(ferrum_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

ferrum_status cuda_error(cudaError_t e, const char* what) {
  return set_error(FERRUM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                        cudaGetErrorString(e) + ")");
}

void clear_error() { g_last_error.clear(); }

DeviceGuard::DeviceGuard(int ordinal) {
  if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
  if (prev_ != ordinal) status_ = cudaSetDevice(ordinal);
}

DeviceGuard::~DeviceGuard() {
  int cur = -1;
  if (prev_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
}

const float2* stage_table(const ferrum_device* dev, int log_n) {
  return dev->tables + dev->stage_off[log_n];
}
const float2* stage_table_p(const ferrum_device* dev, int log_n, int log_p) {
  if (log_p == plan_log_p(log_n)) return stage_table(dev, log_n);
  if (log_p == 5 && tile_p32_table(log_n) && dev->stage32_off[log_n] >= 0)
    return dev->tables + dev->stage32_off[log_n];
  return nullptr;
}
const float2* tw4_lo_table(const ferrum_device* dev, int log_n) {
  return dev->tables + dev->tw4_lo_off[log_n];
}
const float2* tw4_hi_table(const ferrum_device* dev, int log_n) {
  return dev->tables + dev->tw4_hi_off[log_n];
}

namespace {

bool valid_direction(int direction) { return direction == 1 || direction == -1; }

ferrum_status check_device(const ferrum_device* dev) {
  if (dev == nullptr || dev->tables == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "device handle is NULL or destroyed");
  return FERRUM_OK;
}

ferrum_status check_common(int log_n, int lo, int hi, size_t batch, int direction,
                           const char* what, int dims = 1) {
  if (log_n < lo || log_n > hi)
    return set_error(FERRUM_ERR_INVALID_ARG, std::string(what) + ": log_n must be in [" +
                                                 std::to_string(lo) + ", " + std::to_string(hi) +
                                                 "], got " + std::to_string(log_n));
  if (ferrum_status s = check_elements(dims * log_n, batch, what)) return s;
  if (!valid_direction(direction))
    return set_error(FERRUM_ERR_INVALID_ARG,
                     std::string(what) + ": direction must be +1 (forward) or -1 (inverse), got " +
                         std::to_string(direction));
  return FERRUM_OK;
}

bool is_aligned8(const void* p) { return ((uintptr_t)p & 7u) == 0; }

}  // namespace

ferrum_status check_elements(int elem_log, size_t batch, const char* what) {
  if (batch == 0)
    return set_error(FERRUM_ERR_INVALID_ARG, std::string(what) + ": batch must be positive");
  if (elem_log > kMaxLogElems || batch > ((size_t)1 << (kMaxLogElems - elem_log)))
    return set_error(FERRUM_ERR_INVALID_ARG,
                     std::string(what) + ": batch " + std::to_string(batch) +
                         " times the transform size exceeds 2^" + std::to_string(kMaxLogElems) +
                         " complex values per call");
  return FERRUM_OK;
}

size_t workspace_1d_bytes(int log_n, int64_t batch) {
  return (size_t)plan_1d(log_n, batch, false, false).ws_elems * sizeof(float2);
}

size_t workspace_2d_bytes(int log_n, int64_t batch) {
  return (size_t)plan_2d(log_n, batch, false, false).ws_elems * sizeof(float2);
}

ferrum_status run_plan(ferrum_device* dev, const PassPlan& plan, const float2* in, float2* out,
                       float2* ws, cudaStream_t stream) {
  float2* bufs[3] = {const_cast<float2*>(in), out, ws};
  for (int i = 0; i < plan.count; ++i) {
    const PassDesc& d = plan.p[i];
    const float2* src = bufs[(int)d.src];
    float2* dst = bufs[(int)d.dst];
    const float2* stw = stage_table(dev, d.log_n);
    cudaError_t e = cudaSuccess;
    switch (d.kind) {
      case PassKind::Rows:
        e = launch_rows(d.log_n, d.conj_in, d.conj_out, src, dst, stw, d.rows_nfft, d.rows_scale,
                        stream, d.rows_log_block, dev->err_flag, d.rows_block_rows);
        break;
      case PassKind::Pass: {
        PassArgs a = d.pa;
        if (a.log_m > 0) {
          a.tw_lo = tw4_lo_table(dev, a.log_m);
          a.tw_hi = tw4_hi_table(dev, a.log_m);
        }
        e = cudaErrorNotSupported;
        if (d.tile != TileMode::None)
          e = launch_pass_tile(d.tile, d.tile_w, tile_log_p(d), d.log_n, d.conj_in, d.conj_out,
                               a.log_m > 0, src, dst, stage_table_p(dev, d.log_n, tile_log_p(d)),
                               a, dev->err_flag, stream);
        if (e == cudaErrorNotSupported)
          e = launch_pass(d.log_n, d.conj_in, d.conj_out, a.log_m > 0, src, dst, stw, a, stream);
        break;
      }
      case PassKind::RowsT:
        e = cudaErrorNotSupported;
        if (d.tile != TileMode::None)
          e = launch_rows_t_tile(d.tile, d.tile_w, tile_log_p(d), d.log_n, d.conj_in, d.conj_out,
                                 src, dst, stage_table_p(dev, d.log_n, tile_log_p(d)), d.ra,
                                 stream);
        if (e == cudaErrorNotSupported)
          e = launch_rows_t(d.log_n, d.conj_in, d.conj_out, src, dst, stw, d.ra, stream);
        break;
      case PassKind::ColsL2: {
        ColsL2Args a = d.ca;
        a.tw_lo = tw4_lo_table(dev, d.log_n);
        a.tw_hi = tw4_hi_table(dev, d.log_n);
        e = launch_cols_l2(d.log_n, d.conj_in, d.conj_out, src, dst, ws,
                           stage_table(dev, d.cl2_l1), stage_table(dev, d.cl2_l2), a, stream);
        break;
      }
    }
    if (e != cudaSuccess)
      return cuda_error(e, (std::string("pass ") + std::to_string(i) + " launch").c_str());
  }
  return FERRUM_OK;
}

ferrum_status enqueue_1d(ferrum_device* dev, const float2* in, float2* out, int log_n,
                         int64_t batch, int direction, bool normalize, float2* ws,
                         cudaStream_t stream) {
  return run_plan(dev, plan_1d(log_n, batch, direction < 0, normalize), in, out, ws, stream);
}

ferrum_status enqueue_2d(ferrum_device* dev, const float2* in, float2* out, int log_n,
                         int64_t batch, int direction, bool normalize, float2* ws,
                         cudaStream_t stream) {
  return run_plan(dev, plan_2d(log_n, batch, direction < 0, normalize), in, out, ws, stream);
}

ferrum_status check_device_flag(ferrum_device* dev) {
  int flag = 0;
  cudaError_t e = cudaMemcpy(&flag, dev->err_flag, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_error(e, "reading the device error flag");
  if (flag == 0) return FERRUM_OK;
  cudaMemset(dev->err_flag, 0, sizeof(int));
  return set_error(FERRUM_ERR_TIMEOUT,
                   "a kernel's bounded wait for its TMA copy expired (device flag " +
                       std::to_string(flag) + "); its output is incomplete");
}

}  // namespace ferrum

using namespace ferrum;

extern "C" {

const char* ferrum_version(void) { return FERRUM_VERSION; }

const char* ferrum_last_error(void) { return g_last_error.c_str(); }

ferrum_status ferrum_device_create(int ordinal, ferrum_device** out) {
  clear_error();
  if (out == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceCount");
  if (ordinal < 0 || ordinal >= count)
    return set_error(FERRUM_ERR_INVALID_ARG, "device ordinal " + std::to_string(ordinal) +
                                                 " out of range (" + std::to_string(count) +
                                                 " devices)");
  DeviceGuard guard(ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, ordinal);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceProperties");
  if (prop.major != 10 || prop.minor != 0)
    return set_error(FERRUM_ERR_UNSUPPORTED,
                     std::string("ferrum-gpu kernels are built for sm_100a (B200); device is ") +
                         prop.name + " sm_" + std::to_string(prop.major) +
                         std::to_string(prop.minor));

  std::vector<float2> host;
  auto* dev = new ferrum_device();
  dev->ordinal = ordinal;
  for (int l = 0; l <= kMaxSinglePassLogN; ++l) dev->stage_off[l] = dev->stage32_off[l] = -1;
  for (int l = 0; l <= kMaxLogN; ++l) dev->tw4_lo_off[l] = dev->tw4_hi_off[l] = -1;
  for (int l = 2; l <= kMaxSinglePassLogN; ++l) {
    dev->stage_off[l] = (int64_t)host.size();
    append_stage_tables(host, l);
    host.push_back(make_float2(1.f, 0.f));  // keeps every offset valid for 1-stage plans
    if (tile_p32_table(l)) {
      dev->stage32_off[l] = (int64_t)host.size();
      append_stage_tables(host, l, 5);
      host.push_back(make_float2(1.f, 0.f));
    }
  }
  for (int l = 1; l <= kMaxLogN; ++l) {
    std::vector<float2> lo, hi;
    append_four_step_tables(lo, hi, l);
    dev->tw4_lo_off[l] = (int64_t)host.size();
    host.insert(host.end(), lo.begin(), lo.end());
    dev->tw4_hi_off[l] = (int64_t)host.size();
    host.insert(host.end(), hi.begin(), hi.end());
  }
  dev->table_entries = host.size();
  e = cudaMalloc(&dev->tables, host.size() * sizeof(float2));
  if (e != cudaSuccess) {
    delete dev;
    return cuda_error(e, "cudaMalloc(twiddle tables)");
  }
  e = cudaMemcpy(dev->tables, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(dev->tables);
    delete dev;
    return cuda_error(e, "cudaMemcpy(twiddle tables)");
  }
  e = cudaMalloc(&dev->err_flag, 256);
  if (e == cudaSuccess) e = cudaMemset(dev->err_flag, 0, 256);
  if (e != cudaSuccess) {
    cudaFree(dev->tables);
    if (dev->err_flag) cudaFree(dev->err_flag);
    delete dev;
    return cuda_error(e, "cudaMalloc(error flag)");
  }
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.handleTypes = cudaMemHandleTypeNone;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = ordinal;
  e = cudaMemPoolCreate(&dev->pool, &props);
  if (e != cudaSuccess) {
    cudaFree(dev->tables);
    delete dev;
    return cuda_error(e, "cudaMemPoolCreate");
  }
  uint64_t keep = UINT64_MAX;
  cudaMemPoolSetAttribute(dev->pool, cudaMemPoolAttrReleaseThreshold, &keep);
  *out = dev;
  return FERRUM_OK;
}

ferrum_status ferrum_device_destroy(ferrum_device* dev) {
  clear_error();
  if (dev == nullptr) return FERRUM_OK;
  DeviceGuard guard(dev->ordinal);
  if (cudaDeviceSynchronize() == cudaErrorCudartUnloading) {
    // Called from a static destructor after the runtime shut down: the
    // driver has already reclaimed every resource; only free the host side.
    dev->tables = nullptr;
    delete dev;
    return FERRUM_OK;
  }
  for (int i = 0; i < ferrum_device::kHostStreams; ++i) {
    if (dev->host_streams[i]) cudaStreamDestroy(dev->host_streams[i]);
    if (dev->host_dbuf[i]) cudaFree(dev->host_dbuf[i]);
    if (dev->host_ws[i]) cudaFree(dev->host_ws[i]);
    if (dev->host_pin_in[i]) cudaFreeHost(dev->host_pin_in[i]);
    if (dev->host_pin_out[i]) cudaFreeHost(dev->host_pin_out[i]);
  }
  if (dev->pool) cudaMemPoolDestroy(dev->pool);
  if (dev->err_flag) cudaFree(dev->err_flag);
  if (dev->tables) cudaFree(dev->tables);
  dev->tables = nullptr;
  delete dev;
  return FERRUM_OK;
}

ferrum_status ferrum_device_sync(ferrum_device* dev) {
  clear_error();
  if (ferrum_status s = check_device(dev)) return s;
  DeviceGuard guard(dev->ordinal);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_error(e, "cudaDeviceSynchronize");
  return check_device_flag(dev);
}

ferrum_status ferrum_device_ordinal(const ferrum_device* dev, int* ordinal) {
  clear_error();
  if (ferrum_status s = check_device(dev)) return s;
  if (ordinal == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "ordinal is NULL");
  *ordinal = dev->ordinal;
  return FERRUM_OK;
}

ferrum_status ferrum_fft_workspace_bytes(int log_n, size_t batch, int kind, size_t* bytes) {
  clear_error();
  if (bytes == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "bytes is NULL");
  if (kind == 1) {
    if (ferrum_status s = check_common(log_n, 2, kMaxLogN, batch, 1, "workspace")) return s;
    *bytes = workspace_1d_bytes(log_n, (int64_t)batch);
    return FERRUM_OK;
  }
  if (kind == 2) {
    if (ferrum_status s = check_common(log_n, 2, kMaxSinglePassLogN, batch, 1, "workspace", 2))
      return s;
    *bytes = workspace_2d_bytes(log_n, (int64_t)batch);
    return FERRUM_OK;
  }
  return set_error(FERRUM_ERR_INVALID_ARG, "kind must be 1 (1D) or 2 (2D)");
}

ferrum_status ferrum_fft_launch_count(int log_n, size_t batch, int kind, int* launches) {
  clear_error();
  if (launches == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "launches is NULL");
  if (kind == 1) {
    if (ferrum_status s = check_common(log_n, 2, kMaxLogN, batch, 1, "launch_count")) return s;
    *launches = plan_1d(log_n, (int64_t)batch, false, false).count;
    return FERRUM_OK;
  }
  if (kind == 2) {
    if (ferrum_status s = check_common(log_n, 2, kMaxSinglePassLogN, batch, 1, "launch_count", 2))
      return s;
    *launches = plan_2d(log_n, (int64_t)batch, false, false).count;
    return FERRUM_OK;
  }
  return set_error(FERRUM_ERR_INVALID_ARG, "kind must be 1 (1D) or 2 (2D)");
}

ferrum_status ferrum_fft_1d_c2c_pow2_ws(ferrum_device* dev, const void* in_dev, void* out_dev,
                                        int log_n, size_t batch, int direction, int normalize,
                                        void* workspace_dev, size_t workspace_bytes,
                                        void* stream) {
  clear_error();
  if (ferrum_status s = check_device(dev)) return s;
  if (ferrum_status s = check_common(log_n, 2, kMaxLogN, batch, direction, "fft_1d_c2c_pow2"))
    return s;
  if (in_dev == nullptr || out_dev == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2: in/out is NULL");
  if (!is_aligned8(in_dev) || !is_aligned8(out_dev))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2: in/out must be 8-byte aligned");
  const size_t need = workspace_1d_bytes(log_n, (int64_t)batch);
  if (need > 0 && (workspace_dev == nullptr || workspace_bytes < need))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2: workspace needs " +
                                                 std::to_string(need) + " bytes");
  if (need > 0 && !is_aligned8(workspace_dev))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2: workspace must be 8-byte aligned");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  return enqueue_1d(dev, (const float2*)in_dev, (float2*)out_dev, log_n, (int64_t)batch,
                    direction, normalize != 0, (float2*)workspace_dev, (cudaStream_t)stream);
}

ferrum_status ferrum_fft_1d_c2c_pow2(ferrum_device* dev, const void* in_dev, void* out_dev,
                                     int log_n, size_t batch, int direction, int normalize,
                                     void* stream) {
  clear_error();
  if (ferrum_status s = check_device(dev)) return s;
  if (ferrum_status s = check_common(log_n, 2, kMaxLogN, batch, direction, "fft_1d_c2c_pow2"))
    return s;
  const size_t need = workspace_1d_bytes(log_n, (int64_t)batch);
  if (need == 0)
    return ferrum_fft_1d_c2c_pow2_ws(dev, in_dev, out_dev, log_n, batch, direction, normalize,
                                     nullptr, 0, stream);
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  void* ws = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&ws, need, dev->pool, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(workspace)");
  ferrum_status s = ferrum_fft_1d_c2c_pow2_ws(dev, in_dev, out_dev, log_n, batch, direction,
                                              normalize, ws, need, stream);
  e = cudaFreeAsync(ws, (cudaStream_t)stream);
  if (s == FERRUM_OK && e != cudaSuccess) return cuda_error(e, "cudaFreeAsync(workspace)");
  return s;
}

ferrum_status ferrum_fft_1d_c2c_pow2_split(ferrum_device* dev, const float* in_re,
                                           const float* in_im, float* out_re, float* out_im,
                                           int log_n, size_t batch, int direction, int normalize,
                                           void* stream) {
  clear_error();
  if (ferrum_status s = check_device(dev)) return s;
  if (ferrum_status s =
          check_common(log_n, 2, kMaxSinglePassLogN, batch, direction, "fft_1d_c2c_pow2_split"))
    return s;
  if (!in_re || !in_im || !out_re || !out_im)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_1d_c2c_pow2_split: NULL array");
  if ((out_re == in_im && out_re != in_re) || (out_im == in_re && out_im != in_im))
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "fft_1d_c2c_pow2_split: out_re / out_im may only alias in_re / in_im");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  const bool inv = direction < 0;
  const float scale = (inv && normalize) ? 1.0f / (float)((int64_t)1 << log_n) : 1.0f;
  cudaError_t e = launch_rows_split(log_n, inv, inv, in_re, in_im, out_re, out_im,
                                    stage_table(dev, log_n), (int64_t)batch, scale,
                                    (cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "split-layout row pass launch");
}

namespace {
ferrum_status check_elementwise(ferrum_device* dev, size_t n, std::initializer_list<const void*> ptrs,
                                const char* what) {
  if (ferrum_status s = check_device(dev)) return s;
  if (n == 0) return set_error(FERRUM_ERR_INVALID_ARG, std::string(what) + ": n must be positive");
  for (const void* p : ptrs)
    if (p == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, std::string(what) + ": NULL array");
  return FERRUM_OK;
}
}  // namespace

ferrum_status ferrum_cmul_interleaved(ferrum_device* dev, const void* a, const void* b, void* out,
                                      size_t n, void* stream) {
  clear_error();
  if (ferrum_status s = check_elementwise(dev, n, {a, b, out}, "cmul_interleaved")) return s;
  if (!is_aligned8(a) || !is_aligned8(b) || !is_aligned8(out))
    return set_error(FERRUM_ERR_INVALID_ARG, "cmul_interleaved: arrays must be 8-byte aligned");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  cudaError_t e = launch_cmul_interleaved((const float2*)a, (const float2*)b, (float2*)out,
                                          (int64_t)n, (cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "cmul_interleaved launch");
}

ferrum_status ferrum_cmul_split(ferrum_device* dev, const float* a_re, const float* a_im,
                                const float* b_re, const float* b_im, float* out_re,
                                float* out_im, size_t n, void* stream) {
  clear_error();
  if (ferrum_status s =
          check_elementwise(dev, n, {a_re, a_im, b_re, b_im, out_re, out_im}, "cmul_split"))
    return s;
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  cudaError_t e = launch_cmul_split(a_re, a_im, b_re, b_im, out_re, out_im, (int64_t)n,
                                    (cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "cmul_split launch");
}

ferrum_status ferrum_deinterleave(ferrum_device* dev, const void* in, float* out_re, float* out_im,
                                  size_t n, void* stream) {
  clear_error();
  if (ferrum_status s = check_elementwise(dev, n, {in, out_re, out_im}, "deinterleave")) return s;
  if (!is_aligned8(in)) return set_error(FERRUM_ERR_INVALID_ARG, "deinterleave: input must be 8-byte aligned");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  cudaError_t e = launch_deinterleave((const float2*)in, out_re, out_im, (int64_t)n,
                                      (cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "deinterleave launch");
}

ferrum_status ferrum_interleave(ferrum_device* dev, const float* re, const float* im, void* out,
                                size_t n, void* stream) {
  clear_error();
  if (ferrum_status s = check_elementwise(dev, n, {re, im, out}, "interleave")) return s;
  if (!is_aligned8(out)) return set_error(FERRUM_ERR_INVALID_ARG, "interleave: output must be 8-byte aligned");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  cudaError_t e = launch_interleave(re, im, (float2*)out, (int64_t)n, (cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "interleave launch");
}

ferrum_status ferrum_fft_2d_c2c_pow2(ferrum_device* dev, const void* in_dev, void* out_dev,
                                     int log_n, size_t batch, int direction, int normalize,
                                     void* stream) {
  clear_error();
  if (ferrum_status s = check_device(dev)) return s;
  if (ferrum_status s =
          check_common(log_n, 2, kMaxSinglePassLogN, batch, direction, "fft_2d_c2c_pow2", 2))
    return s;
  if (in_dev == nullptr || out_dev == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2: in/out is NULL");
  if (!is_aligned8(in_dev) || !is_aligned8(out_dev))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2: in/out must be 8-byte aligned");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  const size_t need = workspace_2d_bytes(log_n, (int64_t)batch);
  void* ws = nullptr;
  if (need > 0) {
    cudaError_t e = cudaMallocFromPoolAsync(&ws, need, dev->pool, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(2D workspace)");
  }
  ferrum_status s = enqueue_2d(dev, (const float2*)in_dev, (float2*)out_dev, log_n,
                               (int64_t)batch, direction, normalize != 0, (float2*)ws,
                               (cudaStream_t)stream);
  if (ws) {
    cudaError_t e = cudaFreeAsync(ws, (cudaStream_t)stream);
    if (s == FERRUM_OK && e != cudaSuccess) return cuda_error(e, "cudaFreeAsync(2D workspace)");
  }
  return s;
}

}  // extern "C"
