// Distributed 2D FFT over NCCL (one process per GPU). New in this build: the
// reference has no multi-GPU code (every context is CudaContext::new(0),
// crates/ferrum-gpu-py/src/lib.rs:261,385).
//
// A single N x N image is split into P row slabs of B = N/P rows. Per call:
//   1. row FFTs of the local slab; the store writes B x B blocks, one per
//      destination rank, contiguously ([q][row][col]);
//   2. NCCL all-to-all: block q goes to rank q. The received blocks, stacked
//      by source rank, are exactly this rank's N x B column slab, row-major;
//   3. column FFTs of the column slab (length N, row pitch B), one pass or,
//      for N >= 2048, two sub-passes with 16 columns per CTA;
//   4. NCCL all-to-all of the B x B row blocks of the column slab;
//   5. a block gather turns the received [src][row][col] blocks back into the
//      row-major B x N output slab.
// NCCL is opened with dlopen so that the single-GPU library never depends on
// it; when PyTorch is loaded first its libnccl.so.2 is reused. The
// communicator is non-blocking, so set-up and every host wait are bounded by
// the context's timeout, after which the communicator is aborted and
// FERRUM_ERR_TIMEOUT returned.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>

#include "fft_kernels.cuh"
#include "fft_launch.h"
#include "passes.h"
#include "runtime.h"

struct ferrum_dist_ctx {
  ferrum_device* dev = nullptr;
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int timeout_ms = 0;
  bool aborted = false;
};

namespace ferrum {
namespace {

struct NcclApi {
  bool tried = false;
  bool ok = false;
  std::string error;
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclSend) Send = nullptr;
  decltype(&ncclRecv) Recv = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (api.tried) return api;
  api.tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
    return api;
  }
#define FERRUM_SYM(field, name)                                  \
  api.field = (decltype(api.field))dlsym(h, #name);              \
  if (!api.field) {                                              \
    api.error = std::string("libnccl.so.2 lacks ") + #name;      \
    return api;                                                  \
  }
  FERRUM_SYM(GetUniqueId, ncclGetUniqueId)
  FERRUM_SYM(CommInitRankConfig, ncclCommInitRankConfig)
  FERRUM_SYM(CommGetAsyncError, ncclCommGetAsyncError)
  FERRUM_SYM(CommDestroy, ncclCommDestroy)
  FERRUM_SYM(CommAbort, ncclCommAbort)
  FERRUM_SYM(Send, ncclSend)
  FERRUM_SYM(Recv, ncclRecv)
  FERRUM_SYM(GroupStart, ncclGroupStart)
  FERRUM_SYM(GroupEnd, ncclGroupEnd)
  FERRUM_SYM(GetErrorString, ncclGetErrorString)
#undef FERRUM_SYM
  api.ok = true;
  return api;
}

ferrum_status nccl_error(ncclResult_t r, const char* what) {
  NcclApi& api = nccl();
  const char* msg = api.GetErrorString ? api.GetErrorString(r) : "unknown";
  return set_error(FERRUM_ERR_NCCL, std::string(what) + ": " + msg);
}

using Clock = std::chrono::steady_clock;

// Polls a non-blocking communicator until its pending operation completes,
// the deadline passes (abort + FERRUM_ERR_TIMEOUT) or it reports an error.
ferrum_status wait_comm(ferrum_dist_ctx* ctx, const char* what) {
  NcclApi& api = nccl();
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = api.CommGetAsyncError(ctx->comm, &st);
    if (r != ncclSuccess) return nccl_error(r, what);
    if (st == ncclSuccess) return FERRUM_OK;
    if (st != ncclInProgress) return nccl_error(st, what);
    if (Clock::now() > deadline) {
      api.CommAbort(ctx->comm);
      ctx->aborted = true;
      return set_error(FERRUM_ERR_TIMEOUT, std::string(what) + ": timed out after " +
                                               std::to_string(ctx->timeout_ms) + " ms");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

int ilog2(int64_t x) {
  int l = 0;
  while (((int64_t)1 << l) < x) ++l;
  return l;
}

ferrum_status check_ctx(const ferrum_dist_ctx* ctx) {
  if (ctx == nullptr || ctx->comm == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "distributed context is NULL or destroyed");
  if (ctx->aborted)
    return set_error(FERRUM_ERR_NCCL, "communicator was aborted after an earlier timeout");
  return FERRUM_OK;
}

// All-to-all of P contiguous blocks of `elems` complex values.
ferrum_status all_to_all(ferrum_dist_ctx* ctx, const float2* send, float2* recv, int64_t elems,
                         cudaStream_t stream) {
  NcclApi& api = nccl();
  ncclResult_t r = api.GroupStart();
  if (r != ncclSuccess) return nccl_error(r, "ncclGroupStart");
  for (int q = 0; q < ctx->nranks; ++q) {
    r = api.Send(send + q * elems, (size_t)(2 * elems), ncclFloat32, q, ctx->comm, stream);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(r, "ncclSend");
    r = api.Recv(recv + q * elems, (size_t)(2 * elems), ncclFloat32, q, ctx->comm, stream);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(r, "ncclRecv");
  }
  r = api.GroupEnd();
  if (r == ncclInProgress) return wait_comm(ctx, "all-to-all enqueue");
  if (r != ncclSuccess) return nccl_error(r, "ncclGroupEnd");
  return FERRUM_OK;
}

}  // namespace
}  // namespace ferrum

using namespace ferrum;

extern "C" {

ferrum_status ferrum_dist_check(int log_n, int nranks) {
  clear_error();
  if (nranks < 1 || (nranks & (nranks - 1)) != 0)
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "distributed 2D needs a power-of-two rank count, got " + std::to_string(nranks));
  if (log_n < 4 || log_n > kMaxSinglePassLogN)
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "distributed 2D needs log_n in [4, 14], got " + std::to_string(log_n));
  const int64_t n = (int64_t)1 << log_n;
  if (n / nranks < 2)
    return set_error(FERRUM_ERR_INVALID_ARG, "distributed 2D needs N / ranks >= 2 (N = " +
                                                 std::to_string(n) + ", ranks = " +
                                                 std::to_string(nranks) + ")");
  return FERRUM_OK;
}

ferrum_status ferrum_dist_get_unique_id(unsigned char id_out[FERRUM_DIST_ID_BYTES]) {
  clear_error();
  static_assert(sizeof(ncclUniqueId) == FERRUM_DIST_ID_BYTES, "ncclUniqueId size");
  if (id_out == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "id_out is NULL");
  NcclApi& api = nccl();
  if (!api.ok) return set_error(FERRUM_ERR_NCCL, api.error);
  ncclUniqueId id;
  ncclResult_t r = api.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
  memcpy(id_out, &id, sizeof(id));
  return FERRUM_OK;
}

ferrum_status ferrum_dist_init(ferrum_device* dev, const unsigned char id[FERRUM_DIST_ID_BYTES],
                               int nranks, int rank, int timeout_ms, ferrum_dist_ctx** out) {
  clear_error();
  if (out == nullptr || id == nullptr || dev == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "dist_init: NULL argument");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return set_error(FERRUM_ERR_INVALID_ARG, "dist_init: rank " + std::to_string(rank) +
                                                 " out of range for " + std::to_string(nranks) +
                                                 " ranks");
  if (timeout_ms <= 0) return set_error(FERRUM_ERR_INVALID_ARG, "dist_init: timeout_ms must be > 0");
  NcclApi& api = nccl();
  if (!api.ok) return set_error(FERRUM_ERR_NCCL, api.error);
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  auto* ctx = new ferrum_dist_ctx();
  ctx->dev = dev;
  ctx->nranks = nranks;
  ctx->rank = rank;
  ctx->timeout_ms = timeout_ms;
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = api.CommInitRankConfig(&ctx->comm, nranks, uid, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete ctx;
    return nccl_error(r, "ncclCommInitRankConfig");
  }
  ferrum_status s = wait_comm(ctx, "communicator init");
  if (s != FERRUM_OK) {
    if (!ctx->aborted && ctx->comm) api.CommAbort(ctx->comm);
    delete ctx;
    return s;
  }
  *out = ctx;
  return FERRUM_OK;
}

ferrum_status ferrum_dist_destroy(ferrum_dist_ctx* ctx) {
  clear_error();
  if (ctx == nullptr) return FERRUM_OK;
  NcclApi& api = nccl();
  if (ctx->comm && !ctx->aborted && api.ok) {
    DeviceGuard guard(ctx->dev->ordinal);
    api.CommDestroy(ctx->comm);
  }
  delete ctx;
  return FERRUM_OK;
}

ferrum_status ferrum_dist_world(const ferrum_dist_ctx* ctx, int* nranks, int* rank) {
  clear_error();
  if (ctx == nullptr || nranks == nullptr || rank == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "dist_world: NULL argument");
  *nranks = ctx->nranks;
  *rank = ctx->rank;
  return FERRUM_OK;
}

ferrum_status ferrum_dist_workspace_bytes(const ferrum_dist_ctx* ctx, int log_n, size_t* bytes) {
  clear_error();
  if (ctx == nullptr || bytes == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "dist_workspace_bytes: NULL argument");
  if (ferrum_status s = ferrum_dist_check(log_n, ctx->nranks)) return s;
  const int64_t n = (int64_t)1 << log_n;
  *bytes = ctx->nranks == 1 ? workspace_2d_bytes(log_n, 1)
                            : (size_t)(2 * (n / ctx->nranks) * n) * sizeof(float2);
  return FERRUM_OK;
}

ferrum_status ferrum_fft_2d_c2c_pow2_dist(ferrum_dist_ctx* ctx, const void* in_slab_dev,
                                          void* out_slab_dev, int log_n, int direction,
                                          int normalize, void* stream_ptr) {
  clear_error();
  if (ferrum_status s = check_ctx(ctx)) return s;
  if (ferrum_status s = ferrum_dist_check(log_n, ctx->nranks)) return s;
  if (direction != 1 && direction != -1)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2_dist: direction must be +1 or -1");
  if (in_slab_dev == nullptr || out_slab_dev == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2_dist: in/out is NULL");
  if (((uintptr_t)in_slab_dev & 15) || ((uintptr_t)out_slab_dev & 15))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2_dist: in/out must be 16-byte aligned");
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  ferrum_device* dev = ctx->dev;
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  if (ctx->nranks == 1) {
    const size_t need = workspace_2d_bytes(log_n, 1);
    void* ws1 = nullptr;
    if (need > 0) {
      cudaError_t e = cudaMallocFromPoolAsync(&ws1, need, dev->pool, stream);
      if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(2D workspace)");
    }
    ferrum_status s1 = enqueue_2d(dev, (const float2*)in_slab_dev, (float2*)out_slab_dev, log_n, 1,
                                  direction, normalize != 0, (float2*)ws1, stream);
    if (ws1) cudaFreeAsync(ws1, stream);
    return s1;
  }

  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const int64_t b = n / ctx->nranks;
  const int lb = ilog2(b);
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  const float2* tw = stage_table(dev, log_n);
  void* ws = nullptr;
  const size_t slab_bytes = (size_t)(b * n) * sizeof(float2);
  cudaError_t e = cudaMallocFromPoolAsync(&ws, 2 * slab_bytes, dev->pool, stream);
  if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(dist workspace)");
  float2* wa = (float2*)ws;
  float2* wb = wa + b * n;
  ferrum_status s = FERRUM_OK;
  do {
    e = launch_rows(log_n, inv, false, (const float2*)in_slab_dev, wa, tw, b, 1.0f, stream, lb);
    if (e != cudaSuccess) {
      s = cuda_error(e, "distributed row pass launch");
      break;
    }
    if ((s = all_to_all(ctx, wa, wb, b * b, stream)) != FERRUM_OK) break;
    // Column FFTs of the N x B column slab (row pitch B): wb -> wa, one pass or
    // two sub-passes (the first in place on wb).
    PassPlan cols;
    plan_columns(cols, log_n, lb, b, 1, n * b, false, inv, scale, PassBuf::In, PassBuf::In,
                 PassBuf::Out);
    if ((s = run_plan(dev, cols, wb, wa, nullptr, stream)) != FERRUM_OK) break;
    if ((s = all_to_all(ctx, wa, wb, b * b, stream)) != FERRUM_OK) break;
    e = launch_block_gather(wb, (float2*)out_slab_dev, ctx->nranks, b, b, stream);
    if (e != cudaSuccess) {
      s = cuda_error(e, "distributed block gather launch");
      break;
    }
  } while (false);
  cudaError_t ef = cudaFreeAsync(ws, stream);
  if (s == FERRUM_OK && ef != cudaSuccess) return cuda_error(ef, "cudaFreeAsync(dist workspace)");
  return s;
}

ferrum_status ferrum_dist_sync(ferrum_dist_ctx* ctx, void* stream_ptr) {
  clear_error();
  if (ferrum_status s = check_ctx(ctx)) return s;
  DeviceGuard guard(ctx->dev->ordinal);
  NcclApi& api = nccl();
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  for (;;) {
    cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) return FERRUM_OK;
    if (e != cudaErrorNotReady) return cuda_error(e, "dist_sync");
    ncclResult_t st = ncclSuccess;
    if (api.CommGetAsyncError(ctx->comm, &st) == ncclSuccess && st != ncclSuccess &&
        st != ncclInProgress) {
      api.CommAbort(ctx->comm);
      ctx->aborted = true;
      return nccl_error(st, "dist_sync");
    }
    if (Clock::now() > deadline) {
      api.CommAbort(ctx->comm);
      ctx->aborted = true;
      return set_error(FERRUM_ERR_TIMEOUT, "dist_sync: timed out after " +
                                               std::to_string(ctx->timeout_ms) + " ms");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // extern "C"
