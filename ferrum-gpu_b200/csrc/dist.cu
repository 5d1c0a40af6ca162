// Distributed 2D FFT over NCCL (one process per GPU). New in this build: the
// reference has no multi-GPU code (every context is CudaContext::new(0),
// crates/ferrum-gpu-py/src/lib.rs:261,385).
//
// A single N x N image is split over P ranks (B = N/P) as row slabs or
// column slabs (dist_steps.h). Row slab in:
//   1. row FFTs of the local slab, chunk by chunk; the store writes B x B
//      blocks, one per destination rank ([q][row][col]);
//   2. NCCL exchange of each chunk as soon as it is written (own stream), so
//      it overlaps the next chunk's row FFTs. The received blocks, stacked by
//      source rank, are this rank's N x B column slab, row-major;
//   3. column FFTs of the column slab (length N, row pitch B), one pass or,
//      for N >= 2048, two sub-passes with 16 columns per CTA. With a
//      column-slab output the transform ends here (one exchange in total);
//   4. for a row-slab output: exchange of the column slab's B x B row blocks
//      chunk by chunk, each received chunk gathered into the output rows.
// Column slab in (the inverse of a column-slab forward): column FFTs, then
// chunked exchange, gather and row FFTs.
//
// Peer-memory path (the default on up to 8 ranks when CUDA IPC works between
// all of them): every rank holds one receive slab exported with CUDA IPC and
// mapped by the others, so the exchange is fused into the FFT kernels
// (dist_kernels.cuh). Row slab in: the row-FFT kernel stores each B x B block
// straight into the destination rank's slab over NVLink; after a barrier the
// column passes run on the local slab. Column slab in: column passes into the
// local slab, a barrier, then a row-FFT kernel that loads its rows from the
// ranks' slabs. Row -> row adds a peer-load gather of the column results. The
// barriers are one-CTA kernels on flag words in the same IPC allocations
// (bounded waits; a timeout sets a device flag that ferrum_dist_sync
// reports), and every call starts with one so that no rank writes a slab
// another rank still reads. Set-up agreement: the ranks all-gather their IPC
// handles and then whether they could map every peer; if any could not (or
// FERRUM_DIST_P2P=0 is set on any rank) all ranks use the NCCL path.
//
// NCCL is opened with dlopen so that the single-GPU library never depends on
// it; when PyTorch is loaded first its libnccl.so.2 is reused. The
// communicator is non-blocking, so set-up and every host wait are bounded by
// the context's timeout, after which the communicator is aborted and
// FERRUM_ERR_TIMEOUT returned.
#include <cuda_runtime.h>

#include <algorithm>
#include <dlfcn.h>
#include <nccl.h>

#include <stdlib.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "dist_steps.h"
#include "dist_types.h"
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
  // NCCL runs on its own stream so that the exchange of one chunk of rows
  // overlaps the kernels of the next; events hand chunks between the streams.
  cudaStream_t comm_stream = nullptr;
  static constexpr int kEvents = 16;
  cudaEvent_t ev[kEvents] = {};
  // Peer-memory path: one cudaMalloc per rank, [flag words | receive slab],
  // exported with CUDA IPC; peer_base[q] is rank q's allocation as mapped
  // here (peer_base[rank] = p2p_base).
  int p2p = -1;  // -1 undecided (decided collectively at the first call), 0 NCCL path, 1 peer path
  bool p2p_want = true;
  char* p2p_base = nullptr;
  size_t p2p_slab_bytes = 0;
  char* peer_base[ferrum::kMaxPeers] = {};
  uint32_t epoch = 0;
  int* err = nullptr;      // device flag: a peer barrier timed out
  char* stage = nullptr;   // device staging of the set-up all-gathers
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
  decltype(&ncclAllGather) AllGather = nullptr;
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
  FERRUM_SYM(AllGather, ncclAllGather)
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

// Exchange of rows [r0, r1) of every B x B block (dist_steps.h): to rank q
// from src + q*B*B + r0*B, from rank p into dst + p*B*B + r0*B.
ferrum_status all_to_all_rows(ferrum_dist_ctx* ctx, const float2* src, float2* dst, int64_t b,
                              int64_t r0, int64_t r1, cudaStream_t stream) {
  NcclApi& api = nccl();
  const size_t count = (size_t)(2 * (r1 - r0) * b);
  ncclResult_t r = api.GroupStart();
  if (r != ncclSuccess) return nccl_error(r, "ncclGroupStart");
  for (int q = 0; q < ctx->nranks; ++q) {
    r = api.Send(src + dist_block_offset(q, r0, b), count, ncclFloat32, q, ctx->comm, stream);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(r, "ncclSend");
    r = api.Recv(dst + dist_block_offset(q, r0, b), count, ncclFloat32, q, ctx->comm, stream);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(r, "ncclRecv");
  }
  r = api.GroupEnd();
  if (r == ncclInProgress) return wait_comm(ctx, "all-to-all enqueue");
  if (r != ncclSuccess) return nccl_error(r, "ncclGroupEnd");
  return FERRUM_OK;
}

// Polls `stream` until it drains, bounded by the context's timeout; on
// timeout or an NCCL error the communicator is aborted.
ferrum_status wait_stream(ferrum_dist_ctx* ctx, cudaStream_t stream, const char* what) {
  NcclApi& api = nccl();
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  for (;;) {
    cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) return FERRUM_OK;
    if (e != cudaErrorNotReady) return cuda_error(e, what);
    ncclResult_t st = ncclSuccess;
    if (api.CommGetAsyncError(ctx->comm, &st) == ncclSuccess && st != ncclSuccess &&
        st != ncclInProgress) {
      api.CommAbort(ctx->comm);
      ctx->aborted = true;
      return nccl_error(st, what);
    }
    if (Clock::now() > deadline) {
      api.CommAbort(ctx->comm);
      ctx->aborted = true;
      return set_error(FERRUM_ERR_TIMEOUT, std::string(what) + ": timed out after " +
                                               std::to_string(ctx->timeout_ms) + " ms");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Reads (and clears) the device flag a timed-out peer barrier sets. After a
// timeout the ranks are out of step, so the context is marked unusable.
ferrum_status check_barrier_flag(ferrum_dist_ctx* ctx) {
  if (ctx->err == nullptr) return FERRUM_OK;
  int h = 0;
  cudaError_t e = cudaMemcpy(&h, ctx->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_error(e, "reading the peer-barrier flag");
  if (h == 0) return FERRUM_OK;
  cudaMemset(ctx->err, 0, sizeof(int));
  NcclApi& api = nccl();
  if (!ctx->aborted && ctx->comm) api.CommAbort(ctx->comm);
  ctx->aborted = true;
  return set_error(FERRUM_ERR_TIMEOUT, "peer barrier: a rank did not arrive within " +
                                           std::to_string(ctx->timeout_ms) + " ms");
}

// --- peer-memory path --------------------------------------------------------

constexpr size_t kFlagBytes = 4096;  // flag words ahead of the slab (keeps it 256-byte aligned)

struct PeerRecord {
  cudaIpcMemHandle_t handle;
  int32_t ok;
  char pad[60];
};
static_assert(sizeof(PeerRecord) == 128, "PeerRecord layout");

// All-gather of `bytes` per rank through the communicator (stream ordered,
// then waited for with the context's timeout).
ferrum_status allgather_host(ferrum_dist_ctx* ctx, const void* mine, void* all, size_t bytes,
                             cudaStream_t stream) {
  NcclApi& api = nccl();
  char* st = ctx->stage;
  cudaError_t e = cudaMemcpyAsync(st + bytes * ctx->rank, mine, bytes, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return cuda_error(e, "set-up all-gather staging");
  ncclResult_t r = api.AllGather(st + bytes * ctx->rank, st, bytes, ncclUint8, ctx->comm, stream);
  if (r == ncclInProgress) {
    if (ferrum_status s = wait_comm(ctx, "set-up all-gather")) return s;
  } else if (r != ncclSuccess) {
    return nccl_error(r, "ncclAllGather");
  }
  e = cudaMemcpyAsync(all, st, bytes * ctx->nranks, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return cuda_error(e, "set-up all-gather readback");
  return wait_stream(ctx, stream, "set-up all-gather");
}

// Host-waited rendezvous of all ranks through the communicator.
ferrum_status nccl_rendezvous(ferrum_dist_ctx* ctx, cudaStream_t stream, const char* what) {
  std::vector<int32_t> all(ctx->nranks);
  const int32_t mine = 1;
  ferrum_status s = allgather_host(ctx, &mine, all.data(), sizeof(int32_t), stream);
  if (s != FERRUM_OK) return set_error(s, std::string(what) + ": " + ferrum_last_error());
  return FERRUM_OK;
}

// Tears the peer mappings down. `collective`: other ranks have mapped this
// rank's allocation, so first every rank's device work must be finished (no
// kernel may still read or write a peer slab), then the ranks unmap, meet
// again, and only then free: an exporter may free its allocation only after
// every importer has closed its mapping. The rendezvous go through the
// communicator, never through peer memory, so a rank that has already left
// is never written to. When the ranks cannot meet (an aborted communicator)
// the own allocation is left allocated rather than freed under another
// rank's mapping.
void p2p_release(ferrum_dist_ctx* ctx, bool collective, cudaStream_t stream) {
  bool may_free = !collective;
  if (collective) {
    cudaDeviceSynchronize();
    if (!ctx->aborted) may_free = nccl_rendezvous(ctx, stream, "peer teardown") == FERRUM_OK;
  }
  for (int q = 0; q < ctx->nranks && q < kMaxPeers; ++q) {
    if (q != ctx->rank && ctx->peer_base[q]) cudaIpcCloseMemHandle(ctx->peer_base[q]);
    ctx->peer_base[q] = nullptr;
  }
  if (collective && may_free && !ctx->aborted)
    may_free = nccl_rendezvous(ctx, stream, "peer teardown") == FERRUM_OK;
  if (ctx->p2p_base && may_free) cudaFree(ctx->p2p_base);
  ctx->p2p_base = nullptr;
  ctx->p2p_slab_bytes = 0;
  cudaGetLastError();
}

float2* peer_slab(const ferrum_dist_ctx* ctx, int q) {
  return reinterpret_cast<float2*>(ctx->peer_base[q] + kFlagBytes);
}

// Every rank arrives, then every rank proceeds (stream ordered).
ferrum_status p2p_barrier(ferrum_dist_ctx* ctx, cudaStream_t stream) {
  PeerFlags flags{};
  for (int q = 0; q < ctx->nranks; ++q) flags.p[q] = reinterpret_cast<uint32_t*>(ctx->peer_base[q]);
  const uint64_t timeout_ns = (uint64_t)ctx->timeout_ms * 1000000ull;
  cudaError_t e = launch_dist_barrier(flags, ctx->rank, ctx->nranks, ++ctx->epoch, timeout_ns,
                                      ctx->err, stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "peer barrier launch");
}

// Collective: makes the peer path ready for slabs of `slab_bytes`, or settles
// on the NCCL path. Every rank calls it with the same size in the same call.
ferrum_status p2p_prepare(ferrum_dist_ctx* ctx, size_t slab_bytes, cudaStream_t stream) {
  if (ctx->p2p == 0) return FERRUM_OK;
  if (ctx->p2p == 1 && ctx->p2p_slab_bytes >= slab_bytes) return FERRUM_OK;
  // Rebuild (first use, or a larger transform); p2p_release waits until no
  // rank uses the old mappings.
  if (ferrum_status s = wait_stream(ctx, stream, "peer set-up")) return s;
  if (ferrum_status s = check_barrier_flag(ctx)) return s;
  p2p_release(ctx, ctx->p2p == 1, stream);
  if (ctx->aborted) return set_error(FERRUM_ERR_NCCL, "peer set-up: communicator aborted");
  PeerRecord mine{};
  mine.ok = ctx->p2p_want ? 1 : 0;
  if (mine.ok) {
    void* base = nullptr;
    cudaError_t e = cudaMalloc(&base, kFlagBytes + slab_bytes);
    if (e == cudaSuccess) {
      ctx->p2p_base = static_cast<char*>(base);
      e = cudaMemsetAsync(base, 0, kFlagBytes, stream);
    }
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine.handle, base);
    if (e != cudaSuccess) {
      cudaGetLastError();
      mine.ok = 0;
    }
  }
  std::vector<PeerRecord> all(ctx->nranks);
  if (ferrum_status s = allgather_host(ctx, &mine, all.data(), sizeof(PeerRecord), stream)) {
    p2p_release(ctx, false, stream);  // no rank has mapped the new allocation yet
    return s;
  }
  int32_t mapped = mine.ok;
  for (int q = 0; q < ctx->nranks; ++q)
    if (!all[q].ok) mapped = 0;
  for (int q = 0; mapped && q < ctx->nranks; ++q) {
    if (q == ctx->rank) continue;
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, all[q].handle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      mapped = 0;
      break;
    }
    ctx->peer_base[q] = static_cast<char*>(p);
  }
  std::vector<int32_t> oks(ctx->nranks);
  if (ferrum_status s = allgather_host(ctx, &mapped, oks.data(), sizeof(int32_t), stream)) {
    p2p_release(ctx, true, stream);  // the communicator is aborted: unmap, keep the allocation
    return s;
  }
  bool everyone = true;
  for (int32_t v : oks) everyone = everyone && v == 1;
  if (!everyone) {
    p2p_release(ctx, true, stream);
    ctx->p2p = 0;
    return FERRUM_OK;
  }
  ctx->peer_base[ctx->rank] = ctx->p2p_base;
  ctx->p2p_slab_bytes = slab_bytes;
  ctx->epoch = 0;
  ctx->p2p = 1;
  return FERRUM_OK;
}

// The transform over peer memory (see the file comment).
ferrum_status dist_p2p(ferrum_dist_ctx* ctx, const float2* in, float2* out, int log_n, bool inv,
                       float scale, bool row_in, bool row_out, cudaStream_t stream) {
  ferrum_device* dev = ctx->dev;
  const int64_t n = (int64_t)1 << log_n;
  const int64_t b = n / ctx->nranks;
  const int lb = ilog2(b);
  const float2* tw = stage_table(dev, log_n);
  PeerPtrs blocks{};
  for (int q = 0; q < ctx->nranks; ++q) blocks.p[q] = peer_slab(ctx, q) + ctx->rank * b * b;
  float2* mine = peer_slab(ctx, ctx->rank);
  // The column passes of the local slab; their workspace (an intermediate
  // slab, or the fused kernel's scratch slots) is sized from the plan itself.
  PassPlan cols;
  if (row_in)
    plan_columns(cols, log_n, lb, b, 1, n * b, false, inv, scale, PassBuf::In, PassBuf::Ws,
                 PassBuf::Out);
  else
    plan_columns(cols, log_n, lb, b, 1, n * b, inv, false, 1.0f, PassBuf::In, PassBuf::Ws,
                 PassBuf::Out);
  int64_t ws_elems = cols.ws_elems;
  for (int i = 0; i < cols.count; ++i)
    if (cols.p[i].src == PassBuf::Ws || cols.p[i].dst == PassBuf::Ws)
      ws_elems = std::max<int64_t>(ws_elems, b * n);
  void* ws = nullptr;
  if (ws_elems > 0) {
    cudaError_t e = cudaMallocFromPoolAsync(&ws, (size_t)ws_elems * sizeof(float2), dev->pool, stream);
    if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(dist workspace)");
  }
  ferrum_status s = FERRUM_OK;
  auto launched = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && s == FERRUM_OK) s = cuda_error(e, what);
    return s == FERRUM_OK;
  };
  do {
    if ((s = p2p_barrier(ctx, stream)) != FERRUM_OK) break;
    if (row_in) {
      if (!launched(launch_rows_scatter(log_n, inv, in, blocks, tw, b, lb, stream),
                    "distributed row pass (peer stores)"))
        break;
      if ((s = p2p_barrier(ctx, stream)) != FERRUM_OK) break;
      if ((s = run_plan(dev, cols, mine, row_out ? mine : out, (float2*)ws, stream)) != FERRUM_OK)
        break;
      if (!row_out) break;
      if ((s = p2p_barrier(ctx, stream)) != FERRUM_OK) break;
      launched(launch_peer_block_gather(blocks, out, ctx->nranks, b, b, n, stream),
               "row-slab gather (peer loads)");
    } else {
      if ((s = run_plan(dev, cols, in, mine, (float2*)ws, stream)) != FERRUM_OK) break;
      if ((s = p2p_barrier(ctx, stream)) != FERRUM_OK) break;
      launched(launch_rows_gather(log_n, inv, blocks, out, tw, b, scale, lb, stream),
               "distributed row pass (peer loads)");
    }
  } while (false);
  if (ws) {
    cudaError_t ef = cudaFreeAsync(ws, stream);
    if (s == FERRUM_OK && ef != cudaSuccess) return cuda_error(ef, "cudaFreeAsync(dist workspace)");
  }
  return s;
}

// `waiter` waits for the work enqueued so far on `from`.
cudaError_t hand_over(ferrum_dist_ctx* ctx, int slot, cudaStream_t from, cudaStream_t waiter) {
  cudaError_t e = cudaEventRecord(ctx->ev[slot], from);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(waiter, ctx->ev[slot], 0);
  return e;
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
  cudaError_t e = cudaStreamCreateWithFlags(&ctx->comm_stream, cudaStreamNonBlocking);
  for (int i = 0; e == cudaSuccess && i < ferrum_dist_ctx::kEvents; ++i)
    e = cudaEventCreateWithFlags(&ctx->ev[i], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->err, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->stage, (size_t)nranks * sizeof(PeerRecord));
  const char* want = getenv("FERRUM_DIST_P2P");
  ctx->p2p_want = !(want && want[0] == '0');
  ctx->p2p = (nranks > 1 && nranks <= kMaxPeers) ? -1 : 0;
  if (e != cudaSuccess) {
    ferrum_dist_destroy(ctx);
    return cuda_error(e, "dist_init: stream/event creation");
  }
  *out = ctx;
  return FERRUM_OK;
}

ferrum_status ferrum_dist_destroy(ferrum_dist_ctx* ctx) {
  clear_error();
  if (ctx == nullptr) return FERRUM_OK;
  NcclApi& api = nccl();
  DeviceGuard guard(ctx->dev->ordinal);
  if (ctx->comm_stream) cudaStreamSynchronize(ctx->comm_stream);
  // No rank may unmap or free a slab another rank still uses (p2p_release).
  p2p_release(ctx, ctx->p2p == 1, ctx->comm_stream);
  if (ctx->err) cudaFree(ctx->err);
  if (ctx->stage) cudaFree(ctx->stage);
  if (ctx->comm && !ctx->aborted && api.ok) api.CommDestroy(ctx->comm);
  for (int i = 0; i < ferrum_dist_ctx::kEvents; ++i)
    if (ctx->ev[i]) cudaEventDestroy(ctx->ev[i]);
  if (ctx->comm_stream) cudaStreamDestroy(ctx->comm_stream);
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

ferrum_status ferrum_fft_2d_c2c_pow2_dist_layout(ferrum_dist_ctx* ctx, const void* in_dev,
                                                 void* out_dev, int log_n, int direction,
                                                 int normalize, int in_layout, int out_layout,
                                                 void* stream_ptr) {
  clear_error();
  if (ferrum_status s = check_ctx(ctx)) return s;
  if (ferrum_status s = ferrum_dist_check(log_n, ctx->nranks)) return s;
  if (direction != 1 && direction != -1)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2_dist: direction must be +1 or -1");
  const bool row_in = in_layout == FERRUM_DIST_ROW_SLAB, row_out = out_layout == FERRUM_DIST_ROW_SLAB;
  if ((in_layout != FERRUM_DIST_ROW_SLAB && in_layout != FERRUM_DIST_COL_SLAB) ||
      (out_layout != FERRUM_DIST_ROW_SLAB && out_layout != FERRUM_DIST_COL_SLAB) ||
      (!row_in && !row_out))
    return set_error(FERRUM_ERR_INVALID_ARG,
                     "fft_2d_c2c_pow2_dist: layouts must be row->row, row->column or column->row");
  if (in_dev == nullptr || out_dev == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2_dist: in/out is NULL");
  if (((uintptr_t)in_dev & 15) || ((uintptr_t)out_dev & 15))
    return set_error(FERRUM_ERR_INVALID_ARG, "fft_2d_c2c_pow2_dist: in/out must be 16-byte aligned");
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  ferrum_device* dev = ctx->dev;
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  if (ctx->nranks == 1) {
    // One rank: both layouts are the whole image, row-major.
    const size_t need = workspace_2d_bytes(log_n, 1);
    void* ws1 = nullptr;
    if (need > 0) {
      cudaError_t e = cudaMallocFromPoolAsync(&ws1, need, dev->pool, stream);
      if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(2D workspace)");
    }
    ferrum_status s1 = enqueue_2d(dev, (const float2*)in_dev, (float2*)out_dev, log_n, 1,
                                  direction, normalize != 0, (float2*)ws1, stream);
    if (ws1) cudaFreeAsync(ws1, stream);
    return s1;
  }

  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const int64_t b = n / ctx->nranks;
  const int lb = ilog2(b);
  const int chunks = dist_chunks(b);
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  if (ferrum_status sp = p2p_prepare(ctx, (size_t)(b * n) * sizeof(float2), stream)) return sp;
  if (ctx->p2p == 1)
    return dist_p2p(ctx, (const float2*)in_dev, (float2*)out_dev, log_n, inv, scale, row_in,
                    row_out, stream);
  const float2* tw = stage_table(dev, log_n);
  const float2* in = (const float2*)in_dev;
  float2* out = (float2*)out_dev;
  cudaStream_t cs = ctx->comm_stream;
  void* ws = nullptr;
  const size_t slab_bytes = (size_t)(b * n) * sizeof(float2);
  cudaError_t e = cudaMallocFromPoolAsync(&ws, 2 * slab_bytes, dev->pool, stream);
  if (e != cudaSuccess) return cuda_error(e, "cudaMallocFromPoolAsync(dist workspace)");
  float2* wa = (float2*)ws;
  float2* wb = wa + b * n;
  ferrum_status s = FERRUM_OK;
  int ev = 0;
  auto cuda_step = [&](cudaError_t err, const char* what) {
    if (err != cudaSuccess && s == FERRUM_OK) s = cuda_error(err, what);
    return s == FERRUM_OK;
  };
  do {
    if (row_in) {
      // Row FFTs chunk by chunk, each chunk's blocks exchanged while the next
      // chunk computes: in -> wa (blocked) -> wb (column slab).
      for (int c = 0; c < chunks && s == FERRUM_OK; ++c) {
        int64_t r0, r1;
        dist_chunk(b, chunks, c, r0, r1);
        if (!cuda_step(launch_rows(log_n, inv, false, in + r0 * n, wa + r0 * b, tw, r1 - r0, 1.0f,
                                   stream, lb, nullptr, b),
                       "distributed row pass launch"))
          break;
        if (!cuda_step(hand_over(ctx, ev++, stream, cs), "event")) break;
        s = all_to_all_rows(ctx, wa, wb, b, r0, r1, cs);
      }
      if (s != FERRUM_OK || !cuda_step(hand_over(ctx, ev++, cs, stream), "event")) break;
      // Column FFTs of the N x B column slab (row pitch B); they apply the
      // inverse's conjugate and scale.
      PassPlan cols;
      plan_columns(cols, log_n, lb, b, 1, n * b, false, inv, scale, PassBuf::In, PassBuf::In,
                   PassBuf::Out);
      if ((s = run_plan(dev, cols, wb, row_out ? wa : out, nullptr, stream)) != FERRUM_OK) break;
      if (!row_out) break;
      // Back to row slabs: exchange the column slab's B x B row blocks chunk by
      // chunk and gather each received chunk into the output rows.
      if (!cuda_step(hand_over(ctx, ev++, stream, cs), "event")) break;
      for (int c = 0; c < chunks && s == FERRUM_OK; ++c) {
        int64_t r0, r1;
        dist_chunk(b, chunks, c, r0, r1);
        if ((s = all_to_all_rows(ctx, wa, wb, b, r0, r1, cs)) != FERRUM_OK) break;
        if (!cuda_step(hand_over(ctx, ev++, cs, stream), "event")) break;
        cuda_step(launch_block_gather(wb + r0 * b, out + r0 * n, ctx->nranks, r1 - r0, b, b * b, n,
                                      stream),
                  "block gather launch");
      }
    } else {
      // Column slab in: column FFTs (in -> wa -> wb), exchange of row blocks,
      // gather into row slabs and row FFTs, chunk by chunk.
      PassPlan cols;
      plan_columns(cols, log_n, lb, b, 1, n * b, inv, false, 1.0f, PassBuf::In, PassBuf::Out,
                   PassBuf::Ws);
      if ((s = run_plan(dev, cols, in, wa, wb, stream)) != FERRUM_OK) break;
      if (!cuda_step(hand_over(ctx, ev++, stream, cs), "event")) break;
      for (int c = 0; c < chunks && s == FERRUM_OK; ++c) {
        int64_t r0, r1;
        dist_chunk(b, chunks, c, r0, r1);
        if ((s = all_to_all_rows(ctx, wb, wa, b, r0, r1, cs)) != FERRUM_OK) break;
        if (!cuda_step(hand_over(ctx, ev++, cs, stream), "event")) break;
        if (!cuda_step(launch_block_gather(wa + r0 * b, out + r0 * n, ctx->nranks, r1 - r0, b,
                                           b * b, n, stream),
                       "block gather launch"))
          break;
        cuda_step(launch_rows(log_n, false, inv, out + r0 * n, out + r0 * n, tw, r1 - r0, scale,
                              stream, -1, dev->err_flag),
                  "distributed row pass launch");
      }
    }
  } while (false);
  // The pool memory is released on `stream`, which by now waits for every
  // exchange that reads or writes it.
  if (ev > 0 && s != FERRUM_OK) hand_over(ctx, ferrum_dist_ctx::kEvents - 1, cs, stream);
  cudaError_t ef = cudaFreeAsync(ws, stream);
  if (s == FERRUM_OK && ef != cudaSuccess) return cuda_error(ef, "cudaFreeAsync(dist workspace)");
  return s;
}

ferrum_status ferrum_fft_2d_c2c_pow2_dist(ferrum_dist_ctx* ctx, const void* in_slab_dev,
                                          void* out_slab_dev, int log_n, int direction,
                                          int normalize, void* stream) {
  return ferrum_fft_2d_c2c_pow2_dist_layout(ctx, in_slab_dev, out_slab_dev, log_n, direction,
                                            normalize, FERRUM_DIST_ROW_SLAB, FERRUM_DIST_ROW_SLAB,
                                            stream);
}

ferrum_status ferrum_dist_barrier(ferrum_dist_ctx* ctx, void* stream_ptr) {
  clear_error();
  if (ferrum_status s = check_ctx(ctx)) return s;
  DeviceGuard guard(ctx->dev->ordinal);
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  if (ctx->nranks == 1) return FERRUM_OK;
  if (ctx->p2p == 1) return p2p_barrier(ctx, stream);
  NcclApi& api = nccl();
  ncclResult_t r = api.AllGather(ctx->stage + sizeof(int32_t) * ctx->rank, ctx->stage,
                                 sizeof(int32_t), ncclUint8, ctx->comm, stream);
  if (r == ncclInProgress) return wait_comm(ctx, "dist_barrier");
  return r == ncclSuccess ? FERRUM_OK : nccl_error(r, "dist_barrier");
}

int ferrum_dist_peer_path(const ferrum_dist_ctx* ctx) { return ctx ? ctx->p2p : -2; }

ferrum_status ferrum_dist_abort(ferrum_dist_ctx* ctx) {
  clear_error();
  if (ctx == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "dist_abort: NULL ctx");
  if (!ctx->aborted) {
    NcclApi& api = nccl();
    if (ctx->comm && api.ok) api.CommAbort(ctx->comm);
    ctx->aborted = true;
  }
  return FERRUM_OK;
}

ferrum_status ferrum_dist_set_timeout(ferrum_dist_ctx* ctx, int timeout_ms) {
  clear_error();
  if (ctx == nullptr) return set_error(FERRUM_ERR_INVALID_ARG, "dist_set_timeout: NULL ctx");
  if (timeout_ms <= 0) return set_error(FERRUM_ERR_INVALID_ARG, "dist_set_timeout: timeout_ms must be > 0");
  ctx->timeout_ms = timeout_ms;
  return FERRUM_OK;
}

ferrum_status ferrum_dist_sync(ferrum_dist_ctx* ctx, void* stream_ptr) {
  clear_error();
  if (ferrum_status s = check_ctx(ctx)) return s;
  DeviceGuard guard(ctx->dev->ordinal);
  if (ferrum_status s = wait_stream(ctx, (cudaStream_t)stream_ptr, "dist_sync")) return s;
  return check_barrier_flag(ctx);
}

}  // extern "C"
