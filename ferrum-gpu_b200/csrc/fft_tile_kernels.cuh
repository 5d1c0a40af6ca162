// Persistent tile kernels for the long passes of the multi-pass 1D transform
// (sm_100a).
//
// A tile is W transforms that sit next to each other in memory: W adjacent
// columns (fft_cols_tile_kernel, the strided column pass) or W consecutive
// rows stored transposed (fft_rows_t_tile_kernel, the last pass), so every
// global access moves W*8-byte row segments. One CTA of W*T threads runs per
// SM (the tile of a 4096-point pass is 128 KiB, most of the SM's shared
// memory; shorter passes fit two) and walks tiles blockIdx.x,
// blockIdx.x + gridDim.x, ... . With one or two CTAs per SM little overlaps a tile's loads with the butterflies of
// another CTA, so at the start of each tile the CTA asks the L2 for the next
// one: a bulk L2 prefetch (`cp.async.bulk.prefetch`, tiled through a tensor
// map for the strided columns, or one plain bulk prefetch per contiguous row).
// The prefetch is issued by one thread, occupies no registers or shared
// memory, and keeps HBM busy while the tile in hand is transformed; the
// loads of the next tile then hit the L2. Prefetches read this GPU's own
// memory only and never use cluster multicast.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "fft_kernels.cuh"
#include "tma_util.cuh"

namespace ferrum {

// L2 prefetch mode of a tile kernel.
enum : int {
  kPfNone = 0,    // no prefetch
  kPfThreads = 1, // every thread prefetches a few rows of the next tile (prefetch.global.L2)
  kPfTensor = 2,  // one thread, tiled bulk prefetch through a tensor map
};

__device__ __forceinline__ void l2_prefetch_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Rows per box of the tile tensor maps (a TMA box spans at most 256 rows).
constexpr int kTileBoxRows = 256;
FERRUM_HD constexpr int tile_box_rows(int log_n) { return log_n >= 8 ? kTileBoxRows : 1 << log_n; }

template <int LOGN, int LOGP, int W>
struct ColsTileCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = W * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (W < 16 ? W : 16)>::value;
  static constexpr size_t SMEM_BYTES = G::STAGES > 1 ? (size_t)W * RS * sizeof(float2) : 0;
  static_assert(THREADS <= 1024, "one CTA holds a tile");
};

// Strided pass over tiles of W adjacent columns. Transform f = (o, j, c) as in
// fft_pass_kernel (c fastest, in_c = out_c = 1, W divides 2^log_w); tile i
// holds transforms f = i*W .. i*W + W-1. With PF == kPfTensor, `map` is a 2D
// tensor map over the input with rows of in_e elements (8-byte elements), box
// {W, kTileBoxRows}; o*in_o + j*in_j must then be a multiple of in_e.
template <int LOGN, int LOGP, int W, bool CONJ_IN, bool CONJ_OUT, int TW, int PF>
__global__ void __launch_bounds__(ColsTileCfg<LOGN, LOGP, W>::THREADS,
                                  MinBlocks<ColsTileCfg<LOGN, LOGP, W>::THREADS, LOGP>::value)
fft_cols_tile_kernel(const float2* in, float2* out, const float2* __restrict__ tw, PassArgs a,
                     int64_t ntiles, const __grid_constant__ CUtensorMap map) {
  using G = Geom<LOGN, LOGP>;
  using C = ColsTileCfg<LOGN, LOGP, W>;
  extern __shared__ float2 smem[];
  const int cl = threadIdx.x % W;
  const int t = threadIdx.x / W;
  float2* sm = smem + (C::SMEM_BYTES ? cl * C::RS : 0);
  const uint32_t mask = TW ? (1u << a.log_m) - 1u : 0u;
  auto tile_base = [&](int64_t tile, int64_t& o, int64_t& j, int64_t& c) {
    pass_index(tile * W, a.log_w, a.log_j, o, j, c);
  };
  auto prefetch = [&](int64_t tile) {
    int64_t o, j, c;
    tile_base(tile, o, j, c);
    const int64_t off = o * a.in_o + j * a.in_j + c;
    if constexpr (PF == kPfThreads) {
#pragma unroll
      for (int e = threadIdx.x; e < G::N; e += C::THREADS) l2_prefetch_line(in + off + e * a.in_e);
    } else if constexpr (PF == kPfTensor) {
      if (threadIdx.x == 0) {
        const int32_t x = (int32_t)(off % a.in_e);
        const int32_t y = (int32_t)(off / a.in_e);
#pragma unroll 1
        for (int r = 0; r < G::N; r += kTileBoxRows) l2_prefetch_tile2d(&map, x, y + r);
      }
    }
  };
  if constexpr (PF != kPfNone) {
    if (blockIdx.x < ntiles) prefetch(blockIdx.x);
  }
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    if constexpr (PF != kPfNone) {
      if (tile + gridDim.x < ntiles) prefetch(tile + gridDim.x);
    }
    int64_t o, j, c;
    pass_index(tile * W + cl, a.log_w, a.log_j, o, j, c);
    const uint32_t tb = TW ? pass_tw_base((uint32_t)c, (uint32_t)j, a.tcj) : 0u;
    const uint32_t ts = TW ? pass_tw_step((uint32_t)c, (uint32_t)j, a.tc, a.tj) : 0u;
    const float2* src = in + o * a.in_o + j * a.in_j + c;
    float2* dst = out + o * a.out_o + j * a.out_j + c;
    strided_unit<LOGN, LOGP, CONJ_IN, CONJ_OUT, TW != 0, true, true, TW == 2>(
        src, a.in_e, dst, a.out_e, true, t, sm, tw, tb + ts * (uint32_t)t, ts * (uint32_t)G::T,
        a.tw_lo, a.tw_hi, mask, a.scale, SyncBlock{});
    __syncthreads();  // the next tile's first exchange rewrites the regions
  }
}

template <int LOGN, int LOGP, int W>
struct RowsTTileCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = W * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (W < 16 ? W : 16)>::value;
  static constexpr size_t SMEM_BYTES = (size_t)W * RS * sizeof(float2);
  static_assert(THREADS <= 1024, "one CTA holds a tile");
  static_assert(G::STAGES >= 2, "the transposed store rides on an exchange");
};

// Rows stored transposed (as fft_rows_t_kernel) over tiles of W consecutive
// rows f = i*W .. i*W + W-1 (W divides 2^log_w). With PF != kPfNone the next
// tile's rows (contiguous, N*8 bytes each) are prefetched into the L2 with one
// bulk prefetch per row; the row addresses must then be 16-byte aligned.
template <int LOGN, int LOGP, int W, bool CONJ_IN, bool CONJ_OUT, int PF>
__global__ void __launch_bounds__(RowsTTileCfg<LOGN, LOGP, W>::THREADS,
                                  MinBlocks<RowsTTileCfg<LOGN, LOGP, W>::THREADS, LOGP>::value)
fft_rows_t_tile_kernel(const float2* in, float2* out, const float2* __restrict__ tw, RowsTArgs a,
                       int64_t ntiles) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsTTileCfg<LOGN, LOGP, W>;
  extern __shared__ float2 smem[];
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  float2* sm = smem + g * C::RS;
  const int g2 = threadIdx.x % W;
  const int e0 = threadIdx.x / W;
  float2* row = smem + g2 * C::RS;
  auto row_src = [&](int64_t f) {
    int64_t o, j, c;
    pass_index(f, a.log_w, a.log_j, o, j, c);
    return in + o * a.in_o + j * a.in_j + c * a.in_c;
  };
  if constexpr (PF != kPfNone) {
    if (threadIdx.x < W && blockIdx.x < ntiles)
      l2_prefetch_bulk(row_src((int64_t)blockIdx.x * W + threadIdx.x), G::N * sizeof(float2));
  }
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    if constexpr (PF != kPfNone) {
      if (threadIdx.x < W && tile + gridDim.x < ntiles)
        l2_prefetch_bulk(row_src((tile + gridDim.x) * W + threadIdx.x), G::N * sizeof(float2));
    }
    float2 v[G::P];
    {
      const float2* src = row_src(tile * W + g) + t;
#pragma unroll
      for (int m = 0; m < G::P; ++m) v[m] = swap_if(ld_stream(src + G::T * m), CONJ_IN);
    }
    // Exchanges within the row's own warps, the last one regrouped so that
    // the lanes run over the tile's rows for the store.
    if constexpr (G::T <= 32)
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{}, row, e0, SyncBlock{});
    else if constexpr (W > 1 && W <= 15)
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncNamed{1 + g, G::T}, row, e0, SyncBlock{});
    else
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{}, row, e0, SyncBlock{});
    int64_t o, j, c;
    pass_index(tile * W + g2, a.log_w, a.log_j, o, j, c);
    float2* dst = out + o * a.out_o + j * a.out_j + c;
#pragma unroll
    for (int q = 0; q < G::P; ++q)
      st_stream(dst + a.out_e * (e0 + G::T * q), epilogue<CONJ_OUT>(v[q], a.scale));
    __syncthreads();  // the next tile's first exchange rewrites the regions
  }
}

// ----------------------------------------------------------------------------
// TMA tile kernels. The strided accesses of a tile (W*8-byte row segments,
// one per row) cost the load/store pipeline a cache-line lookup each when
// threads issue them; here the tensor-copy engine moves them instead, between
// global memory and a shared-memory tile buffer laid out [row][W]
// (TMA boxes of W x tile_box_rows elements), and the threads read and write
// that buffer 256 contiguous bytes per warp instruction. The same buffer
// holds the padded exchange regions while the stages run. One thread issues
// every copy; the load completes on an mbarrier whose wait is bounded
// (kWaitTimeoutNs; on expiry the CTA sets *err and returns after a bounded
// wait for its copies in flight). Tensor maps describe this GPU's own memory
// and no copy uses cluster multicast.

template <int LOGN, int LOGP, int W>
struct TmaTileCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = W * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (W < 16 ? W : 16)>::value;
  static constexpr size_t XCHG_BYTES = G::STAGES > 1 ? (size_t)W * RS * sizeof(float2) : 0;
  static constexpr size_t TILE_BYTES = (size_t)W * G::N * sizeof(float2);
  static constexpr size_t BUF_BYTES = XCHG_BYTES > TILE_BYTES ? XCHG_BYTES : TILE_BYTES;
  static constexpr size_t SMEM_BYTES = BUF_BYTES + 16;  // + mbarrier
  static constexpr int BOX_ROWS = tile_box_rows(LOGN);
  static constexpr int BOXES = G::N / BOX_ROWS;
  static_assert(THREADS <= 1024, "one CTA holds a tile");
  static_assert((W * sizeof(float2)) % 16 == 0, "TMA rows are multiples of 16 bytes");
};

// TMA coordinates {x, y} of element `off` of a 2D map whose rows hold `ld`
// elements.
FERRUM_HD __forceinline__ void tile_coords(int64_t off, int64_t ld, int32_t& x, int32_t& y) {
  x = (int32_t)(off % ld);
  y = (int32_t)(off / ld);
}

// Strided pass (fft_pass_kernel's transform indexing, in_c = out_c = 1) over
// tiles of W adjacent columns, loaded and stored by TMA: `in_map` is a 2D map
// over the input with rows of in_e elements, `out_map` over the output with
// rows of out_e elements, both with 8-byte elements and boxes
// {W, tile_box_rows(LOGN)}; o*in_o + j*in_j must be a multiple of in_e and
// o*out_o + j*out_j of out_e. The next tile is prefetched into the L2 while
// the current one is transformed, so its load from the L2 is short.
template <int LOGN, int LOGP, int W, bool CONJ_IN, bool CONJ_OUT, int TW>
__global__ void __launch_bounds__(TmaTileCfg<LOGN, LOGP, W>::THREADS,
                                  MinBlocks<TmaTileCfg<LOGN, LOGP, W>::THREADS, LOGP>::value)
fft_cols_tma_kernel(const float2* __restrict__ tw, PassArgs a, int64_t ntiles,
                    const __grid_constant__ CUtensorMap in_map,
                    const __grid_constant__ CUtensorMap out_map, int* err) {
  using G = Geom<LOGN, LOGP>;
  using C = TmaTileCfg<LOGN, LOGP, W>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float2* buf = reinterpret_cast<float2*>(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw + C::BUF_BYTES);
  const int cl = threadIdx.x % W;
  const int t = threadIdx.x / W;
  float2* sm = buf + cl * C::RS;
  const uint32_t mask = TW ? (1u << a.log_m) - 1u : 0u;
  auto first = [&](int64_t tile, int64_t so, int64_t sj) {
    int64_t o, j, c;
    pass_index(tile * W, a.log_w, a.log_j, o, j, c);
    return o * so + j * sj + c;
  };
  auto issue_load = [&](int64_t tile) {
    int32_t x, y;
    tile_coords(first(tile, a.in_o, a.in_j), a.in_e, x, y);
    mbar_arrive_expect_tx(bar, (uint32_t)C::TILE_BYTES);
#pragma unroll 1
    for (int b = 0; b < C::BOXES; ++b)
      tma_load_tile2d(buf + b * C::BOX_ROWS * W, &in_map, x, y + b * C::BOX_ROWS, bar);
  };
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  int64_t tile = blockIdx.x;
  if (threadIdx.x == 0 && tile < ntiles) issue_load(tile);
  uint32_t phase = 0;
  for (; tile < ntiles; tile += gridDim.x) {
    const int64_t next = tile + gridDim.x;
    if (threadIdx.x == 0 && next < ntiles) {
      int32_t x, y;
      tile_coords(first(next, a.in_o, a.in_j), a.in_e, x, y);
#pragma unroll 1
      for (int b = 0; b < C::BOXES; ++b) l2_prefetch_tile2d(&in_map, x, y + b * C::BOX_ROWS);
    }
    const bool ok = mbar_wait_bounded(bar, phase);
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) {
        atomicOr(err, kErrWaitTimeout);
        mbar_wait_bounded(bar, phase);
        bulk_wait_all();
      }
      return;
    }
    phase ^= 1u;
    float2 v[G::P];
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = swap_if(buf[(t + G::T * m) * W + cl], CONJ_IN);
    __syncthreads();  // the tile is in registers; the exchanges reuse the buffer
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{});
    if constexpr (TW != 0) {
      int64_t o, j, c;
      pass_index(tile * W + cl, a.log_w, a.log_j, o, j, c);
      const uint32_t tb = pass_tw_base((uint32_t)c, (uint32_t)j, a.tcj);
      const uint32_t ts = pass_tw_step((uint32_t)c, (uint32_t)j, a.tc, a.tj);
      apply_progression_twiddles<G::P>(v, a.tw_lo, a.tw_hi, tb + ts * (uint32_t)t,
                                       ts * (uint32_t)G::T, mask, TW == 2);
    }
    if constexpr (G::STAGES > 1) __syncthreads();  // every read of the last exchange is done
#pragma unroll
    for (int m = 0; m < G::P; ++m) buf[(t + G::T * m) * W + cl] = epilogue<CONJ_OUT>(v[m], a.scale);
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      int32_t x, y;
      tile_coords(first(tile, a.out_o, a.out_j), a.out_e, x, y);
#pragma unroll 1
      for (int b = 0; b < C::BOXES; ++b)
        tma_store_tile2d(&out_map, x, y + b * C::BOX_ROWS, buf + b * C::BOX_ROWS * W);
      bulk_commit();
      if (next < ntiles) {
        bulk_wait_read_all();  // the store has read the buffer
        issue_load(next);
      }
    }
  }
  if (threadIdx.x == 0) bulk_wait_all();
}

// Rows stored transposed (fft_rows_t_kernel's indexing) over tiles of W
// consecutive rows: contiguous loads by the threads (the next tile's rows
// prefetched into the L2 with bulk prefetches), the W x N output tile staged
// in the buffer as [k][W] and stored by TMA through `out_map`, a 2D map over
// the output with rows of out_e elements and boxes {W, tile_box_rows(LOGN)};
// o*out_o + j*out_j must be a multiple of out_e. Row addresses must be
// 16-byte aligned for the prefetch.
template <int LOGN, int LOGP, int W, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(TmaTileCfg<LOGN, LOGP, W>::THREADS,
                                  MinBlocks<TmaTileCfg<LOGN, LOGP, W>::THREADS, LOGP>::value)
fft_rows_t_tma_kernel(const float2* in, const float2* __restrict__ tw, RowsTArgs a, int64_t ntiles,
                      const __grid_constant__ CUtensorMap out_map) {
  using G = Geom<LOGN, LOGP>;
  using C = TmaTileCfg<LOGN, LOGP, W>;
  static_assert(G::STAGES >= 2, "the transposed store rides on an exchange");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float2* buf = reinterpret_cast<float2*>(smem_raw);
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  float2* sm = buf + g * C::RS;
  const int g2 = threadIdx.x % W;
  const int e0 = threadIdx.x / W;
  float2* row = buf + g2 * C::RS;
  auto row_src = [&](int64_t f) {
    int64_t o, j, c;
    pass_index(f, a.log_w, a.log_j, o, j, c);
    return in + o * a.in_o + j * a.in_j + c * a.in_c;
  };
  if (threadIdx.x < W && blockIdx.x < ntiles)
    l2_prefetch_bulk(row_src((int64_t)blockIdx.x * W + threadIdx.x), G::N * sizeof(float2));
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    if (threadIdx.x < W && tile + gridDim.x < ntiles)
      l2_prefetch_bulk(row_src((tile + gridDim.x) * W + threadIdx.x), G::N * sizeof(float2));
    float2 v[G::P];
    {
      const float2* src = row_src(tile * W + g) + t;
#pragma unroll
      for (int m = 0; m < G::P; ++m) v[m] = swap_if(ld_stream(src + G::T * m), CONJ_IN);
    }
    if (threadIdx.x == 0) bulk_wait_read_all();  // the previous tile's store has read the buffer
    __syncthreads();
    if constexpr (G::T <= 32)
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{}, row, e0, SyncBlock{});
    else if constexpr (W > 1 && W <= 15)
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncNamed{1 + g, G::T}, row, e0, SyncBlock{});
    else
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{}, row, e0, SyncBlock{});
    __syncthreads();  // every read of the last exchange is done
#pragma unroll
    for (int q = 0; q < G::P; ++q)
      buf[(e0 + G::T * q) * W + g2] = epilogue<CONJ_OUT>(v[q], a.scale);
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      int64_t o, j, c;
      pass_index(tile * W, a.log_w, a.log_j, o, j, c);
      int32_t x, y;
      tile_coords(o * a.out_o + j * a.out_j + c, a.out_e, x, y);
#pragma unroll 1
      for (int b = 0; b < C::BOXES; ++b)
        tma_store_tile2d(&out_map, x, y + b * C::BOX_ROWS, buf + b * C::BOX_ROWS * W);
      bulk_commit();
    }
  }
  if (threadIdx.x == 0) bulk_wait_all();
}

}  // namespace ferrum
