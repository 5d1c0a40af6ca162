// Bulk-copy (TMA) helpers and the persistent prefetching rows kernel
// (sm_100a).
//
// fft_rows_pf_kernel: each CTA owns a strided sequence of tiles (FPB
// contiguous transforms). Once the last exchange of tile i has been read, one
// elected thread moves tile i+1 from HBM into the CTA's exchange buffer with
// a single `cp.async.bulk.shared::cluster.global` copy (no multicast; the
// source is this GPU's own memory) that completes on an mbarrier, so the HBM
// read overlaps the last stage and the stores of tile i. Every mbarrier wait
// is bounded (%globaltimer, 1 s): on expiry the CTA raises a device error
// flag that the host reads, waits (again bounded) for its own copy in flight,
// and returns.
#pragma once

#include <stdint.h>

#include "fft_kernels.cuh"
#include "tma_util.cuh"

namespace ferrum {

// ----------------------------------------------------------------------------
// Persistent rows kernel that prefetches into the exchange buffer itself.
// No extra shared memory: once the last exchange of tile i has been read, the
// group's padded exchange regions are free, so one elected thread starts the
// bulk copy of tile i+1 into them (unpadded, contiguous) and the copy overlaps
// the last stage and the stores of tile i. Stage 0 of tile i+1 reads its
// values from shared memory; a barrier then separates those reads from the
// first exchange writes. For N = 8192 / 16384 (one or two CTAs per SM, whose
// load phase is otherwise exposed).
template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
struct RowsPfCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, 1>::value;
  static constexpr size_t TILE_ELEMS = (size_t)FPB * G::N;
  static constexpr size_t TILE_BYTES = TILE_ELEMS * sizeof(float2);
  static constexpr size_t XCHG_BYTES = (size_t)FPB * RS * sizeof(float2);
  static constexpr size_t SMEM_BYTES = XCHG_BYTES + 16;
  static_assert(XCHG_BYTES >= TILE_BYTES, "the tile must fit the exchange regions");
  static_assert(G::STAGES >= 2, "needs at least one exchange");
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsPfCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsPfCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS, LOGP>::value)
fft_rows_pf_kernel(const float2* __restrict__ in, float2* out, const float2* __restrict__ tw,
                   int64_t nfft, float scale, int* err) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsPfCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float2* xchg = reinterpret_cast<float2*>(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw + C::XCHG_BYTES);

  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  const int64_t ntiles = (nfft + FPB - 1) / FPB;
  float2* sm = xchg + g * C::RS;

  auto tile_bytes = [&](int64_t tile) -> uint32_t {
    const int64_t rows = (nfft - tile * FPB) < FPB ? (nfft - tile * FPB) : FPB;
    return (uint32_t)(rows * G::N * sizeof(float2));
  };

  int64_t tile = blockIdx.x;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0 && tile < ntiles) {
    const uint32_t b = tile_bytes(tile);
    mbar_arrive_expect_tx(bar, b);
    bulk_g2s(xchg, in + tile * C::TILE_ELEMS, b, bar);
  }

  uint32_t phase = 0;
  for (; tile < ntiles; tile += gridDim.x) {
    const bool ok = mbar_wait_bounded(bar, phase);
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) {
        atomicOr(err, kErrWaitTimeout);
        mbar_wait_bounded(bar, phase);
      }
      return;
    }
    phase ^= 1u;
    const int64_t f = tile * FPB + g;
    const bool valid = f < nfft;
    float2 v[G::P];
    const float2* src = xchg + g * G::N + t;  // the tile, unpadded
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = swap_if(src[G::T * m], CONJ_IN);
    __syncthreads();  // tile reads done before the first exchange writes
    const int64_t next = tile + gridDim.x;
    auto prefetch = [&]() {
      // Exchange regions free: order the generic reads before the async-proxy
      // write, then start the next tile's copy.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (threadIdx.x == 0 && next < ntiles) {
        const uint32_t b = tile_bytes(next);
        mbar_arrive_expect_tx(bar, b);
        bulk_g2s(xchg, in + next * C::TILE_ELEMS, b, bar);
      }
    };
    if constexpr (G::T <= 32)
      run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{}, prefetch);
    else
      run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{}, prefetch);
    if (valid) {
      float2* dst = out + f * G::N + t;
#pragma unroll
      for (int m = 0; m < G::P; ++m) st_stream(dst + G::T * m, epilogue<CONJ_OUT>(v[m], scale));
    }
  }
}

}  // namespace ferrum
