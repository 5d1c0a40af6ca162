// Kernels of the distributed 2D transform that move data over NVLink
// themselves (one process per GPU, peer pointers from CUDA IPC):
//
//   fft_rows_scatter_kernel  row FFTs whose store writes each B x B block
//                            straight into the destination rank's receive
//                            slab (peer stores), so the exchange overlaps the
//                            butterflies of the same kernel;
//   fft_rows_gather_kernel   row FFTs whose load reads each row's B-wide
//                            pieces from the ranks that hold them (peer
//                            loads), the inverse direction;
//   peer_block_gather_kernel the row-slab gather without an FFT (the second
//                            exchange of a row -> row transform);
//   dist_barrier_kernel      a barrier across the ranks' GPUs through flags
//                            in peer memory, with a bounded wait.
//
// Plain loads and stores to peer memory only: no TMA and no multicast.
// Block layout (the receive slab of rank q is its N x B column slab,
// row-major): row f of rank p's slab, columns [q*B, (q+1)*B), lives at
// slab_q + p*B*B + f*B. The PeerPtrs tables passed to the kernels hold
// slab_q + p*B*B for the calling rank p, so element e of local row f is at
// p[e >> log_b] + (f << log_b) + (e & (B - 1)).
#pragma once

#include <stdint.h>

#include "dist_steps.h"
#include "dist_types.h"
#include "fft_kernels.cuh"
#include "fft_rows_tma.cuh"

namespace ferrum {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Copies the pointer table into shared memory with compile-time indices (a
// kernel parameter indexed at run time would be copied to local memory by
// every thread) and makes it visible to the CTA.
__device__ __forceinline__ void load_peer_table(float2** tab, const PeerPtrs& ptrs) {
  if (threadIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < kMaxPeers; ++k) tab[k] = ptrs.p[k];
  }
  __syncthreads();
}

template <int LOGN, int LOGP, int FPB, bool CONJ_IN>
__global__ void __launch_bounds__(RowsCfg<LOGN, LOGP, FPB, CONJ_IN, false>::THREADS,
                                  MinBlocks<RowsCfg<LOGN, LOGP, FPB, CONJ_IN, false>::THREADS, LOGP>::value)
fft_rows_scatter_kernel(const float2* __restrict__ in, PeerPtrs dst, const float2* __restrict__ tw,
                        int64_t nfft, int log_b) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsCfg<LOGN, LOGP, FPB, CONJ_IN, false>;
  extern __shared__ float2 smem[];
  __shared__ float2* peer_tab[kMaxPeers];
  load_peer_table(peer_tab, dst);
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  const int64_t f = (int64_t)blockIdx.x * FPB + g;
  const bool valid = f < nfft;
  float2 v[G::P];
  if (valid) {
    const float2* src = in + f * G::N + t;
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = swap_if(ld_stream(src + G::T * m), CONJ_IN);
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  float2* sm = smem + (C::NEEDS_SMEM ? g * C::RS : 0);
  if constexpr (G::T <= 32)
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
  else
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{});
  if (valid) {
#pragma unroll
    for (int m = 0; m < G::P; ++m) {
      const int e = t + G::T * m;
      peer_tab[e >> log_b][peer_offset(f, e, log_b)] = v[m];
    }
  }
}

template <int LOGN, int LOGP, int FPB, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsCfg<LOGN, LOGP, FPB, false, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsCfg<LOGN, LOGP, FPB, false, CONJ_OUT>::THREADS, LOGP>::value)
fft_rows_gather_kernel(PeerPtrs src, float2* __restrict__ out, const float2* __restrict__ tw,
                       int64_t nfft, float scale, int log_b) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsCfg<LOGN, LOGP, FPB, false, CONJ_OUT>;
  extern __shared__ float2 smem[];
  __shared__ float2* peer_tab[kMaxPeers];
  load_peer_table(peer_tab, src);
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  const int64_t f = (int64_t)blockIdx.x * FPB + g;
  const bool valid = f < nfft;
  float2 v[G::P];
  if (valid) {
#pragma unroll
    for (int m = 0; m < G::P; ++m) {
      const int e = t + G::T * m;
      v[m] = ld_stream(peer_tab[e >> log_b] + peer_offset(f, e, log_b));
    }
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  float2* sm = smem + (C::NEEDS_SMEM ? g * C::RS : 0);
  if constexpr (G::T <= 32)
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
  else
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{});
  if (valid) {
    float2* dst = out + f * G::N + t;
#pragma unroll
    for (int m = 0; m < G::P; ++m) st_stream(dst + G::T * m, epilogue<CONJ_OUT>(v[m], scale));
  }
}

// out[r*out_ld + q*B + c] = src.p[q][r*B + c] for q < nranks, r < rows, c < B;
// one thread moves two complex values (B even, 16-byte aligned bases).
__global__ void __launch_bounds__(256) peer_block_gather_kernel(PeerPtrs src, float4* __restrict__ out,
                                                                int nranks, int64_t rows,
                                                                int64_t b2, int64_t out_ld2) {
  __shared__ float2* peer_tab[kMaxPeers];
  load_peer_table(peer_tab, src);
  const int64_t total2 = (int64_t)nranks * rows * b2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total2; i += stride) {
    const int64_t c = i % b2;
    const int64_t r = (i / b2) % rows;
    const int q = (int)(i / (b2 * rows));
    const float4* s = reinterpret_cast<const float4*>(peer_tab[q]);
    out[r * out_ld2 + q * b2 + c] = __ldcs(s + r * b2 + c);
  }
}

// Barrier across the ranks' GPUs. Thread q < nranks publishes this rank's
// arrival in rank q's flag word [rank] (release, system scope, after a
// system-scope fence so that every earlier write of this GPU, including the
// peer stores of the kernels before it on the stream, is visible first) and
// then waits for rank q's arrival in its own word [q] (acquire). A wait that
// exceeds timeout_ns sets *err and returns, so a rank that never arrives
// leaves an error the host reads instead of a hung GPU.
__global__ void __launch_bounds__(32) dist_barrier_kernel(PeerFlags flags, int rank, int nranks,
                                                          uint32_t epoch, uint64_t timeout_ns,
                                                          int* err) {
  const int q = threadIdx.x;
  if (q >= nranks) return;
  __threadfence_system();
  st_release_sys(flags.p[q] + rank, epoch);
  const uint32_t* mine = flags.p[rank] + q;
  const uint64_t t0 = global_ns();
  while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
    if (global_ns() - t0 > timeout_ns) {
      atomicExch(err, 1);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace ferrum
