// Split (planar) complex layout: real and imaginary parts in two float arrays.
// The reference keeps split twins of its radix kernels and a set of layout
// helpers for its layout study (crates/ferrum-gpu-fft-kernels/src/
// kernels_body.rs:508-626 fft_c2c_1024_split, 1614-1672 cmul_interleaved,
// cmul_split, deinterleave, interleave). Here:
//   fft_rows_split_kernel  the single-pass batched 1D transform reading and
//                          writing the two float streams directly (same
//                          butterflies and exchanges as fft_rows_kernel);
//   cmul_*, (de)interleave elementwise, one complex value per thread step.
#pragma once

#include <stdint.h>

#include "fft_kernels.cuh"

namespace ferrum {

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS, LOGP>::value)
fft_rows_split_kernel(const float* __restrict__ in_re, const float* __restrict__ in_im,
                      float* __restrict__ out_re, float* __restrict__ out_im,
                      const float2* __restrict__ tw, int64_t nfft, float scale) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>;
  extern __shared__ float2 smem[];
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  const int64_t f = (int64_t)blockIdx.x * FPB + g;
  const bool valid = f < nfft;
  float2* sm = smem + (C::NEEDS_SMEM ? g * C::RS : 0);
  float2 v[G::P];
  if constexpr (C::STAGED) {
    // As fft_rows_kernel: the CTA's contiguous tile through padded shared
    // memory, so the two float streams are read and written lane-contiguous.
    const int64_t base = (int64_t)blockIdx.x * C::TILE;
    const int64_t total = nfft * G::N;
    // (the inverse's input step applied on the read-out, as in fft_rows_kernel)
#pragma unroll
    for (int i = threadIdx.x; i < C::TILE; i += C::THREADS)
      smem[tile_pad(i)] = base + i < total
                              ? make_float2(__ldcs(in_re + base + i), __ldcs(in_im + base + i))
                              : make_float2(0.f, 0.f);
    __syncthreads();
#pragma unroll
    for (int m = 0; m < G::P; ++m)
      v[m] = swap_if(smem[tile_pad(g * G::N + t + G::T * m)], CONJ_IN);
    __syncthreads();
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
    __syncthreads();
#pragma unroll
    for (int m = 0; m < G::P; ++m)
      smem[tile_pad(g * G::N + t + G::T * m)] = epilogue<CONJ_OUT>(v[m], scale);
    __syncthreads();
#pragma unroll
    for (int i = threadIdx.x; i < C::TILE; i += C::THREADS)
      if (base + i < total) {
        const float2 r = smem[tile_pad(i)];
        __stcs(out_re + base + i, r.x);
        __stcs(out_im + base + i, r.y);
      }
  } else {
    if (valid) {
      const int64_t o = f * G::N + t;
#pragma unroll
      for (int m = 0; m < G::P; ++m)
        v[m] = swap_if(make_float2(__ldcs(in_re + o + G::T * m), __ldcs(in_im + o + G::T * m)),
                       CONJ_IN);
    } else {
#pragma unroll
      for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
    }
    if constexpr (G::T <= 32)
      run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
    else if constexpr (FPB > 1 && FPB <= 15)
      run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncNamed{1 + g, G::T});
    else
      run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{});
    if (valid) {
      const int64_t o = f * G::N + t;
#pragma unroll
      for (int m = 0; m < G::P; ++m) {
        const float2 r = epilogue<CONJ_OUT>(v[m], scale);
        __stcs(out_re + o + G::T * m, r.x);
        __stcs(out_im + o + G::T * m, r.y);
      }
    }
  }
}

// (ar + i ai)(br + i bi) with each product and sum rounded separately (the
// reference's expression, not fused into FMAs).
__device__ __forceinline__ float2 cmul_rn(float ar, float ai, float br, float bi) {
  return make_float2(__fsub_rn(__fmul_rn(ar, br), __fmul_rn(ai, bi)),
                     __fadd_rn(__fmul_rn(ar, bi), __fmul_rn(ai, br)));
}

__global__ void __launch_bounds__(256) cmul_interleaved_kernel(const float2* __restrict__ a,
                                                               const float2* __restrict__ b,
                                                               float2* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 x = __ldcs(a + i), y = __ldcs(b + i);
    __stcs(out + i, cmul_rn(x.x, x.y, y.x, y.y));
  }
}

__global__ void __launch_bounds__(256) cmul_split_kernel(const float* __restrict__ a_re,
                                                         const float* __restrict__ a_im,
                                                         const float* __restrict__ b_re,
                                                         const float* __restrict__ b_im,
                                                         float* __restrict__ o_re,
                                                         float* __restrict__ o_im, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 r = cmul_rn(__ldcs(a_re + i), __ldcs(a_im + i), __ldcs(b_re + i), __ldcs(b_im + i));
    __stcs(o_re + i, r.x);
    __stcs(o_im + i, r.y);
  }
}

__global__ void __launch_bounds__(256) deinterleave_kernel(const float2* __restrict__ in,
                                                           float* __restrict__ re,
                                                           float* __restrict__ im, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = __ldcs(in + i);
    __stcs(re + i, v.x);
    __stcs(im + i, v.y);
  }
}

__global__ void __launch_bounds__(256) interleave_kernel(const float* __restrict__ re,
                                                         const float* __restrict__ im,
                                                         float2* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    __stcs(out + i, make_float2(__ldcs(re + i), __ldcs(im + i)));
}

}  // namespace ferrum
