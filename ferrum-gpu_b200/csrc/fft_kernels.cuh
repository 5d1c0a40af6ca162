// sm_100a FFT pass kernels. Each kernel is one HBM read and one HBM write of
// every element it touches; all butterflies run in registers and the groups
// exchange values through padded shared memory (stockham.cuh).
//
//   fft_rows_kernel    FPB contiguous length-N transforms per CTA
//                      (batched 1D, the 2D row pass, the distributed row pass)
//   fft_cols_kernel    FPB adjacent columns per CTA, elements `ld` apart
//                      (2D column pass, four-step pass A with the
//                      W_N^(n2*k1) twiddle fused into the store)
//   fft_rows_t_kernel  FPB contiguous rows per CTA, stored transposed through
//                      shared memory (four-step pass B: X[k1 + N1*k2])
//
// Inverse transforms use the reference's conjugation identity
// IFFT(x) = conj(FFT(conj(x))) (crates/ferrum-gpu-fft/src/cpu.rs:106-121),
// fused into the loads (CONJ_IN) and the stores (CONJ_OUT, which also applies
// the optional 1/N scale), so no extra pass runs.
#pragma once

#include <stdint.h>

#include "stockham.cuh"

namespace ferrum {

struct SyncBlock {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
struct SyncWarp {
  __device__ __forceinline__ void operator()() const { __syncwarp(); }
};

// Per-group shared-memory stride (complex slots). `G` groups share one
// half-warp (16 lanes, one 128-byte wavefront of 8-byte accesses); a stride
// congruent to 16/G mod 16 puts their accesses on disjoint bank pairs.
template <int LOGN, int G>
struct RegionStride {
  static constexpr int base = PaddedLen<LOGN>::value;
  static constexpr int want = (G <= 1) ? (base & 15) : ((16 / G) & 15);
  static constexpr int value = base + ((want - (base & 15) + 16) & 15);
};

__device__ __forceinline__ float2 ld_stream(const float2* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float2* p, float2 v) { __stcs(p, v); }

__device__ __forceinline__ float2 conj_if(float2 v, bool c) { return c ? make_float2(v.x, -v.y) : v; }

template <bool CONJ_OUT>
__device__ __forceinline__ float2 epilogue(float2 v, float scale) {
  if constexpr (CONJ_OUT) return make_float2(v.x * scale, -v.y * scale);
  return v;
}

template <int THREADS>
struct MinBlocks {
  static constexpr int value = (THREADS >= 1024) ? 1 : (1024 / THREADS);
};

// ----------------------------------------------------------------------------
// Contiguous rows: transform f occupies in[f*N, (f+1)*N).
template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
struct RowsCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int GROUPS_PER_HALFWARP = (G::T >= 16) ? 1 : (16 / G::T);
  static constexpr int RS = RegionStride<LOGN, GROUPS_PER_HALFWARP>::value;
  static constexpr bool NEEDS_SMEM = G::STAGES > 1;
  static constexpr size_t SMEM_BYTES = NEEDS_SMEM ? (size_t)FPB * RS * sizeof(float2) : 0;
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS>::value)
fft_rows_kernel(const float2* in, float2* out, const float2* __restrict__ tw, int64_t nfft,
                float scale, int log_block) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>;
  extern __shared__ float2 smem[];
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  const int64_t f = (int64_t)blockIdx.x * FPB + g;
  const bool valid = f < nfft;

  float2 v[G::P];
  if (valid) {
    const float2* src = in + f * G::N + t;
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = conj_if(ld_stream(src + G::T * m), CONJ_IN);
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
    if (log_block >= LOGN) {
      float2* dst = out + f * G::N + t;
#pragma unroll
      for (int m = 0; m < G::P; ++m) st_stream(dst + G::T * m, epilogue<CONJ_OUT>(v[m], scale));
    } else {
      // Blocked store for the distributed 2D transform: element e of row f goes
      // to block q = e >> log_block, laid out [q][f][e mod 2^log_block], so
      // each destination rank's block is contiguous.
#pragma unroll
      for (int m = 0; m < G::P; ++m)
        st_stream(out + blocked_index(f, t + G::T * m, log_block, nfft),
                  epilogue<CONJ_OUT>(v[m], scale));
    }
  }
}

// ----------------------------------------------------------------------------
// Strided columns. Transform f = img * cols + col has element e at
// in[img * img_stride + col + e * ld]. Lanes run over the FPB adjacent
// columns first so each row segment of FPB values is one coalesced access.
struct ColsArgs {
  int64_t nfft;        // images * cols
  int64_t img_stride;  // elements between images
  int64_t ld;          // elements between consecutive elements of a column
  int log_cols;        // log2(columns per image)
  float scale;
  const float2* tw4_lo;  // four-step twiddle W_Ntot^e, e in [0, 4096)
  const float2* tw4_hi;  // four-step twiddle W_Ntot^(4096 h)
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT, bool TW4>
struct ColsCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, (FPB < 16 ? FPB : 16)>::value;
  static constexpr size_t SMEM_BYTES = (size_t)FPB * RS * sizeof(float2);
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT, bool TW4>
__global__ void __launch_bounds__(ColsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT, TW4>::THREADS,
                                  MinBlocks<ColsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT, TW4>::THREADS>::value)
fft_cols_kernel(const float2* in, float2* out, const float2* __restrict__ tw, ColsArgs a) {
  using G = Geom<LOGN, LOGP>;
  using C = ColsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT, TW4>;
  extern __shared__ float2 smem[];
  const int c = threadIdx.x % FPB;
  const int t = threadIdx.x / FPB;
  const int64_t f = (int64_t)blockIdx.x * FPB + c;
  const bool valid = f < a.nfft;
  const int64_t img = f >> a.log_cols;
  const int64_t col = f & (((int64_t)1 << a.log_cols) - 1);
  const int64_t base = img * a.img_stride + col;

  float2 v[G::P];
  if (valid) {
    const float2* src = in + base + (int64_t)t * a.ld;
    const int64_t step = (int64_t)G::T * a.ld;
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = conj_if(ld_stream(src + step * m), CONJ_IN);
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  run_stages<LOGN, LOGP, 0>(v, smem + c * C::RS, t, tw, SyncBlock{});
  if (valid) {
    float2* dst = out + base + (int64_t)t * a.ld;
    const int64_t step = (int64_t)G::T * a.ld;
#pragma unroll
    for (int m = 0; m < G::P; ++m) {
      float2 r = v[m];
      if constexpr (TW4) {
        // Output k1 = t + T*m of column n2 = col: multiply by W_Ntot^(n2*k1).
        const uint32_t e = (uint32_t)col * (uint32_t)(t + G::T * m);
        r = c_mul(r, four_step_twiddle(a.tw4_lo, a.tw4_hi, e));
      }
      st_stream(dst + step * m, epilogue<CONJ_OUT>(r, a.scale));
    }
  }
}

// ----------------------------------------------------------------------------
// Rows stored transposed. Transform b holds `rows` contiguous rows of length N;
// output element k2 of row k1 goes to out[b * rows * N + k1 + rows * k2].
struct RowsTArgs {
  int64_t nfft;  // transforms * rows
  int log_rows;  // log2(rows per transform)
  float scale;
};

template <int LOGN, int LOGP, int FPB, bool CONJ_OUT>
struct RowsTCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, (FPB < 16 ? FPB : 16)>::value;
  static constexpr size_t SMEM_BYTES = (size_t)FPB * RS * sizeof(float2);
};

template <int LOGN, int LOGP, int FPB, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsTCfg<LOGN, LOGP, FPB, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsTCfg<LOGN, LOGP, FPB, CONJ_OUT>::THREADS>::value)
fft_rows_t_kernel(const float2* in, float2* out, const float2* __restrict__ tw, RowsTArgs a) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsTCfg<LOGN, LOGP, FPB, CONJ_OUT>;
  extern __shared__ float2 smem[];
  const int g = threadIdx.x / G::T;
  const int t = threadIdx.x % G::T;
  const int64_t f = (int64_t)blockIdx.x * FPB + g;
  const bool valid = f < a.nfft;

  float2 v[G::P];
  if (valid) {
    const float2* src = in + f * G::N + t;
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = ld_stream(src + G::T * m);
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  float2* sm = smem + g * C::RS;
  if constexpr (G::T <= 32)
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
  else
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{});

  // Transpose FPB rows through shared memory so that lanes run over rows.
  __syncthreads();
#pragma unroll
  for (int m = 0; m < G::P; ++m) sm[smem_pad(t + G::T * m)] = v[m];
  __syncthreads();
  const int g2 = threadIdx.x % FPB;
  const int e0 = threadIdx.x / FPB;
  const int64_t f2 = (int64_t)blockIdx.x * FPB + g2;
  if (f2 < a.nfft) {
    const int64_t rows = (int64_t)1 << a.log_rows;
    const int64_t img = f2 >> a.log_rows;
    const int64_t k1 = f2 & (rows - 1);
    float2* dst = out + img * rows * G::N + k1;
    const float2* row = smem + g2 * C::RS;
#pragma unroll
    for (int q = 0; q < G::P; ++q) {
      const int e = e0 + G::T * q;
      st_stream(dst + rows * e, epilogue<CONJ_OUT>(row[smem_pad(e)], a.scale));
    }
  }
}

}  // namespace ferrum
