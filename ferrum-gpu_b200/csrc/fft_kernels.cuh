// sm_100a FFT pass kernels. Each kernel is one HBM read and one HBM write of
// every element it touches; all butterflies run in registers and the groups
// exchange values through padded shared memory (stockham.cuh).
//
//   fft_rows_kernel    FPB contiguous length-N transforms per CTA
//                      (batched 1D, the 2D row pass, the distributed row pass)
//   fft_pass_kernel    FPB adjacent columns per CTA, strided elements, an
//                      optional twiddle fused into the store (2D column
//                      passes, column passes of the multi-pass 1D transform)
//   fft_rows_t_kernel  FPB contiguous rows per CTA, stored transposed through
//                      shared memory (last pass of the multi-pass 1D
//                      transform: X[k1 + N1*k2 + ...] in natural order)
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
template <int LOGN, int LOGP, int G>
struct RegionStride {
  static constexpr int base = PaddedLen<LOGN, LOGP>::value;
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

// Resident CTAs per SM to target: 1024 threads' worth (64 registers per
// thread), at most 32 CTAs; threads owning 32 values get 128 registers.
template <int THREADS, int LOGP = 4>
struct MinBlocks {
  static constexpr int threads_per_sm = LOGP >= 5 ? 512 : 1024;
  static constexpr int value = (THREADS >= threads_per_sm)
                                   ? 1
                                   : (threads_per_sm / THREADS > 32 ? 32 : threads_per_sm / THREADS);
};

// ----------------------------------------------------------------------------
// Contiguous rows: transform f occupies in[f*N, (f+1)*N).
template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
struct RowsCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int GROUPS_PER_HALFWARP = (G::T >= 16) ? 1 : (16 / G::T);
  static constexpr int RS = RegionStride<LOGN, LOGP, GROUPS_PER_HALFWARP>::value;
  static constexpr bool NEEDS_SMEM = G::STAGES > 1;
  static constexpr size_t SMEM_BYTES = NEEDS_SMEM ? (size_t)FPB * RS * sizeof(float2) : 0;
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS, LOGP>::value)
fft_rows_kernel(const float2* in, float2* out, const float2* __restrict__ tw, int64_t nfft,
                float scale, int log_block, int64_t block_rows) {
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
      // to block q = e >> log_block, laid out [q][f][e mod 2^log_block] with
      // block_rows rows per block, so each destination rank's block is
      // contiguous (a chunk of rows writes the middle of every block).
#pragma unroll
      for (int m = 0; m < G::P; ++m)
        st_stream(out + blocked_index(f, t + G::T * m, log_block, block_rows),
                  epilogue<CONJ_OUT>(v[m], scale));
    }
  }
}

// ----------------------------------------------------------------------------
// Strided pass. `nfft` length-N transforms, transform f = (o, j, c) with c the
// fastest index (c < 2^log_w, j < 2^log_j): element e is read at
//   in [o*in_o  + j*in_j  + c + e*in_e]
// and output k is written to
//   out[o*out_o + j*out_j + c + k*out_e],
// multiplied, when log_m > 0, by the twiddle W_M^((c*j*tcj + (c*tc + j*tj)*k) mod M),
// M = 2^log_m. Adjacent columns c are adjacent in memory on both sides, so a
// CTA of FPB columns reads and writes FPB*8-byte row segments; lanes run over
// the columns first. Used for 2D column passes (one or two sub-passes), the
// column passes of the multi-pass 1D transform and the distributed column
// pass.
struct PassArgs {
  int64_t nfft;
  int log_w;
  int log_j;
  int64_t in_o, in_j, in_e;
  int64_t out_o, out_j, out_e;
  uint32_t tcj, tc, tj;
  int log_m;
  const float2* tw_lo;
  const float2* tw_hi;
  float scale;
};

FERRUM_HD __forceinline__ void pass_index(int64_t f, int log_w, int log_j, int64_t& o, int64_t& j,
                                          int64_t& c) {
  c = f & (((int64_t)1 << log_w) - 1);
  j = (f >> log_w) & (((int64_t)1 << log_j) - 1);
  o = f >> (log_w + log_j);
}

// Twiddle exponent of output k (mod 2^32; the caller masks to M).
FERRUM_HD __forceinline__ uint32_t pass_tw_base(uint32_t c, uint32_t j, uint32_t tcj) {
  return c * j * tcj;
}
FERRUM_HD __forceinline__ uint32_t pass_tw_step(uint32_t c, uint32_t j, uint32_t tc, uint32_t tj) {
  return c * tc + j * tj;
}

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT, bool TW>
struct PassCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (FPB < 16 ? FPB : 16)>::value;
  static constexpr size_t SMEM_BYTES = G::STAGES > 1 ? (size_t)FPB * RS * sizeof(float2) : 0;
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT, bool TW>
__global__ void __launch_bounds__(PassCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT, TW>::THREADS,
                                  MinBlocks<PassCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT, TW>::THREADS, LOGP>::value)
fft_pass_kernel(const float2* in, float2* out, const float2* __restrict__ tw, PassArgs a) {
  using G = Geom<LOGN, LOGP>;
  using C = PassCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT, TW>;
  extern __shared__ float2 smem[];
  const int cl = threadIdx.x % FPB;
  const int t = threadIdx.x / FPB;
  const int64_t f = (int64_t)blockIdx.x * FPB + cl;
  const bool valid = f < a.nfft;
  int64_t o, j, c;
  pass_index(f, a.log_w, a.log_j, o, j, c);

  float2 v[G::P];
  if (valid) {
    const float2* src = in + o * a.in_o + j * a.in_j + c + (int64_t)t * a.in_e;
    const int64_t step = (int64_t)G::T * a.in_e;
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = conj_if(ld_stream(src + step * m), CONJ_IN);
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  if constexpr (FPB == 1 && G::T <= 32)
    run_stages<LOGN, LOGP, 0>(v, smem + (C::SMEM_BYTES ? cl * C::RS : 0), t, tw, SyncWarp{});
  else
    run_stages<LOGN, LOGP, 0>(v, smem + (C::SMEM_BYTES ? cl * C::RS : 0), t, tw, SyncBlock{});
  if (valid) {
    float2* dst = out + o * a.out_o + j * a.out_j + c + (int64_t)t * a.out_e;
    const int64_t step = (int64_t)G::T * a.out_e;
    if constexpr (TW) {
      // Output k = t + T*m takes W_M^(tb + ts*k): a progression in m.
      const uint32_t tb = pass_tw_base((uint32_t)c, (uint32_t)j, a.tcj);
      const uint32_t ts = pass_tw_step((uint32_t)c, (uint32_t)j, a.tc, a.tj);
      apply_progression_twiddles<G::P>(v, a.tw_lo, a.tw_hi, tb + ts * (uint32_t)t,
                                       ts * (uint32_t)G::T, (1u << a.log_m) - 1u);
    }
#pragma unroll
    for (int m = 0; m < G::P; ++m) st_stream(dst + step * m, epilogue<CONJ_OUT>(v[m], a.scale));
  }
}

// ----------------------------------------------------------------------------
// Rows stored transposed. Transform f = (o, j, c), c fastest: its N elements
// are contiguous at in[o*in_o + j*in_j + c*in_c], and output k goes to
// out[o*out_o + j*out_j + c + k*out_e]. FPB adjacent c share a CTA, which
// transposes them through shared memory so that stores run over c
// (FPB*8-byte segments). Used for the last pass of the multi-pass 1D
// transform, where X[k1 + N1*k2 + ...] must land in natural order.
struct RowsTArgs {
  int64_t nfft;
  int log_w;
  int log_j;
  int64_t in_o, in_j, in_c;
  int64_t out_o, out_j, out_e;
  float scale;
};

template <int LOGN, int LOGP, int FPB, bool CONJ_OUT>
struct RowsTCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (FPB < 16 ? FPB : 16)>::value;
  static constexpr size_t SMEM_BYTES = (size_t)FPB * RS * sizeof(float2);
};

template <int LOGN, int LOGP, int FPB, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsTCfg<LOGN, LOGP, FPB, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsTCfg<LOGN, LOGP, FPB, CONJ_OUT>::THREADS, LOGP>::value)
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
    int64_t o, j, c;
    pass_index(f, a.log_w, a.log_j, o, j, c);
    const float2* src = in + o * a.in_o + j * a.in_j + c * a.in_c + t;
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
  for (int m = 0; m < G::P; ++m) sm[stage_read_addr<LOGN, LOGP>(t, m)] = v[m];
  __syncthreads();
  const int g2 = threadIdx.x % FPB;
  const int e0 = threadIdx.x / FPB;
  const int64_t f2 = (int64_t)blockIdx.x * FPB + g2;
  if (f2 < a.nfft) {
    int64_t o, j, c;
    pass_index(f2, a.log_w, a.log_j, o, j, c);
    float2* dst = out + o * a.out_o + j * a.out_j + c;
    const float2* row = smem + g2 * C::RS;
#pragma unroll
    for (int q = 0; q < G::P; ++q) {
      const int e = e0 + G::T * q;
      st_stream(dst + a.out_e * e, epilogue<CONJ_OUT>(row[stage_read_addr<LOGN, LOGP>(e0, q)], a.scale));
    }
  }
}

}  // namespace ferrum
