// sm_100a FFT pass kernels. Each kernel is one HBM read and one HBM write of
// every element it touches; all butterflies run in registers and the groups
// exchange values through padded shared memory (stockham.cuh).
//
//   fft_rows_kernel    FPB contiguous length-N transforms per CTA
//                      (batched 1D, the 2D row pass, the distributed row pass)
//   fft_pass_kernel    FPB adjacent columns per CTA, strided elements, an
//                      optional twiddle fused into the store (2D column
//                      passes, column passes of the multi-pass 1D transform)
//   fft_rows_t_kernel  FPB contiguous rows per CTA, stored transposed (the
//                      last stage runs with lanes over the rows; last pass of
//                      the multi-pass 1D transform: X[k1 + N1*k2 + ...] in
//                      natural order)
//
// Inverse transforms use the reference's conjugation identity
// IFFT(x) = conj(FFT(conj(x))) (crates/ferrum-gpu-fft/src/cpu.rs:106-121),
// fused into the loads (CONJ_IN) and the stores (CONJ_OUT, which also applies
// the optional 1/N scale), so no extra pass runs. On the device the two steps
// swap the real and imaginary parts instead of negating one: with
// swap(z) = i*conj(z) and F the (C-linear) forward transform of all passes,
// swap(F(swap(x))) = i*conj(i*F(conj(x))) = conj(F(conj(x))), and a swap is
// only a choice of registers where a conjugate costs a negation per value
// (measured: the inverse of 2^21 x 128 +8.2 % over the forward with negations,
// +1.5 % with swaps).
#pragma once

#include <stdint.h>

#include <type_traits>

#include "stockham.cuh"

namespace ferrum {

struct SyncBlock {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
struct SyncWarp {
  __device__ __forceinline__ void operator()() const { __syncwarp(); }
};
// Barrier of the `count` threads (whole warps) of one thread group, on named
// barrier `id` (1..15; 0 is __syncthreads).
struct SyncNamed {
  int id, count;
  __device__ __forceinline__ void operator()() const {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
  }
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

// The inverse's input step (CONJ_IN): swap the real and imaginary parts.
__device__ __forceinline__ float2 swap_if(float2 v, bool c) { return c ? make_float2(v.y, v.x) : v; }

// The inverse's output step (CONJ_OUT): swap, times the scale.
template <bool CONJ_OUT>
__device__ __forceinline__ float2 epilogue(float2 v, float scale) {
  if constexpr (CONJ_OUT) return make_float2(v.y * scale, v.x * scale);
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
  // With at most four threads per transform (N <= 64) the CTA's FPB contiguous
  // transforms are loaded and stored through shared memory: lane-contiguous
  // global accesses (256 bytes per warp instruction) instead of lanes N
  // values apart, which cost a cache line per lane and made these sizes
  // L1-bound. The tile is padded by one slot per 16 values, so each thread's
  // own values (stride N) also read without bank conflicts.
  static constexpr bool STAGED = G::T <= 4;
  static constexpr int TILE = FPB * G::N;
  static constexpr size_t XCHG_BYTES = NEEDS_SMEM ? (size_t)FPB * RS * sizeof(float2) : 0;
  static constexpr size_t STAGE_BYTES = STAGED ? (size_t)(TILE + TILE / 16) * sizeof(float2) : 0;
  static constexpr size_t SMEM_BYTES = XCHG_BYTES > STAGE_BYTES ? XCHG_BYTES : STAGE_BYTES;
};

__device__ __forceinline__ int tile_pad(int i) { return i + (i >> 4); }

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
  float2* sm = smem + (C::NEEDS_SMEM ? g * C::RS : 0);

  float2 v[G::P];
  if constexpr (C::STAGED) {
    if (log_block >= LOGN) {  // unblocked store (the blocked one keeps the direct path)
      const int64_t base = (int64_t)blockIdx.x * C::TILE;
      const int64_t total = nfft * G::N;
      // The copy stays a plain load/store loop; the inverse's input step is
      // applied as each thread reads its own values (a negation inside the
      // copy halved the N = 16 inverse: 0.318 vs 0.159 ms per 512 MiB).
#pragma unroll
      for (int i = threadIdx.x; i < C::TILE; i += C::THREADS)
        smem[tile_pad(i)] = base + i < total ? ld_stream(in + base + i) : make_float2(0.f, 0.f);
      __syncthreads();
#pragma unroll
      for (int m = 0; m < G::P; ++m)
        v[m] = swap_if(smem[tile_pad(g * G::N + t + G::T * m)], CONJ_IN);
      __syncthreads();  // the exchange regions overlay the tile
      run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
      __syncthreads();
#pragma unroll
      for (int m = 0; m < G::P; ++m)
        smem[tile_pad(g * G::N + t + G::T * m)] = epilogue<CONJ_OUT>(v[m], scale);
      __syncthreads();
#pragma unroll
      for (int i = threadIdx.x; i < C::TILE; i += C::THREADS)
        if (base + i < total) st_stream(out + base + i, smem[tile_pad(i)]);
      return;
    }
  }
  if (valid) {
    const float2* src = in + f * G::N + t;
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = swap_if(ld_stream(src + G::T * m), CONJ_IN);
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  // A transform spanning several warps orders its exchanges with a named
  // barrier of its own warps (N = 2048: 4 % faster than block barriers).
  if constexpr (G::T <= 32)
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
  else if constexpr (FPB > 1 && FPB <= 15)
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncNamed{1 + g, G::T});
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
//   in [o*in_o  + j*in_j  + c*in_c  + e*in_e]
// and output k is written to
//   out[o*out_o + j*out_j + c*out_c + k*out_e],
// multiplied, when log_m > 0, by the twiddle W_M^((c*j*tcj + (c*tc + j*tj)*k) mod M),
// M = 2^log_m. Usually adjacent columns c are adjacent in memory on both
// sides (in_c = out_c = 1, what every plan uses), so a CTA of FPB columns
// reads and writes FPB*8-byte row segments; lanes run over the columns first.
// (Contiguous rows stored transposed, in_c = N, in_e = 1, measured slower than
// fft_rows_t_kernel for the two-pass 1D rows: 32-byte input segments.) Used for 2D column passes (one or two sub-passes), the
// column passes of the multi-pass 1D transform and the distributed column
// pass.
struct PassArgs {
  int64_t nfft;
  int log_w;
  int log_j;
  int64_t in_o, in_j, in_e;
  int64_t out_o, out_j, out_e;
  int64_t in_c, out_c;  // column strides (1 for adjacent columns)
  uint32_t tcj, tc, tj;
  int log_m;
  const float2* tw_lo;
  const float2* tw_hi;
  float scale;
  int tw_sfu;  // with a twiddle: its factors from the SFU (kernel TW = 2), not the table
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

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT, int TW>
struct PassCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (FPB < 16 ? FPB : 16)>::value;
  static constexpr size_t SMEM_BYTES = G::STAGES > 1 ? (size_t)FPB * RS * sizeof(float2) : 0;
};

// One strided length-2^LOGN transform per thread group: thread t loads
// src[(t + T*m) * in_e], runs the stages, multiplies output k = t + T*m by
// W_M^(tw_e0 + tw_d*m) when TW (factors from the SFU when TW_SFU, else from
// the two-level table), and stores dst[(t + T*m) * out_e]. With
// LD_STREAM / ST_STREAM the data is read or written once and takes the
// streaming (evict-first) hints; otherwise it is scratch kept in L2 between a
// store and one later load: stores carry an L2 evict-last policy and loads an
// evict-first one (the line is dead after it), which cut the scratch lines
// written back to HBM.
template <int LOGN, int LOGP, bool CONJ_IN, bool CONJ_OUT, bool TW, bool LD_STREAM, bool ST_STREAM,
          bool TW_SFU, class Sync>
__device__ __forceinline__ void strided_unit(const float2* src, int64_t in_e, float2* dst,
                                             int64_t out_e, bool valid, int t, float2* sm,
                                             const float2* __restrict__ tw, uint32_t tw_e0,
                                             uint32_t tw_d, const float2* tw_lo,
                                             const float2* tw_hi, uint32_t tw_mask, float scale,
                                             Sync sync) {
  using G = Geom<LOGN, LOGP>;
  float2 v[G::P];
  if (valid) {
    src += (int64_t)t * in_e;
    const int64_t step = (int64_t)G::T * in_e;
    uint64_t pol_first = 0;
    if constexpr (!LD_STREAM) asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_first));
#pragma unroll
    for (int m = 0; m < G::P; ++m) {
      float2 x;
      if constexpr (LD_STREAM) {
        x = ld_stream(src + step * m);
      } else {
        asm volatile("ld.global.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
                     : "=f"(x.x), "=f"(x.y) : "l"(src + step * m), "l"(pol_first));
      }
      v[m] = swap_if(x, CONJ_IN);
    }
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  run_stages<LOGN, LOGP, 0>(v, sm, t, tw, sync);
  if (valid) {
    if constexpr (TW) apply_progression_twiddles<G::P>(v, tw_lo, tw_hi, tw_e0, tw_d, tw_mask, TW_SFU);
    dst += (int64_t)t * out_e;
    const int64_t step = (int64_t)G::T * out_e;
#pragma unroll
    for (int m = 0; m < G::P; ++m) {
      const float2 r = epilogue<CONJ_OUT>(v[m], scale);
      if constexpr (ST_STREAM) {
        st_stream(dst + step * m, r);
      } else {
        uint64_t pol_last;
        asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_last));
        asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(dst + step * m),
                     "f"(r.x), "f"(r.y), "l"(pol_last) : "memory");
      }
    }
  }
}

// TW: 0 no twiddle, 1 twiddle factors from the table, 2 from the SFU.
template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT, int TW>
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
  // Output k = t + T*m takes W_M^(tb + ts*k): a progression in m.
  const uint32_t tb = TW ? pass_tw_base((uint32_t)c, (uint32_t)j, a.tcj) : 0u;
  const uint32_t ts = TW ? pass_tw_step((uint32_t)c, (uint32_t)j, a.tc, a.tj) : 0u;
  const uint32_t mask = TW ? (1u << a.log_m) - 1u : 0u;
  float2* sm = smem + (C::SMEM_BYTES ? cl * C::RS : 0);
  const float2* src = in + o * a.in_o + j * a.in_j + c * a.in_c;
  float2* dst = out + o * a.out_o + j * a.out_j + c * a.out_c;
  if constexpr (FPB == 1 && G::T <= 32)
    strided_unit<LOGN, LOGP, CONJ_IN, CONJ_OUT, TW != 0, true, true, TW == 2>(
        src, a.in_e, dst, a.out_e, valid, t, sm, tw, tb + ts * (uint32_t)t, ts * (uint32_t)G::T,
        a.tw_lo, a.tw_hi, mask, a.scale, SyncWarp{});
  else
    strided_unit<LOGN, LOGP, CONJ_IN, CONJ_OUT, TW != 0, true, true, TW == 2>(
        src, a.in_e, dst, a.out_e, valid, t, sm, tw, tb + ts * (uint32_t)t, ts * (uint32_t)G::T,
        a.tw_lo, a.tw_hi, mask, a.scale, SyncBlock{});
}

// ----------------------------------------------------------------------------
// Column FFTs of length N = 2^(L1 + L2) as both sub-passes in one persistent
// kernel (N = A*B, A = 2^L2, B = 2^L1, column element n = a + A*b):
//   sub-pass 1, unit a < A: DFT over b of rows a + A*b, times W_N^(a*kb),
//               stored to rows a + A*kb of the CTA's scratch slot;
//   sub-pass 2, unit kb < B: DFT over a of slot rows A*kb + a, stored to
//               output row kb + B*ka.
// A CTA takes tiles of W adjacent columns of one image (all N rows) in turn;
// its slot (N x W values, row pitch W) is rewritten for every tile, so the
// slots of all CTAs (a few tens of MiB) stay in L2 and HBM sees one read and
// one write per element instead of two of each for two separate passes.
// The input is read with evict-first hints, the slot with normal ones. A unit
// (W columns x T threads) is one warp or a few whole warps, and runs its
// rounds on its own with a warp barrier or a named barrier of its warps, so
// the units of a CTA overlap each other's memory latency; only the two
// sub-pass boundaries of a tile are block-wide barriers.
struct ColsL2Args {
  int64_t tiles;           // images * (width / W)
  int log_tiles_per_img;   // log2(width / W)
  int64_t img_stride;      // input and output image stride (elements)
  int64_t ld;              // input and output row pitch (elements)
  const float2* tw_lo;     // two-level W_N tables
  const float2* tw_hi;
  float scale;
};

template <int L1, int L2, int W, int THREADS>
struct ColsL2Cfg {
  static constexpr int LP1 = plan_log_p(L1), LP2 = plan_log_p(L2);
  using G1 = Geom<L1, LP1>;
  using G2 = Geom<L2, LP2>;
  static constexpr int U1 = THREADS / (W * G1::T);  // sub-pass-1 units per round
  static constexpr int U2 = THREADS / (W * G2::T);
  static constexpr int A = 1 << L2, B = 1 << L1;
  static_assert(U1 >= 1 && U2 >= 1 && THREADS % (W * G1::T) == 0 && THREADS % (W * G2::T) == 0,
                "a round must be whole units");
  static_assert(A % U1 == 0 && B % U2 == 0, "whole rounds per sub-pass");
  static constexpr int RS1 = RegionStride<L1, LP1, (W < 16 ? W : 16)>::value;
  static constexpr int RS2 = RegionStride<L2, LP2, (W < 16 ? W : 16)>::value;
  static constexpr size_t SM1 = G1::STAGES > 1 ? (size_t)U1 * W * RS1 : 0;
  static constexpr size_t SM2 = G2::STAGES > 1 ? (size_t)U2 * W * RS2 : 0;
  static constexpr size_t SMEM_BYTES = (SM1 > SM2 ? SM1 : SM2) * sizeof(float2);
  static constexpr int64_t SLOT = (int64_t)W << (L1 + L2);  // complex values per CTA
};

template <int L1, int L2, int W, int THREADS, int MINB, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(THREADS, MINB)
fft_cols_l2_kernel(const float2* in, float2* out, float2* ws, const float2* __restrict__ tw1,
                   const float2* __restrict__ tw2, ColsL2Args a) {
  using C = ColsL2Cfg<L1, L2, W, THREADS>;
  extern __shared__ float2 smem[];
  constexpr int A = C::A, B = C::B;
  constexpr uint32_t kMask = (1u << (L1 + L2)) - 1u;
  constexpr int kUnit1 = W * C::G1::T, kUnit2 = W * C::G2::T;
  static_assert(kUnit1 <= 32 || (kUnit1 % 32 == 0 && C::U1 <= 15), "unit barriers");
  static_assert(kUnit2 <= 32 || (kUnit2 % 32 == 0 && C::U2 <= 15), "unit barriers");
  float2* slot = ws + (int64_t)blockIdx.x * C::SLOT;
  const int cl = threadIdx.x % W;
  const int64_t tile_mask = ((int64_t)1 << a.log_tiles_per_img) - 1;
  for (int64_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    const int64_t base = (tile >> a.log_tiles_per_img) * a.img_stride + (tile & tile_mask) * W + cl;
    {
      const int t1 = (threadIdx.x / W) % C::G1::T, u1 = threadIdx.x / (W * C::G1::T);
      float2* sm1 = smem + (u1 * W + cl) * C::RS1;
      using Sync1 = typename std::conditional<(kUnit1 <= 32), SyncWarp, SyncNamed>::type;
      Sync1 sync1;
      if constexpr (kUnit1 > 32) sync1 = SyncNamed{1 + u1, kUnit1};
#pragma unroll 1
      for (int r = 0; r < A / C::U1; ++r) {
        const int j = r * C::U1 + u1;  // a
        // The stage twiddles depend on the thread only; an opaque table
        // pointer keeps them from being hoisted out of the loop and held in
        // registers across rounds (which spilled at 64 registers).
        const float2* twr = tw1;
        asm volatile("" : "+l"(twr));
        strided_unit<L1, C::LP1, CONJ_IN, false, true, true, false, false>(
            in + base + j * a.ld, (int64_t)A * a.ld, slot + j * W + cl, (int64_t)A * W, true, t1,
            sm1, twr, (uint32_t)j * (uint32_t)t1, (uint32_t)j * (uint32_t)C::G1::T, a.tw_lo,
            a.tw_hi, kMask, 1.0f, sync1);
        sync1();  // the next round's first exchange reuses the unit's shared region
      }
    }
    __syncthreads();  // the tile's slot is complete
    {
      const int t2 = (threadIdx.x / W) % C::G2::T, u2 = threadIdx.x / (W * C::G2::T);
      float2* sm2 = smem + (u2 * W + cl) * C::RS2;
      using Sync2 = typename std::conditional<(kUnit2 <= 32), SyncWarp, SyncNamed>::type;
      Sync2 sync2;
      if constexpr (kUnit2 > 32) sync2 = SyncNamed{1 + u2, kUnit2};
#pragma unroll 1
      for (int r = 0; r < B / C::U2; ++r) {
        const int j = r * C::U2 + u2;  // kb
        const float2* twr = tw2;
        asm volatile("" : "+l"(twr));
        strided_unit<L2, C::LP2, false, CONJ_OUT, false, false, true, false>(
            slot + (int64_t)A * j * W + cl, (int64_t)W, out + base + j * a.ld, (int64_t)B * a.ld,
            true, t2, sm2, twr, 0u, 0u, nullptr, nullptr, 0u, a.scale, sync2);
        sync2();
      }
    }
    __syncthreads();  // every read of the slot is done before the next tile rewrites it
  }
}

// ----------------------------------------------------------------------------
// Rows stored transposed (the input optionally conjugated on load, CONJ_IN).
// Transform f = (o, j, c), c fastest: its N elements
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

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
struct RowsTCfg {
  using G = Geom<LOGN, LOGP>;
  static constexpr int THREADS = FPB * G::T;
  static constexpr int RS = RegionStride<LOGN, LOGP, (FPB < 16 ? FPB : 16)>::value;
  static constexpr size_t SMEM_BYTES = (size_t)FPB * RS * sizeof(float2);
};

template <int LOGN, int LOGP, int FPB, bool CONJ_IN, bool CONJ_OUT>
__global__ void __launch_bounds__(RowsTCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS,
                                  MinBlocks<RowsTCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>::THREADS, LOGP>::value)
fft_rows_t_kernel(const float2* in, float2* out, const float2* __restrict__ tw, RowsTArgs a) {
  using G = Geom<LOGN, LOGP>;
  using C = RowsTCfg<LOGN, LOGP, FPB, CONJ_IN, CONJ_OUT>;
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
    for (int m = 0; m < G::P; ++m) v[m] = swap_if(ld_stream(src + G::T * m), CONJ_IN);
  } else {
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = make_float2(0.f, 0.f);
  }
  float2* sm = smem + g * C::RS;
  // The store runs with lanes over rows: thread (g2, e0) ends with outputs
  // e0 + T*q of row g2, so FPB adjacent rows give FPB-value output segments.
  const int g2 = threadIdx.x % FPB;
  const int e0 = threadIdx.x / FPB;
  float2* row = smem + g2 * C::RS;
  if constexpr (G::STAGES >= 2) {
    // The last stage reads its inputs in the lanes-over-rows arrangement
    // (one block barrier, as every row's region is read by other warps).
    // The exchanges before it stay within the row's own warps (a named
    // barrier per row when a row spans several warps).
    if constexpr (G::T <= 32)
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{}, row, e0, SyncBlock{});
    else if constexpr (FPB > 1 && FPB <= 15)
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncNamed{1 + g, G::T}, row, e0, SyncBlock{});
    else
      run_stages_regroup<LOGN, LOGP, 0>(v, sm, t, tw, SyncBlock{}, row, e0, SyncBlock{});
  } else {
    // One stage, no exchange: transpose through shared memory.
    run_stages<LOGN, LOGP, 0>(v, sm, t, tw, SyncWarp{});
#pragma unroll
    for (int m = 0; m < G::P; ++m) sm[stage_read_addr<LOGN, LOGP>(t, m)] = v[m];
    __syncthreads();
#pragma unroll
    for (int q = 0; q < G::P; ++q) v[q] = row[stage_read_addr<LOGN, LOGP>(e0, q)];
  }
  const int64_t f2 = (int64_t)blockIdx.x * FPB + g2;
  if (f2 < a.nfft) {
    int64_t o, j, c;
    pass_index(f2, a.log_w, a.log_j, o, j, c);
    float2* dst = out + o * a.out_o + j * a.out_j + c;
#pragma unroll
    for (int q = 0; q < G::P; ++q)
      st_stream(dst + a.out_e * (e0 + G::T * q), epilogue<CONJ_OUT>(v[q], a.scale));
  }
}

}  // namespace ferrum
