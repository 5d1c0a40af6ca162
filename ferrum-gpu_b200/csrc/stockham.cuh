// Stockham stage machinery for one thread group.
//
// A group of T = N/P threads transforms one length-N sequence. Thread t owns
// the P values at positions t + T*m (m in [0, P)); before stage 0 these are
// the inputs x[t + T*m], after the last stage they are the outputs
// X[t + T*m]. Stage s (radix R, NS = product of the earlier radices) runs
// B = P/R butterflies per thread; butterfly i of thread t is j = t + T*i and
//   reads      positions j + r*N/R            (= register slot i + r*B)
//   multiplies input r by W_{NS*R}^{r*(j mod NS)}     (s >= 1)
//   writes     position (j div NS)*NS*R + (j mod NS) + r*NS
// which is the radix-R form of the reference's radix-2 Stockham butterfly
// (crates/ferrum-gpu-fft/src/cpu.rs:30-45). Between stages the group swaps
// values through shared memory; in the last stage the write position is
// j + r*N/R, i.e. the same register slot, so no exchange is needed.
//
// The helpers are __host__ __device__ so that the CPU emulator in the test
// suite runs exactly this index arithmetic and butterfly code.
#pragma once

#include "dft.cuh"
#include "plan.h"

namespace ferrum {

// Shared-memory padding: one empty slot after every 16 complex values. Stage
// 0 writes with a stride of 16 values, which would otherwise put a half-warp
// on a single pair of banks.
FERRUM_HD __forceinline__ int smem_pad(int i) { return i + (i >> 4); }

template <int LOGN>
struct PaddedLen {
  static constexpr int value = (1 << LOGN) + ((1 << LOGN) >> 4);
};

FERRUM_HD __forceinline__ float2 tw_load(const float2* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}

template <int LOGN, int LOGP>
struct Geom {
  static constexpr int N = 1 << LOGN;
  static constexpr int P = 1 << LOGP;
  static constexpr int T = N / P;
  static constexpr int STAGES = plan_num_stages(LOGN, LOGP);
};

// Twiddle multiply (stage s >= 1) and the radix-R butterflies of stage S,
// in registers.
template <int LOGN, int LOGP, int S>
FERRUM_HD __forceinline__ void stage_compute(float2 (&v)[1 << LOGP], int t, const float2* tw) {
  using G = Geom<LOGN, LOGP>;
  constexpr int LR = plan_log_radix(LOGN, LOGP, S);
  constexpr int R = 1 << LR;
  constexpr int B = G::P / R;
  constexpr int LNS = plan_log_ns(LOGP, S);
  constexpr int NS = 1 << LNS;
  if constexpr (S > 0) {
    const float2* tws = tw + plan_stage_tw_offset(LOGN, LOGP, S);
#pragma unroll
    for (int i = 0; i < B; ++i) {
      const int k = (t + G::T * i) & (NS - 1);
#pragma unroll
      for (int r = 1; r < R; ++r) v[i + r * B] = c_mul(v[i + r * B], tw_load(tws + (r - 1) * NS + k));
    }
  }
#pragma unroll
  for (int i = 0; i < B; ++i) {
    float2 u[R];
#pragma unroll
    for (int r = 0; r < R; ++r) u[r] = v[i + r * B];
    dft<R>(u);
#pragma unroll
    for (int r = 0; r < R; ++r) v[i + r * B] = u[r];
  }
}

// Destination position of output r of butterfly i (thread t) in stage S.
template <int LOGN, int LOGP, int S>
FERRUM_HD __forceinline__ int stage_out_pos(int t, int i, int r) {
  using G = Geom<LOGN, LOGP>;
  constexpr int LR = plan_log_radix(LOGN, LOGP, S);
  constexpr int LNS = plan_log_ns(LOGP, S);
  constexpr int NS = 1 << LNS;
  const int j = t + G::T * i;
  return ((j >> LNS) << (LNS + LR)) + (j & (NS - 1)) + r * NS;
}

// Register slot holding output r of butterfly i in stage S.
template <int LOGN, int LOGP, int S>
FERRUM_HD constexpr int stage_slot(int i, int r) {
  return i + r * ((1 << LOGP) >> plan_log_radix(LOGN, LOGP, S));
}

// Four-step twiddle W_N^e from the two-level tables (e < N <= 2^26).
FERRUM_HD __forceinline__ float2 four_step_twiddle(const float2* lo, const float2* hi, uint32_t e) {
  return c_mul(tw_load(hi + (e >> kFourStepLoBits)),
               tw_load(lo + (e & ((1u << kFourStepLoBits) - 1))));
}

// Blocked layout of the distributed row pass: element e of row f (of nrows)
// lives at (e >> lb) * nrows * 2^lb + f * 2^lb + (e mod 2^lb).
FERRUM_HD __forceinline__ int64_t blocked_index(int64_t f, int64_t e, int lb, int64_t nrows) {
  return (e >> lb) * (nrows << lb) + (f << lb) + (e & (((int64_t)1 << lb) - 1));
}

#if defined(__CUDACC__)
// Runs stages S.. to the end. On entry v holds stage S's inputs; on return
// v[m] = X[t + T*m]. `sm` is this group's padded shared-memory region and
// `sync` orders the group's shared-memory traffic.
template <int LOGN, int LOGP, int S, class Sync>
__device__ __forceinline__ void run_stages(float2 (&v)[1 << LOGP], float2* sm, int t,
                                           const float2* tw, Sync sync) {
  using G = Geom<LOGN, LOGP>;
  stage_compute<LOGN, LOGP, S>(v, t, tw);
  if constexpr (S + 1 < G::STAGES) {
    constexpr int LR = plan_log_radix(LOGN, LOGP, S);
    constexpr int R = 1 << LR;
    constexpr int B = G::P / R;
    if constexpr (S > 0) sync();  // every read of the previous exchange is done
#pragma unroll
    for (int i = 0; i < B; ++i)
#pragma unroll
      for (int r = 0; r < R; ++r)
        sm[smem_pad(stage_out_pos<LOGN, LOGP, S>(t, i, r))] = v[stage_slot<LOGN, LOGP, S>(i, r)];
    sync();
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = sm[smem_pad(t + G::T * m)];
    run_stages<LOGN, LOGP, S + 1>(v, sm, t, tw, sync);
  }
}
#endif

}  // namespace ferrum
