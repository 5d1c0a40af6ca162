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

// Shared-memory padding: one empty slot after every 16 complex values, and
// with 32 values per thread one more after every 32. Stage 0 writes with a
// stride of P values; unpadded, a half-warp of 8-byte stores would land on
// one pair of banks. The padded strides, 17 (P = 16) and 35 (P = 32) slots,
// are odd, so the 16 lanes of a half-warp cover all 32 banks once.
template <int LOGP>
FERRUM_HD __forceinline__ constexpr int smem_pad(int i) {
  return i + (i >> 4) + (LOGP >= 5 ? (i >> 5) : 0);
}

template <int LOGN, int LOGP>
struct PaddedLen {
  static constexpr int value = smem_pad<LOGP>(1 << LOGN);
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
  if constexpr (S > 0 && (R == 16 || R == 32) && B == 1) {
    // Radix-16/32 input twiddles w^r, w = W_{R NS}^k, from the table entries
    // w, w^2, w^4, w^8 (and w^16) and products instead of R-1 loads. The
    // L1/shared pipe is the kernel's tightest unit on B200, the FMA pipe has
    // room (measured +4 % sustained throughput at N = 4096); each power is a
    // product of at most five correctly rounded table entries. For radix 32,
    // w^(16+r) = w^16 * w^r is formed as it is applied, to bound registers.
    const float2* tws = tw + plan_stage_tw_offset(LOGN, LOGP, S);
    const int k = t & (NS - 1);
    float2 w[16];
    w[1] = tw_load(tws + 0 * NS + k);
    w[2] = tw_load(tws + 1 * NS + k);
    w[4] = tw_load(tws + 3 * NS + k);
    w[8] = tw_load(tws + 7 * NS + k);
    w[3] = c_mul(w[1], w[2]);
    w[5] = c_mul(w[1], w[4]);
    w[6] = c_mul(w[2], w[4]);
    w[7] = c_mul(w[3], w[4]);
#pragma unroll
    for (int r = 9; r < 16; ++r) w[r] = c_mul(w[r - 8], w[8]);
#pragma unroll
    for (int r = 1; r < 16; ++r) v[r] = c_mul(v[r], w[r]);
    if constexpr (R == 32) {
      const float2 w16 = tw_load(tws + 15 * NS + k);
      v[16] = c_mul(v[16], w16);
#pragma unroll
      for (int r = 17; r < 32; ++r) v[r] = c_mul(v[r], c_mul(w16, w[r - 16]));
    }
  } else if constexpr (S > 0 && (G::P == 32 && R < 16)) {
    // 32 values per thread and a last radix of 8 or less: most of the
    // rotations below would be general angles (measured slower at N = 8192),
    // so every butterfly loads its own twiddles.
    const float2* tws = tw + plan_stage_tw_offset(LOGN, LOGP, S);
#pragma unroll
    for (int i = 0; i < B; ++i) {
      const int k = (t + G::T * i) & (NS - 1);
#pragma unroll
      for (int r = 1; r < R; ++r) v[i + r * B] = c_mul(v[i + r * B], tw_load(tws + (r - 1) * NS + k));
    }
  } else if constexpr (S > 0) {
    // Last stage with a smaller radix (R < P, B = P/R butterflies per thread;
    // NS*R = N and T <= NS): butterfly i has k = t + T*i, so
    //   W_N^(r k) = W_N^(r t) * W_N^(r T i) = W_N^(r t) * W_P^(r i),
    // R - 1 table loads for all B butterflies and constant rotations (quarter
    // turns by swaps) instead of (R - 1) * B lane-scattered loads, which made
    // the strided passes L1-bound (N = 1024: 0.65 -> 0.63 ms, N = 16384:
    // 0.85 -> 0.79 ms per 2 GiB).
    static_assert(G::T <= NS, "last stage: T <= NS");
    const float2* tws = tw + plan_stage_tw_offset(LOGN, LOGP, S);
    const int k = t & (NS - 1);
    if constexpr (R == 16) {
      float2 w[16];
      w[1] = tw_load(tws + 0 * NS + k);
      w[2] = tw_load(tws + 1 * NS + k);
      w[4] = tw_load(tws + 3 * NS + k);
      w[8] = tw_load(tws + 7 * NS + k);
      w[3] = c_mul(w[1], w[2]);
      w[5] = c_mul(w[1], w[4]);
      w[6] = c_mul(w[2], w[4]);
      w[7] = c_mul(w[3], w[4]);
#pragma unroll
      for (int r = 9; r < 16; ++r) w[r] = c_mul(w[r - 8], w[8]);
#pragma unroll
      for (int i = 0; i < B; ++i)
#pragma unroll
        for (int r = 1; r < R; ++r)
          v[i + r * B] = c_mul(c_mul_w32(v[i + r * B], (r * i) * (32 / G::P)), w[r]);
    } else {
      // One twiddle live at a time: it serves input r of all B butterflies.
#pragma unroll
      for (int r = 1; r < R; ++r) {
        const float2 w = tw_load(tws + (r - 1) * NS + k);
#pragma unroll
        for (int i = 0; i < B; ++i)
          v[i + r * B] = c_mul(c_mul_w32(v[i + r * B], (r * i) * (32 / G::P)), w);
      }
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

// Padded shared-memory address of output r of butterfly i (thread t) in
// stage S, as base + offset(r): one address per butterfly and compile-time
// offsets for the R stores. Stage 0 (NS = 1) writes positions j*R + r with
// R | 16 or R = 32, so pad(j*R + r) = pad(j*R) + pad(r); later stages have NS
// a multiple of the padding period (16, or 32 when P = 32), so
// pad(pos0 + r*NS) = pad(pos0) + r*pad(NS).
template <int LOGN, int LOGP, int S>
FERRUM_HD __forceinline__ int stage_write_base(int t, int i) {
  return smem_pad<LOGP>(stage_out_pos<LOGN, LOGP, S>(t, i, 0));
}
template <int LOGN, int LOGP, int S>
FERRUM_HD constexpr int stage_write_offset(int r) {
  return plan_log_ns(LOGP, S) == 0 ? smem_pad<LOGP>(r)
                                   : r * smem_pad<LOGP>(1 << plan_log_ns(LOGP, S));
}
template <int LOGN, int LOGP, int S>
FERRUM_HD __forceinline__ int stage_write_addr(int t, int i, int r) {
  static_assert(plan_log_ns(LOGP, S) == 0 || plan_log_ns(LOGP, S) >= (LOGP >= 5 ? 5 : 4),
                "NS must be a multiple of the padding period");
  return stage_write_base<LOGN, LOGP, S>(t, i) + stage_write_offset<LOGN, LOGP, S>(r);
}

// Padded shared-memory address of the value thread t reads into slot m
// (position t + T*m): pad(t) + m*pad(T) when T is a multiple of the padding
// period.
template <int LOGN, int LOGP>
FERRUM_HD __forceinline__ int stage_read_addr(int t, int m) {
  constexpr int T = Geom<LOGN, LOGP>::T;
  if constexpr (T % (LOGP >= 5 ? 32 : 16) == 0)
    return smem_pad<LOGP>(t) + m * smem_pad<LOGP>(T);
  else
    return smem_pad<LOGP>(t + T * m);
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

// v[m] *= W_M^(e0 + d*m) for m < P, with W_M^e0 and W_M^(d*2^b) from
// `factor` (1 + log2 P evaluations instead of P): W_M^(e0 + d*m) is their
// product over the set bits b of m, at most 1 + log2 P factors.
template <int P, class Factor>
FERRUM_HD __forceinline__ void progression_twiddles_by(float2 (&v)[P], uint32_t e0, uint32_t d,
                                                       Factor factor) {
  constexpr int H = P / 2;
  float2 w[H > 0 ? H : 1];
  w[0] = factor(e0);
  if constexpr (P == 1) {
    v[0] = c_mul(v[0], w[0]);
  } else {
#pragma unroll
    for (int b = 1; b < H; b <<= 1) {
      const float2 p = factor(d * (uint32_t)b);
#pragma unroll
      for (int m = 0; m < b; ++m) w[m + b] = c_mul(w[m], p);
    }
    const float2 top = factor(d * (uint32_t)H);
#pragma unroll
    for (int m = 0; m < H; ++m) {
      v[m + H] = c_mul(v[m + H], c_mul(w[m], top));
      v[m] = c_mul(v[m], w[m]);
    }
  }
}

#if defined(__CUDACC__)
// W_M^e, M = 2^(32 - sh), from the special-function unit: e << sh is the
// exponent as a signed 32-bit fixed-point fraction of a turn, so the angle
// -2*pi*e/M is taken in [-pi, pi), where __sinf / __cosf are within 2^-21.4
// absolute; with the rounding of the integer-to-float conversion and of the
// scaling each component is within ~7e-7 of exp(-2*pi*i*e/M) (a correctly
// rounded table entry: ~6e-8).
__device__ __forceinline__ float2 sfu_twiddle(uint32_t e, int sh) {
  float s, c;
  __sincosf((float)(int32_t)(e << sh) * -1.46291808e-9f, &s, &c);  // -2*pi / 2^32
  return make_float2(c, s);
}
#endif

// v[m] *= W_M^(e0 + d*m) for m < P (M = mask + 1, a power of two, M >= 2):
// the twiddles of one thread's outputs k = t + T*m in a strided pass, whose
// exponents form an arithmetic progression. The factors come from the
// two-level table (two lookups each), or, with `sfu` on the device, from the
// special-function unit. The passes of the multi-pass 1D transform take the
// SFU path: the lookups of their four-step twiddles filled the L1 data pipe
// (lanes of different columns gather from different cache lines), and the
// SFU factors measured faster for every length (1D 2^18 x 1024: 1.83 ->
// 1.66 ms, 2^24 x 4: 0.597 -> 0.581 ms per transform). The 2D column
// sub-passes keep the table, where they measured faster (their twiddle
// W_N^(a*kb) is the same for all columns, so the lanes of a warp share the
// entries). The host (CPU emulator) always uses the table.
template <int P>
FERRUM_HD __forceinline__ void apply_progression_twiddles(float2 (&v)[P], const float2* lo,
                                                          const float2* hi, uint32_t e0,
                                                          uint32_t d, uint32_t mask,
                                                          bool sfu = false) {
#if defined(__CUDA_ARCH__)
  if (sfu) {
    const int sh = __clz(mask);
    progression_twiddles_by(v, e0, d, [sh](uint32_t e) { return sfu_twiddle(e, sh); });
    return;
  }
#else
  (void)sfu;
#endif
  progression_twiddles_by(v, e0, d,
                          [lo, hi, mask](uint32_t e) { return four_step_twiddle(lo, hi, e & mask); });
}

// Blocked layout of the distributed row pass: element e of row f (of nrows)
// lives at (e >> lb) * nrows * 2^lb + f * 2^lb + (e mod 2^lb).
FERRUM_HD __forceinline__ int64_t blocked_index(int64_t f, int64_t e, int lb, int64_t nrows) {
  return (e >> lb) * (nrows << lb) + (f << lb) + (e & (((int64_t)1 << lb) - 1));
}

#if defined(__CUDACC__)
struct NoHook {
  __device__ __forceinline__ void operator()() const {}
};

// Runs stages S.. to the end. On entry v holds stage S's inputs; on return
// v[m] = X[t + T*m]. `sm` is this group's padded shared-memory region and
// `sync` orders the group's shared-memory traffic. `after_last_read` runs (in
// every thread) once the last exchange has been read, when the shared region
// is no longer needed.
template <int LOGN, int LOGP, int S, class Sync, class Hook = NoHook>
__device__ __forceinline__ void run_stages(float2 (&v)[1 << LOGP], float2* sm, int t,
                                           const float2* tw, Sync sync,
                                           Hook after_last_read = Hook{}) {
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
        sm[stage_write_addr<LOGN, LOGP, S>(t, i, r)] = v[stage_slot<LOGN, LOGP, S>(i, r)];
    sync();
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = sm[stage_read_addr<LOGN, LOGP>(t, m)];
    if constexpr (S + 2 == G::STAGES) after_last_read();
    run_stages<LOGN, LOGP, S + 1>(v, sm, t, tw, sync, after_last_read);
  }
}

// As run_stages, but the last stage runs in another thread arrangement: its
// inputs are read by thread t_last from region sm_last (which may belong to
// another group of the CTA), after `last_sync`, which must order the writes
// of every group whose region that can be. On return v[m] = X[t_last + T*m] of
// sm_last's transform. A stage's butterflies depend on the thread only through
// the position t it reads, so the values are those run_stages gives thread
// t_last of that group; the regrouping replaces a separate transpose exchange.
template <int LOGN, int LOGP, int S, class Sync, class LastSync>
__device__ __forceinline__ void run_stages_regroup(float2 (&v)[1 << LOGP], float2* sm, int t,
                                                   const float2* tw, Sync sync, float2* sm_last,
                                                   int t_last, LastSync last_sync) {
  using G = Geom<LOGN, LOGP>;
  static_assert(G::STAGES >= 2, "regrouping needs an exchange");
  stage_compute<LOGN, LOGP, S>(v, t, tw);
  constexpr int LR = plan_log_radix(LOGN, LOGP, S);
  constexpr int R = 1 << LR;
  constexpr int B = G::P / R;
  if constexpr (S > 0) sync();  // every read of the previous exchange is done
#pragma unroll
  for (int i = 0; i < B; ++i)
#pragma unroll
    for (int r = 0; r < R; ++r)
      sm[stage_write_addr<LOGN, LOGP, S>(t, i, r)] = v[stage_slot<LOGN, LOGP, S>(i, r)];
  if constexpr (S + 2 == G::STAGES) {
    last_sync();
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = sm_last[stage_read_addr<LOGN, LOGP>(t_last, m)];
    stage_compute<LOGN, LOGP, S + 1>(v, t_last, tw);
  } else {
    sync();
#pragma unroll
    for (int m = 0; m < G::P; ++m) v[m] = sm[stage_read_addr<LOGN, LOGP>(t, m)];
    run_stages_regroup<LOGN, LOGP, S + 1>(v, sm, t, tw, sync, sm_last, t_last, last_sync);
  }
}
#endif

}  // namespace ferrum
