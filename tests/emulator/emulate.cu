// CPU emulator of the sm_100a FFT kernels — test infrastructure only.
//
// Runs, on the host, the exact per-thread code the kernels run: the radix
// plans (plan.h), the twiddle tables the runtime uploads (twiddle_tables.h),
// stage_compute / stage_out_pos / stage_slot / smem_pad (stockham.cuh), the
// four-step twiddle lookup and the distributed blocked layout. Each thread
// group is simulated thread by thread between barriers, and every shared
// memory exchange is checked to be a permutation (each padded slot written
// exactly once and read exactly once). The tests compare its output with the
// CPU oracle, so index-arithmetic bugs show up without a GPU.
#include <stdint.h>
#include <string.h>

#include <vector>

#include "../../ferrum-gpu_b200/csrc/stockham.cuh"
#include "../../ferrum-gpu_b200/csrc/twiddle_tables.h"

using namespace ferrum;

namespace {

template <int LOGN>
struct Group {
  static constexpr int LOGP = plan_log_p(LOGN);
  using G = Geom<LOGN, LOGP>;
  struct Regs {
    float2 v[G::P];
  };

  template <int S>
  static int stages(std::vector<Regs>& regs, const float2* tw) {
    for (int t = 0; t < G::T; ++t) stage_compute<LOGN, LOGP, S>(regs[t].v, t, tw);
    if constexpr (S + 1 < G::STAGES) {
      constexpr int LR = plan_log_radix(LOGN, LOGP, S);
      constexpr int R = 1 << LR;
      constexpr int B = G::P / R;
      const int slots = PaddedLen<LOGN>::value + 16;
      std::vector<float2> sm(slots);
      std::vector<int> writes(slots, 0), reads(slots, 0);
      for (int t = 0; t < G::T; ++t)
        for (int i = 0; i < B; ++i)
          for (int r = 0; r < R; ++r) {
            const int idx = smem_pad(stage_out_pos<LOGN, LOGP, S>(t, i, r));
            if (idx < 0 || idx >= slots) return -10 - S;
            sm[idx] = regs[t].v[stage_slot<LOGN, LOGP, S>(i, r)];
            writes[idx]++;
          }
      for (int t = 0; t < G::T; ++t)
        for (int m = 0; m < G::P; ++m) {
          const int idx = smem_pad(t + G::T * m);
          if (idx < 0 || idx >= slots || writes[idx] != 1) return -20 - S;
          reads[idx]++;
          regs[t].v[m] = sm[idx];
        }
      for (int k = 0; k < slots; ++k)
        if (reads[k] != writes[k]) return -30 - S;
      return stages<S + 1>(regs, tw);
    }
    return 0;
  }

  // y[e] = DFT(x)[e] with the kernel's thread layout (y may alias x).
  static int run(const float2* x, float2* y, const float2* tw) {
    std::vector<Regs> regs(G::T);
    for (int t = 0; t < G::T; ++t)
      for (int m = 0; m < G::P; ++m) regs[t].v[m] = x[t + G::T * m];
    const int rc = stages<0>(regs, tw);
    for (int t = 0; t < G::T; ++t)
      for (int m = 0; m < G::P; ++m) y[t + G::T * m] = regs[t].v[m];
    return rc;
  }
};

int run_group(int log_n, const float2* x, float2* y, const float2* tw) {
  switch (log_n) {
#define X(L) \
  case L:    \
    return Group<L>::run(x, y, tw);
    X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)
#undef X
    default:
      return -1;
  }
}

struct Tables {
  std::vector<float2> stage[kMaxSinglePassLogN + 1];
  std::vector<float2> lo, hi;
  Tables(int log_n) {
    for (int l = 2; l <= kMaxSinglePassLogN; ++l) {
      append_stage_tables(stage[l], l);
      stage[l].push_back(make_float2(1.f, 0.f));
    }
    if (log_n > kMaxSinglePassLogN) append_four_step_tables(lo, hi, log_n);
  }
};

float2 conj_if(float2 v, bool c) { return c ? make_float2(v.x, -v.y) : v; }
float2 epi(float2 v, bool conj_out, float scale) {
  return conj_out ? make_float2(v.x * scale, -v.y * scale) : v;
}

}  // namespace

extern "C" {

// In-place batched 1D transform, laid out like ferrum_fft_1d_c2c_pow2.
int emu_fft_1d(float* data, int log_n, int64_t batch, int direction, int normalize) {
  if (log_n < 2 || log_n > kMaxLogN || batch <= 0) return -1;
  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const float scale = (inv && normalize) ? 1.0f / (float)n : 1.0f;
  float2* d = (float2*)data;
  Tables tab(log_n);
  if (log_n <= kMaxSinglePassLogN) {
    std::vector<float2> x(n);
    for (int64_t b = 0; b < batch; ++b) {
      for (int64_t e = 0; e < n; ++e) x[e] = conj_if(d[b * n + e], inv);
      int rc = run_group(log_n, x.data(), x.data(), tab.stage[log_n].data());
      if (rc) return rc;
      for (int64_t e = 0; e < n; ++e) d[b * n + e] = epi(x[e], inv, scale);
    }
    return 0;
  }
  const int l1 = four_step_log_n1(log_n), l2 = four_step_log_n2(log_n);
  const int64_t n1 = (int64_t)1 << l1, n2 = (int64_t)1 << l2;
  std::vector<float2> ws(n), col(n1), row(n2);
  for (int64_t b = 0; b < batch; ++b) {
    float2* xb = d + b * n;
    // Pass A (fft_cols_kernel with TW4): column n2 of the N1 x N2 view.
    for (int64_t c = 0; c < n2; ++c) {
      for (int64_t e = 0; e < n1; ++e) col[e] = conj_if(xb[e * n2 + c], inv);
      int rc = run_group(l1, col.data(), col.data(), tab.stage[l1].data());
      if (rc) return rc;
      for (int64_t k1 = 0; k1 < n1; ++k1)
        ws[k1 * n2 + c] = c_mul(col[k1], four_step_twiddle(tab.lo.data(), tab.hi.data(),
                                                           (uint32_t)(c * k1)));
    }
    // Pass B (fft_rows_t_kernel): row k1, stored to X[k1 + N1*k2].
    for (int64_t k1 = 0; k1 < n1; ++k1) {
      int rc = run_group(l2, ws.data() + k1 * n2, row.data(), tab.stage[l2].data());
      if (rc) return rc;
      for (int64_t k2 = 0; k2 < n2; ++k2) xb[k1 + n1 * k2] = epi(row[k2], inv, scale);
    }
  }
  return 0;
}

// In-place batched 2D transform, laid out like ferrum_fft_2d_c2c_pow2.
int emu_fft_2d(float* data, int log_n, int64_t batch, int direction, int normalize) {
  if (log_n < 2 || log_n > kMaxSinglePassLogN || batch <= 0) return -1;
  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  float2* d = (float2*)data;
  Tables tab(log_n);
  const float2* tw = tab.stage[log_n].data();
  std::vector<float2> x(n);
  for (int64_t b = 0; b < batch; ++b) {
    float2* img = d + b * n * n;
    for (int64_t r = 0; r < n; ++r) {
      for (int64_t e = 0; e < n; ++e) x[e] = conj_if(img[r * n + e], inv);
      int rc = run_group(log_n, x.data(), img + r * n, tw);
      if (rc) return rc;
    }
    for (int64_t c = 0; c < n; ++c) {
      for (int64_t e = 0; e < n; ++e) x[e] = img[e * n + c];
      int rc = run_group(log_n, x.data(), x.data(), tw);
      if (rc) return rc;
      for (int64_t e = 0; e < n; ++e) img[e * n + c] = epi(x[e], inv, scale);
    }
  }
  return 0;
}

// The distributed 2D transform on `nranks` emulated ranks; `data` is the
// whole N x N image, rank p owning rows [p*N/P, (p+1)*N/P).
int emu_fft_2d_dist(float* data, int log_n, int nranks, int direction, int normalize) {
  if (log_n < 2 || log_n > kMaxSinglePassLogN || nranks < 1) return -1;
  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const int64_t b = n / nranks;
  int lb = 0;
  while (((int64_t)1 << lb) < b) ++lb;
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  float2* d = (float2*)data;
  Tables tab(log_n);
  const float2* tw = tab.stage[log_n].data();
  std::vector<std::vector<float2>> wa(nranks, std::vector<float2>(b * n)),
      wb(nranks, std::vector<float2>(b * n));
  std::vector<float2> x(n);
  // 1. row pass, blocked store (fft_rows_kernel with log_block = lb)
  for (int p = 0; p < nranks; ++p)
    for (int64_t f = 0; f < b; ++f) {
      for (int64_t e = 0; e < n; ++e) x[e] = conj_if(d[(p * b + f) * n + e], inv);
      int rc = run_group(log_n, x.data(), x.data(), tw);
      if (rc) return rc;
      for (int64_t e = 0; e < n; ++e) wa[p][blocked_index(f, e, lb, b)] = x[e];
    }
  // 2. all-to-all: block q of rank p -> block p of rank q
  for (int p = 0; p < nranks; ++p)
    for (int q = 0; q < nranks; ++q)
      memcpy(wb[q].data() + p * b * b, wa[p].data() + q * b * b, b * b * sizeof(float2));
  // 3. column pass in place on the N x B column slab (ld = B)
  for (int q = 0; q < nranks; ++q)
    for (int64_t c = 0; c < b; ++c) {
      for (int64_t e = 0; e < n; ++e) x[e] = wb[q][e * b + c];
      int rc = run_group(log_n, x.data(), x.data(), tw);
      if (rc) return rc;
      for (int64_t e = 0; e < n; ++e) wb[q][e * b + c] = epi(x[e], inv, scale);
    }
  // 4. all-to-all of the B x B row blocks
  for (int p = 0; p < nranks; ++p)
    for (int q = 0; q < nranks; ++q)
      memcpy(wa[q].data() + p * b * b, wb[p].data() + q * b * b, b * b * sizeof(float2));
  // 5. block gather: out[r][p*B + c] = in[p][r][c]
  for (int q = 0; q < nranks; ++q)
    for (int p = 0; p < nranks; ++p)
      for (int64_t r = 0; r < b; ++r)
        for (int64_t c = 0; c < b; ++c)
          d[(q * b + r) * n + p * b + c] = wa[q][p * b * b + r * b + c];
  return 0;
}

}  // extern "C"
