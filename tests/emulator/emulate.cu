// CPU emulator of the sm_100a FFT kernels — test infrastructure only.
//
// Executes, on the host, the same pass plans the runtime launches
// (ferrum-gpu_b200/csrc/passes.h) with the exact per-thread code of the
// kernels: the radix plans (plan.h), the twiddle tables the runtime uploads
// (twiddle_tables.h), stage_compute / stage_out_pos / stage_slot / smem_pad
// (stockham.cuh), pass_index / pass_tw_base / pass_tw_step and the two-level
// twiddle lookup (fft_kernels.cuh), and the distributed blocked layout (the
// device takes the multi-pass 1D twiddle factors from the SFU instead of the
// table; the emulator checks that those passes have a compiled length). Each
// thread group is simulated thread by thread between barriers, and every
// shared-memory exchange is checked to be a permutation (each padded slot
// written exactly once and read exactly once). The tests compare its output
// with the CPU oracle, so planner and index-arithmetic bugs show up without a
// GPU.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "../../ferrum-gpu_b200/csrc/dist_steps.h"
#include "../../ferrum-gpu_b200/csrc/passes.h"
#include "../../ferrum-gpu_b200/csrc/twiddle_tables.h"

using namespace ferrum;

namespace {

template <int LOGN, int LOGP_ = plan_log_p(LOGN)>
struct Group {
  static constexpr int LOGP = LOGP_;
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
      const int slots = PaddedLen<LOGN, LOGP>::value + 16;
      std::vector<float2> sm(slots);
      std::vector<int> writes(slots, 0), reads(slots, 0);
      for (int t = 0; t < G::T; ++t)
        for (int i = 0; i < B; ++i)
          for (int r = 0; r < R; ++r) {
            const int idx = stage_write_addr<LOGN, LOGP, S>(t, i, r);
            if (idx != smem_pad<LOGP>(stage_out_pos<LOGN, LOGP, S>(t, i, r))) return -40 - S;
            if (idx < 0 || idx >= slots) return -10 - S;
            sm[idx] = regs[t].v[stage_slot<LOGN, LOGP, S>(i, r)];
            writes[idx]++;
          }
      for (int t = 0; t < G::T; ++t)
        for (int m = 0; m < G::P; ++m) {
          const int idx = stage_read_addr<LOGN, LOGP>(t, m);
          if (idx != smem_pad<LOGP>(t + G::T * m)) return -50 - S;
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

// The strided-pass twiddle epilogue, thread by thread: thread t owns outputs
// k = t + T*m and multiplies them by W_M^(tb + ts*k) as fft_pass_kernel does.
template <int LOGN>
int pass_twiddles_group(float2* x, const float2* lo, const float2* hi, uint32_t tb, uint32_t ts,
                        uint32_t mask) {
  using G = Geom<LOGN, plan_log_p(LOGN)>;
  for (int t = 0; t < G::T; ++t) {
    float2 v[G::P];
    for (int m = 0; m < G::P; ++m) v[m] = x[t + G::T * m];
    apply_progression_twiddles<G::P>(v, lo, hi, tb + ts * (uint32_t)t, ts * (uint32_t)G::T, mask);
    for (int m = 0; m < G::P; ++m) x[t + G::T * m] = v[m];
  }
  return 0;
}

int apply_pass_twiddles(int log_n, float2* x, const float2* lo, const float2* hi, uint32_t tb,
                        uint32_t ts, uint32_t mask) {
  switch (log_n) {
#define X(L) \
  case L:    \
    return pass_twiddles_group<L>(x, lo, hi, tb, ts, mask);
    X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14)
#undef X
    default:
      return -1;
  }
}

struct Tables {
  std::vector<float2> stage[kMaxSinglePassLogN + 1];
  std::vector<float2> lo[kMaxLogN + 1], hi[kMaxLogN + 1];
  Tables() {
    for (int l = 2; l <= kMaxSinglePassLogN; ++l) {
      append_stage_tables(stage[l], l);
      stage[l].push_back(make_float2(1.f, 0.f));
    }
    for (int l = 1; l <= kMaxLogN; ++l) append_four_step_tables(lo[l], hi[l], l);
  }
};

const Tables& tables() {
  static Tables t;
  return t;
}

// The inverse's input and output steps as the kernels take them
// (fft_kernels.cuh swap_if / epilogue): real and imaginary parts swapped,
// which over the whole transform equals conjugating both ends.
float2 conj_if(float2 v, bool c) { return c ? make_float2(v.y, v.x) : v; }
float2 epi(float2 v, bool conj_out, float scale) {
  return conj_out ? make_float2(v.y * scale, v.x * scale) : v;
}

// fft_cols_l2_kernel: per tile of W columns, sub-pass 1 (units a < A) into
// the tile's scratch slot (row pitch W), then sub-pass 2 (units kb < B) from
// the slot to the output. The GPU grid is min(tiles, slots) CTAs and CTA c
// takes tiles c, c + grid, ... with slot c, so tile t uses slot t mod grid;
// each tile rewrites its slot before reading it.
int run_cols_l2(const PassDesc& d, const float2* src, float2* dst, float2* ws) {
  if (ws == nullptr) return -70;
  const Tables& tab = tables();
  const int l1 = d.cl2_l1, l2 = d.cl2_l2, w = cols_l2_width(d.log_n);
  if (l1 + l2 != d.log_n || w == 0) return -71;
  const int64_t A = (int64_t)1 << l2, B = (int64_t)1 << l1, n = A * B;
  const uint32_t mask = (uint32_t)(n - 1);
  const ColsL2Args& a = d.ca;
  const int64_t grid = a.tiles < cols_l2_slots(d.log_n) ? a.tiles : cols_l2_slots(d.log_n);
  std::vector<float2> x(n);
  for (int64_t tile = 0; tile < a.tiles; ++tile) {
    const int64_t tpi = (int64_t)1 << a.log_tiles_per_img;
    const int64_t base = (tile / tpi) * a.img_stride + (tile % tpi) * w;
    float2* slot = ws + (tile % grid) * (int64_t)w * n;
    for (int64_t j = 0; j < A; ++j)
      for (int cl = 0; cl < w; ++cl) {
        for (int64_t e = 0; e < B; ++e)
          x[e] = conj_if(src[base + cl + (j + A * e) * a.ld], d.conj_in);
        if (int rc = run_group(l1, x.data(), x.data(), tab.stage[l1].data())) return rc;
        if (int rc = apply_pass_twiddles(l1, x.data(), tab.lo[d.log_n].data(),
                                         tab.hi[d.log_n].data(), 0u, (uint32_t)j, mask))
          return rc;
        for (int64_t k = 0; k < B; ++k) slot[(j + A * k) * w + cl] = x[k];
      }
    for (int64_t j = 0; j < B; ++j)
      for (int cl = 0; cl < w; ++cl) {
        for (int64_t e = 0; e < A; ++e) x[e] = slot[(A * j + e) * w + cl];
        if (int rc = run_group(l2, x.data(), x.data(), tab.stage[l2].data())) return rc;
        for (int64_t k = 0; k < A; ++k)
          dst[base + cl + (j + B * k) * a.ld] = epi(x[k], d.conj_out, a.scale);
      }
  }
  return 0;
}

// Layout conditions of the tile kernels (launch_tile.cu checks the same at
// run time and falls back to the plain kernel when one fails; a plan should
// never need that fallback for its own buffers).
int check_tile_pass(const PassDesc& d) {
  if (d.tile == TileMode::None) return 0;
  if (d.tile_w <= 0) return -80;
  if (d.kind == PassKind::Pass) {
    const PassArgs& a = d.pa;
    if (a.in_c != 1 || a.out_c != 1 || (((int64_t)1 << a.log_w) % d.tile_w) != 0) return -81;
    if (a.in_o % a.in_e != 0 || a.in_j % a.in_e != 0) return -82;
    if (d.tile == TileMode::Tma && (a.out_o % a.out_e != 0 || a.out_j % a.out_e != 0)) return -83;
    if (d.conj_out || a.log_m == 0 || !a.tw_sfu) return -84;  // compiled combinations
    const int lp = tile_log_p(d);
    const bool compiled = (d.tile == TileMode::Prefetch && d.tile_w == 16 && lp == 5 &&
                           (d.log_n == 9 || d.log_n == 10)) ||
                          (d.tile == TileMode::Tma && d.tile_w == 4 && d.log_n == 11 && lp == 4);
    if (lp != plan_log_p(d.log_n) && !(lp == 5 && tile_p32_table(d.log_n))) return -92;
    return compiled ? 0 : -85;
  }
  if (d.kind == PassKind::RowsT) {
    const RowsTArgs& a = d.ra;
    if ((((int64_t)1 << a.log_w) % d.tile_w) != 0) return -86;
    if (a.in_c % 2 != 0 || a.in_o % 2 != 0 || a.in_j % 2 != 0) return -87;
    if (d.tile == TileMode::Tma && (a.out_o % a.out_e != 0 || a.out_j % a.out_e != 0)) return -88;
    const int lp = tile_log_p(d);
    const bool compiled = (d.tile == TileMode::Prefetch && d.tile_w == 8 &&
                           ((d.log_n == 10 && lp == 5) || (d.log_n == 11 && lp == 4))) ||
                          (d.tile == TileMode::Tma && d.tile_w == 4 && d.log_n == 12 && lp == 4);
    if (lp != plan_log_p(d.log_n) && !(lp == 5 && tile_p32_table(d.log_n))) return -92;
    return compiled ? 0 : -89;
  }
  return -90;
}

// One pass of a plan, FFT by FFT (each touches disjoint elements, so in-place
// passes behave as on the GPU).
int run_pass(const PassDesc& d, const float2* src, float2* dst, float2* ws) {
  if (int rc = check_tile_pass(d)) return rc;
  const Tables& tab = tables();
  const int64_t n = (int64_t)1 << d.log_n;
  const float2* stw = tab.stage[d.log_n].data();
  std::vector<float2> x(n);
  switch (d.kind) {
    case PassKind::Rows: {
      const int lb = (d.rows_log_block < 0 || d.rows_log_block > d.log_n) ? d.log_n
                                                                          : d.rows_log_block;
      for (int64_t f = 0; f < d.rows_nfft; ++f) {
        for (int64_t e = 0; e < n; ++e) x[e] = conj_if(src[f * n + e], d.conj_in);
        if (int rc = run_group(d.log_n, x.data(), x.data(), stw)) return rc;
        for (int64_t e = 0; e < n; ++e) {
          const int64_t rows = d.rows_block_rows > 0 ? d.rows_block_rows : d.rows_nfft;
          const int64_t at = lb >= d.log_n ? f * n + e : blocked_index(f, e, lb, rows);
          dst[at] = epi(x[e], d.conj_out, d.rows_scale);
        }
      }
      return 0;
    }
    case PassKind::Pass: {
      const PassArgs& a = d.pa;
      if (!pass_flags_supported(d.conj_in, d.conj_out, a.log_m > 0)) return -60;
      if (a.tw_sfu && (a.log_m == 0 || !pass_sfu_supported(d.log_n))) return -62;
      const uint32_t mask = a.log_m > 0 ? (1u << a.log_m) - 1u : 0u;
      for (int64_t f = 0; f < a.nfft; ++f) {
        int64_t o, j, c;
        pass_index(f, a.log_w, a.log_j, o, j, c);
        const int64_t ib = o * a.in_o + j * a.in_j + c * a.in_c,
                      ob = o * a.out_o + j * a.out_j + c * a.out_c;
        for (int64_t e = 0; e < n; ++e) x[e] = conj_if(src[ib + e * a.in_e], d.conj_in);
        if (int rc = run_group(d.log_n, x.data(), x.data(), stw)) return rc;
        if (a.log_m > 0) {
          // fft_pass_kernel: thread t owns outputs k = t + T*m and applies
          // W_M^(tb + ts*k) through apply_progression_twiddles.
          const uint32_t tb = pass_tw_base((uint32_t)c, (uint32_t)j, a.tcj);
          const uint32_t ts = pass_tw_step((uint32_t)c, (uint32_t)j, a.tc, a.tj);
          if (int rc = apply_pass_twiddles(d.log_n, x.data(), tab.lo[a.log_m].data(),
                                           tab.hi[a.log_m].data(), tb, ts, mask))
            return rc;
        }
        for (int64_t k = 0; k < n; ++k) dst[ob + k * a.out_e] = epi(x[k], d.conj_out, a.scale);
      }
      return 0;
    }
    case PassKind::ColsL2:
      return run_cols_l2(d, src, dst, ws);
    case PassKind::RowsT: {
      const RowsTArgs& a = d.ra;
      // fft_rows_t_kernel: 4 <= log_n <= 14, not both conj_in and conj_out
      if ((d.conj_in && d.conj_out) || d.log_n < 4) return -61;
      for (int64_t f = 0; f < a.nfft; ++f) {
        int64_t o, j, c;
        pass_index(f, a.log_w, a.log_j, o, j, c);
        const int64_t ib = o * a.in_o + j * a.in_j + c * a.in_c, ob = o * a.out_o + j * a.out_j + c;
        for (int64_t e = 0; e < n; ++e) x[e] = conj_if(src[ib + e], d.conj_in);
        if (int rc = run_group(d.log_n, x.data(), x.data(), stw)) return rc;
        for (int64_t k = 0; k < n; ++k) dst[ob + k * a.out_e] = epi(x[k], d.conj_out, a.scale);
      }
      return 0;
    }
  }
  return -2;
}

int run_plan(const PassPlan& pl, const float2* in, float2* out, float2* ws) {
  float2* bufs[3] = {const_cast<float2*>(in), out, ws};
  for (int i = 0; i < pl.count; ++i) {
    const PassDesc& d = pl.p[i];
    if (int rc = run_pass(d, bufs[(int)d.src], bufs[(int)d.dst], ws)) return rc;
  }
  return 0;
}

}  // namespace

extern "C" {

// In-place batched 1D transform, laid out like ferrum_fft_1d_c2c_pow2.
int emu_fft_1d(float* data, int log_n, int64_t batch, int direction, int normalize) {
  if (log_n < 2 || log_n > kMaxLogN || batch <= 0) return -1;
  PassPlan pl = plan_1d(log_n, batch, direction < 0, normalize != 0);
  std::vector<float2> ws(pl.ws_elems);
  float2* d = (float2*)data;
  return run_plan(pl, d, d, ws.data());
}

// One forward transform of length 2^log_n in place with 2^log_p values per
// thread and that split's stage tables: the 32-value split the tile kernels
// run at lengths 2^9..2^12 (tile_p32_table).
int emu_group_lp(float* data, int log_n, int log_p) {
  std::vector<float2> tw;
  append_stage_tables(tw, log_n, log_p);
  tw.push_back(make_float2(1.f, 0.f));
  float2* d = (float2*)data;
  switch (log_n * 8 + log_p) {
#define X(L, P) \
  case L * 8 + P: \
    return Group<L, P>::run(d, d, tw.data());
    X(9, 5) X(10, 5) X(11, 5) X(12, 5)
#undef X
    default:
      return -1;
  }
}

// Number of passes the plan for this 1D size uses (for the tests).
int emu_plan_1d_passes(int log_n) { return plan_1d(log_n, 1, false, false).count; }

// In-place batched 2D transform, laid out like ferrum_fft_2d_c2c_pow2.
int emu_fft_2d(float* data, int log_n, int64_t batch, int direction, int normalize) {
  if (log_n < 2 || log_n > kMaxSinglePassLogN || batch <= 0) return -1;
  PassPlan pl = plan_2d(log_n, batch, direction < 0, normalize != 0);
  std::vector<float2> ws(pl.ws_elems);
  float2* d = (float2*)data;
  return run_plan(pl, d, d, ws.data());
}

// The distributed 2D transform on `nranks` emulated ranks, following the
// same steps, chunks and offsets as ferrum_fft_2d_c2c_pow2_dist_layout.
// `data` is the whole N x N image, row-major; it is split into row slabs
// (layout 0) or column slabs (layout 1) on input and reassembled from the
// output layout.
// The peer-memory path of dist.cu (dist_p2p): each rank's receive slab is
// written by the row-FFT scatter (or read by the row-FFT gather) through
// peer_offset, the column passes run on the local slab.
int emu_fft_2d_dist_p2p(float* data, int log_n, int nranks, int direction, int normalize,
                        int in_layout, int out_layout) {
  if (log_n < 4 || log_n > kMaxSinglePassLogN || nranks < 1) return -1;
  const bool row_in = in_layout == 0, row_out = out_layout == 0;
  if (!row_in && !row_out) return -1;
  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const int64_t b = n / nranks;
  int lb = 0;
  while (((int64_t)1 << lb) < b) ++lb;
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  const float2* stw = tables().stage[log_n].data();
  float2* d = (float2*)data;
  const size_t slab = (size_t)(b * n);
  std::vector<std::vector<float2>> in(nranks, std::vector<float2>(slab)),
      out(nranks, std::vector<float2>(slab)), recv(nranks, std::vector<float2>(slab)),
      ws(nranks, std::vector<float2>(std::max<size_t>(slab, (size_t)cols_l2_ws_elems(log_n))));
  for (int p = 0; p < nranks; ++p)
    for (int64_t r = 0; r < (row_in ? b : n); ++r)
      for (int64_t c = 0; c < (row_in ? n : b); ++c)
        in[p][r * (row_in ? n : b) + c] = row_in ? d[(p * b + r) * n + c] : d[r * n + p * b + c];
  std::vector<float2> x(n);
  if (row_in) {
    // fft_rows_scatter_kernel on every rank, then the barrier.
    for (int p = 0; p < nranks; ++p)
      for (int64_t f = 0; f < b; ++f) {
        for (int64_t e = 0; e < n; ++e) {
          const float2 v = in[p][f * n + e];
          x[e] = conj_if(v, inv);  // CONJ_IN of the scatter kernel
        }
        if (int rc = run_group(log_n, x.data(), x.data(), stw)) return rc;
        for (int64_t e = 0; e < n; ++e)
          recv[e >> lb][p * b * b + peer_offset(f, e, lb)] = x[e];
      }
    for (int p = 0; p < nranks; ++p) {
      PassPlan cols;
      plan_columns(cols, log_n, lb, b, 1, n * b, false, inv, scale, PassBuf::In, PassBuf::Ws,
                   PassBuf::Out);
      if (int rc = run_plan(cols, recv[p].data(), row_out ? recv[p].data() : out[p].data(),
                            ws[p].data()))
        return rc;
    }
    if (row_out)  // peer_block_gather_kernel after a barrier
      for (int p = 0; p < nranks; ++p)
        for (int q = 0; q < nranks; ++q)
          for (int64_t r = 0; r < b; ++r)
            for (int64_t c = 0; c < b; ++c)
              out[p][r * n + q * b + c] = recv[q][p * b * b + r * b + c];
  } else {
    for (int p = 0; p < nranks; ++p) {
      PassPlan cols;
      plan_columns(cols, log_n, lb, b, 1, n * b, inv, false, 1.0f, PassBuf::In, PassBuf::Ws,
                   PassBuf::Out);
      if (int rc = run_plan(cols, in[p].data(), recv[p].data(), ws[p].data())) return rc;
    }
    // fft_rows_gather_kernel after the barrier.
    for (int p = 0; p < nranks; ++p)
      for (int64_t f = 0; f < b; ++f) {
        for (int64_t e = 0; e < n; ++e) x[e] = recv[e >> lb][p * b * b + peer_offset(f, e, lb)];
        if (int rc = run_group(log_n, x.data(), x.data(), stw)) return rc;
        for (int64_t e = 0; e < n; ++e) out[p][f * n + e] = epi(x[e], inv, scale);
      }
  }
  for (int p = 0; p < nranks; ++p)
    for (int64_t r = 0; r < (row_out ? b : n); ++r)
      for (int64_t c = 0; c < (row_out ? n : b); ++c) {
        const float2 v = out[p][r * (row_out ? n : b) + c];
        if (row_out)
          d[(p * b + r) * n + c] = v;
        else
          d[r * n + p * b + c] = v;
      }
  return 0;
}

int emu_fft_2d_dist_layout(float* data, int log_n, int nranks, int direction, int normalize,
                           int in_layout, int out_layout) {
  if (log_n < 2 || log_n > kMaxSinglePassLogN || nranks < 1) return -1;
  const bool row_in = in_layout == 0, row_out = out_layout == 0;
  if (!row_in && !row_out) return -1;
  const bool inv = direction < 0;
  const int64_t n = (int64_t)1 << log_n;
  const int64_t b = n / nranks;
  int lb = 0;
  while (((int64_t)1 << lb) < b) ++lb;
  const int chunks = dist_chunks(b);
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  float2* d = (float2*)data;
  const size_t slab = (size_t)(b * n);
  std::vector<std::vector<float2>> in(nranks, std::vector<float2>(slab)),
      out(nranks, std::vector<float2>(slab)), wa(nranks, std::vector<float2>(slab)),
      wb(nranks, std::vector<float2>(slab));
  for (int p = 0; p < nranks; ++p)
    for (int64_t r = 0; r < (row_in ? b : n); ++r)
      for (int64_t c = 0; c < (row_in ? n : b); ++c)
        in[p][r * (row_in ? n : b) + c] = row_in ? d[(p * b + r) * n + c] : d[r * n + p * b + c];
  // Exchange of rows [r0, r1) of every block: rank p sends from src[p] to q.
  auto exchange = [&](std::vector<std::vector<float2>>& src, std::vector<std::vector<float2>>& dst,
                      int64_t r0, int64_t r1) {
    for (int p = 0; p < nranks; ++p)
      for (int q = 0; q < nranks; ++q)
        memcpy(dst[q].data() + dist_block_offset(p, r0, b), src[p].data() + dist_block_offset(q, r0, b),
               (size_t)((r1 - r0) * b) * sizeof(float2));
  };
  auto gather = [&](const float2* src, float2* dst, int64_t rows) {
    for (int p = 0; p < nranks; ++p)
      for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < b; ++c) dst[r * n + p * b + c] = src[p * b * b + r * b + c];
  };
  if (row_in) {
    for (int c = 0; c < chunks; ++c) {
      int64_t r0, r1;
      dist_chunk(b, chunks, c, r0, r1);
      for (int p = 0; p < nranks; ++p) {
        PassDesc rows = make_rows(log_n, r1 - r0, inv, false, 1.0f, PassBuf::In, PassBuf::Out, lb, b);
        if (int rc = run_pass(rows, in[p].data() + r0 * n, wa[p].data() + r0 * b, nullptr)) return rc;
      }
      exchange(wa, wb, r0, r1);
    }
    for (int p = 0; p < nranks; ++p) {
      PassPlan cols;
      plan_columns(cols, log_n, lb, b, 1, n * b, false, inv, scale, PassBuf::In, PassBuf::In,
                   PassBuf::Out);
      if (int rc = run_plan(cols, wb[p].data(), row_out ? wa[p].data() : out[p].data(), nullptr))
        return rc;
    }
    if (row_out)
      for (int c = 0; c < chunks; ++c) {
        int64_t r0, r1;
        dist_chunk(b, chunks, c, r0, r1);
        exchange(wa, wb, r0, r1);
        for (int p = 0; p < nranks; ++p) gather(wb[p].data() + r0 * b, out[p].data() + r0 * n, r1 - r0);
      }
  } else {
    for (int p = 0; p < nranks; ++p) {
      PassPlan cols;
      plan_columns(cols, log_n, lb, b, 1, n * b, inv, false, 1.0f, PassBuf::In, PassBuf::Out,
                   PassBuf::Ws);
      if (int rc = run_plan(cols, in[p].data(), wa[p].data(), wb[p].data())) return rc;
    }
    for (int c = 0; c < chunks; ++c) {
      int64_t r0, r1;
      dist_chunk(b, chunks, c, r0, r1);
      exchange(wb, wa, r0, r1);
      for (int p = 0; p < nranks; ++p) {
        gather(wa[p].data() + r0 * b, out[p].data() + r0 * n, r1 - r0);
        PassDesc rows = make_rows(log_n, r1 - r0, false, inv, scale, PassBuf::In, PassBuf::Out);
        if (int rc = run_pass(rows, out[p].data() + r0 * n, out[p].data() + r0 * n, nullptr)) return rc;
      }
    }
  }
  for (int p = 0; p < nranks; ++p)
    for (int64_t r = 0; r < (row_out ? b : n); ++r)
      for (int64_t c = 0; c < (row_out ? n : b); ++c) {
        const float2 v = out[p][r * (row_out ? n : b) + c];
        if (row_out)
          d[(p * b + r) * n + c] = v;
        else
          d[r * n + p * b + c] = v;
      }
  return 0;
}

int emu_fft_2d_dist(float* data, int log_n, int nranks, int direction, int normalize) {
  return emu_fft_2d_dist_layout(data, log_n, nranks, direction, normalize, 0, 0);
}

}  // extern "C"
