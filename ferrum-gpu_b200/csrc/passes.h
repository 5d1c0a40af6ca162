// Pass planner: turns a transform request into an ordered list of kernel
// passes over HBM. Shared by the runtime (capi.cu, dist.cu) and the CPU
// emulator in the test suite, which executes the same plans.
//
// Every pass reads and writes each element once, with row segments of at
// least 64-128 bytes:
//   * 1D, N <= 2^14: one fft_rows_kernel pass.
//   * 1D, 2^15..2^23: two passes, N = N1*N2 (N1 = 2^(log_n/2), except
//     2^22 = 1024 x 4096), x[n2 + N2*n1]:
//       A  DFT over n1 (columns of the N1 x N2 view), times W_N^(n2*k1);
//       B  DFT over n2 (rows), stored transposed to X[k1 + N1*k2].
//     (2^19..2^23 run both passes in the persistent tile kernels).
//   * 1D, 2^24..2^26: three passes, N = N1*N2*N3, x[n3 + N3*n2 + N3*N2*n1]:
//       1  DFT over n1, times W_{N1 N2}^(n2*k1);
//       2  DFT over n2, times W_N^(n3*(k1 + N1*k2));
//       3  DFT over n3 (rows), stored to X[k1 + N1*k2 + N1*N2*k3].
//   * 2D N x N, N <= 512: row pass, then one column pass in place.
//   * 2D, N = 1024..4096: two transposed-row passes through a workspace
//     (rows of each image stored transposed, then the rows of that stored
//     transposed back), in the persistent tile kernels.
//   * 2D, N >= 8192: columns first as two sub-passes (N = A*B, row a + A*b:
//     DFT over b times W_N^(a*kb), then DFT over a stored to row kb + B*ka),
//     then the row pass, which also applies the inverse's conjugate and
//     scale. (The fused two-sub-pass column kernel, fft_cols_l2_kernel, keeps
//     the intermediate of each tile of 4096-point columns in an L2-resident
//     scratch slot; the distributed transform's column passes use it.)
// The index identities are the Cooley-Tukey splits; the reference's CPU
// Stockham (crates/ferrum-gpu-fft/src/cpu.rs) defines the results they must
// reproduce.
#pragma once

#include <stdint.h>

#include "fft_kernels.cuh"
#include "plan.h"

namespace ferrum {

enum class PassKind : int { Rows = 0, Pass = 1, RowsT = 2, ColsL2 = 3 };
enum class PassBuf : int { In = 0, Out = 1, Ws = 2 };

// Kernel family of a Pass / RowsT pass. The tile kernels (fft_tile_kernels.cuh)
// compute exactly what the plain kernels do over the same PassArgs /
// RowsTArgs, in persistent CTAs that each take tiles of `tile_w` adjacent
// transforms. They need 16-byte aligned buffers (the runtime falls back to the
// plain kernel otherwise).
enum class TileMode : int {
  None = 0,     // fft_pass_kernel / fft_rows_t_kernel
  Prefetch = 1, // fft_cols_tile_kernel (tensor-map L2 prefetch) / fft_rows_t_tile_kernel
  Tma = 2,      // fft_cols_tma_kernel (TMA tile load and store) / fft_rows_t_tma_kernel (TMA store)
};

struct PassDesc {
  PassKind kind;
  int log_n;  // transform length of the pass
  TileMode tile = TileMode::None;
  int tile_w = 0;
  int tile_lp = 0;  // log2 values per thread of the tile kernel (0: plan_log_p(log_n))
  bool conj_in, conj_out;
  PassBuf src, dst;
  // Rows
  int64_t rows_nfft;
  int rows_log_block;
  int64_t rows_block_rows;
  float rows_scale;
  // Pass / RowsT (twiddle tables are filled in by the executor from log_m)
  PassArgs pa;
  RowsTArgs ra;
  // ColsL2: sub-pass lengths 2^l1 (first) and 2^l2 (second), log_n = l1 + l2;
  // the executor fills the twiddle tables. Scratch slots live in PassBuf::Ws.
  int cl2_l1, cl2_l2;
  ColsL2Args ca;
};

struct PassPlan {
  int count = 0;
  PassDesc p[4];
  int64_t ws_elems = 0;  // workspace (complex values) the plan needs
};

// (conj_in, conj_out, twiddle) combinations of fft_pass_kernel that are
// compiled: a twiddled pass is never last (no conj_out), and no single pass
// both conjugates its input and its output.
constexpr bool pass_flags_supported(bool ci, bool co, bool tw) {
  return tw ? !co : !(ci && co);
}

// Pass lengths compiled with SFU twiddle factors (the column passes of the
// multi-pass 1D transform, 2^15..2^26, have lengths 2^7..2^11).
constexpr bool pass_sfu_supported(int log_n) { return log_n >= 7 && log_n <= 11; }

inline PassDesc make_rows(int log_n, int64_t nfft, bool ci, bool co, float scale, PassBuf src,
                          PassBuf dst, int log_block = -1, int64_t block_rows = 0) {
  PassDesc d{};
  d.kind = PassKind::Rows;
  d.log_n = log_n;
  d.conj_in = ci;
  d.conj_out = co;
  d.src = src;
  d.dst = dst;
  d.rows_nfft = nfft;
  d.rows_log_block = log_block;
  d.rows_block_rows = block_rows;
  d.rows_scale = scale;
  return d;
}

inline PassDesc make_pass(int log_n, bool ci, bool co, PassBuf src, PassBuf dst, const PassArgs& a) {
  PassDesc d{};
  d.kind = PassKind::Pass;
  d.log_n = log_n;
  d.conj_in = ci;
  d.conj_out = co;
  d.src = src;
  d.dst = dst;
  d.pa = a;
  return d;
}

inline PassDesc make_rows_t(int log_n, bool co, PassBuf src, PassBuf dst, const RowsTArgs& a,
                            bool ci = false) {
  PassDesc d{};
  d.kind = PassKind::RowsT;
  d.log_n = log_n;
  d.conj_in = ci;
  d.conj_out = co;
  d.src = src;
  d.dst = dst;
  d.ra = a;
  return d;
}

inline PassArgs pass_args(int64_t nfft, int log_w, int log_j, int64_t in_o, int64_t in_j,
                          int64_t in_e, int64_t out_o, int64_t out_j, int64_t out_e) {
  PassArgs a{};
  a.nfft = nfft;
  a.log_w = log_w;
  a.log_j = log_j;
  a.in_o = in_o;
  a.in_j = in_j;
  a.in_e = in_e;
  a.out_o = out_o;
  a.out_j = out_j;
  a.out_e = out_e;
  a.in_c = 1;
  a.out_c = 1;
  a.scale = 1.0f;
  return a;
}


// The fused column kernel (fft_cols_l2_kernel) per column length: columns per
// tile W (0 = the length keeps two separate sub-passes), threads and resident
// CTAs per SM, and scratch slots (one per resident CTA on a 148-SM B200).
// Measured on 2D N x N transforms (2 GiB): the sub-pass loop needs ~127
// registers (at 64 it spilled); one 512-thread CTA per SM with W = 8 at
// N = 4096 (a 37 MiB slot set) beat the separate sub-passes (1.88 vs 2.10 ms
// for 4096^2 x 16), while a 74 MiB slot set (two CTAs per SM, or W = 8 at
// N = 8192) lost to them: the L2 keeps the slots only well below its 126 MB.
// 32-byte row segments (W = 4) at N >= 8192 were worse still, so N >= 8192
// keeps the separate sub-passes.
constexpr int cols_l2_width(int log_n) { return log_n == 12 ? 8 : 0; }
constexpr int cols_l2_threads(int) { return 512; }
constexpr int cols_l2_ctas_per_sm(int) { return 1; }
constexpr int cols_l2_slots(int log_n) { return 148 * cols_l2_ctas_per_sm(log_n); }

inline PassDesc make_cols_l2(int log_n, int log_width, int64_t ld, int64_t images,
                             int64_t img_stride, bool ci, bool co, float scale, PassBuf src,
                             PassBuf dst) {
  PassDesc d{};
  d.kind = PassKind::ColsL2;
  d.log_n = log_n;
  d.conj_in = ci;
  d.conj_out = co;
  d.src = src;
  d.dst = dst;
  d.cl2_l2 = log_n / 2;
  d.cl2_l1 = log_n - d.cl2_l2;
  int lw = 0;
  while ((1 << lw) < cols_l2_width(log_n)) ++lw;
  d.ca.tiles = images << (log_width - lw);
  d.ca.log_tiles_per_img = log_width - lw;
  d.ca.img_stride = img_stride;
  d.ca.ld = ld;
  d.ca.scale = scale;
  return d;
}

inline int64_t cols_l2_ws_elems(int log_n) {
  return (int64_t)cols_l2_slots(log_n) * cols_l2_width(log_n) * ((int64_t)1 << log_n);
}

// Passes of a multi-pass 1D transform.
inline int plan_1d_passes(int log_n) { return log_n <= kMaxSinglePassLogN ? 1 : (log_n <= 23 ? 2 : 3); }

// Column length 2^l1 of the two-pass split N = N1 * N2: half of log_n, except
// 2^22 = 1024 x 4096, which takes the 16-column tiles of the 1024-point
// column pass and the 4096-point transposed-row pass instead of the 4-column
// (32-byte segment) 2048-point column pass (per 512 MiB: 0.210 + 0.214 vs
// 0.250 + 0.194 ms; the whole 2 GiB transform 1.731 -> 1.678 ms forward,
// 1.791 -> 1.759 inverse on one B200).
inline int four_step_split_l1(int log_n) { return log_n == 22 ? 10 : log_n / 2; }

// Kernels of the two passes of the 2^19..2^23 transforms: per pass the tile
// kernel family and the tile width (transforms per tile), chosen by measured
// per-pass time on B200 (512 MiB batches, per pass in ms: the plain strided
// pass vs the tile kernels; whole transforms 2^19 0.417 -> 0.404,
// 2^20 0.466 -> 0.425, 2^21 0.510 -> 0.439, 2^22 0.522 -> 0.472,
// 2^23 (three passes before) 0.542 -> 0.482). Column passes of 512 and 1024
// take 16 columns per tile (128-byte row segments; the next tile is
// prefetched into the L2 through a tensor map), 2048 takes 4 columns moved by
// TMA (its 32-byte segments cost the load/store pipeline a line lookup each;
// two CTAs per SM); transposed-store row passes of 1024 and 2048 take 8 rows
// per tile, 4096 takes 4 rows stored by TMA. Below 2^19 the plain kernels,
// with many CTAs per SM, measured faster; 2^24 and up keep three passes of
// 128-byte segments (two passes of 4096 with 32-byte segments measured 3 %
// slower).
// The 512- and 1024-point column tiles and the 1024-point transposed-row
// tiles run with 32 values per thread (one exchange fewer at 1024; per
// 512 MiB: 1024-point columns 0.228 -> 0.210 ms, 512-point 0.215 -> 0.207,
// 1024-point rows 0.189 -> 0.184); the 2048- and 4096-point tiles keep 16
// (32 measured 3-13 % slower).
struct TileChoice {
  TileMode mode;
  int w;
  int lp;  // 0: plan_log_p
};
inline TileChoice tile_cols_choice(int log_n1) {
  if (log_n1 == 9 || log_n1 == 10) return {TileMode::Prefetch, 16, 5};
  if (log_n1 == 11) return {TileMode::Tma, 4, 0};
  return {TileMode::None, 0, 0};
}
inline TileChoice tile_rows_t_choice(int log_n2) {
  if (log_n2 == 10) return {TileMode::Prefetch, 8, 5};
  if (log_n2 == 11) return {TileMode::Prefetch, 8, 0};
  if (log_n2 == 12) return {TileMode::Tma, 4, 0};
  return {TileMode::None, 0, 0};
}
// Values per thread (log2) a pass's tile kernel runs with.
inline int tile_log_p(const PassDesc& d) { return d.tile_lp > 0 ? d.tile_lp : plan_log_p(d.log_n); }
constexpr int kTileFromLogN = 19;

inline PassPlan plan_1d(int log_n, int64_t batch, bool inv, bool normalize) {
  PassPlan pl;
  const int64_t n = (int64_t)1 << log_n;
  const float scale = (inv && normalize) ? 1.0f / (float)n : 1.0f;
  const int np = plan_1d_passes(log_n);
  if (np == 1) {
    pl.p[pl.count++] = make_rows(log_n, batch, inv, inv, scale, PassBuf::In, PassBuf::Out);
    return pl;
  }
  pl.ws_elems = n * batch;
  if (np == 2) {
    const int l1 = four_step_split_l1(log_n), l2 = log_n - l1;
    const int64_t n1 = (int64_t)1 << l1, n2 = (int64_t)1 << l2;
    PassArgs a = pass_args(batch * n2, l2, 0, n, 0, n2, n, 0, n2);
    a.tc = 1;
    a.log_m = log_n;
    a.tw_sfu = pass_sfu_supported(l1);
    pl.p[pl.count++] = make_pass(l1, inv, false, PassBuf::In, PassBuf::Ws, a);
    if (log_n >= kTileFromLogN) {
      const TileChoice c = tile_cols_choice(l1);
      pl.p[pl.count - 1].tile = c.mode;
      pl.p[pl.count - 1].tile_w = c.w;
      pl.p[pl.count - 1].tile_lp = c.lp;
    }
    RowsTArgs b{};
    b.nfft = batch * n1;
    b.log_w = l1;
    b.log_j = 0;
    b.in_o = n;
    b.in_c = n2;
    b.out_o = n;
    b.out_e = n1;
    b.scale = scale;
    pl.p[pl.count++] = make_rows_t(l2, inv, PassBuf::Ws, PassBuf::Out, b);
    if (log_n >= kTileFromLogN) {
      const TileChoice c = tile_rows_t_choice(l2);
      pl.p[pl.count - 1].tile = c.mode;
      pl.p[pl.count - 1].tile_w = c.w;
      pl.p[pl.count - 1].tile_lp = c.lp;
    }
    return pl;
  }
  // Three passes: the row pass (last) gets the largest factor.
  const int l1 = log_n / 3, l2 = (log_n - l1) / 2, l3 = log_n - l1 - l2;
  const int64_t n1 = (int64_t)1 << l1, n2 = (int64_t)1 << l2, n3 = (int64_t)1 << l3;
  PassArgs a1 = pass_args(batch * n2 * n3, l3, l2, n, n3, n2 * n3, n, n3, n2 * n3);
  a1.tj = 1;
  a1.log_m = l1 + l2;
  a1.tw_sfu = pass_sfu_supported(l1);
  pl.p[pl.count++] = make_pass(l1, inv, false, PassBuf::In, PassBuf::Ws, a1);
  PassArgs a2 = pass_args(batch * n1 * n3, l3, l1, n, n2 * n3, n3, n, n2 * n3, n3);
  a2.tcj = 1;
  a2.tc = (uint32_t)n1;
  a2.log_m = log_n;
  a2.tw_sfu = pass_sfu_supported(l2);
  pl.p[pl.count++] = make_pass(l2, false, false, PassBuf::Ws, PassBuf::Ws, a2);
  RowsTArgs b{};
  b.nfft = batch * n1 * n2;
  b.log_w = l1;
  b.log_j = l2;
  b.in_o = n;
  b.in_j = n3;
  b.in_c = n2 * n3;
  b.out_o = n;
  b.out_j = n1;
  b.out_e = n1 * n2;
  b.scale = scale;
  pl.p[pl.count++] = make_rows_t(l3, inv, PassBuf::Ws, PassBuf::Out, b);
  return pl;
}

// Longest column FFT done in one strided pass.
constexpr int kMaxOnePassColumnLogN = 11;

// Column FFTs of length 2^log_n over `width` adjacent columns (row pitch
// `ld`), for `images` blocks `img_stride` apart, from `src` to `dst`. One pass
// when the pass kernel covers >= 4 columns per CTA with at most 512 threads
// (N <= 2048), otherwise two sub-passes through `mid`; a one-pass N = 4096
// column kernel (4 columns, 1024 threads, one CTA per SM) measured slower than
// the two sub-passes. The last pass applies conj_out / scale.
inline void plan_columns(PassPlan& pl, int log_n, int log_width, int64_t ld, int64_t images,
                         int64_t img_stride, bool ci, bool co, float scale, PassBuf src,
                         PassBuf mid, PassBuf dst) {
  const int64_t width = (int64_t)1 << log_width;
  // Both sub-passes in one kernel when the plan has a workspace for the slots
  // (mid == Ws) and the columns split into whole tiles.
  if (log_n > kMaxOnePassColumnLogN && mid == PassBuf::Ws && cols_l2_width(log_n) > 0 &&
      width >= cols_l2_width(log_n)) {
    pl.p[pl.count++] = make_cols_l2(log_n, log_width, ld, images, img_stride, ci, co, scale, src,
                                    dst);
    if (pl.ws_elems < cols_l2_ws_elems(log_n)) pl.ws_elems = cols_l2_ws_elems(log_n);
    return;
  }
  if (log_n <= kMaxOnePassColumnLogN) {
    PassArgs a = pass_args(images * width, log_width, 0, img_stride, 0, ld, img_stride, 0, ld);
    a.scale = scale;
    pl.p[pl.count++] = make_pass(log_n, ci, co, src, dst, a);
    return;
  }
  const int la = log_n / 2, lb = log_n - la;
  const int64_t na = (int64_t)1 << la, nb = (int64_t)1 << lb;
  // Sub-pass 1: DFT over b of rows a + A*b, times W_N^(a*kb), same positions.
  PassArgs a1 = pass_args(images * width * na, log_width, la, img_stride, ld, na * ld, img_stride,
                          ld, na * ld);
  a1.tj = 1;
  a1.log_m = log_n;
  pl.p[pl.count++] = make_pass(lb, ci, false, src, mid, a1);
  // Sub-pass 2: DFT over a of rows A*kb + a, stored to row kb + B*ka.
  PassArgs a2 = pass_args(images * width * nb, log_width, lb, img_stride, na * ld, ld, img_stride,
                          ld, nb * ld);
  a2.scale = scale;
  pl.p[pl.count++] = make_pass(la, false, co, mid, dst, a2);
}

// 2D lengths run as two transposed-row passes (2^log_n x 2^log_n images):
// per pass the tile kernel and rows per tile. Measured on B200 for 512 MiB of
// images, forward (ms): N = 1024 0.394 -> 0.381, 2048 0.465 -> 0.397,
// 4096 0.471 -> 0.434 against a row pass plus column passes; up to 512 the
// row pass plus one column pass is faster (more CTAs per SM), and from 8192
// a tile of 4 rows no longer fits one SM's shared memory.
inline TileChoice tile_2d_choice(int log_n) {
  if (log_n == 10) return {TileMode::Prefetch, 8, 5};  // 1024^2: 0.383 -> 0.370 ms with P = 32
  if (log_n == 11) return {TileMode::Prefetch, 8, 0};
  if (log_n == 12) return {TileMode::Tma, 4, 0};
  return {TileMode::None, 0, 0};
}

inline RowsTArgs rows_t_2d_args(int log_n, int64_t batch, float scale) {
  const int64_t n = (int64_t)1 << log_n;
  RowsTArgs b{};
  b.nfft = batch * n;
  b.log_w = log_n;
  b.log_j = 0;
  b.in_o = n * n;
  b.in_c = n;
  b.out_o = n * n;
  b.out_e = n;
  b.scale = scale;
  return b;
}

inline PassPlan plan_2d(int log_n, int64_t batch, bool inv, bool normalize) {
  PassPlan pl;
  const int64_t n = (int64_t)1 << log_n;
  // cpu_2d.rs:56-62: one 1/(n*n) scale computed in float.
  const float scale = (inv && normalize) ? 1.0f / ((float)n * (float)n) : 1.0f;
  const TileChoice tc = tile_2d_choice(log_n);
  if (tc.mode != TileMode::None) {
    // Row FFTs of every image stored transposed into the workspace (the
    // transposed image's rows are the columns), then row FFTs of those stored
    // transposed back: the columns' FFTs in natural layout.
    pl.ws_elems = batch * n * n;
    pl.p[pl.count++] = make_rows_t(log_n, false, PassBuf::In, PassBuf::Ws,
                                   rows_t_2d_args(log_n, batch, 1.0f), inv);
    pl.p[pl.count++] = make_rows_t(log_n, inv, PassBuf::Ws, PassBuf::Out,
                                   rows_t_2d_args(log_n, batch, scale));
    for (int i = 0; i < 2; ++i) {
      pl.p[i].tile = tc.mode;
      pl.p[i].tile_w = tc.w;
      pl.p[i].tile_lp = tc.lp;
    }
    return pl;
  }
  if (log_n <= kMaxOnePassColumnLogN) {
    pl.p[pl.count++] = make_rows(log_n, batch * n, inv, false, 1.0f, PassBuf::In, PassBuf::Out);
    plan_columns(pl, log_n, log_n, n, batch, n * n, false, inv, scale, PassBuf::Out, PassBuf::Out,
                 PassBuf::Out);
    return pl;
  }
  if (cols_l2_width(log_n) > 0) {
    // Fused column kernel (slots in the workspace), then rows in place.
    plan_columns(pl, log_n, log_n, n, batch, n * n, inv, false, 1.0f, PassBuf::In, PassBuf::Ws,
                 PassBuf::Out);
    pl.p[pl.count++] = make_rows(log_n, batch * n, false, inv, scale, PassBuf::Out, PassBuf::Out);
    return pl;
  }
  pl.ws_elems = batch * n * n;
  plan_columns(pl, log_n, log_n, n, batch, n * n, inv, false, 1.0f, PassBuf::In, PassBuf::Out,
               PassBuf::Ws);
  pl.p[pl.count++] = make_rows(log_n, batch * n, false, inv, scale, PassBuf::Ws, PassBuf::Out);
  return pl;
}

}  // namespace ferrum
