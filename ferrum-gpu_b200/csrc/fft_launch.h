// Host-side launchers for the sm_100a FFT pass kernels (fft_kernels.cuh).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ferrum {

struct PassArgs;
struct RowsTArgs;
struct ColsL2Args;
struct PeerPtrs;
struct PeerFlags;
enum class TileMode : int;

// Batched contiguous transforms of length 2^log_n (2 <= log_n <= 14). With
// 0 <= log_block < log_n the output is stored blocked: element e of row f at
// (e >> log_block) * R * 2^log_block + f * 2^log_block + (e mod 2^log_block),
// R = block_rows (default nfft).
// With `err_flag` (a device int), N = 16384, an unblocked store and a
// 16-byte aligned input, the persistent prefetching kernel runs; it sets
// *err_flag if a bounded wait expires.
cudaError_t launch_rows(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                        const float2* tw, int64_t nfft, float scale, cudaStream_t stream,
                        int log_block = -1, int* err_flag = nullptr, int64_t block_rows = 0);

// Gathers `nblocks` row-major (rows x bw) blocks, block p starting at
// in + p*in_block_stride, into rows of pitch out_ld:
// out[r*out_ld + p*bw + c] = in[p*in_block_stride + r*bw + c].
cudaError_t launch_block_gather(const float2* in, float2* out, int64_t nblocks, int64_t rows,
                                int64_t bw, int64_t in_block_stride, int64_t out_ld,
                                cudaStream_t stream);

// Strided pass (fft_pass_kernel) of length 2^log_n, 2 <= log_n <= 14; with
// tw the twiddle described by the PassArgs is fused into the store. The
// (conj_in, conj_out, tw) combinations are those pass_flags_supported()
// (passes.h) accepts; others return cudaErrorInvalidValue. With tw,
// args.tw_sfu selects the kernel that takes the twiddle factors from the SFU
// instead of the two-level table.
cudaError_t launch_pass(int log_n, bool conj_in, bool conj_out, bool tw, const float2* in,
                        float2* out, const float2* stage_tw, const PassArgs& args,
                        cudaStream_t stream);

// Both column sub-passes of length 2^log_n (the lengths cols_l2_width() in
// passes.h enables) in one persistent kernel; `ws` holds
// cols_l2_slots(log_n) scratch slots, tw1 / tw2 are the stage tables of the
// sub-pass lengths 2^(log_n - log_n/2) and 2^(log_n/2).
cudaError_t launch_cols_l2(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                           float2* ws, const float2* tw1, const float2* tw2, const ColsL2Args& args,
                           cudaStream_t stream);

// The same strided pass in a persistent tile kernel (launch_tile.cu) of the
// given family, tile width and values per thread (2^log_p; `stage_tw` is the
// stage table for that split, stage_table_p); cudaErrorNotSupported when that kernel is not
// compiled for these arguments or the layout does not meet its conditions
// (the caller then runs launch_pass). `err` is the device flag of the TMA
// kernel's bounded waits.
cudaError_t launch_pass_tile(TileMode mode, int w, int log_p, int log_n, bool conj_in,
                             bool conj_out, bool tw, const float2* in, float2* out,
                             const float2* stage_tw, const PassArgs& args, int* err,
                             cudaStream_t stream);

// Rows of length 2^log_n (4 <= log_n <= 14) stored transposed; not both
// conj_in and conj_out.
cudaError_t launch_rows_t(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                          const float2* tw, const RowsTArgs& args, cudaStream_t stream);
// The same in a persistent tile kernel; cudaErrorNotSupported as for
// launch_pass_tile (the caller then runs launch_rows_t).
cudaError_t launch_rows_t_tile(TileMode mode, int w, int log_p, int log_n, bool conj_in,
                               bool conj_out, const float2* in, float2* out, const float2* tw,
                               const RowsTArgs& args, cudaStream_t stream);

// Distributed 2D over peer memory (dist_kernels.cuh); 4 <= log_n <= 14,
// B = 2^log_b columns per rank. Row FFTs of `nfft` local rows whose output
// element e goes to dst.p[e >> log_b] + f*B + (e mod B):
cudaError_t launch_rows_scatter(int log_n, bool conj_in, const float2* in, const PeerPtrs& dst,
                                const float2* tw, int64_t nfft, int log_b, cudaStream_t stream);
// Row FFTs whose input element e of row f comes from
// src.p[e >> log_b] + f*B + (e mod B); contiguous output rows.
cudaError_t launch_rows_gather(int log_n, bool conj_out, const PeerPtrs& src, float2* out,
                               const float2* tw, int64_t nfft, float scale, int log_b,
                               cudaStream_t stream);
// out[r*out_ld + q*B + c] = src.p[q][r*B + c] (q < nranks, r < rows, c < B).
cudaError_t launch_peer_block_gather(const PeerPtrs& src, float2* out, int nranks, int64_t rows,
                                     int64_t b, int64_t out_ld, cudaStream_t stream);
// Cross-GPU barrier through peer flag words; sets *err after timeout_ns.
cudaError_t launch_dist_barrier(const PeerFlags& flags, int rank, int nranks, uint32_t epoch,
                                uint64_t timeout_ns, int* err, cudaStream_t stream);

// Split (planar) layout, layout_kernels.cuh: batched single-pass transform
// (2 <= log_n <= 14) on separate real / imaginary float arrays, and the
// elementwise helpers over n complex values.
cudaError_t launch_rows_split(int log_n, bool conj_in, bool conj_out, const float* in_re,
                              const float* in_im, float* out_re, float* out_im, const float2* tw,
                              int64_t nfft, float scale, cudaStream_t stream);
cudaError_t launch_cmul_interleaved(const float2* a, const float2* b, float2* out, int64_t n,
                                    cudaStream_t stream);
cudaError_t launch_cmul_split(const float* a_re, const float* a_im, const float* b_re,
                              const float* b_im, float* o_re, float* o_im, int64_t n,
                              cudaStream_t stream);
cudaError_t launch_deinterleave(const float2* in, float* re, float* im, int64_t n,
                                cudaStream_t stream);
cudaError_t launch_interleave(const float* re, const float* im, float2* out, int64_t n,
                              cudaStream_t stream);

}  // namespace ferrum
