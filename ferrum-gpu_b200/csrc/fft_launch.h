// Host-side launchers for the sm_100a FFT pass kernels (fft_kernels.cuh).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ferrum {

struct ColsArgs;
struct RowsTArgs;

// Number of CTAs and threads one pass launch uses (for the bench's launch
// count and for tests).
struct LaunchShape {
  int64_t blocks;
  int threads;
  size_t smem_bytes;
};

// Batched contiguous transforms of length 2^log_n (2 <= log_n <= 14). With
// 0 <= log_block < log_n the output is stored blocked: element e of row f at
// (e >> log_block) * nfft * 2^log_block + f * 2^log_block + (e mod 2^log_block).
cudaError_t launch_rows(int log_n, bool conj_in, bool conj_out, const float2* in, float2* out,
                        const float2* tw, int64_t nfft, float scale, cudaStream_t stream,
                        int log_block = -1);

// Copies `nblocks` row-major (rows x bw) blocks stored one after another into a
// row-major (rows x nblocks*bw) matrix: out[r][p*bw + c] = in[p][r][c].
cudaError_t launch_block_gather(const float2* in, float2* out, int64_t nblocks, int64_t rows,
                                int64_t bw, cudaStream_t stream);
LaunchShape rows_shape(int log_n, int64_t nfft);

// Strided column transforms of length 2^log_n (2 <= log_n <= 14); with tw4
// the four-step twiddle is fused into the store (7 <= log_n <= 13).
cudaError_t launch_cols(int log_n, bool conj_in, bool conj_out, bool tw4, const float2* in,
                        float2* out, const float2* tw, const ColsArgs& args, cudaStream_t stream);
LaunchShape cols_shape(int log_n, int64_t nfft);

// Rows of length 2^log_n (8 <= log_n <= 13) stored transposed.
cudaError_t launch_rows_t(int log_n, bool conj_out, const float2* in, float2* out,
                          const float2* tw, const RowsTArgs& args, cudaStream_t stream);
LaunchShape rows_t_shape(int log_n, int64_t nfft);

}  // namespace ferrum
