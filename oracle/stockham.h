/*
 * CPU ORACLE (test infrastructure only). Restatement of the reference's CPU
 * radix-2 Stockham FFT; see stockham.c for the file:line map.
 * Buffers are interleaved complex64 [re, im] floats, row-major [batch][N].
 * Every function returns 0 on success, -1 on invalid arguments or allocation
 * failure.
 */
#ifndef FERRUM_ORACLE_STOCKHAM_H
#define FERRUM_ORACLE_STOCKHAM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Number of complex entries in the radix-2 stage table: 2^log_n - 1. */
size_t oracle_twiddle_count(uint32_t log_n);
/* Fill `out` (2 * oracle_twiddle_count floats) like twiddles.rs:10-23. */
void oracle_twiddles(uint32_t log_n, float *out);
/* In-place batched 1D C2C (cpu.rs:90-124). dir: +1 forward, -1 inverse. */
int oracle_fft_1d(float *buf, uint32_t log_n, size_t batch, int dir, int normalize);
/* Same arithmetic, lanes split over `threads` POSIX threads. */
int oracle_fft_1d_mt(float *buf, uint32_t log_n, size_t batch, int dir,
                     int normalize, int threads);
/* In-place 2D C2C on `batch` square images (cpu_2d.rs:9-73); the row passes
 * use `threads` threads. */
int oracle_fft_2d(float *buf, uint32_t log_n, size_t batch, int dir,
                  int normalize, int threads);

#ifdef __cplusplus
}
#endif

#endif
