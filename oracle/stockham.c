/*
 * CPU ORACLE — test infrastructure only, never part of the product path.
 *
 * A plain-C restatement of the reference's CPU radix-2 Stockham FFT
 * (alejandro-soto-franco/ferrum-gpu, crate `ferrum-gpu-fft`). Only the test
 * suite, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference`
 * legs of `bench.py` load this library, as the checker and the timed CPU
 * baseline. The CUDA product path never calls it.
 *
 * Arithmetic follows the reference operation by operation, in float32:
 *   - twiddle table: crates/ferrum-gpu-fft/src/twiddles.rs:10-23
 *       scale = -2*PI / n_stage in f32, theta = scale * k in f32,
 *       (cosf(theta), sinf(theta)); stages descending (largest first).
 *   - stage offsets: crates/ferrum-gpu-fft/src/cpu.rs:15-23
 *   - butterfly:     crates/ferrum-gpu-fft/src/cpu.rs:30-45
 *       a = src[j*m/2 + k], b = src[j*m/2 + k + N/2], wb = w*b,
 *       dst[j*m + k] = a + wb, dst[j*m + k + m/2] = a - wb
 *   - complex mul:   crates/ferrum-gpu-fft/src/complex.rs:33-38
 *       (w.re*b.re - w.im*b.im, w.re*b.im + w.im*b.re), no fused multiply-add
 *   - lane driver:   crates/ferrum-gpu-fft/src/cpu.rs:51-81 (ping-pong, copy back
 *       when log_n is odd) and :90-124 (inverse = conj(FFT(conj x)), optional
 *       multiply by 1.0f/N)
 *   - 2D:            crates/ferrum-gpu-fft/src/cpu_2d.rs:9-73 (row pass, in-place
 *       square transpose, row pass, transpose back, conj + one 1/(N*N) scale)
 * The reference asserts log_n <= 12 (plan.rs:58,111); the algorithm itself has
 * no such limit, so this restatement accepts 1 <= log_n <= 26.
 *
 * Build with -ffp-contract=off so that a*b - c*d is not contracted into an FMA:
 * rustc never contracts, and bit-for-bit agreement with the Rust code depends
 * on it.
 */
#include "stockham.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* core::f32::consts::PI */
static const float PI_F32 = 3.14159265358979323846264338327950288f;

size_t oracle_twiddle_count(uint32_t log_n) {
    return ((size_t)1 << log_n) - 1;
}

/* twiddles.rs:10-23 */
void oracle_twiddles(uint32_t log_n, float *out) {
    size_t idx = 0;
    for (uint32_t stage = log_n; stage >= 1; --stage) {
        uint64_t n_stage = (uint64_t)1 << stage;
        size_t half = (size_t)(n_stage / 2);
        float scale = -2.0f * PI_F32 / (float)n_stage;
        for (size_t k = 0; k < half; ++k) {
            float theta = scale * (float)k;
            out[2 * idx] = cosf(theta);
            out[2 * idx + 1] = sinf(theta);
            ++idx;
        }
    }
}

/* cpu.rs:15-23: offs[s] = start of stage s's block (s in 1..=log_n). */
static void stage_offsets(uint32_t log_n, size_t *offs) {
    size_t off = 0;
    offs[0] = 0;
    for (uint32_t s = log_n; s >= 1; --s) {
        offs[s] = off;
        off += (size_t)1 << (s - 1);
    }
}

/* cpu.rs:30-45 */
static void stockham_stage(const float *src, float *dst, size_t n, uint32_t s,
                           const float *tw) {
    size_t m = (size_t)1 << s;
    size_t m_half = (size_t)1 << (s - 1);
    size_t l = n / m;
    size_t half_n = n / 2;
    for (size_t j = 0; j < l; ++j) {
        for (size_t k = 0; k < m_half; ++k) {
            float wr = tw[2 * k], wi = tw[2 * k + 1];
            size_t ia = j * m_half + k;
            size_t ib = ia + half_n;
            float ar = src[2 * ia], ai = src[2 * ia + 1];
            float br = src[2 * ib], bi = src[2 * ib + 1];
            /* complex.rs:33-38, self = w, other = b */
            float wbr = wr * br - wi * bi;
            float wbi = wr * bi + wi * br;
            size_t o0 = j * m + k;
            size_t o1 = o0 + m_half;
            dst[2 * o0] = ar + wbr;
            dst[2 * o0 + 1] = ai + wbi;
            dst[2 * o1] = ar - wbr;
            dst[2 * o1 + 1] = ai - wbi;
        }
    }
}

/* cpu.rs:51-81 */
static void forward_lane(float *buf, float *scratch, uint32_t log_n,
                         const float *tw, const size_t *offs) {
    size_t n = (size_t)1 << log_n;
    int from_buf_to_scratch = 1;
    for (uint32_t s = 1; s <= log_n; ++s) {
        const float *tws = tw + 2 * offs[s];
        if (from_buf_to_scratch)
            stockham_stage(buf, scratch, n, s, tws);
        else
            stockham_stage(scratch, buf, n, s, tws);
        from_buf_to_scratch = !from_buf_to_scratch;
    }
    if (log_n % 2 == 1) memcpy(buf, scratch, n * 2 * sizeof(float));
}

static void conj_lane(float *lane, size_t n) {
    for (size_t i = 0; i < n; ++i) lane[2 * i + 1] = -lane[2 * i + 1];
}

/* cpu.rs:90-124, one lane */
static void execute_lane(float *lane, float *scratch, uint32_t log_n, int dir,
                         int normalize, const float *tw, const size_t *offs) {
    size_t n = (size_t)1 << log_n;
    if (dir >= 0) {
        forward_lane(lane, scratch, log_n, tw, offs);
        return;
    }
    conj_lane(lane, n);
    forward_lane(lane, scratch, log_n, tw, offs);
    conj_lane(lane, n);
    if (normalize) {
        float inv_n = 1.0f / (float)n;
        for (size_t i = 0; i < 2 * n; ++i) lane[i] *= inv_n;
    }
}

int oracle_fft_1d(float *buf, uint32_t log_n, size_t batch, int dir,
                  int normalize) {
    return oracle_fft_1d_mt(buf, log_n, batch, dir, normalize, 1);
}

typedef struct {
    float *buf;
    uint32_t log_n;
    size_t lane_begin, lane_end;
    int dir, normalize;
    const float *tw;
    const size_t *offs;
    int status;
} lane_job;

static void *lane_worker(void *arg) {
    lane_job *job = (lane_job *)arg;
    size_t n = (size_t)1 << job->log_n;
    float *scratch = (float *)malloc(n * 2 * sizeof(float));
    if (!scratch) {
        job->status = -1;
        return NULL;
    }
    for (size_t lane = job->lane_begin; lane < job->lane_end; ++lane)
        execute_lane(job->buf + 2 * n * lane, scratch, job->log_n, job->dir,
                     job->normalize, job->tw, job->offs);
    free(scratch);
    job->status = 0;
    return NULL;
}

/* Lane-parallel form of cpu.rs:90-124: the same per-lane arithmetic, lanes
 * split into contiguous ranges over `threads` POSIX threads. Results are
 * identical to the single-threaded call. */
int oracle_fft_1d_mt(float *buf, uint32_t log_n, size_t batch, int dir,
                     int normalize, int threads) {
    if (log_n < 1 || log_n > 26 || batch == 0 || buf == NULL) return -1;
    size_t offs[27];
    stage_offsets(log_n, offs);
    float *tw = (float *)malloc(oracle_twiddle_count(log_n) * 2 * sizeof(float));
    if (!tw) return -1;
    oracle_twiddles(log_n, tw);
    if (threads < 1) threads = 1;
    if ((size_t)threads > batch) threads = (int)batch;
    lane_job *jobs = (lane_job *)calloc((size_t)threads, sizeof(lane_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int rc = 0;
    if (!jobs || !tids) {
        rc = -1;
        goto done;
    }
    for (int t = 0; t < threads; ++t) {
        jobs[t].buf = buf;
        jobs[t].log_n = log_n;
        jobs[t].lane_begin = batch * (size_t)t / (size_t)threads;
        jobs[t].lane_end = batch * (size_t)(t + 1) / (size_t)threads;
        jobs[t].dir = dir;
        jobs[t].normalize = normalize;
        jobs[t].tw = tw;
        jobs[t].offs = offs;
        jobs[t].status = -1;
    }
    if (threads == 1) {
        lane_worker(&jobs[0]);
    } else {
        for (int t = 0; t < threads; ++t)
            pthread_create(&tids[t], NULL, lane_worker, &jobs[t]);
        for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
    }
    for (int t = 0; t < threads; ++t)
        if (jobs[t].status != 0) rc = -1;
done:
    free(jobs);
    free(tids);
    free(tw);
    return rc;
}

/* cpu_2d.rs:67-73 */
static void transpose_square(float *buf, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        for (size_t j = i + 1; j < n; ++j) {
            size_t a = i * n + j, b = j * n + i;
            float tr = buf[2 * a], ti = buf[2 * a + 1];
            buf[2 * a] = buf[2 * b];
            buf[2 * a + 1] = buf[2 * b + 1];
            buf[2 * b] = tr;
            buf[2 * b + 1] = ti;
        }
    }
}

/* cpu_2d.rs:9-64 for one (N, N) image. */
static int fft_2d_image(float *buf, uint32_t log_n, int dir, int normalize,
                        int threads) {
    size_t n = (size_t)1 << log_n;
    if (dir < 0) conj_lane(buf, n * n);
    int rc = oracle_fft_1d_mt(buf, log_n, n, +1, 0, threads);
    if (rc) return rc;
    transpose_square(buf, n);
    rc = oracle_fft_1d_mt(buf, log_n, n, +1, 0, threads);
    if (rc) return rc;
    transpose_square(buf, n);
    if (dir < 0) {
        conj_lane(buf, n * n);
        if (normalize) {
            float scale = 1.0f / ((float)n * (float)n);
            for (size_t i = 0; i < 2 * n * n; ++i) buf[i] *= scale;
        }
    }
    return 0;
}

int oracle_fft_2d(float *buf, uint32_t log_n, size_t batch, int dir,
                  int normalize, int threads) {
    if (log_n < 1 || log_n > 14 || batch == 0 || buf == NULL) return -1;
    size_t n = (size_t)1 << log_n;
    for (size_t b = 0; b < batch; ++b) {
        int rc = fft_2d_image(buf + 2 * n * n * b, log_n, dir, normalize, threads);
        if (rc) return rc;
    }
    return 0;
}
