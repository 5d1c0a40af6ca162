/*
 * ferrum_fft.h — C ABI of the B200 (sm_100a) FFT path.
 *
 * This is the drop-in boundary for the reference's FFT hot path
 * (alejandro-soto-franco/ferrum-gpu). Every entry point takes plain pointers
 * and sizes, returns a status code, and records a message for
 * ferrum_last_error(). The kernels are hand-written CUDA for sm_100a; there is
 * no CPU fallback: without a usable B200 every compute entry point returns
 * FERRUM_ERR_CUDA.
 *
 * Data layout (crates/ferrum-gpu-fft/src/complex.rs:10-18): complex64
 * interleaved [re, im] float pairs, row-major [batch][N] for 1D and
 * [batch][N][N] for 2D. `direction` is +1 forward / -1 inverse
 * (crates/ferrum-gpu-core/src/dim.rs:49-64). Forward is the unnormalised DFT
 * X[k] = sum_n x[n] exp(-2 pi i n k / N); inverse is conj(FFT(conj(x))),
 * multiplied by 1/N (1D) or 1/N^2 (2D) only when `normalize` is non-zero
 * (crates/ferrum-gpu-fft/src/cpu.rs:106-121, cpu_2d.rs:51-63).
 *
 * Every `*_dev` pointer is device memory on the handle's device; `stream` is a
 * cudaStream_t (NULL = the legacy default stream). Device-pointer calls are
 * asynchronous with respect to the host; the host-pointer (`_host`) calls
 * return when the result is in host memory. `in` may equal `out` (in place).
 */
#ifndef FERRUM_FFT_H
#define FERRUM_FFT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int ferrum_status;
enum {
  FERRUM_OK = 0,
  FERRUM_ERR_INVALID_ARG = 1,
  FERRUM_ERR_CUDA = 2,
  FERRUM_ERR_NCCL = 3,
  FERRUM_ERR_TIMEOUT = 4,
  FERRUM_ERR_ALLOC = 5,
  FERRUM_ERR_UNSUPPORTED = 6
};

enum { FERRUM_FORWARD = 1, FERRUM_INVERSE = -1 };

/* Supported sizes. 1D lengths up to 2^14 run as one HBM pass; 2^15..2^23 run
 * the two-pass four-step and 2^24..2^26 a three-pass split. 2D images are
 * N x N with N up to 2^14. Every call covers at most 2^36 complex values
 * (N * batch, or N * N * batch for 2D); larger requests return
 * FERRUM_ERR_INVALID_ARG. Buffers need 8-byte alignment; the fastest
 * multi-pass and 2D kernels read and write through TMA and need 16-byte
 * aligned buffers (8-byte aligned ones run slower kernels with the same
 * results). */
#define FERRUM_MIN_LOG_N 2
#define FERRUM_MAX_LOG_N_SINGLE_PASS 14
#define FERRUM_MAX_LOG_N_1D 26
#define FERRUM_MAX_LOG_N_2D 14

typedef struct ferrum_device ferrum_device;

/* Library version string ("0.3.0-b200"); replaces `version()`
 * (crates/ferrum-gpu-py/src/lib.rs:419-423). */
const char *ferrum_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char *ferrum_last_error(void);

/* Open CUDA device `ordinal`, upload every twiddle table and return a handle.
 * Replaces `Device::new(ordinal)` (crates/ferrum-gpu-py/src/lib.rs:398-408,
 * crates/ferrum-gpu/src/lib.rs:143-150). Thread-safe. */
ferrum_status ferrum_device_create(int ordinal, ferrum_device **out);
ferrum_status ferrum_device_destroy(ferrum_device *dev);
/* Wait for all work on the device (crates/ferrum-gpu-py/src/lib.rs:410-416). */
ferrum_status ferrum_device_sync(ferrum_device *dev);
/* Ordinal of the device behind the handle. */
ferrum_status ferrum_device_ordinal(const ferrum_device *dev, int *ordinal);

/* Batched 1D C2C on device memory: `batch` transforms of N = 2^log_n.
 * Device-resident form of `fft_1d_c2c_pow2` / `run_fft_flat_with_device`
 * (crates/ferrum-gpu-py/src/lib.rs:445-504, :86-250); log_n in [2, 26].
 * Lengths above 2^14 need a workspace of N*batch*8 bytes, taken from the
 * device's stream-ordered memory pool. A kernel's bounded wait that runs out
 * sets a device flag that ferrum_device_sync reports as FERRUM_ERR_TIMEOUT. */
ferrum_status ferrum_fft_1d_c2c_pow2(ferrum_device *dev, const void *in_dev, void *out_dev,
                                     int log_n, size_t batch, int direction, int normalize,
                                     void *stream);

/* Same, with a caller-owned workspace of at least
 * ferrum_fft_workspace_bytes(log_n, batch, 1) bytes (may be NULL when that is 0). */
ferrum_status ferrum_fft_1d_c2c_pow2_ws(ferrum_device *dev, const void *in_dev, void *out_dev,
                                        int log_n, size_t batch, int direction, int normalize,
                                        void *workspace_dev, size_t workspace_bytes,
                                        void *stream);

/* Allocation-free form of ferrum_fft_1d_c2c_pow2 (no counterpart in the
 * reference). For callers that cannot allocate device memory at call time:
 * applications whose memory belongs to their own allocator or to a pool
 * reserved at start-up, and latency-critical loops where an allocation may
 * block in the driver. Lengths above 2^14 use a 32 MiB file-scope __device__
 * scratch array instead of a workspace, so N * batch must be <= 2^22 there
 * (larger calls return FERRUM_ERR_INVALID_ARG); every GPU that loads the
 * library keeps that array until exit. The array is shared by all calls on a
 * device: calls that overlap on the GPU race, and none needs it zeroed. The
 * first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) and caches it; make that first call on a device
 * before any stream capture. */
ferrum_status ferrum_fft_1d_c2c_pow2_noalloc(ferrum_device *dev, const void *in_dev,
                                             void *out_dev, int log_n, size_t batch,
                                             int direction, int normalize, void *stream);

/* Batched 2D C2C on device memory: `batch` images of N x N, N = 2^log_n,
 * log_n in [2, 14]. Replaces `fft_2d_c2c_pow2` / `run_fft_2d_flat`
 * (crates/ferrum-gpu-py/src/lib.rs:527-588, :273-375); the reference's 2D takes
 * one image and log_n in [4, 12]. Up to N = 512 a row pass and a column pass
 * in place; N = 1024..4096 two transposed-row passes through an image-sized
 * workspace; N >= 8192 two column sub-passes and a row pass (workspace from
 * the device's stream-ordered pool). */
ferrum_status ferrum_fft_2d_c2c_pow2(ferrum_device *dev, const void *in_dev, void *out_dev,
                                     int log_n, size_t batch, int direction, int normalize,
                                     void *stream);

/* Host-memory forms: copy in, transform, copy out, return when done. Inputs
 * are processed in chunks so that copies overlap the kernels; pinned host
 * buffers give full PCIe bandwidth. These are the entry points behind the
 * Python `fft_1d_c2c_pow2` / `fft_2d_c2c_pow2` (lib.rs:445-588). */
ferrum_status ferrum_fft_1d_c2c_pow2_host(ferrum_device *dev, const void *in_host,
                                          void *out_host, int log_n, size_t batch,
                                          int direction, int normalize);
ferrum_status ferrum_fft_2d_c2c_pow2_host(ferrum_device *dev, const void *in_host,
                                          void *out_host, int log_n, size_t batch,
                                          int direction, int normalize);

/* ---------------------------------------------------------------------------
 * Split (planar) complex layout: real and imaginary parts in two float
 * arrays. Replaces the reference's split twins and layout helpers
 * (crates/ferrum-gpu-fft-kernels/src/kernels_body.rs:508-626
 * fft_c2c_1024_split; 1614-1672 cmul_interleaved, cmul_split, deinterleave,
 * interleave), which it only launches from its layout benchmarks.
 */
/* Batched 1D transform on [batch][N] float arrays, single pass:
 * 2 <= log_n <= 14. Same results as ferrum_fft_1d_c2c_pow2 on the
 * interleaved data. out_re / out_im may be in_re / in_im (in place). */
ferrum_status ferrum_fft_1d_c2c_pow2_split(ferrum_device *dev, const float *in_re,
                                           const float *in_im, float *out_re, float *out_im,
                                           int log_n, size_t batch, int direction, int normalize,
                                           void *stream);
/* out[i] = a[i] * b[i] for n interleaved complex values (products and sums
 * rounded separately, as the reference's kernel writes them). */
ferrum_status ferrum_cmul_interleaved(ferrum_device *dev, const void *a, const void *b, void *out,
                                      size_t n, void *stream);
/* The same on split arrays. */
ferrum_status ferrum_cmul_split(ferrum_device *dev, const float *a_re, const float *a_im,
                                const float *b_re, const float *b_im, float *out_re,
                                float *out_im, size_t n, void *stream);
/* n interleaved complex values to two float arrays, and back. */
ferrum_status ferrum_deinterleave(ferrum_device *dev, const void *in, float *out_re,
                                  float *out_im, size_t n, void *stream);
ferrum_status ferrum_interleave(ferrum_device *dev, const float *re, const float *im, void *out,
                                size_t n, void *stream);

/* ---------------------------------------------------------------------------
 * Kernel-module substrate: the operations of the reference's backend contract
 * (crates/ferrum-gpu-core/src/backend.rs:12-77 alloc_zeros, copy_h2d,
 * copy_d2h, load_module, get_kernel, launch, sync_stream) for callers that
 * bring their own kernels, as its vector-add examples do.
 */
typedef struct ferrum_module ferrum_module;
/* `bytes` of device memory, zero-filled; release with ferrum_buffer_free. */
ferrum_status ferrum_buffer_alloc_zeros(ferrum_device *dev, size_t bytes, void **out);
ferrum_status ferrum_buffer_free(ferrum_device *dev, void *buf);
/* Synchronous copies between host and device memory. */
ferrum_status ferrum_copy_h2d(ferrum_device *dev, void *dst_dev, const void *src_host, size_t bytes);
ferrum_status ferrum_copy_d2h(ferrum_device *dev, void *dst_host, const void *src_dev, size_t bytes);
/* Loads a module image: NUL-terminated PTX text (compiled for the device
 * when loaded) or a cubin / fatbin image. */
ferrum_status ferrum_module_load(ferrum_device *dev, const void *image, ferrum_module **out);
ferrum_status ferrum_module_unload(ferrum_module *module);
/* Kernel `name` (its mangled name for C++ kernels) of a loaded module; the
 * handle stays valid until the module is unloaded. */
ferrum_status ferrum_module_kernel(ferrum_module *module, const char *name, void **kernel_out);
/* Launches `kernel` with grid / block dimensions (x, y, z), dynamic shared
 * bytes and `args` (an array of pointers to each argument value), on
 * `stream` (NULL: the default stream). Asynchronous. */
ferrum_status ferrum_launch(ferrum_device *dev, void *kernel, const unsigned grid[3],
                            const unsigned block[3], unsigned shared_bytes, void **args,
                            void *stream);
/* Waits for all work on `stream`. */
ferrum_status ferrum_stream_sync(ferrum_device *dev, void *stream);

/* Workspace bytes a call needs: kind 1 = 1D, kind 2 = 2D. */
ferrum_status ferrum_fft_workspace_bytes(int log_n, size_t batch, int kind, size_t *bytes);

/* Number of kernel launches one device-pointer call makes (kind 1 = 1D,
 * kind 2 = 2D): 1 for single-pass 1D, 2 for four-step 1D and for 2D. */
ferrum_status ferrum_fft_launch_count(int log_n, size_t batch, int kind, int *launches);

/* ---------------------------------------------------------------------------
 * Distributed 2D (one process per GPU over NVLink). New in this build: the
 * reference is single-GPU. A single N x N image is split into row slabs of
 * N/P rows; each rank holds its slab row-major. On up to 8 ranks whose GPUs
 * can map each other's memory (CUDA IPC) the exchange is fused into the FFT
 * kernels: the row-FFT kernel stores each (N/P) x (N/P) block directly into
 * the destination rank's receive slab, the column FFTs run on the received
 * column slab, and the return to row slabs is a row-FFT (or copy) kernel
 * that loads from the ranks' slabs. Otherwise (or with FERRUM_DIST_P2P=0 in
 * the environment of any rank) an NCCL all-to-all moves the blocks.
 */
typedef struct ferrum_dist_ctx ferrum_dist_ctx;

/* Bytes of the opaque id rank 0 creates and every rank passes to init. */
#define FERRUM_DIST_ID_BYTES 128
ferrum_status ferrum_dist_get_unique_id(unsigned char id_out[FERRUM_DIST_ID_BYTES]);
/* Collective: every rank calls it with the same id. `timeout_ms` bounds
 * communicator set-up and every later collective wait. */
ferrum_status ferrum_dist_init(ferrum_device *dev, const unsigned char id[FERRUM_DIST_ID_BYTES],
                               int nranks, int rank, int timeout_ms, ferrum_dist_ctx **out);
ferrum_status ferrum_dist_destroy(ferrum_dist_ctx *ctx);
ferrum_status ferrum_dist_world(const ferrum_dist_ctx *ctx, int *nranks, int *rank);
/* Workspace bytes per rank for an N x N distributed transform. */
ferrum_status ferrum_dist_workspace_bytes(const ferrum_dist_ctx *ctx, int log_n, size_t *bytes);
/* Collective: in/out are this rank's (N/P) x N row slab (row-major, device
 * memory, 16-byte aligned; in == out allowed). Every rank calls it with the
 * same arguments, on a stream of its own device. Enqueues and returns; the
 * workspace (ferrum_dist_workspace_bytes) comes from the device's pool. */
ferrum_status ferrum_fft_2d_c2c_pow2_dist(ferrum_dist_ctx *ctx, const void *in_slab_dev,
                                          void *out_slab_dev, int log_n, int direction,
                                          int normalize, void *stream);
/* Layout-aware form: FERRUM_DIST_ROW_SLAB = rank r holds rows [rB, rB+B)
 * (B x N, row-major); FERRUM_DIST_COL_SLAB = rank r holds columns [rB, rB+B)
 * of all rows (N x B, row-major). Row -> column needs one all-to-all (the
 * usual forward), column -> row one (its inverse), row -> row two.
 * Column -> column is not supported. */
enum { FERRUM_DIST_ROW_SLAB = 0, FERRUM_DIST_COL_SLAB = 1 };
ferrum_status ferrum_fft_2d_c2c_pow2_dist_layout(ferrum_dist_ctx *ctx, const void *in_dev,
                                                 void *out_dev, int log_n, int direction,
                                                 int normalize, int in_layout, int out_layout,
                                                 void *stream);
/* Waits for `stream` with the context's timeout. On timeout, an NCCL error or
 * a peer barrier that timed out on the device (FERRUM_ERR_TIMEOUT) the
 * communicator is aborted and the context becomes unusable. */
ferrum_status ferrum_dist_sync(ferrum_dist_ctx *ctx, void *stream);
/* Collective, stream ordered: no rank's work after it on `stream` starts
 * before every rank's work before it has finished. On the peer-memory path a
 * one-CTA kernel on flag words in peer memory whose wait is bounded by the
 * context's timeout (expiry is reported by ferrum_dist_sync); on the NCCL
 * path a 4-byte all-gather. No counterpart in the reference. */
ferrum_status ferrum_dist_barrier(ferrum_dist_ctx *ctx, void *stream);
/* Which data path the context uses: 1 = peer memory (CUDA IPC over NVLink,
 * exchange fused into the FFT kernels), 0 = NCCL send/recv, -1 = not decided
 * yet (it is decided collectively by the first transform), -2 = NULL ctx. */
int ferrum_dist_peer_path(const ferrum_dist_ctx *ctx);
/* Host-side abort, for a rank that learns by its own means (a process group,
 * a heartbeat) that another rank has failed: aborts the communicator without
 * waiting for any rank; the context is unusable afterwards and
 * ferrum_dist_destroy then only releases local resources (a peer-memory slab
 * other ranks may still map is left allocated, not freed under them). */
ferrum_status ferrum_dist_abort(ferrum_dist_ctx *ctx);
/* Replaces the timeout that bounds later host waits and device-side peer
 * barriers (set-up often needs a longer bound than the steady state). */
ferrum_status ferrum_dist_set_timeout(ferrum_dist_ctx *ctx, int timeout_ms);
/* FERRUM_OK when (log_n, nranks) is a supported distributed shape: nranks a
 * power of two, log_n in [4, 14], N / nranks >= 2. */
ferrum_status ferrum_dist_check(int log_n, int nranks);

#ifdef __cplusplus
}
#endif

#endif /* FERRUM_FFT_H */
