/*
 * bmo_kernels.h -- device-pointer kernel layer of libbmo.so.
 *
 * The counterpart of the reference's launch_* functions (utkarshyadav009/
 * bmo_jetson src/bmo.h:348-445): each call takes device buffers and a
 * cudaStream_t (as void*), launches the sm_100a kernels that the decode step
 * uses, and returns 0 or a CUDA error code.  Callers own every buffer,
 * including the scratch the split kernels need (size from the *_scratch_bytes
 * queries).  Calls are asynchronous on `stream`.
 */
#ifndef BMO_KERNELS_H
#define BMO_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#include "bmo_api.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { BMO_PERM_IDENTITY = 0, BMO_PERM_SWIGLU = 1 };

/* Q8_1 quantisation of n floats (n % 32 == 0) into 36-byte blocks
 * (fp16 d, fp16 sum, 32 int8).  Replaces bmo_quantize_row_q8_1_kernel as
 * launched by launch_gemv_q4_0_q8_1 (bmo_cuda_kernels.cu:685-699). */
BMO_API int bmo_k_quantize_q8_1(const float *x_dev, void *out_dev, int n, void *stream);

/* Bytes of the tiled layout of a rows x cols Q4_0 matrix. */
BMO_API size_t bmo_k_q4_0_tiled_bytes(int rows, int cols, int perm, int swiglu_f);
/* ggml Q4_0 row-major blocks -> tiled layout (done once at model load). */
BMO_API int bmo_k_repack_q4_0(const void *ggml_dev, void *tiled_dev, int rows, int cols, int perm, int swiglu_f,
                              void *stream);

/* Scratch bytes bmo_k_gemv_q4_0 needs for a rows x cols matrix. */
BMO_API size_t bmo_k_gemv_scratch_bytes(int rows, int cols, int perm, int swiglu_f);
/* y = W x with the reference's Q4_0 x Q8_1 arithmetic (replaces
 * launch_gemv_q4_0_q8_1, bmo.h:405-412).  W is the tiled layout.
 * gamma_dev != NULL: x is RMS-normalised and scaled by gamma first (fused
 * launch_rmsnorm, bmo.h:358-364).  perm == SWIGLU: y receives
 * silu(gate) * up of length swiglu_f (fused launch_swiglu_split).
 * resid_dev != NULL: y = resid + W x (fused launch_residual_add).
 * q8_out_dev / xn_out_dev (optional) receive the Q8_1 blocks and the
 * normalised fp32 vector the kernel used.  scratch_dev must be zero on the
 * first call and is left zero by every call that returns 0.  x_dev and
 * xn_out_dev are 16-byte aligned; with gamma_dev, cols <= 5120.  grid 0
 * picks the launch (whole row tiles per CTA where that balances); grid > 0
 * runs that many CTAs over an even split of the (row tile, 8-block chunk)
 * units, combining straddled tiles through scratch_dev. */
BMO_API int bmo_k_gemv_q4_0(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f,
                            const float *x_dev, const float *gamma_dev, float eps, const float *resid_dev,
                            float *y_dev, void *q8_out_dev, float *xn_out_dev, void *scratch_dev,
                            size_t scratch_bytes, int grid, void *stream);

/* y = W x computed in the reference kernel's own fp32 order: every row is
 * bit-identical to launch_gemv_q4_0_q8_1 (bmo.h:405-412, kernel
 * bmo_cuda_kernels.cu:560-683) on the same ggml weights and x, and with
 * gamma_dev the RMSNorm is launch_rmsnorm's (bmo.h:358-364) in its own
 * order, the SwiGLU (perm SWIGLU) launch_swiglu_split's with __expf and the
 * residual (resid_dev) launch_residual_add's.  Arguments as in
 * bmo_k_gemv_q4_0; no scratch (each CTA owns whole row tiles); with
 * gamma_dev, cols <= 4096.  status_dev (optional, device int) receives bit
 * 1 if a weight copy did not land within the wait bound. */
BMO_API int bmo_k_gemv_q4_0_ref(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f,
                                const float *x_dev, const float *gamma_dev, float eps, const float *resid_dev,
                                float *y_dev, void *q8_out_dev, float *xn_out_dev, int *status_dev, void *stream);

/* Size of the fixed scratch buffer behind bmo_k_gemv_q4_0_static (4 MiB: every
 * temporal and depformer layer matrix of the 7B Moshi shapes fits; the
 * 32000-row text head does not). */
#define BMO_K_GEMV_STATIC_SCRATCH_BYTES (4u << 20)
/* Returned by bmo_k_gemv_q4_0_static when the matrix needs more scratch than
 * BMO_K_GEMV_STATIC_SCRATCH_BYTES (see bmo_k_gemv_scratch_bytes). */
#define BMO_K_ERR_SCRATCH_TOO_SMALL (-2)

/* bmo_k_gemv_q4_0 for callers that cannot allocate device memory when they
 * run it (a real-time callback that must not block in cudaMalloc, a host
 * framework that owns all allocations, a process under a device-memory cap).
 * No counterpart in the reference.  The split-K scratch is a fixed 4 MiB
 * buffer inside libbmo (held by every GPU that loads the library until
 * exit) instead of scratch_dev; nothing is allocated or freed.  Arguments
 * and results are those of bmo_k_gemv_q4_0.  The buffer is shared by every
 * call on a device and keeps the last call's contents (its counters are
 * cleared on `stream` before each launch), so calls that can overlap on the
 * GPU race: keep them on one stream or order them.  The first call on a
 * device looks up the buffer's address; make it before any stream capture.
 * That address is kept for the life of the process, so after cudaDeviceReset
 * on a device this entry point must not be used on it again.  Arguments are
 * checked before the shared buffer is touched.  Returns
 * BMO_K_ERR_SCRATCH_TOO_SMALL for matrices beyond the buffer. */
BMO_API int bmo_k_gemv_q4_0_static(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f,
                                   const float *x_dev, const float *gamma_dev, float eps, const float *resid_dev,
                                   float *y_dev, void *q8_out_dev, float *xn_out_dev, int grid, void *stream);

/* Scratch bytes bmo_k_batch_gemm_q4_0 needs (on the current device). */
BMO_API size_t bmo_k_batch_gemm_scratch_bytes(int rows, int cols, int perm, int swiglu_f, int n_sess);
/* The batched decode's GEMM (no reference counterpart: the reference decodes
 * one session): for each of n_sess (1..64) sessions, y[s] = W x[s] with the
 * Q4_0 x Q8_1 arithmetic of bmo_k_gemv_q4_0.  x_dev [n_sess][cols], y_dev
 * [n_sess][rows] ([n_sess][swiglu_f] for perm SWIGLU); gamma_dev and
 * resid_dev ([n_sess][rows]) as in bmo_k_gemv_q4_0.  tensor_cores = 1: int8
 * tcgen05 MMA per 32-column block into tensor memory, the reference's
 * half-block terms summed error-free (the rounding of bmo_k_gemv_q4_0 up to
 * rare ties); 2: tensor cores with full-block terms summed in fp32
 * (fp32-accurate, not reproducible bit for bit); 0: CUDA cores with the
 * batch-1 GEMV's rounding.  scratch_dev must be zero on the first call and
 * is left reusable by every call that returns 0. */
BMO_API int bmo_k_batch_gemm_q4_0(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f,
                                  const float *x_dev, const float *gamma_dev, float eps, const float *resid_dev,
                                  float *y_dev, int n_sess, int tensor_cores, void *scratch_dev,
                                  size_t scratch_bytes, void *stream);

/* Appends k, v (fp32, [n_kv_heads][head_dim]) at ring slot pos % n_ctx of
 * `layer`, then attends q over the window (replaces launch_decode_attention,
 * bmo.h:414-428).  Caches are [n_layers][n_kv_heads][n_ctx][head_dim] in
 * fp16 (kv_type 0) or Q4_0 nibble planes with fp16 scale planes (kv_type 1;
 * *_scale_dev).  pos_dev is a device int; n_ctx <= 8192.  No scratch: the
 * window splits of a head exchange partial results through distributed
 * shared memory. */
BMO_API int bmo_k_decode_attention(const float *q_dev, const float *k_dev, const float *v_dev, void *k_cache_dev,
                                   void *v_cache_dev, void *k_scale_dev, void *v_scale_dev, float *out_dev,
                                   int head_dim, int n_heads, int n_kv_heads, int n_ctx, const int *pos_dev,
                                   int layer, int kv_type, void *stream);

/* bmo_k_decode_attention over an fp16 ring, computed in the reference
 * kernel's own fp32 order: bit-identical to launch_decode_attention
 * (bmo.h:414-428, kernel bmo_cuda_kernels.cu:713-848) on the same ring,
 * q, k and v, including the appended slot.  head_dim 64 or 128; n_ctx <= 1024
 * (the reference kernel's own score buffer).  No scratch. */
BMO_API int bmo_k_decode_attention_ref(const float *q_dev, const float *k_dev, const float *v_dev, void *k_cache_dev,
                                       void *v_cache_dev, float *out_dev, int head_dim, int n_heads, int n_kv_heads,
                                       int n_ctx, const int *pos_dev, int layer, void *stream);

/* One tensor-parallel exchange over peer memory (the kernel bmo_init_tp
 * handles run after each split projection): parts[r] is rank r's buffer of n
 * double partial sums (device or peer-mapped pointers, r < size <= 8),
 * flag_out[r] this rank's 64-bit arrival word in rank r's block (ignored for
 * r == rank), flag_in this rank's words (one per source rank), seq a device
 * counter starting at 0 that the exchanges of a group share, status a device
 * int.  Publishes exchange number e into flag_out, waits (at most 2 s) for
 * flag_in[r] >= e from every peer, then y[i] = resid[i] + fl(sum over r in
 * rank order of parts[r][i]).  A wait that runs out sets bit 4 of *status and
 * leaves y untouched; while that bit is set, exchanges return at once.
 * n <= 8192. */
BMO_API int bmo_k_tp_exchange(const double *const *parts, unsigned long long *const *flag_out,
                              const unsigned long long *flag_in_dev, unsigned long long *seq_dev,
                              const float *resid_dev, float *y_dev, int *status_dev, int rank, int size, int n,
                              void *stream);

/* One draw of the daemon's token sampler (sample_token_cpp,
 * bmo_daemon.cpp:147-175) over logits_dev[0, n) on the device: first argmax
 * when top_k <= 0 or temp <= 1e-4, else the top_k logits (ties by lower
 * index), exp(l_i / temp - l_0 / temp) in float and std::discrete_distribution's
 * draw from std::mt19937.  pause_rule 1 adds the daemon's text rule
 * (:758-762): a first argmax of 3 or 0 is kept without a draw.  rng_dev holds
 * 625 words, the generator's 624 state words then its position (624 right
 * after seeding), and is advanced in place.  n <= 32768, min(top_k, n) <=
 * 2048.  One CTA. */
BMO_API int bmo_k_sample_token(const float *logits_dev, int n, float temp, int top_k, int pause_rule,
                               uint32_t *rng_dev, int32_t *out_dev, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BMO_KERNELS_H */
