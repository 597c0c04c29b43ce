// launch.h -- host-side launchers of the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "layout.h"

namespace bmo {

// GEMV, exact-reduction order (kernels/gemv_q4.cu).  `grid` CTAs split the
// (tile, chunk) units; `pdl` enables programmatic dependent launch on the stream.
cudaError_t launch_gemv(const GemvArgs &a, int prologue, int epilogue, int grid, cudaStream_t s, bool pdl);
size_t gemv_smem_bytes();
// Argument rules of the kernel-layer GEMV (kernel_api.cu) other than its scratch.
bool gemv_kernel_args_ok(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f, const float *x_dev,
                         const float *gamma_dev, const float *y_dev, const float *xn_out_dev);
int gemv_max_tiles_per_cta();
int gemv_max_nbx();
int gemv_max_norm_cols();
// GEMV in the reference kernel's fp32 order (kernels/gemv_ref.cu): `grid`
// CTAs (at most the tile count, gemv_ref_grid) each own whole row tiles.
cudaError_t launch_gemv_ref(const GemvArgs &a, int prologue, int epilogue, int grid, cudaStream_t s, bool pdl);
int gemv_ref_grid(const QMatDesc &m, int sms);
size_t gemv_ref_smem_bytes();
int gemv_ref_max_norm_cols();
// Grid and split for a matrix on a device with `sms` SMs: whole row tiles per
// CTA unless that leaves the busiest CTA much more work than an even split.
struct GemvPlan {
    int grid;
    int tile_aligned;
};
GemvPlan plan_gemv(const QMatDesc &m, int sms);

// Ring decode attention (kernels/attention.cu): one cluster of `splits` CTAs per head.
// n_sess > 1: grid z runs that many sessions (AttnArgs strides).
cudaError_t launch_attention(const AttnArgs &a, int head_dim, int splits, cudaStream_t s, bool pdl, int n_sess = 1);
int attn_splits_for(int n_ctx);
int attn_max_ctx();
// Decode attention over an fp16 ring in the reference kernel's fp32 order
// (kernels/attention_ref.cu): split = a cluster of 8 CTAs per head (rings up
// to 1024 slots), else one CTA per head (rings up to 64 slots).
cudaError_t launch_attention_ref(const AttnArgs &a, int head_dim, bool split, cudaStream_t s, bool pdl);
bool attn_ref_supported(int head_dim, int n_ctx, bool split);
int attn_ref_max_ctx();

// The depformer's greedy cascade as one launch on a cluster of `heads` CTAs
// (kernels/dep_cascade.cu), reference fp32 order.
cudaError_t launch_dep_cascade(const DepCascadeArgs &a, size_t smem_bytes, cudaStream_t s, bool pdl);
size_t dep_cascade_smem_bytes(int dim, int ffn, int n_embd, int n_layers, int n_ctx);
int dep_cascade_configure(int heads, size_t smem_bytes);  // resident clusters on the current device (0: cannot run)
int dep_cascade_part_slots();
int dep_cascade_max_cluster();
int dep_cascade_max_local_tiles();
int dep_cascade_head_dim();
// The same cascade as one cooperative launch over `grid` CTAs (one per SM)
// exchanging op outputs through epoch-tagged words in global memory
// (kernels/dep_cascade_ll.cu).
cudaError_t launch_dep_cascade_ll(const DepCascadeArgs &a, int grid, size_t smem_bytes, cudaStream_t s);
size_t dep_cascade_ll_smem_bytes(int dim, int ffn, int n_embd, int n_layers, int n_ctx);
int dep_cascade_ll_configure(size_t smem_bytes, int sms);  // CTAs that can run co-resident (0: cannot run)
int dep_cascade_ll_items();
int dep_cascade_ll_max_local_tiles();
int dep_cascade_ll_max_in();
int dep_cascade_ll_head_dim();
int dep_cascade_ll_phases();
int dep_cascade_ll_max_grid();
int dep_cascade_ll_max_ops();

// Batched sessions (kernels/batch.cu).  Stage: per-session RMSNorm + Q8_1
// into the block-major layout (and the embedding token); GEMM: the skinny
// Q4_0 x Q8_1 product of all sessions with a fused epilogue, `grid` CTAs
// owning whole row tiles (at most W.n_tiles).
cudaError_t launch_batch_stage(const BatchStageArgs &a, cudaStream_t s);
cudaError_t launch_batch_gemm(const BatchGemmArgs &a, int epilogue, int grid, cudaStream_t s);
size_t batch_gemm_smem_bytes();
int batch_gemm_grid(const QMatDesc &m, int sms);
// Tensor-core form of the batched GEMM (kernels/batch_mma.cu): one CTA per SM
// (at most the unit count), stream-K over (128-row block, chunk) units.
// exact: the reference's half-block terms summed error-free (the batch-1
// rounding); otherwise full-block terms summed in fp32.  Split row blocks
// need a.ws (batch_mma_ws_floats) and a.cnt (one zeroed int per 128-row
// block) with a.max_contrib >= batch_mma_max_contrib.
cudaError_t launch_batch_mma(const BatchGemmArgs &a, int epilogue, int sms, bool exact, cudaStream_t s);
int batch_mma_grid(const QMatDesc &m, int sms);
int batch_mma_max_contrib(const QMatDesc &m, int sms);
size_t batch_mma_ws_floats(const QMatDesc &m, int sms);
size_t batch_mma_smem_bytes();
// Embedding sums out[s][n_embd] of the first n_sess rows of `in` and their
// RoPE tables rope[s][head_dim / 2].
cudaError_t launch_batch_embed(const EmbTable *tables, int n_tables, const BatchIn *in, int n_embd, float *out,
                               int n_sess, float theta, int head_dim, float2 *rope, cudaStream_t s);
// Fills `in` from device arrays sess[n] (null: 0..n-1), tokens[n][K], pos[n].
cudaError_t launch_batch_set_inputs(BatchIn *in, const int *sess, const int *tokens, int K, const int *pos, int n,
                                    cudaStream_t s);
// Greedy token of each session: first maximum of pairs[s * pairs_stride + 0..n_pairs).
cudaError_t launch_batch_finalize(const float2 *pairs, int pairs_stride, int n_pairs, int *out, int out_stride,
                                  int n_sess, cudaStream_t s);

// Tensor parallel: y = resid + (float)part (kernels/misc.cu).
cudaError_t launch_tp_resid(const double *part, const float *resid, float *y, int n, cudaStream_t s);
cudaError_t launch_tp_exchange(const TpExchangeArgs &a, cudaStream_t s, bool pdl);

// Frame-start embedding sum + RoPE table (kernels/misc.cu); ref: the table
// by the reference's intrinsics (__powf, __sincosf).
cudaError_t launch_embed(const EmbTable *tables, int n_tables, const int *tokens, const int *n_tok_dev, int n_embd,
                         float *out, const int *pos, float theta, int head_dim, float2 *rope_cs, bool ref,
                         cudaStream_t s);
cudaError_t launch_set_frame(int *fin_tokens, int *fin_n_tok, int *fin_pos, const int *tokens, int K, int pos,
                             cudaStream_t s);
cudaError_t launch_set_int(int *dst, int v, cudaStream_t s);
cudaError_t launch_finalize_token(const float2 *pairs, int n, int *out, cudaStream_t s, bool pdl);
// Sets the shared-memory opt-in of every kernel variant on the current device.
// The caller's frame loop on the device (kernels/loop.cu).
cudaError_t launch_loop_begin(LoopState *st, const LoopConfig &cfg, int *tokens, int *n_tok, int *pos,
                              cudaStream_t s);
cudaError_t launch_loop_end(LoopState *st, cudaStream_t s);
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s, bool pdl);

cudaError_t configure_kernels();
cudaError_t launch_repack_q4_0(const void *src, void *dst, int rows, int cols, const QMatDesc &m, cudaStream_t s);
cudaError_t launch_quantize_q8_1(const float *x, void *out, int n, cudaStream_t s);

}  // namespace bmo
