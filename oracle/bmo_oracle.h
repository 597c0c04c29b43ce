/*
 * bmo_oracle.h -- CPU oracle for the Moshi decode step (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the checker, never the product: only tests/, the smoke()
 * entry and bench.py's cpu_baseline / --impl reference legs may load it.
 * It restates, in plain C, the arithmetic of the reference's GPU path
 * (utkarshyadav009/bmo_jetson, src/bmo_cuda_kernels.cu and the graph order in
 * src/bmo_compute.cpp); every function cites the reference lines it follows.
 *
 * Parity pins: the Q4_0 quantiser is checked bit-exact against gguf.quants
 * (the upstream numpy restatement of ggml's quantize_row_q4_0_ref); the Q8_1
 * quantiser, GEMV, RMSNorm, RoPE, SwiGLU and ring attention are checked
 * against golden vectors produced by the reference's own CUDA kernels
 * (compiled unmodified for sm_100a into oracle/_ref) on a B200.
 */
#ifndef BMO_ORACLE_H
#define BMO_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml block_q4_0: fp16 scale + 16 bytes of nibbles; element j is the low
 * nibble of qs[j], element j+16 the high nibble (bmo_cuda_kernels.cu:496-499). */
#pragma pack(push, 1)
typedef struct { uint16_t d; uint8_t qs[16]; } orc_block_q4_0;
/* bmo_block_q8_1: half2 ds = (d, sum) + 32 int8 (bmo_cuda_kernels.cu:501-504). */
typedef struct { uint16_t d; uint16_t s; int8_t qs[32]; } orc_block_q8_1;
#pragma pack(pop)

enum { ORC_KV_F16 = 0, ORC_KV_Q4_0 = 1 };

float    orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);

/* ---- kernel-level restatements ------------------------------------------ */
void orc_quantize_row_q8_1(const float *x, orc_block_q8_1 *y, int n);
void orc_quantize_row_q4_0(const float *x, orc_block_q4_0 *y, int n);
void orc_dequantize_row_q4_0(const orc_block_q4_0 *x, float *y, int n);
void orc_gemv_q4_0_q8_1(const orc_block_q4_0 *W, const orc_block_q8_1 *x,
                        float *y, int rows, int cols);
void orc_rmsnorm(const float *x, const float *w, float eps, int n, float *y);
void orc_rope_interleaved(const float *x, int n_heads, int head_dim, int pos,
                          float theta, float *y);
void orc_swiglu(const float *h, int d_ff, float *y);
/* Ring decode attention over an fp16 cache laid out [layer][head][slot][hd]. */
void orc_decode_attention_f16(const float *q, const float *k, const float *v,
                              uint16_t *k_cache, uint16_t *v_cache, float *out,
                              int head_dim, int n_heads, int n_kv_heads,
                              int n_ctx, int pos, int layer);
/* Same over a Q4_0 cache: per (layer, head, slot) head_dim/32 blocks. */
void orc_decode_attention_q4(const float *q, const float *k, const float *v,
                             orc_block_q4_0 *k_cache, orc_block_q4_0 *v_cache,
                             float *out, int head_dim, int n_heads,
                             int n_kv_heads, int n_ctx, int pos, int layer);
int  orc_argmax(const float *x, int n);
/* The same three kernels restated in the reference kernels' own fp32 order
 * (the GEMV bit-exact; the RMSNorm and attention up to the reference's
 * approximate rsqrtf / CUDA's expf). */
void orc_gemv_q4_0_q8_1_reforder(const orc_block_q4_0 *W, const orc_block_q8_1 *x, float *y, int rows, int cols);
void orc_rmsnorm_reforder(const float *x, const float *w, float eps, int n, float *y);
void orc_decode_attention_f16_reforder(const float *q, const float *k, const float *v, uint16_t *k_cache,
                                       uint16_t *v_cache, float *out, int head_dim, int n_heads, int n_kv_heads,
                                       int n_ctx, int pos, int layer);

/* ---- model-level restatement --------------------------------------------- */
typedef struct orc_model orc_model;

orc_model *orc_model_load(const char *gguf_path, int n_ctx, int kv_type);
void       orc_model_free(orc_model *m);
/* geometry: n_layers, n_embd, n_heads, head_dim, n_codebooks, dep_q,
 * text_vocab, audio_vocab, n_ctx, n_kv_heads, ffn_hidden, dep_dim */
int        orc_model_geometry(const orc_model *m, int32_t *out, int n_out);
void       orc_model_set_threads(orc_model *m, int n_threads);
void       orc_reset(orc_model *m);
void       orc_reset_depth_kv(orc_model *m);
/* Temporal step for one token (bmo_api.cpp:384-511 + bmo_compute.cpp:2124-2739).
 * capture_out receives post-layer residuals of the listed layers. Layers in
 * [layer_begin, layer_end) only; the out_norm/head run when layer_end==n_layers. */
int orc_forward_temporal(orc_model *m, const int32_t *tokens, int K, int pos,
                         float *out_z, float *out_logits,
                         const int32_t *capture, int n_capture,
                         float *capture_out);
int orc_forward_layers(orc_model *m, const float *x_in, int pos,
                       int layer_begin, int layer_end, float *x_out);
int orc_embed(orc_model *m, const int32_t *tokens, int K, float *out);
/* out_norm and text head applied to a given final residual. */
int orc_text_head(orc_model *m, const float *x_final, float *out_z, float *out_logits);
int orc_forward_depth(orc_model *m, int cb, int32_t prev_token,
                      const float *z, float *out_logits);
int orc_forward_depth_cascade_greedy(orc_model *m, int32_t text_token,
                                     const float *z, int32_t *out_tokens);
/* Write fp32 K/V rows (already rotated, as stored) into ring slots
 * [slot0, slot0+n) of one temporal layer; rows are [n][n_kv_heads*head_dim]. */
int orc_kv_import(orc_model *m, int layer, int slot0, int n,
                  const float *k_rows, const float *v_rows);
/* Batched sessions: orc_sessions(m, n) gives the model n independent
 * temporal rings (ring 0 is its existing one, the others start empty);
 * orc_select_session(m, s) points every call above at ring s. */
int orc_sessions(orc_model *m, int n);
int orc_select_session(orc_model *m, int s);
/* Read the temporal cache back as fp32 [n][n_kv_heads*head_dim] (which: 0=K, 1=V). */
int orc_kv_export(orc_model *m, int which, int layer, int slot0, int n,
                  float *out);

/* ---- synthetic model data (the benchmark models' generator, bit for bit) - */
void orc_synth_normal_f32(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, float *out);
void orc_synth_f16(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, uint16_t *out);
void orc_synth_q4_0(uint64_t seed, uint64_t stream, long long rows, long long cols, float sigma, uint8_t *out);

#ifdef __cplusplus
}
#endif
#endif
