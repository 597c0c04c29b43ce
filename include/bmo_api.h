/*
 * bmo_api.h -- C ABI of libbmo.so, the B200 decode-step engine.
 *
 * Drop-in for utkarshyadav009/bmo_jetson src/bmo_api.h: every entry point
 * below has the reference's name, signature, return codes and threading
 * rules, so bmo_daemon, bmo_engine and ctypes callers (bmo_engine.py) link
 * and run unchanged.  Each declaration cites the reference line it replaces.
 * Extensions that have no counterpart in the reference live in bmo_ext.h.
 */
#ifndef BMO_API_H
#define BMO_API_H

#include <stdint.h>

#if defined(_WIN32)
#if defined(BMO_BUILDING_SHARED)
#define BMO_API __declspec(dllexport)
#else
#define BMO_API __declspec(dllimport)
#endif
#elif defined(__GNUC__) || defined(__clang__)
#define BMO_API __attribute__((visibility("default")))
#else
#define BMO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque engine handle (reference bmo_api.h:33). */
typedef struct bmo_handle bmo_handle_t;

/* Loads a GGUF model into HBM of the current CUDA device (or BMO_DEVICE) and
 * allocates an n_ctx-slot KV ring (n_ctx <= 0 means 2048).  Returns NULL on
 * failure with the reason on stderr.  Replaces bmo_api.h:39. */
BMO_API bmo_handle_t *bmo_init(const char *gguf_path, int n_ctx);

/* Releases everything the handle owns; NULL-safe (bmo_api.h:43). */
BMO_API void bmo_free(bmo_handle_t *h);

/* pos := 0, temporal KV ring zeroed, error cleared (bmo_api.h:47). */
BMO_API void bmo_reset(bmo_handle_t *h);

/* Geometry getters; 0 for a NULL handle (bmo_api.h:50-57). */
BMO_API int bmo_get_n_layers(bmo_handle_t *h);
BMO_API int bmo_get_n_embd(bmo_handle_t *h);
BMO_API int bmo_get_n_codebooks(bmo_handle_t *h);
BMO_API int bmo_get_dep_q(bmo_handle_t *h);
BMO_API int bmo_get_text_vocab(bmo_handle_t *h);
BMO_API int bmo_get_audio_vocab(bmo_handle_t *h);
BMO_API int bmo_get_n_attn_heads(bmo_handle_t *h);
BMO_API int bmo_get_head_dim(bmo_handle_t *h);

/* Copies ring slots [t_start, t_start+n_positions) of one layer's K cache as
 * float32 [position][head][dim].  Returns the count written, -1 bad
 * arguments, -2 buffer too small, -3 range (bmo_api.h:61). */
BMO_API int bmo_copy_k_cache_f32(bmo_handle_t *h, int layer, int t_start, int n_positions, float *out,
                                 int max_floats);

/* Captures the per-frame CUDA graphs; 0 on success (bmo_api.h:71-72). */
BMO_API int bmo_capture_graphs(bmo_handle_t *h);
BMO_API int bmo_has_cuda_graphs(bmo_handle_t *h);

/* One temporal decode step: embeds input_tokens[0..num_codebooks), runs all
 * layers at absolute position pos, writes the final-normed hidden state
 * (n_embd floats) and the text logits (text_vocab floats).  rc 1 null
 * argument, 2 bad num_codebooks/pos, 3 missing output head, 9 device error
 * (bmo_api.h:86). */
BMO_API int bmo_forward_temporal(bmo_handle_t *h, const int32_t *input_tokens, int num_codebooks, int pos,
                                 float *out_transformer, float *out_text_logits);

/* As above, plus copies of the post-layer residual stream of the listed
 * layers into capture_out (n_capture_layers * n_embd floats); rc 6 for a
 * layer index outside the model (bmo_api.h:99). */
BMO_API int bmo_forward_temporal2(bmo_handle_t *h, const int32_t *input_tokens, int num_codebooks, int pos,
                                  float *out_transformer, float *out_text_logits, const int32_t *capture_layers,
                                  int n_capture_layers, float *capture_out);

/* One depformer step for codebook cb_index in [0, dep_q); resets the depth KV
 * at cb_index == 0; writes audio_vocab logits (bmo_api.h:125). */
BMO_API int bmo_forward_depth(bmo_handle_t *h, int cb_index, int32_t prev_token, const float *transformer_out,
                              float *out_audio_logits);

/* All dep_q depformer steps with sampling between them: greedy (first
 * maximum) when top_k_audio <= 0 or temp_audio <= 1e-4, else top-k softmax
 * sampling with a per-thread mt19937 seeded 42 (bmo_api.h:134). */
BMO_API int bmo_forward_depth_cascade(bmo_handle_t *h, int32_t text_token, const float *transformer_out,
                                      float temp_audio, int top_k_audio, int32_t *out_audio_tokens);

/* Description of the last error on this handle, or NULL (bmo_api.h:145). */
BMO_API const char *bmo_last_error(bmo_handle_t *h);

/* Mimi RVQ decode / encode on caller device buffers (bmo_api.h:148-160). */
BMO_API int bmo_rvq_decode(const int32_t *codes_dev, const float *proj_tables_dev, float *out_dev, void *stream);
BMO_API int bmo_rvq_encode(const float *in_vec_dev, const float *w_in0_dev, const float *e0_dev,
                           const float *norm0_dev, const float *w_in_rest_dev, const float *e_rest_dev,
                           const float *norm_rest_dev, int32_t *out_codes_dev, float *scratch_dev, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BMO_API_H */
