/*
 * bmo_ext.h -- extensions of libbmo.so beyond the reference C ABI.
 *
 * None of these has a counterpart in utkarshyadav009/bmo_jetson; the
 * reference entry points in bmo_api.h are unchanged by them.
 */
#ifndef BMO_EXT_H
#define BMO_EXT_H

#include <stddef.h>
#include <stdint.h>

#include "bmo_api.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { BMO_KV_F16 = 0, BMO_KV_Q4_0 = 1 };

/* Flags of bmo_init_ex. */
enum {
    BMO_FLAG_NO_GRAPHS = 1, /* launch kernels eagerly instead of replaying CUDA graphs */
    BMO_FLAG_NO_PDL = 2,    /* no programmatic dependent launch between kernels */
    /* Summation order of the decode step.  Default: the reference kernels'
     * own fp32 operations in their own order (RMSNorm, Q4_0 x Q8_1 GEMV,
     * RoPE, decode attention, SwiGLU, residual adds), so that hidden states,
     * logits and tokens are bit-identical to the reference's chain of
     * kernels; used where it applies (fp16 ring of at most 1024 slots, head
     * sizes 64 or 128, one GPU), else the exact-reduction order.  The
     * environment variable BMO_SEMANTICS=exact|ref overrides the flags. */
    BMO_FLAG_EXACT = 8,      /* exact-reduction order: every sum in double, rounded once */
    BMO_FLAG_REF_ORDER = 16, /* the reference order, or fail when the model or ring does not allow it */
    /* Reference order: run the greedy depformer cascade as one launch on a
     * thread-block cluster (one CTA per depformer head) instead of one kernel
     * per op, when the model fits it.  Same results; slower on B200 for the
     * 7B depformer (its 16 SMs are compute-bound), so off by default. */
    BMO_FLAG_DEP_CLUSTER = 32,
};

/* bmo_init with an explicit CUDA device, KV ring format and flags.
 * device < 0 selects BMO_DEVICE or the current device. */
BMO_API bmo_handle_t *bmo_init_ex(const char *gguf_path, int n_ctx, int device, int kv_type, int flags);

BMO_API int bmo_get_kv_type(bmo_handle_t *h);
BMO_API int bmo_get_n_ctx(bmo_handle_t *h);
BMO_API int bmo_get_n_kv_heads(bmo_handle_t *h);
BMO_API int bmo_get_device(bmo_handle_t *h);
BMO_API int bmo_get_pos(bmo_handle_t *h);
/* CUDA stream (cudaStream_t) the handle launches on. */
BMO_API void *bmo_get_stream(bmo_handle_t *h);
/* Bytes of device memory the handle holds (weights, KV, buffers). */
BMO_API size_t bmo_get_device_bytes(bmo_handle_t *h);
/* 1 when the handle computes in the reference kernels' fp32 order, 0 for
 * the exact-reduction order (see BMO_FLAG_EXACT). */
BMO_API int bmo_get_ref_order(bmo_handle_t *h);
/* How greedy depformer cascades run: 0 one kernel per op, 1 one launch on a
 * thread-block cluster (BMO_FLAG_DEP_CLUSTER), 2 one cooperative launch over
 * every SM exchanging op outputs through global memory. */
BMO_API int bmo_get_dep_mode(bmo_handle_t *h);
/* Kernels one greedy frame (bmo_forward_frame_greedy / bmo_enqueue_frame)
 * launches on the device, or -1. */
BMO_API int bmo_get_frame_launches(bmo_handle_t *h);

/* Writes fp32 K/V rows (already rotated, as the ring stores them) into ring
 * slots [slot0, slot0+n) of temporal layer `layer`; rows are
 * [n][n_kv_heads * head_dim].  Converts to the ring format (fp16 or Q4_0).
 * Returns 0, or 2 for a bad range. */
BMO_API int bmo_kv_import_f32(bmo_handle_t *h, int layer, int slot0, int n, const float *k_rows,
                              const float *v_rows);
/* Same contract as bmo_copy_k_cache_f32 for the V ring. */
BMO_API int bmo_copy_v_cache_f32(bmo_handle_t *h, int layer, int t_start, int n_positions, float *out,
                                 int max_floats);
/* Raw ring bytes of one layer: which 0 = K, 1 = V; for Q4_0 rings part 0 is
 * the nibble plane and part 1 the fp16 scale plane. Returns bytes copied. */
BMO_API long long bmo_copy_kv_raw(bmo_handle_t *h, int which, int part, int layer, void *out, long long max_bytes);

/* One whole frame in a single graph: temporal step at `pos`, greedy text
 * token (argmax over the text logits), then the greedy depformer cascade
 * from that token.  Any output pointer may be NULL. */
BMO_API int bmo_forward_frame_greedy(bmo_handle_t *h, const int32_t *input_tokens, int num_codebooks, int pos,
                                     float *out_transformer, float *out_text_logits, int32_t *out_text_token,
                                     int32_t *out_audio_tokens);

/* Temporal layers [layer_begin, layer_end) on an fp32 hidden vector at
 * absolute position pos (no embedding, no final norm or head), as the
 * reference harness's per-layer cascade mode drives them.  Appends K/V of
 * those layers to the ring like a full step.  Returns 0, 1 null, 2 range. */
BMO_API int bmo_forward_layers(bmo_handle_t *h, const float *x_in, int pos, int layer_begin, int layer_end,
                               float *x_out);

/* Debug taps (the role of the reference's BMO_DUMP_* dumps): copies the
 * engine's activation buffer `which` as left by the last call into out
 * (max_floats).  which: 0 rotated q, 1 raw v, 2 attention output, 3
 * post-attention residual, 4 SwiGLU activation, 5 normed hidden z, 6 RoPE
 * (cos, sin) table, 7 the audio logits of every depformer step [dep_q][audio
 * vocabulary] (the last cascade's, or of the steps run since).  Returns
 * floats copied or -1. */
BMO_API int bmo_debug_tap(bmo_handle_t *h, int which, float *out, int max_floats);

/* Asynchronous device-resident frame: tokens_dev (device int32[num_codebooks])
 * are copied on the device, the frame graph is enqueued on the handle's
 * stream, and the text token + dep_q audio tokens land in out_tokens_dev
 * (device int32[1 + dep_q]).  No host synchronisation. */
BMO_API int bmo_enqueue_frame(bmo_handle_t *h, const int32_t *tokens_dev, int num_codebooks, int pos,
                              int32_t *out_tokens_dev);
/* Asynchronous parts of a frame, for timing: the temporal step alone
 * (tokens_dev as in bmo_enqueue_frame) and the greedy depformer cascade
 * alone (on the last temporal output, starting from text_token). */
BMO_API int bmo_enqueue_temporal(bmo_handle_t *h, const int32_t *tokens_dev, int num_codebooks, int pos);
BMO_API int bmo_enqueue_cascade(bmo_handle_t *h, int32_t text_token);

/* ---- tensor parallel (batch-1 latency mode) ---------------------------------
 * tp_size processes, one per GPU, each open a handle with bmo_init_tp on the
 * same GGUF and the same group id (from bmo_tp_unique_id on one process,
 * passed to the others).  Rank r holds attention heads [r H/T, (r+1) H/T),
 * their KV ring and O-projection columns, and FFN columns [r F/T, (r+1) F/T)
 * of every temporal and depformer layer; embeddings, norms and heads are
 * replicated.  After the O-projection and the FFN-out of every layer the
 * ranks sum their partial outputs in double -- over NVLink peer memory (the
 * ranks' exchange buffers mapped through CUDA IPC at init), or an NCCL
 * all-reduce with BMO_TP_P2P=0; both in the frame's CUDA graph -- and round
 * once, so every rank holds the same hidden state and the tokens equal the
 * single-GPU handle's.  Every rank must make the same calls
 * in the same order.  The handle's geometry getters report its shard's head
 * and FFN counts; bmo_kv_import_f32 takes the shard's KV heads.  Needs H, the
 * KV heads, the depformer heads and both FFN widths to split into
 * 32-column shards.  Returns NULL (reason on stderr) on failure. */
BMO_API int bmo_tp_unique_id(void *out_id /* 128 bytes */);
BMO_API bmo_handle_t *bmo_init_tp(const char *gguf_path, int n_ctx, int device, int kv_type, int flags, int tp_rank,
                                  int tp_size, const void *tp_id);
BMO_API int bmo_get_tp_size(bmo_handle_t *h);
BMO_API int bmo_get_tp_rank(bmo_handle_t *h);
/* 1 when the ranks sum their partial projections over NVLink peer memory
 * (every rank's exchange buffers mapped through CUDA IPC, one fused sum +
 * residual kernel per split projection); 0 on the NCCL all-reduce path (one
 * rank, BMO_TP_P2P=0, or a rank that could not map its peers). */
BMO_API int bmo_get_tp_exchange(bmo_handle_t *h);

/* ---- batched sessions ----------------------------------------------------
 * Up to 64 independent sessions share the handle's weights; each has its own
 * temporal ring (n_ctx slots, the handle's KV format).  One batched frame
 * steps any subset of them together, streaming every weight once for all. */

/* Allocates the rings of n_sessions sessions (1..64), empty.  Returns 0; 2 for
 * a bad count; 3 if sessions were already allocated with another count. */
BMO_API int bmo_batch_init(bmo_handle_t *h, int n_sessions);
BMO_API int bmo_batch_sessions(bmo_handle_t *h);
/* One greedy frame (as bmo_forward_frame_greedy) for each of n_rows rows: row
 * r runs session sess_ids[r] (NULL: r; ids distinct) at absolute position
 * pos[r] on input_tokens[r * num_codebooks + 0..num_codebooks).
 * out_tokens[r * (1 + dep_q)] receives the text token, then the dep_q audio
 * tokens.  out_transformer [n_rows][n_embd] (the normed hidden z) and
 * out_text_logits [n_rows][text_vocab] may be NULL.  The handle's own
 * single-session position and ring are untouched. */
BMO_API int bmo_forward_frame_batch(bmo_handle_t *h, int n_rows, const int32_t *sess_ids,
                                    const int32_t *input_tokens, int num_codebooks, const int32_t *pos,
                                    float *out_transformer, float *out_text_logits, int32_t *out_tokens);
/* Asynchronous form with device arrays (sess_ids_dev may be NULL); tokens
 * land in out_tokens_dev [n_rows][1 + dep_q] on the handle's stream. */
BMO_API int bmo_enqueue_frame_batch(bmo_handle_t *h, int n_rows, const int32_t *sess_ids_dev,
                                    const int32_t *tokens_dev, int num_codebooks, const int32_t *pos_dev,
                                    int32_t *out_tokens_dev);
/* bmo_kv_import_f32 into the ring of one session. */
BMO_API int bmo_batch_kv_import_f32(bmo_handle_t *h, int session, int layer, int slot0, int n,
                                    const float *k_rows, const float *v_rows);
/* Empties one session's ring (session < 0: all).  Returns 0, 2 for a bad id. */
BMO_API int bmo_batch_reset(bmo_handle_t *h, int session);

/* ---- the caller's frame loop on the device (replaces the per-frame host
 * logic of bmo_daemon.cpp:727-816: the 17-channel interleave with its delay,
 * bmo_forward_temporal, the text sample with pause tokens 3 and 0 kept
 * greedy, 8 x bmo_forward_depth each followed by its audio sample, the codec
 * input and the delay-line update).  Each frame is one CUDA graph; a call
 * of n frames synchronises with the host once. ---- */
/* Starts a conversation: frame 0, empty KV rings, the daemon's delay-line
 * start state and its sampler generator std::mt19937(seed) (the daemon seeds
 * 1337).  Returns 0; 3 when the model has no text head or depformer, its
 * depformer takes other than 8 steps, it reads other than 9 or 17 input
 * channels, or the handle is tensor parallel; 9 on a device error. */
BMO_API int bmo_loop_reset(bmo_handle_t *h, uint32_t seed);
/* Runs n_frames (1 to 64) frames.  user_tokens: [n_frames][8] the user's
 * audio tokens, or NULL for the daemon's silence tokens.  use_sampling 0:
 * first argmax everywhere; otherwise sample_token_cpp's top-k / temperature
 * draw (min(top_k, logits drawn from) up to 2048; top_k <= 0 or temp <=
 * 1e-4 is greedy).  out:
 * [n_frames][17] = text token, 8 audio tokens, 8 codec tokens (the daemon
 * decodes nothing at frame 0).  Returns 0; 1 null pointer; 2 bad count or
 * top_k; 4 not reset; 9 device error. */
BMO_API int bmo_loop_run(bmo_handle_t *h, int n_frames, const int32_t *user_tokens, int use_sampling,
                         float temp_text, int top_k_text, float temp_audio, int top_k_audio, int32_t *out);
/* 1 when the model runs the frame loop (the conditions of bmo_loop_reset). */
BMO_API int bmo_loop_supported(bmo_handle_t *h);
/* Frames run since bmo_loop_reset, or -1. */
BMO_API int bmo_loop_frame(bmo_handle_t *h);

/* Waits for the handle's stream; returns the device status word (0 = ok). */
BMO_API int bmo_sync(bmo_handle_t *h);

/* Deterministic synthetic data for benchmark models (counter-based RNG,
 * Box-Muller normals).  q4_0 quantises rows of N(0, sigma) with ggml's
 * reference Q4_0 rule; f16/f32 fill N(mean, sigma). */
BMO_API void bmo_synth_normal_f32(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, float *out);
BMO_API void bmo_synth_f16(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, uint16_t *out);
BMO_API void bmo_synth_q4_0(uint64_t seed, uint64_t stream, long long rows, long long cols, float sigma,
                            uint8_t *out);
/* ggml Q4_0 reference quantiser (18-byte blocks) over n floats. */
BMO_API void bmo_quantize_q4_0_ref(const float *x, long long n, uint8_t *out);

/* ---- offline repacking (bmo_jetson_b200/repack.py) ----
 * A repacked GGUF carries the key bmo.tiled.version = 1 and, for each Q4_0
 * matrix N, the I8 tensor "bmo.tiled:N" holding N in the device's row-tile
 * layout and the I32 tensor "bmo.tiled_desc:N" = {cols, rows, perm,
 * swiglu_f} (perm 0 rows in order, 1 the SwiGLU gate/up pairing with
 * F = swiglu_f); N itself is dropped unless the file was repacked with its
 * raw rows kept.  The loader copies such tiles into the weight arena as they
 * are (no staging, no repack kernel); slices that are not whole row tiles of
 * the stored form (tensor-parallel shards) need the raw rows. */
/* Tiles a rows x cols Q4_0 matrix (ggml's row-major 18-byte blocks) on the
 * host into the layout the load-time repack produces on the device, byte for
 * byte.  dst NULL: returns the bytes needed.  Returns the bytes written, or
 * -1 for a shape the GEMV does not take. */
BMO_API long long bmo_q4_0_tile_host(const uint8_t *raw, long long rows, long long cols, int perm, int swiglu_f,
                                     uint8_t *dst);
/* Weights of the handle's model that were loaded from pre-tiled tensors. */
BMO_API int bmo_get_tiled_weights(bmo_handle_t *h);

#ifdef __cplusplus
}
#endif

#endif /* BMO_EXT_H */
