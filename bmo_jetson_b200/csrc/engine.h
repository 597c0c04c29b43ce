// engine.h -- device-side decode-step engine behind the C ABI.
//
// Owns the model in HBM (Q4_0 matrices repacked into row tiles, embedding
// tables and norms as stored), the temporal KV ring, the depformer KV, the
// activation buffers, and one CUDA graph per entry point:
//   temporal      embed -> 32 x {QKV, attention, O, FFN-in, FFN-out} -> head
//   depth[cb]     one depformer step (reference bmo_forward_depth)
//   cascade       dep_q depformer steps with greedy argmax chaining on device
//                 (opt-in: one cluster kernel, kernels/dep_cascade.cu)
//   frame         temporal + greedy text token + cascade
// Each op list runs one kernel per op, chained with programmatic dependent
// launch inside CUDA graphs.  Two summation orders exist for the GEMV and
// the attention: the reference kernels' own fp32 order (default; bit-identical
// to the reference's chain of kernels) and the exact-reduction order (double
// sums rounded once; used by Q4_0 rings, tensor parallel and batched
// sessions, whose arithmetic has no fp32 counterpart in the reference).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "gguf.h"
#include "layout.h"
#include "tp_comm.h"

namespace bmo {

constexpr int kDepQMax = 8;
constexpr int kDepLayers = 6;
constexpr int kMaxTokens = 64;

struct EngineConfig {
    int device = -1;   // < 0: BMO_DEVICE or current device
    int n_ctx = 0;     // <= 0: 2048
    int kv_type = -1;  // < 0: BMO_KV_TYPE or fp16
    bool graphs = true;
    bool pdl = true;
    // -1: the reference kernels' fp32 order where the model and ring allow,
    // else the exact-reduction order; 0: exact-reduction order; 1: the
    // reference order or an error
    int semantics = -1;
    // reference order: run the greedy depformer cascade as one launch on a
    // thread-block cluster instead of one kernel per op (same results; opt-in:
    // measured slower on B200, its 16 SMs are compute-bound)
    bool dep_cluster = false;
    // tensor parallel (batch-1 latency mode): tp_size >= 1 makes this engine
    // rank tp_rank of tp_size, holding the attention heads and FFN columns of
    // its shard; tp_id is the group's NCCL unique id
    int tp_rank = 0, tp_size = 0;
    unsigned char tp_id[128] = {};
};

// Per-call inputs, copied to the device in one transfer.
struct FrameIn {
    int32_t tokens[kMaxTokens];
    int32_t n_tok;
    int32_t pos;
    int32_t prev_token;
    int32_t pad;
};

class Engine {
public:
    Engine(const std::string &gguf_path, const EngineConfig &cfg);
    ~Engine();
    Engine(const Engine &) = delete;
    Engine &operator=(const Engine &) = delete;

    // ---- geometry (reference names, src/bmo.h:263-291) ----
    int n_layers = 0, n_embd = 0, n_heads = 0, head_dim = 0, n_kv_heads = 0, ffn = 0;
    int n_ctx = 0, kv_type = kKvF16, n_q = 0, num_codebooks = 0, dep_q = 0;
    int text_vocab = 0, audio_vocab = 0;
    float rope_theta = 10000.0f, norm_eps = 1e-8f;
    int dep_dim = 0, dep_heads = 16, dep_hd = 0, dep_ffn = 0, dep_n_ctx = 0;
    bool has_text_head = false;
    bool has_dep_head[kDepQMax] = {};
    bool has_dep_tables = false;
    int device = 0, sm_count = 148;
    cudaStream_t stream = nullptr;
    size_t device_bytes = 0;
    // tensor parallel: head, KV-head and FFN counts above are this rank's shard
    bool tensor_parallel = false;
    int tp_rank = 0, tp_size = 1;

    // ---- synchronous operations (caller serialises) ----
    void run_temporal(const int32_t *tokens, int K, int pos);
    const float *z_host() const { return z_h_; }
    const float *logits_host() const { return logits_h_; }
    void copy_resid(int layer, float *out);  // post-layer residual of the last temporal step
    void run_layers(const float *x_in, int pos, int layer_begin, int layer_end, float *x_out);
    void run_depth(int cb, int32_t prev, const float *z);
    const float *depth_logits_host() const { return dlogits_h_; }
    void run_cascade_greedy(int32_t text_tok, const float *z, int32_t *out_tokens);
    void run_frame_greedy(const int32_t *tokens, int K, int pos, int32_t *out_text_tok, int32_t *out_audio);
    void enqueue_frame_device(const int32_t *tokens_dev, int K, int pos, int32_t *out_tokens_dev);
    void enqueue_temporal_device(const int32_t *tokens_dev, int K, int pos);
    void enqueue_cascade_device(int32_t text_token);
    int sync_status();
    void reset_kv();
    void reset_depth_kv();
    int kv_import(int layer, int slot0, int n, const float *k_rows, const float *v_rows);
    int copy_cache_f32(int which, int layer, int t_start, int n_positions, float *out);
    long long copy_kv_raw(int which, int part, int layer, void *out, long long max_bytes);
    int debug_tap(int which, float *out, int max_floats);
    void capture_all();
    bool graphs_captured() const { return graphs_ready_; }
    bool ref_order() const { return ref_order_; }
    bool dep_cluster() const { return dep_cluster_; }
    int frame_launches() const;  // kernels one greedy frame launches (embed, temporal ops, cascade)
    bool dep_grid() const { return dep_grid_; }
    bool tp_exchange() const { return tp_p2p_; }
    int tiled_weights() const { return tiled_weights_; }  // weights copied from a repacked file's tiles

    // ---- the caller's frame loop on the device (bmo_daemon.cpp:641-816):
    // interleave, temporal step, text sample, dep_q depformer steps with
    // their audio samples and the codec input of each frame, as one graph ----
    bool loop_supported() const;  // a text head, 8 depformer steps, 9 or 17 input channels, one GPU
    void loop_reset(uint32_t seed);  // frame 0, the daemon's start state, mt19937(seed), fresh KV rings
    // top-k values the device sampler takes: min(top_k, logits considered) <= kLoopTopKMax
    bool loop_params_ok(const LoopParams &in) const;
    // Frames f .. f + n - 1 (n <= kLoopRing) with in[i] as frame f + i's
    // inputs; out[i][kLoopOut] their results.  One host synchronisation.
    void loop_run(int n, const LoopParams *in, int32_t *out);
    int loop_frame() const { return loop_st_ ? loop_frame_ : -1; }  // -1 before loop_reset

    // ---- batched sessions: up to kBatchMax independent sessions stepped
    // together, each with its own temporal ring, sharing one weight stream ----
    int batch_init(int n_sessions);  // allocates the rings once (0 ok, 1 bad count, 3 already other size)
    int batch_sessions() const;
    // One greedy frame for rows s < n: session sess_ids[s] at pos[s] on
    // tokens[s * K + 0..K).  out_tokens[s * (1 + dep_q)] = text token, then
    // the dep_q audio tokens; out_z [n][n_embd] and out_logits
    // [n][text_vocab] are optional.
    void run_frame_batch(int n, const int32_t *sess_ids, const int32_t *tokens, int K, const int32_t *pos,
                         float *out_z, float *out_logits, int32_t *out_tokens);
    // Same with device inputs and outputs; no host synchronisation.
    void enqueue_frame_batch_device(int n, const int32_t *sess_dev, const int32_t *tokens_dev, int K,
                                    const int32_t *pos_dev, int32_t *out_tokens_dev);
    int batch_kv_import(int sess, int layer, int slot0, int n, const float *k_rows, const float *v_rows);
    int batch_reset(int sess);  // sess < 0: every session

private:
    struct Layer {
        QMatDesc qkv{}, wo{}, ffn_in{}, ffn_out{};
        float *norm1 = nullptr, *norm2 = nullptr;
    };
    struct DepLayer {
        QMatDesc qkv[kDepQMax] = {}, wo[kDepQMax] = {}, ffn_in[kDepQMax] = {}, ffn_out[kDepQMax] = {};
        float *norm1 = nullptr, *norm2 = nullptr;
    };

    void load(const std::string &path);
    void alloc_state();
    void *arena(size_t bytes);
    QMatDesc upload_q4(const GgufTensor *t, int perm, int swiglu_f, int64_t row0, int64_t rows);
    // rows from several ranges (concatenated) and 32-aligned columns [col0, col0 + ncols)
    QMatDesc upload_q4_sel(const GgufTensor *t, int perm, int swiglu_f,
                           const std::vector<std::pair<int64_t, int64_t>> &row_ranges, int64_t col0, int64_t ncols);
    QMatDesc upload_q4_raw(const std::string &name, const uint8_t *src, int64_t rows, int64_t cols, int perm,
                           int swiglu_f);
    QMatDesc upload_q4_tiled(const std::string &name, const uint8_t *tiles, int64_t rows, int64_t cols, int perm,
                             int swiglu_f);
    int tiled_weights_ = 0;
    float *upload_f32(const GgufTensor *t, int64_t n);
    EmbTable upload_table(const GgufTensor *t);
    GemvArgs gemv_base(const QMatDesc &m) const;

    // a frame's steps as op lists (layout.h FramePhase)
    void ops_layer(std::vector<FramePhase> &v, int l) const;
    void ops_text_head(std::vector<FramePhase> &v) const;
    std::vector<FramePhase> ops_temporal() const;
    void ops_depth_step(std::vector<FramePhase> &v, int cb, const float *z, const TokenSrc &tok) const;
    void ops_cascade(std::vector<FramePhase> &v, const float *z, const TokenSrc &first) const;
    // per-op path
    void enqueue_ops(cudaStream_t s, const std::vector<FramePhase> &ops);
    void enqueue_embed(cudaStream_t s);
    void enqueue_temporal(cudaStream_t s);
    void enqueue_layer(cudaStream_t s, int l);
    void enqueue_depth_step(cudaStream_t s, int cb, const float *z, const TokenSrc &tok);
    void enqueue_cascade(cudaStream_t s, const float *z, const TokenSrc &first, bool reset_kv = true);
    void enqueue_frame_greedy(cudaStream_t s);
    void reset_depth_kv_async(cudaStream_t s);
    void choose_semantics(int want);
    // tensor parallel
    std::unique_ptr<TpComm> tp_comm_;
    double *tp_part_ = nullptr;  // partial sums of the split projections, summed over the ranks (NCCL path)
    // peer-memory exchange (kPhTpExchange): this rank's block and every rank's
    // block mapped here (tp_peer_[tp_rank] == tp_block_), and the exchange count
    bool tp_p2p_ = false;
    void *tp_block_ = nullptr;
    void *tp_peer_[kTpMaxRanks] = {};
    unsigned long long *tp_seq_ = nullptr;
    void setup_tp_exchange();
    void teardown_tp_exchange();
    double *tp_buf(int rank, int buf) const {
        return static_cast<double *>(tp_peer_[rank]) + static_cast<size_t>(buf) * kTpBufDoubles;
    }
    void ops_tp_reduce(std::vector<FramePhase> &v, const GemvArgs &g, const float *resid, float *y, int n,
                       int buf) const;
    // batched sessions (batch_engine.cpp)
    struct BatchState;
    struct BatchDeleter {
        void operator()(BatchState *b) const;
    };
    std::unique_ptr<BatchState, BatchDeleter> batch_;
    void enqueue_batch_frame(cudaStream_t s, int n);
    void batch_clear_counters(cudaStream_t s);  // after a device error
    void enqueue_batch_temporal(cudaStream_t s, int n);
    void enqueue_batch_cascade(cudaStream_t s, int n);
    void batch_stage(cudaStream_t s, int n, const float *x, int cols, const QMatDesc &W, const float *gamma,
                     float *xn_out, const TokenSrc *tok, int pairs_stride, int *tok_out);
    void batch_gemm(cudaStream_t s, const BatchGemmArgs &a, int epi);
    int kv_import_into(void *kc, void *vc, uint8_t *ks, uint8_t *vs, int layer, int slot0, int n, const float *k_rows,
                       const float *v_rows);

    // frame loop (kernels/loop.cu)
    LoopState *loop_st_ = nullptr;
    LoopParams *loop_in_h_ = nullptr;  // pinned [kLoopRing]
    int32_t *loop_out_h_ = nullptr;    // pinned [kLoopRing][kLoopOut]
    int loop_frame_ = 0;
    cudaGraphExec_t g_loop_ = nullptr;
    void enqueue_loop_frame(cudaStream_t s);

    cudaGraphExec_t capture(const std::function<void(cudaStream_t)> &fn);
    void launch(cudaGraphExec_t &g, const std::function<void(cudaStream_t)> &fn);
    void finish_call();

    EngineConfig cfg_;
    GgufFile file_;
    std::vector<void *> allocs_;
    uint8_t *arena_ = nullptr;
    size_t arena_size_ = 0, arena_used_ = 0;
    uint8_t *staging_d_ = nullptr;
    size_t staging_bytes_ = 0;

    // weights
    std::vector<Layer> L_;
    QMatDesc text_head_{};
    float *text_bias_ = nullptr, *out_norm_ = nullptr;
    QMatDesc dep_in_[kDepQMax] = {}, dep_head_[kDepQMax] = {};
    DepLayer D_[kDepLayers];
    EmbTable *ttables_d_ = nullptr;
    int n_ttables_ = 0;
    EmbTable dep_text_emb_{}, dep_emb_[kDepQMax] = {};

    // temporal state and activations
    void *k_cache_ = nullptr, *v_cache_ = nullptr;
    uint8_t *k_scale_ = nullptr, *v_scale_ = nullptr;
    size_t kv_plane_bytes_ = 0, kv_scale_bytes_ = 0;
    float *resid_ = nullptr, *xmid_ = nullptr, *q_ = nullptr, *vraw_ = nullptr, *attn_ = nullptr, *act_ = nullptr;
    float *z_ = nullptr, *logits_ = nullptr;
    float2 *rope_ = nullptr, *tpairs_ = nullptr;
    // depformer state and activations
    __half *dk_cache_ = nullptr, *dv_cache_ = nullptr;
    size_t dkv_bytes_ = 0;
    float *dz_ = nullptr, *dxa_ = nullptr, *dxb_ = nullptr, *dq_ = nullptr, *dvraw_ = nullptr, *dattn_ = nullptr;
    float *dact_ = nullptr, *dlogits_ = nullptr;
    float2 *dpairs_ = nullptr;
    int dpairs_stride_ = 0;
    int *dep_pos_ = nullptr;
    int *tok_out_ = nullptr;  // [1 + kDepQMax]: text token, audio tokens
    // scratch
    double *gpart_ = nullptr;
    int *gcount_ = nullptr;
    size_t gpart_bytes_ = 0, gcount_bytes_ = 0;
    int attn_splits_ = 1;
    int *status_ = nullptr;
    FrameIn *fin_d_ = nullptr;

    // pinned host staging
    FrameIn *fin_h_ = nullptr;
    float *z_h_ = nullptr, *logits_h_ = nullptr, *zin_h_ = nullptr, *dlogits_h_ = nullptr;
    int *tok_h_ = nullptr, *status_h_ = nullptr;

    // graphs
    cudaGraphExec_t g_temporal_ = nullptr, g_depth_[kDepQMax] = {}, g_cascade_ = nullptr, g_frame_ = nullptr;
    cudaGraphExec_t g_layers_ = nullptr, g_cascade_z_ = nullptr;
    int g_layers_range_[2] = {-1, -1};
    bool graphs_ready_ = false;

    // summation order of the single-session path (see the header comment)
    bool ref_order_ = false;

    // the greedy cascade as one launch (reference order): on one
    // thread-block cluster, or over every SM with epoch-tagged exchanges
    bool dep_cluster_ = false, dep_grid_ = false;
    int dep_grid_ctas_ = 0;
    DepOp *dep_ops_d_ = nullptr;
    DepCascadeArgs dep_args_{};
    size_t dep_smem_ = 0;
    void setup_dep_cascade();
};

}  // namespace bmo
