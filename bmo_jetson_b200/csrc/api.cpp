// api.cpp -- the C ABI (include/bmo_api.h, include/bmo_ext.h) over the
// device engine.  Argument checks, return codes, the per-handle mutex and
// last-error semantics follow the reference bridge (src/bmo_api.cpp);
// exceptions never cross the ABI.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <utility>
#include <vector>

#include "../../include/bmo_api.h"
#include "../../include/bmo_ext.h"
#include "engine.h"

struct bmo_handle {
    std::unique_ptr<bmo::Engine> eng;
    int pos = 0;
    std::string last_error;
    std::mutex mu;
};

namespace {

void set_err(bmo_handle_t *h, const std::string &m) {
    if (h) h->last_error = m;
}

bmo_handle_t *create(const char *path, int n_ctx, const bmo::EngineConfig &cfg) {
    if (!path) {
        std::fprintf(stderr, "[bmo_api] bmo_init: gguf_path is null\n");
        return nullptr;
    }
    try {
        auto h = std::make_unique<bmo_handle>();
        bmo::EngineConfig c = cfg;
        c.n_ctx = n_ctx;
        h->eng = std::make_unique<bmo::Engine>(path, c);
        return h.release();
    } catch (const std::exception &e) {
        std::fprintf(stderr, "[bmo_api] init failed: %s\n", e.what());
    } catch (...) {
        std::fprintf(stderr, "[bmo_api] init failed: unknown exception\n");
    }
    return nullptr;
}

// Sampling of the reference cascade (bmo_api.cpp:638-666): greedy when
// top_k <= 0 or temp <= 1e-4, else top-k softmax with std::discrete_distribution.
int sample_token(const float *logits, int n_vocab, float temp, int top_k, std::vector<std::pair<float, int>> &scratch,
                 std::mt19937 &rng) {
    if (top_k <= 0 || temp <= 1e-4f) return static_cast<int>(std::max_element(logits, logits + n_vocab) - logits);
    scratch.resize(static_cast<size_t>(n_vocab));
    for (int i = 0; i < n_vocab; ++i) scratch[static_cast<size_t>(i)] = {logits[i], i};
    const int k = std::min(top_k, n_vocab);
    std::partial_sort(scratch.begin(), scratch.begin() + k, scratch.end(),
                      [](const std::pair<float, int> &a, const std::pair<float, int> &b) { return a.first > b.first; });
    const float max_l = scratch[0].first / temp;
    std::vector<float> probs(static_cast<size_t>(k));
    float sum_p = 0.0f;
    for (int i = 0; i < k; ++i) {
        probs[static_cast<size_t>(i)] = std::exp(scratch[static_cast<size_t>(i)].first / temp - max_l);
        sum_p += probs[static_cast<size_t>(i)];
    }
    if (sum_p <= 0.0f || std::isnan(sum_p)) return scratch[0].second;
    std::discrete_distribution<int> dist(probs.begin(), probs.end());
    return scratch[static_cast<size_t>(dist(rng))].second;
}

int copy_cache(bmo_handle_t *h, int which, int layer, int t_start, int n_positions, float *out, int max_floats) {
    if (!h || !out || n_positions <= 0 || max_floats <= 0) return -1;
    bmo::Engine *e = h->eng.get();
    if (!e) return -1;
    if (layer < 0 || layer >= e->n_layers || e->n_heads <= 0 || e->head_dim <= 0) return -3;
    if (t_start < 0 || t_start + n_positions > e->n_ctx) return -3;
    const long long need = static_cast<long long>(n_positions) * e->n_kv_heads * e->head_dim;
    if (need > max_floats) return -2;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return e->copy_cache_f32(which, layer, t_start, n_positions, out);
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return -1;
    }
}

}  // namespace

extern "C" {

bmo_handle_t *bmo_init(const char *gguf_path, int n_ctx) { return create(gguf_path, n_ctx, bmo::EngineConfig{}); }

bmo_handle_t *bmo_init_ex(const char *gguf_path, int n_ctx, int device, int kv_type, int flags) {
    bmo::EngineConfig c;
    c.device = device;
    c.kv_type = kv_type;
    c.graphs = !(flags & BMO_FLAG_NO_GRAPHS);
    c.pdl = !(flags & BMO_FLAG_NO_PDL);
    if (flags & BMO_FLAG_EXACT) c.semantics = 0;
    else if (flags & BMO_FLAG_REF_ORDER) c.semantics = 1;
    c.dep_cluster = (flags & BMO_FLAG_DEP_CLUSTER) != 0;
    return create(gguf_path, n_ctx, c);
}

int bmo_tp_unique_id(void *out_id) {
    if (!out_id) return 1;
    try {
        bmo::tp_unique_id(out_id);
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "[bmo_api] bmo_tp_unique_id: %s\n", e.what());
        return 9;
    }
}

bmo_handle_t *bmo_init_tp(const char *gguf_path, int n_ctx, int device, int kv_type, int flags, int tp_rank,
                          int tp_size, const void *tp_id) {
    if (!tp_id || tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) {
        std::fprintf(stderr, "[bmo_api] bmo_init_tp: invalid rank, size or id\n");
        return nullptr;
    }
    bmo::EngineConfig c;
    c.device = device;
    c.kv_type = kv_type;
    c.graphs = !(flags & BMO_FLAG_NO_GRAPHS);
    c.pdl = !(flags & BMO_FLAG_NO_PDL);
    c.tp_rank = tp_rank;
    c.tp_size = tp_size;
    std::memcpy(c.tp_id, tp_id, sizeof c.tp_id);
    return create(gguf_path, n_ctx, c);
}

int bmo_get_tp_size(bmo_handle_t *h) { return (h && h->eng) ? h->eng->tp_size : 0; }
int bmo_get_tp_rank(bmo_handle_t *h) { return (h && h->eng) ? h->eng->tp_rank : 0; }
int bmo_get_tp_exchange(bmo_handle_t *h) { return (h && h->eng && h->eng->tp_exchange()) ? 1 : 0; }

void bmo_free(bmo_handle_t *h) {
    if (!h) return;
    try {
        h->eng.reset();
    } catch (...) {
    }
    delete h;
}

void bmo_reset(bmo_handle_t *h) {
    if (!h) return;
    std::lock_guard<std::mutex> lk(h->mu);
    h->pos = 0;
    try {
        if (h->eng) h->eng->reset_kv();
    } catch (const std::exception &e) {
        h->last_error = e.what();
        return;
    }
    h->last_error.clear();
}

int bmo_get_n_layers(bmo_handle_t *h) { return h ? h->eng->n_layers : 0; }
int bmo_get_n_embd(bmo_handle_t *h) { return h ? h->eng->n_embd : 0; }
int bmo_get_n_codebooks(bmo_handle_t *h) { return h ? h->eng->num_codebooks : 0; }
int bmo_get_dep_q(bmo_handle_t *h) { return h ? h->eng->dep_q : 0; }
int bmo_get_text_vocab(bmo_handle_t *h) { return h ? h->eng->text_vocab : 0; }
int bmo_get_audio_vocab(bmo_handle_t *h) { return h ? h->eng->audio_vocab : 0; }
int bmo_get_n_attn_heads(bmo_handle_t *h) { return h ? h->eng->n_heads : 0; }
int bmo_get_head_dim(bmo_handle_t *h) { return h ? h->eng->head_dim : 0; }
int bmo_get_kv_type(bmo_handle_t *h) { return h ? h->eng->kv_type : -1; }
int bmo_get_n_ctx(bmo_handle_t *h) { return h ? h->eng->n_ctx : 0; }
int bmo_get_n_kv_heads(bmo_handle_t *h) { return h ? h->eng->n_kv_heads : 0; }
int bmo_get_device(bmo_handle_t *h) { return h ? h->eng->device : -1; }
int bmo_get_pos(bmo_handle_t *h) { return h ? h->pos : 0; }
void *bmo_get_stream(bmo_handle_t *h) { return h ? static_cast<void *>(h->eng->stream) : nullptr; }
size_t bmo_get_device_bytes(bmo_handle_t *h) { return h ? h->eng->device_bytes : 0; }

int bmo_copy_k_cache_f32(bmo_handle_t *h, int layer, int t_start, int n_positions, float *out, int max_floats) {
    return copy_cache(h, 0, layer, t_start, n_positions, out, max_floats);
}

int bmo_copy_v_cache_f32(bmo_handle_t *h, int layer, int t_start, int n_positions, float *out, int max_floats) {
    return copy_cache(h, 1, layer, t_start, n_positions, out, max_floats);
}

long long bmo_copy_kv_raw(bmo_handle_t *h, int which, int part, int layer, void *out, long long max_bytes) {
    if (!h || !out || layer < 0 || layer >= h->eng->n_layers) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->copy_kv_raw(which, part, layer, out, max_bytes);
    } catch (const std::exception &e) {
        h->last_error = e.what();
        return -1;
    }
}

int bmo_debug_tap(bmo_handle_t *h, int which, float *out, int max_floats) {
    if (!h || !out) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->debug_tap(which, out, max_floats);
    } catch (const std::exception &e) {
        h->last_error = e.what();
        return -1;
    }
}

int bmo_kv_import_f32(bmo_handle_t *h, int layer, int slot0, int n, const float *k_rows, const float *v_rows) {
    if (!h || !k_rows || !v_rows) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->kv_import(layer, slot0, n, k_rows, v_rows);
    } catch (const std::exception &e) {
        h->last_error = e.what();
        return 9;
    }
}

int bmo_capture_graphs(bmo_handle_t *h) {
    if (!h) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        h->eng->capture_all();
        return h->eng->graphs_captured() ? 0 : 1;
    } catch (const std::exception &e) {
        h->last_error = e.what();
        return 1;
    }
}

int bmo_has_cuda_graphs(bmo_handle_t *h) { return (h && h->eng->graphs_captured()) ? 1 : 0; }

int bmo_get_ref_order(bmo_handle_t *h) { return (h && h->eng->ref_order()) ? 1 : 0; }

int bmo_get_frame_launches(bmo_handle_t *h) {
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->frame_launches();
    } catch (const std::exception &e) {
        h->last_error = e.what();
        return -1;
    }
}

int bmo_loop_reset(bmo_handle_t *h, uint32_t seed) {
    if (!h) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    bmo::Engine *e = h->eng.get();
    if (!e->loop_supported()) {
        h->last_error = "bmo_loop_reset: the model has no frame loop (text head, 8 depformer steps, 9 or 17 channels, one GPU)";
        return 3;
    }
    try {
        e->loop_reset(seed);
    } catch (const std::exception &ex) {
        h->last_error = ex.what();
        return 9;
    }
    h->last_error.clear();
    return 0;
}

int bmo_loop_run(bmo_handle_t *h, int n_frames, const int32_t *user_tokens, int use_sampling, float temp_text,
                 int top_k_text, float temp_audio, int top_k_audio, int32_t *out) {
    if (!h || !out) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    bmo::Engine *e = h->eng.get();
    if (n_frames < 1 || n_frames > bmo::kLoopRing) {
        h->last_error = "bmo_loop_run: 1 to 64 frames per call";
        return 2;
    }
    if (e->loop_frame() < 0 || !e->loop_supported()) return 4;
    bmo::LoopParams in[bmo::kLoopRing] = {};
    for (int i = 0; i < n_frames; ++i) {
        in[i].sampling = use_sampling ? 1 : 0;
        in[i].temp_text = temp_text;
        in[i].temp_audio = temp_audio;
        in[i].top_k_text = top_k_text;
        in[i].top_k_audio = top_k_audio;
        in[i].user_valid = user_tokens ? 1 : 0;
        for (int c = 0; c < bmo::kLoopCb; ++c) in[i].user[c] = user_tokens ? user_tokens[i * bmo::kLoopCb + c] : 0;
    }
    if (!e->loop_params_ok(in[0])) {
        h->last_error = "bmo_loop_run: top_k above 2048 over more than 2048 logits";
        return 2;
    }
    try {
        e->loop_run(n_frames, in, out);
    } catch (const std::exception &ex) {
        h->last_error = ex.what();
        return std::strstr(ex.what(), "not reset") ? 4 : 9;
    }
    h->last_error.clear();
    return 0;
}

int bmo_get_tiled_weights(bmo_handle_t *h) { return h ? h->eng->tiled_weights() : 0; }

int bmo_loop_supported(bmo_handle_t *h) { return (h && h->eng->loop_supported()) ? 1 : 0; }

int bmo_loop_frame(bmo_handle_t *h) {
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    return h->eng->loop_frame();
}

int bmo_get_dep_mode(bmo_handle_t *h) {
    if (!h) return 0;
    return h->eng->dep_grid() ? 2 : h->eng->dep_cluster() ? 1 : 0;
}

const char *bmo_last_error(bmo_handle_t *h) { return (!h || h->last_error.empty()) ? nullptr : h->last_error.c_str(); }

int bmo_forward_temporal(bmo_handle_t *h, const int32_t *input_tokens, int num_codebooks, int pos,
                         float *out_transformer, float *out_text_logits) {
    return bmo_forward_temporal2(h, input_tokens, num_codebooks, pos, out_transformer, out_text_logits, nullptr, 0,
                                 nullptr);
}

// bmo_forward_temporal2, reference bmo_api.cpp:384-511.
int bmo_forward_temporal2(bmo_handle_t *h, const int32_t *input_tokens, int num_codebooks, int pos,
                          float *out_transformer, float *out_text_logits, const int32_t *capture_layers,
                          int n_capture_layers, float *capture_out) {
    if (!h || !input_tokens || !out_transformer || !out_text_logits) {
        set_err(h, "bmo_forward_temporal2: null pointer argument");
        return 1;
    }
    bmo::Engine *e = h->eng.get();
    if (num_codebooks <= 0 || num_codebooks > e->num_codebooks) {
        set_err(h, "bmo_forward_temporal2: invalid num_codebooks");
        return 2;
    }
    if (pos < 0) {
        set_err(h, "bmo_forward_temporal2: pos must be non-negative");
        return 2;
    }
    if (n_capture_layers < 0) {
        set_err(h, "bmo_forward_temporal2: invalid n_capture_layers");
        return 2;
    }
    if (n_capture_layers > 0 && (!capture_layers || !capture_out)) {
        set_err(h, "bmo_forward_temporal2: capture_layers/capture_out required when n_capture_layers > 0");
        return 2;
    }
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        e->run_temporal(input_tokens, num_codebooks, pos);
        std::memcpy(out_transformer, e->z_host(), sizeof(float) * static_cast<size_t>(e->n_embd));
        if (!e->has_text_head) {
            set_err(h, "bmo_forward_temporal2: text_logits tensor missing (model.text_linear may be null)");
            return 3;
        }
        std::memcpy(out_text_logits, e->logits_host(), sizeof(float) * static_cast<size_t>(e->text_vocab));
        for (int i = 0; i < n_capture_layers; ++i) {
            const int L = capture_layers[i];
            if (L < 0 || L >= e->n_layers) {
                set_err(h, "bmo_forward_temporal2: missing capture tensor out_layer_" + std::to_string(L));
                return 6;
            }
            e->copy_resid(L, capture_out + static_cast<size_t>(i) * e->n_embd);
        }
        h->pos = pos + 1;
        h->last_error.clear();
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    } catch (...) {
        set_err(h, "bmo_forward_temporal2: unknown exception");
        return 9;
    }
}

// bmo_forward_depth, reference bmo_api.cpp:513-636.
int bmo_forward_depth(bmo_handle_t *h, int cb_index, int32_t prev_token, const float *transformer_out,
                      float *out_audio_logits) {
    if (!h || !transformer_out || !out_audio_logits) {
        set_err(h, "bmo_forward_depth: null pointer argument");
        return 1;
    }
    bmo::Engine *e = h->eng.get();
    if (cb_index < 0 || cb_index >= e->dep_q) {
        set_err(h, "bmo_forward_depth: cb_index out of range");
        return 2;
    }
    if (e->dep_n_ctx <= 0 || cb_index >= e->dep_n_ctx) {
        set_err(h, "bmo_forward_depth: depth KV cache not initialised or cb_index too large");
        return 2;
    }
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        if (e->dep_dim <= 0 || !e->has_dep_tables || (cb_index > 0 && e->n_q == 0)) {
            set_err(h, "bmo_forward_depth: depformer weights or embedding tables missing");
            return 9;
        }
        if (!e->has_dep_head[cb_index]) {
            set_err(h, "bmo_forward_depth: audio_logits tensor missing (model.audio_heads[cb_index] may be null)");
            return 3;
        }
        e->run_depth(cb_index, prev_token, transformer_out);
        std::memcpy(out_audio_logits, e->depth_logits_host(), sizeof(float) * static_cast<size_t>(e->audio_vocab));
        h->last_error.clear();
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    } catch (...) {
        set_err(h, "bmo_forward_depth: unknown exception");
        return 9;
    }
}

// bmo_forward_depth_cascade, reference bmo_api.cpp:668-743.
int bmo_forward_depth_cascade(bmo_handle_t *h, int32_t text_token, const float *transformer_out, float temp_audio,
                              int top_k_audio, int32_t *out_audio_tokens) {
    if (!h || !transformer_out || !out_audio_tokens) {
        set_err(h, "bmo_forward_depth_cascade: null pointer argument");
        return 1;
    }
    bmo::Engine *e = h->eng.get();
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        if (e->dep_dim <= 0 || !e->has_dep_tables) {
            set_err(h, "bmo_forward_depth_cascade: depformer weights or embedding tables missing");
            return 9;
        }
        for (int cb = 0; cb < e->dep_q; ++cb)
            if (!e->has_dep_head[cb]) {
                set_err(h, "bmo_forward_depth_cascade: audio_logits tensor missing");
                return 3;
            }
        if (top_k_audio <= 0 || temp_audio <= 1e-4f) {
            e->run_cascade_greedy(text_token, transformer_out, out_audio_tokens);
        } else {
            static thread_local std::mt19937 rng(42);
            static thread_local std::vector<std::pair<float, int>> scratch(2048);
            std::vector<float> logits(static_cast<size_t>(std::max(e->audio_vocab, 2049)));
            int32_t prev = text_token;
            e->reset_depth_kv();
            for (int cb = 0; cb < e->dep_q; ++cb) {
                e->run_depth(cb, prev, transformer_out);
                std::memcpy(logits.data(), e->depth_logits_host(), sizeof(float) * static_cast<size_t>(e->audio_vocab));
                if (e->audio_vocab > 2048) logits[2048] = -1e9f;
                const int tok = sample_token(logits.data(), std::min(e->audio_vocab, 2048), temp_audio, top_k_audio,
                                             scratch, rng);
                out_audio_tokens[cb] = tok;
                prev = tok;
            }
        }
        h->last_error.clear();
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    } catch (...) {
        set_err(h, "bmo_forward_depth_cascade: unknown exception");
        return 9;
    }
}

int bmo_forward_frame_greedy(bmo_handle_t *h, const int32_t *input_tokens, int num_codebooks, int pos,
                             float *out_transformer, float *out_text_logits, int32_t *out_text_token,
                             int32_t *out_audio_tokens) {
    if (!h || !input_tokens) {
        set_err(h, "bmo_forward_frame_greedy: null pointer argument");
        return 1;
    }
    bmo::Engine *e = h->eng.get();
    if (num_codebooks <= 0 || num_codebooks > e->num_codebooks || pos < 0) {
        set_err(h, "bmo_forward_frame_greedy: invalid num_codebooks or pos");
        return 2;
    }
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        if (!e->has_text_head || e->dep_dim <= 0 || !e->has_dep_tables) {
            set_err(h, "bmo_forward_frame_greedy: text head or depformer missing");
            return 3;
        }
        e->run_frame_greedy(input_tokens, num_codebooks, pos, out_text_token, out_audio_tokens);
        if (out_transformer) std::memcpy(out_transformer, e->z_host(), sizeof(float) * static_cast<size_t>(e->n_embd));
        if (out_text_logits)
            std::memcpy(out_text_logits, e->logits_host(), sizeof(float) * static_cast<size_t>(e->text_vocab));
        h->pos = pos + 1;
        h->last_error.clear();
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_forward_layers(bmo_handle_t *h, const float *x_in, int pos, int layer_begin, int layer_end, float *x_out) {
    if (!h || !x_in || !x_out) {
        set_err(h, "bmo_forward_layers: null pointer argument");
        return 1;
    }
    bmo::Engine *e = h->eng.get();
    if (pos < 0 || layer_begin < 0 || layer_end > e->n_layers || layer_begin >= layer_end) {
        set_err(h, "bmo_forward_layers: invalid layer range or position");
        return 2;
    }
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        e->run_layers(x_in, pos, layer_begin, layer_end, x_out);
        h->last_error.clear();
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_enqueue_frame(bmo_handle_t *h, const int32_t *tokens_dev, int num_codebooks, int pos,
                      int32_t *out_tokens_dev) {
    if (!h || !tokens_dev) return 1;
    bmo::Engine *e = h->eng.get();
    if (num_codebooks <= 0 || num_codebooks > e->num_codebooks || pos < 0) return 2;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        if (!e->has_text_head || e->dep_dim <= 0 || !e->has_dep_tables) return 3;
        e->enqueue_frame_device(tokens_dev, num_codebooks, pos, out_tokens_dev);
        h->pos = pos + 1;
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_enqueue_temporal(bmo_handle_t *h, const int32_t *tokens_dev, int num_codebooks, int pos) {
    if (!h || !tokens_dev) return 1;
    bmo::Engine *e = h->eng.get();
    if (num_codebooks <= 0 || num_codebooks > e->num_codebooks || pos < 0) return 2;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        e->enqueue_temporal_device(tokens_dev, num_codebooks, pos);
        h->pos = pos + 1;
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_enqueue_cascade(bmo_handle_t *h, int32_t text_token) {
    if (!h) return 1;
    bmo::Engine *e = h->eng.get();
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        if (e->dep_dim <= 0 || !e->has_dep_tables) return 3;
        e->enqueue_cascade_device(text_token);
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_batch_init(bmo_handle_t *h, int n_sessions) {
    if (!h) return 1;
    bmo::Engine *e = h->eng.get();
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        const int rc = e->batch_init(n_sessions);
        if (rc == 1) set_err(h, "bmo_batch_init: session count outside [1, 64]");
        if (rc == 3) set_err(h, "bmo_batch_init: sessions already allocated with another count");
        return rc == 1 ? 2 : rc;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_batch_sessions(bmo_handle_t *h) { return (h && h->eng) ? h->eng->batch_sessions() : 0; }

int bmo_forward_frame_batch(bmo_handle_t *h, int n_rows, const int32_t *sess_ids, const int32_t *input_tokens,
                            int num_codebooks, const int32_t *pos, float *out_transformer, float *out_text_logits,
                            int32_t *out_tokens) {
    if (!h || !input_tokens || !pos || !out_tokens) {
        set_err(h, "bmo_forward_frame_batch: null pointer argument");
        return 1;
    }
    bmo::Engine *e = h->eng.get();
    if (num_codebooks <= 0 || num_codebooks > e->num_codebooks) {
        set_err(h, "bmo_forward_frame_batch: invalid num_codebooks");
        return 2;
    }
    std::lock_guard<std::mutex> lk(h->mu);
    if (n_rows < 1 || n_rows > e->batch_sessions()) {
        set_err(h, "bmo_forward_frame_batch: row count outside [1, sessions] (bmo_batch_init first)");
        return 2;
    }
    try {
        e->run_frame_batch(n_rows, sess_ids, input_tokens, num_codebooks, pos, out_transformer, out_text_logits,
                           out_tokens);
        h->last_error.clear();
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_enqueue_frame_batch(bmo_handle_t *h, int n_rows, const int32_t *sess_ids_dev, const int32_t *tokens_dev,
                            int num_codebooks, const int32_t *pos_dev, int32_t *out_tokens_dev) {
    if (!h || !tokens_dev || !pos_dev) return 1;
    bmo::Engine *e = h->eng.get();
    if (num_codebooks <= 0 || num_codebooks > e->num_codebooks) return 2;
    std::lock_guard<std::mutex> lk(h->mu);
    if (n_rows < 1 || n_rows > e->batch_sessions()) return 2;
    try {
        e->enqueue_frame_batch_device(n_rows, sess_ids_dev, tokens_dev, num_codebooks, pos_dev, out_tokens_dev);
        return 0;
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_batch_kv_import_f32(bmo_handle_t *h, int session, int layer, int slot0, int n, const float *k_rows,
                            const float *v_rows) {
    if (!h || !k_rows || !v_rows) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->batch_kv_import(session, layer, slot0, n, k_rows, v_rows);
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_batch_reset(bmo_handle_t *h, int session) {
    if (!h) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->batch_reset(session);
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

int bmo_sync(bmo_handle_t *h) {
    if (!h) return 1;
    std::lock_guard<std::mutex> lk(h->mu);
    try {
        return h->eng->sync_status();
    } catch (const std::exception &ex) {
        set_err(h, ex.what());
        return 9;
    }
}

}  // extern "C"
