// batch_engine.cpp -- batched sessions: up to kBatchMax independent decode
// sessions stepped together over one weight stream.
//
// Each session owns a temporal KV ring ([layer][kv_head][slot][hd], the
// single-session layout, one ring after another) and its row of every
// activation buffer ([row][dim]).  A batched frame is, per row, exactly the
// single-session greedy frame: embedding sum -> n_layers x {RMSNorm, QKV +
// RoPE + ring append, ring attention, O-proj + residual, RMSNorm, FFN-in +
// SwiGLU, FFN-out + residual} -> out_norm + text head + greedy text token ->
// dep_q depformer steps with greedy chaining.  Every GEMV of the
// single-session path becomes a stage kernel (RMSNorm + Q8_1 of all rows) and
// a skinny GEMM over all rows (kernels/batch.cu).  Rows map to sessions
// through BatchIn::sess, so any subset of sessions can step in one call.
#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>

#include "engine.h"
#include "launch.h"

namespace bmo {

namespace {

void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

struct Engine::BatchState {
    int n_max = 0;
    // temporal rings of every session
    void *k = nullptr, *v = nullptr;
    uint8_t *ks = nullptr, *vs = nullptr;
    long long sess_elems = 0;  // ring elements of one session (all layers)
    size_t plane_bytes = 0, scale_bytes = 0;  // of one session
    // inputs
    BatchIn *in_d = nullptr, *in_h = nullptr;
    // activations, [row][dim]
    float *res[2] = {}, *xmid = nullptr, *q = nullptr, *vraw = nullptr, *attn = nullptr, *act = nullptr;
    float *z = nullptr, *logits = nullptr;
    float2 *rope = nullptr, *tpairs = nullptr;
    int tpairs_stride = 1;
    int8_t *xq = nullptr;
    float *xds = nullptr;
    int *tok = nullptr;
    // depformer, per row
    __half *dk = nullptr, *dv = nullptr;
    long long dsess_elems = 0;
    float *dxa = nullptr, *dxb = nullptr, *dq = nullptr, *dvraw = nullptr, *dattn = nullptr, *dact = nullptr;
    float *dlogits = nullptr;
    float2 *dpairs = nullptr;
    int dpairs_stride = 1;  // per step; a row holds dep_q steps
    int *tok_out = nullptr;  // [row][1 + dep_q]
    // host outputs (pinned)
    int *tok_h = nullptr;
    float *z_h = nullptr, *logits_h = nullptr;
    // tensor-core GEMM: split-row-block partials and their counters
    float *ws = nullptr;
    int *cnt = nullptr;
    int n_cnt = 0;
    int gemm = 1;  // 0 CUDA cores, 1 tensor cores (batch-1 rounding), 2 tensor cores (fp32 block sums)
    std::vector<void *> dev, host;
    std::map<int, cudaGraphExec_t> graphs;  // batched frame by row count
};

void Engine::BatchDeleter::operator()(BatchState *b) const {
    if (!b) return;
    for (auto &g : b->graphs)
        if (g.second) cudaGraphExecDestroy(g.second);
    for (void *p : b->dev) cudaFree(p);
    for (void *p : b->host) cudaFreeHost(p);
    delete b;
}

int Engine::batch_sessions() const { return batch_ ? batch_->n_max : 0; }

void Engine::batch_clear_counters(cudaStream_t s) {
    if (!batch_) return;
    cudaMemsetAsync(batch_->cnt, 0, sizeof(int) * batch_->n_cnt, s);
}

int Engine::batch_init(int n_sessions) {
    if (n_sessions < 1 || n_sessions > kBatchMax) return 1;
    if (batch_) return batch_->n_max == n_sessions ? 0 : 3;
    if (!has_text_head || !has_dep_tables || dep_dim <= 0 || dep_q <= 0)
        throw std::runtime_error("batched frames need the text head and the depformer");
    if (tensor_parallel) throw std::runtime_error("batched frames are not available on a tensor-parallel handle");
    ck(cudaSetDevice(device), "cudaSetDevice");
    std::unique_ptr<BatchState, BatchDeleter> b(new BatchState);
    const int S = kBatchMax;  // activation rows are sized for the largest batch
    auto dalloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        ck(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc batch state");
        b->dev.push_back(p);
        ck(cudaMemset(p, 0, std::max<size_t>(bytes, 16)), "cudaMemset batch state");
        device_bytes += bytes;
        return p;
    };
    auto halloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        ck(cudaHostAlloc(&p, std::max<size_t>(bytes, 16), cudaHostAllocDefault), "cudaHostAlloc batch");
        b->host.push_back(p);
        std::memset(p, 0, std::max<size_t>(bytes, 16));
        return p;
    };
    b->n_max = n_sessions;
    b->sess_elems = static_cast<long long>(n_layers) * n_kv_heads * n_ctx * head_dim;
    if (kv_type == kKvF16) {
        b->plane_bytes = static_cast<size_t>(b->sess_elems) * 2;
    } else {
        b->plane_bytes = static_cast<size_t>(b->sess_elems) / 2;
        b->scale_bytes = static_cast<size_t>(b->sess_elems) / 32 * 2;
        b->ks = static_cast<uint8_t *>(dalloc(b->scale_bytes * n_sessions));
        b->vs = static_cast<uint8_t *>(dalloc(b->scale_bytes * n_sessions));
    }
    b->k = dalloc(b->plane_bytes * n_sessions);
    b->v = dalloc(b->plane_bytes * n_sessions);

    const int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    b->in_d = static_cast<BatchIn *>(dalloc(sizeof(BatchIn)));
    b->in_h = static_cast<BatchIn *>(halloc(sizeof(BatchIn)));
    for (int r = 0; r < 2; ++r) b->res[r] = static_cast<float *>(dalloc(sizeof(float) * S * n_embd));
    b->xmid = static_cast<float *>(dalloc(sizeof(float) * S * n_embd));
    b->q = static_cast<float *>(dalloc(sizeof(float) * S * q_dim));
    b->vraw = static_cast<float *>(dalloc(sizeof(float) * S * kv_dim));
    b->attn = static_cast<float *>(dalloc(sizeof(float) * S * q_dim));
    b->act = static_cast<float *>(dalloc(sizeof(float) * S * ffn));
    b->z = static_cast<float *>(dalloc(sizeof(float) * S * n_embd));
    b->logits = static_cast<float *>(dalloc(sizeof(float) * S * text_vocab));
    b->rope = static_cast<float2 *>(dalloc(sizeof(float2) * S * (head_dim / 2)));
    b->tpairs_stride = std::max(text_head_.n_tiles, 1);
    b->tpairs = static_cast<float2 *>(dalloc(sizeof(float2) * S * b->tpairs_stride));
    // Q8_1 staging for the widest input of any matrix
    int nbx = 0;
    auto widest = [&](const QMatDesc &m) {
        if (m.tiles) nbx = std::max(nbx, m.nbx);
    };
    for (auto &l : L_) { widest(l.qkv); widest(l.wo); widest(l.ffn_in); widest(l.ffn_out); }
    widest(text_head_);
    for (int k = 0; k < kDepQMax; ++k) { widest(dep_in_[k]); widest(dep_head_[k]); }
    for (auto &d : D_)
        for (int s = 0; s < kDepQMax; ++s) { widest(d.qkv[s]); widest(d.wo[s]); widest(d.ffn_in[s]); widest(d.ffn_out[s]); }
    // tensor-core GEMM workspace for the most split matrix
    size_t ws_floats = 0;
    int n_super = 1;
    auto ws_need = [&](const QMatDesc &m) {
        if (!m.tiles) return;
        ws_floats = std::max(ws_floats, batch_mma_ws_floats(m, sm_count));
        n_super = std::max(n_super, (m.n_tiles + 3) / 4);
    };
    for (auto &l : L_) { ws_need(l.qkv); ws_need(l.wo); ws_need(l.ffn_in); ws_need(l.ffn_out); }
    ws_need(text_head_);
    for (int k = 0; k < kDepQMax; ++k) { ws_need(dep_in_[k]); ws_need(dep_head_[k]); }
    for (auto &d : D_)
        for (int s = 0; s < kDepQMax; ++s) { ws_need(d.qkv[s]); ws_need(d.wo[s]); ws_need(d.ffn_in[s]); ws_need(d.ffn_out[s]); }
    b->ws = static_cast<float *>(dalloc(sizeof(float) * ws_floats));
    b->cnt = static_cast<int *>(dalloc(sizeof(int) * n_super));
    b->n_cnt = n_super;
    // BMO_BATCH_GEMM: "tc" (default) tensor cores with the batch-1 rounding,
    // "simt" the CUDA-core form of the same arithmetic, "tc_fast" tensor cores
    // with full-block terms summed in fp32
    const char *mode = std::getenv("BMO_BATCH_GEMM");
    const std::string m = mode ? mode : "tc";
    if (m == "simt") b->gemm = 0;
    else if (m == "tc_fast") b->gemm = 2;
    else if (m == "tc") b->gemm = 1;
    else throw std::runtime_error("BMO_BATCH_GEMM must be tc, tc_fast or simt");
    b->xq = static_cast<int8_t *>(dalloc(static_cast<size_t>(nbx) * S * 64));
    b->xds = static_cast<float *>(dalloc(sizeof(float) * 3 * static_cast<size_t>(nbx) * S));
    b->tok = static_cast<int *>(dalloc(sizeof(int) * S));

    b->dsess_elems = static_cast<long long>(kDepLayers) * dep_heads * std::max(dep_n_ctx, 1) * dep_hd;
    b->dk = static_cast<__half *>(dalloc(sizeof(__half) * S * b->dsess_elems));
    b->dv = static_cast<__half *>(dalloc(sizeof(__half) * S * b->dsess_elems));
    b->dxa = static_cast<float *>(dalloc(sizeof(float) * S * dep_dim));
    b->dxb = static_cast<float *>(dalloc(sizeof(float) * S * dep_dim));
    b->dq = static_cast<float *>(dalloc(sizeof(float) * S * dep_dim));
    b->dvraw = static_cast<float *>(dalloc(sizeof(float) * S * dep_dim));
    b->dattn = static_cast<float *>(dalloc(sizeof(float) * S * dep_dim));
    b->dact = static_cast<float *>(dalloc(sizeof(float) * S * std::max(dep_ffn, 32)));
    b->dlogits = static_cast<float *>(dalloc(sizeof(float) * S * audio_vocab));
    b->dpairs_stride = 1;
    for (int k = 0; k < kDepQMax; ++k) b->dpairs_stride = std::max(b->dpairs_stride, dep_head_[k].n_tiles);
    b->dpairs = static_cast<float2 *>(dalloc(sizeof(float2) * S * dep_q * b->dpairs_stride));
    b->tok_out = static_cast<int *>(dalloc(sizeof(int) * S * (1 + dep_q)));
    b->tok_h = static_cast<int *>(halloc(sizeof(int) * S * (1 + dep_q)));
    b->z_h = static_cast<float *>(halloc(sizeof(float) * S * n_embd));
    b->logits_h = static_cast<float *>(halloc(sizeof(float) * S * text_vocab));
    ck(cudaDeviceSynchronize(), "batch alloc sync");
    batch_ = std::move(b);
    return 0;
}

// ---------------------------------------------------------------------------
// enqueue
// ---------------------------------------------------------------------------
void Engine::batch_stage(cudaStream_t s, int n, const float *x, int cols, const QMatDesc &W, const float *gamma,
                         float *xn_out, const TokenSrc *tok, int pairs_stride, int *tok_out) {
    BatchState &b = *batch_;
    if (W.cols != cols) throw std::runtime_error("internal: batched stage width differs from the matrix");
    BatchStageArgs a{};
    a.x = x;
    a.x_stride = cols;
    a.cols = cols;
    a.nbx = W.nbx;
    a.n_sess = n;
    a.gamma = gamma;
    a.eps = norm_eps;
    a.xn_out = xn_out;
    a.xn_stride = cols;
    a.xq = b.xq;
    a.xds = b.xds;
    if (tok) {
        a.pairs = tok->pairs;
        a.pairs_stride = pairs_stride;
        a.n_pairs = tok->n_pairs;
        a.tok_in = tok->tok;
        a.tok = b.tok;
        a.tok_out = tok_out;
        a.tok_out_stride = 1 + dep_q;
    }
    ck(launch_batch_stage(a, s), "launch batch stage");
}

void Engine::batch_gemm(cudaStream_t s, const BatchGemmArgs &a, int epi) {
    BatchState &b = *batch_;
    if (b.gemm == 0) {
        ck(launch_batch_gemm(a, epi, batch_gemm_grid(a.W, sm_count), s), "launch batch gemm");
        return;
    }
    BatchGemmArgs m = a;
    m.ws = b.ws;
    m.cnt = b.cnt;
    m.max_contrib = batch_mma_max_contrib(a.W, sm_count);
    ck(launch_batch_mma(m, epi, sm_count, b.gemm == 1, s), "launch batch mma");
}

void Engine::enqueue_batch_temporal(cudaStream_t s, int n) {
    BatchState &b = *batch_;
    const int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    ck(launch_batch_embed(ttables_d_, n_ttables_, b.in_d, n_embd, b.res[0], n, rope_theta, head_dim, b.rope, s),
       "launch batch embed");
    // ring attention: one CTA per (head, row), so that a row's arithmetic does
    // not depend on how many rows share the frame
    const int splits = 1;
    auto base = [&](const QMatDesc &W) {
        BatchGemmArgs g{};
        g.W = W;
        g.n_sess = n;
        g.xq = b.xq;
        g.xds = b.xds;
        g.argmax_limit = INT_MAX;
        g.status = status_;
        return g;
    };
    for (int l = 0; l < n_layers; ++l) {
        float *x_in = b.res[l & 1], *x_out = b.res[(l + 1) & 1];
        const long long layer_off = static_cast<long long>(l) * n_kv_heads * n_ctx * head_dim;
        batch_stage(s, n, x_in, n_embd, L_[l].qkv, L_[l].norm1, nullptr, nullptr, 0, nullptr);
        BatchGemmArgs a = base(L_[l].qkv);
        a.y = b.q;
        a.y_stride = q_dim;
        a.q_dim = q_dim;
        a.kv_dim = kv_dim;
        a.head_dim = head_dim;
        a.rope = b.rope;
        a.k_cache = b.k;
        a.v_cache = b.v;
        a.k_scale = b.ks;
        a.v_scale = b.vs;
        a.kv_sess_stride = b.sess_elems;
        a.kv_layer_off = layer_off;
        a.kv_type = kv_type;
        a.n_ctx = n_ctx;
        a.pos = b.in_d->pos;
        a.pos_stride = 1;
        a.ring_of = b.in_d->sess;
        a.v_out = b.vraw;
        a.v_out_stride = kv_dim;
        batch_gemm(s, a, kEpiQKV);

        AttnArgs at{};
        at.q = b.q;
        at.v_raw = b.vraw;
        at.k_cache = b.k;
        at.v_cache = b.v;
        at.k_scale = b.ks;
        at.v_scale = b.vs;
        at.kv_layer_off = layer_off;
        at.n_heads = n_heads;
        at.n_kv_heads = n_kv_heads;
        at.n_ctx = n_ctx;
        at.kv_type = kv_type;
        at.pos = b.in_d->pos;
        at.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
        at.out = b.attn;
        at.status = status_;
        at.kv_sess_stride = b.sess_elems;
        at.qo_stride = q_dim;
        at.vraw_stride = kv_dim;
        at.pos_stride = 1;
        at.ring_of = b.in_d->sess;
        ck(launch_attention(at, head_dim, splits, s, false, n), "launch batch attention");

        batch_stage(s, n, b.attn, q_dim, L_[l].wo, nullptr, nullptr, nullptr, 0, nullptr);
        BatchGemmArgs o = base(L_[l].wo);
        o.y = b.xmid;
        o.y_stride = n_embd;
        o.resid = x_in;
        o.resid_stride = n_embd;
        batch_gemm(s, o, kEpiResid);

        batch_stage(s, n, b.xmid, n_embd, L_[l].ffn_in, L_[l].norm2, nullptr, nullptr, 0, nullptr);
        BatchGemmArgs fi = base(L_[l].ffn_in);
        fi.y = b.act;
        fi.y_stride = ffn;
        batch_gemm(s, fi, kEpiSwiGLU);

        batch_stage(s, n, b.act, ffn, L_[l].ffn_out, nullptr, nullptr, nullptr, 0, nullptr);
        BatchGemmArgs fo = base(L_[l].ffn_out);
        fo.y = x_out;
        fo.y_stride = n_embd;
        fo.resid = b.xmid;
        fo.resid_stride = n_embd;
        batch_gemm(s, fo, kEpiResid);
    }
    // out_norm (normalised vector = z) + text head + per-tile argmax
    batch_stage(s, n, b.res[n_layers & 1], n_embd, text_head_, out_norm_, b.z, nullptr, 0, nullptr);
    BatchGemmArgs h = base(text_head_);
    h.y = b.logits;
    h.y_stride = text_vocab;
    h.bias = text_bias_;
    h.pairs = b.tpairs;
    h.pairs_stride = b.tpairs_stride;
    h.argmax_limit = text_vocab;
    batch_gemm(s, h, kEpiLogits);
}

void Engine::enqueue_batch_cascade(cudaStream_t s, int n) {
    BatchState &b = *batch_;
    const int pstride = dep_q * b.dpairs_stride;  // pairs of one row
    ck(cudaMemsetAsync(b.dk, 0, sizeof(__half) * n * b.dsess_elems, s), "reset batch depth kv");
    ck(cudaMemsetAsync(b.dv, 0, sizeof(__half) * n * b.dsess_elems, s), "reset batch depth kv");
    auto base = [&](const QMatDesc &W) {
        BatchGemmArgs g{};
        g.W = W;
        g.n_sess = n;
        g.xq = b.xq;
        g.xds = b.xds;
        g.argmax_limit = INT_MAX;
        g.status = status_;
        return g;
    };
    for (int cb = 0; cb < dep_q; ++cb) {
        // the step's token: the greedy text token, then the previous step's audio token
        TokenSrc t{};
        int stride;
        if (cb == 0) {
            t.pairs = b.tpairs;
            t.n_pairs = text_head_.n_tiles;
            stride = b.tpairs_stride;
        } else {
            t.pairs = b.dpairs + static_cast<size_t>(cb - 1) * b.dpairs_stride;
            t.n_pairs = dep_head_[cb - 1].n_tiles;
            stride = pstride;
        }
        batch_stage(s, n, b.z, n_embd, dep_in_[cb], nullptr, nullptr, &t, stride, b.tok_out + cb);
        BatchGemmArgs w = base(dep_in_[cb]);
        w.y = b.dxa;
        w.y_stride = dep_dim;
        w.emb = cb == 0 ? dep_text_emb_ : dep_emb_[cb - 1];
        w.tok = b.tok;
        batch_gemm(s, w, kEpiEmbAdd);
        for (int i = 0; i < kDepLayers; ++i) {
            const long long layer_off = static_cast<long long>(i) * dep_heads * dep_n_ctx * dep_hd;
            batch_stage(s, n, b.dxa, dep_dim, D_[i].qkv[cb], D_[i].norm1, nullptr, nullptr, 0, nullptr);
            BatchGemmArgs a = base(D_[i].qkv[cb]);
            a.y = b.dq;
            a.y_stride = dep_dim;
            a.q_dim = dep_dim;
            a.kv_dim = dep_dim;
            a.head_dim = dep_hd;
            a.k_cache = b.dk;
            a.v_cache = b.dv;
            a.kv_sess_stride = b.dsess_elems;
            a.kv_layer_off = layer_off;
            a.kv_type = kKvF16;
            a.n_ctx = dep_n_ctx;
            a.pos = dep_pos_ + cb;
            a.pos_stride = 0;
            a.v_out = b.dvraw;
            a.v_out_stride = dep_dim;
            batch_gemm(s, a, kEpiQKV);

            AttnArgs at{};
            at.q = b.dq;
            at.v_raw = b.dvraw;
            at.k_cache = b.dk;
            at.v_cache = b.dv;
            at.kv_layer_off = layer_off;
            at.n_heads = dep_heads;
            at.n_kv_heads = dep_heads;
            at.n_ctx = dep_n_ctx;
            at.kv_type = kKvF16;
            at.pos = dep_pos_ + cb;
            at.scale = 1.0f / std::sqrt(static_cast<float>(dep_hd));
            at.out = b.dattn;
            at.status = status_;
            at.kv_sess_stride = b.dsess_elems;
            at.qo_stride = dep_dim;
            at.vraw_stride = dep_dim;
            at.pos_stride = 0;
            ck(launch_attention(at, dep_hd, 1, s, false, n), "launch batch depth attention");

            batch_stage(s, n, b.dattn, dep_dim, D_[i].wo[cb], nullptr, nullptr, nullptr, 0, nullptr);
            BatchGemmArgs o = base(D_[i].wo[cb]);
            o.y = b.dxb;
            o.y_stride = dep_dim;
            o.resid = b.dxa;
            o.resid_stride = dep_dim;
            batch_gemm(s, o, kEpiResid);

            batch_stage(s, n, b.dxb, dep_dim, D_[i].ffn_in[cb], D_[i].norm2, nullptr, nullptr, 0, nullptr);
            BatchGemmArgs fi = base(D_[i].ffn_in[cb]);
            fi.y = b.dact;
            fi.y_stride = dep_ffn;
            batch_gemm(s, fi, kEpiSwiGLU);

            batch_stage(s, n, b.dact, dep_ffn, D_[i].ffn_out[cb], nullptr, nullptr, nullptr, 0, nullptr);
            BatchGemmArgs fo = base(D_[i].ffn_out[cb]);
            fo.y = b.dxa;
            fo.y_stride = dep_dim;
            fo.resid = b.dxb;
            fo.resid_stride = dep_dim;
            batch_gemm(s, fo, kEpiResid);
        }
        batch_stage(s, n, b.dxa, dep_dim, dep_head_[cb], nullptr, nullptr, nullptr, 0, nullptr);
        BatchGemmArgs h = base(dep_head_[cb]);
        h.y = b.dlogits;
        h.y_stride = audio_vocab;
        h.pairs = b.dpairs + static_cast<size_t>(cb) * b.dpairs_stride;
        h.pairs_stride = pstride;
        h.argmax_limit = std::min(audio_vocab, 2048);
        batch_gemm(s, h, kEpiLogits);
    }
    ck(launch_batch_finalize(b.dpairs + static_cast<size_t>(dep_q - 1) * b.dpairs_stride, pstride,
                             dep_head_[dep_q - 1].n_tiles, b.tok_out + dep_q, 1 + dep_q, n, s),
       "launch batch finalize");
}

void Engine::enqueue_batch_frame(cudaStream_t s, int n) {
    enqueue_batch_temporal(s, n);
    enqueue_batch_cascade(s, n);
}

// ---------------------------------------------------------------------------
// calls
// ---------------------------------------------------------------------------
static void check_batch_rows(int n, int n_max, int K) {
    if (n < 1 || n > n_max) throw std::runtime_error("batched frame: row count outside [1, sessions]");
    if (K < 0 || K > kBatchMaxTokens) throw std::runtime_error("batched frame: token count outside [0, 64]");
}

void Engine::run_frame_batch(int n, const int32_t *sess_ids, const int32_t *tokens, int K, const int32_t *pos,
                             float *out_z, float *out_logits, int32_t *out_tokens) {
    if (!batch_) throw std::runtime_error("batched frame before batch_init");
    BatchState &b = *batch_;
    check_batch_rows(n, b.n_max, K);
    std::vector<char> seen(b.n_max, 0);
    for (int r = 0; r < n; ++r) {
        const int sid = sess_ids ? sess_ids[r] : r;
        if (sid < 0 || sid >= b.n_max || seen[sid]) throw std::runtime_error("batched frame: bad or repeated session id");
        seen[sid] = 1;
        if (pos[r] < 0) throw std::runtime_error("batched frame: negative position");
    }
    ck(cudaSetDevice(device), "cudaSetDevice");
    for (int r = 0; r < n; ++r) {
        b.in_h->sess[r] = sess_ids ? sess_ids[r] : r;
        b.in_h->pos[r] = pos[r];
        for (int k = 0; k < kBatchMaxTokens; ++k)
            b.in_h->tokens[r * kBatchMaxTokens + k] = k < K ? tokens[static_cast<size_t>(r) * K + k] : 0;
    }
    b.in_h->n_tok = K;
    ck(cudaMemcpyAsync(b.in_d, b.in_h, sizeof(BatchIn), cudaMemcpyHostToDevice, stream), "batch input copy");
    cudaGraphExec_t &g = b.graphs[n];
    launch(g, [this, n](cudaStream_t s) { enqueue_batch_frame(s, n); });
    ck(cudaMemcpyAsync(b.tok_h, b.tok_out, sizeof(int) * n * (1 + dep_q), cudaMemcpyDeviceToHost, stream),
       "batch tokens copy");
    if (out_z)
        ck(cudaMemcpyAsync(b.z_h, b.z, sizeof(float) * n * n_embd, cudaMemcpyDeviceToHost, stream), "batch z copy");
    if (out_logits)
        ck(cudaMemcpyAsync(b.logits_h, b.logits, sizeof(float) * n * text_vocab, cudaMemcpyDeviceToHost, stream),
           "batch logits copy");
    finish_call();
    std::memcpy(out_tokens, b.tok_h, sizeof(int) * n * (1 + dep_q));
    if (out_z) std::memcpy(out_z, b.z_h, sizeof(float) * n * n_embd);
    if (out_logits) std::memcpy(out_logits, b.logits_h, sizeof(float) * n * text_vocab);
}

void Engine::enqueue_frame_batch_device(int n, const int32_t *sess_dev, const int32_t *tokens_dev, int K,
                                        const int32_t *pos_dev, int32_t *out_tokens_dev) {
    if (!batch_) throw std::runtime_error("batched frame before batch_init");
    BatchState &b = *batch_;
    check_batch_rows(n, b.n_max, K);
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(launch_batch_set_inputs(b.in_d, sess_dev, tokens_dev, K, pos_dev, n, stream), "batch set inputs");
    cudaGraphExec_t &g = b.graphs[n];
    launch(g, [this, n](cudaStream_t s) { enqueue_batch_frame(s, n); });
    if (out_tokens_dev)
        ck(cudaMemcpyAsync(out_tokens_dev, b.tok_out, sizeof(int) * n * (1 + dep_q), cudaMemcpyDeviceToDevice, stream),
           "batch tokens copy");
}

int Engine::batch_kv_import(int sess, int layer, int slot0, int n, const float *k_rows, const float *v_rows) {
    if (!batch_ || sess < 0 || sess >= batch_->n_max) return 2;
    BatchState &b = *batch_;
    uint8_t *kc = static_cast<uint8_t *>(b.k) + b.plane_bytes * sess;
    uint8_t *vc = static_cast<uint8_t *>(b.v) + b.plane_bytes * sess;
    uint8_t *ks = b.ks ? b.ks + b.scale_bytes * sess : nullptr;
    uint8_t *vs = b.vs ? b.vs + b.scale_bytes * sess : nullptr;
    return kv_import_into(kc, vc, ks, vs, layer, slot0, n, k_rows, v_rows);
}

int Engine::batch_reset(int sess) {
    if (!batch_ || sess >= batch_->n_max) return 2;
    BatchState &b = *batch_;
    ck(cudaSetDevice(device), "cudaSetDevice");
    const int s0 = sess < 0 ? 0 : sess, cnt = sess < 0 ? b.n_max : 1;
    ck(cudaMemsetAsync(static_cast<uint8_t *>(b.k) + b.plane_bytes * s0, 0, b.plane_bytes * cnt, stream), "batch reset");
    ck(cudaMemsetAsync(static_cast<uint8_t *>(b.v) + b.plane_bytes * s0, 0, b.plane_bytes * cnt, stream), "batch reset");
    if (b.ks) {
        ck(cudaMemsetAsync(b.ks + b.scale_bytes * s0, 0, b.scale_bytes * cnt, stream), "batch reset");
        ck(cudaMemsetAsync(b.vs + b.scale_bytes * s0, 0, b.scale_bytes * cnt, stream), "batch reset");
    }
    ck(cudaStreamSynchronize(stream), "batch reset sync");
    return 0;
}

}  // namespace bmo
