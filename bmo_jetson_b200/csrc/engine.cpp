// engine.cpp -- model loading into HBM, device state, per-frame enqueue
// sequences and CUDA graphs.  See engine.h for the overall structure.
#include "engine.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "launch.h"

extern "C" void bmo_quantize_q4_0_ref(const float *x, long long n, uint8_t *out);

namespace bmo {

namespace {

void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

int env_int(const char *name, int fallback) {
    const char *v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : fallback;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

std::string fmt(const char *f, int i) {
    char b[160];
    std::snprintf(b, sizeof b, f, i);
    return b;
}
std::string fmt2(const char *f, int i, int j) {
    char b[160];
    std::snprintf(b, sizeof b, f, i, j);
    return b;
}

}  // namespace

// ---------------------------------------------------------------------------
// construction
// ---------------------------------------------------------------------------
Engine::Engine(const std::string &gguf_path, const EngineConfig &cfg) : cfg_(cfg) {
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev <= 0) {
        cudaGetLastError();
        throw std::runtime_error("no CUDA device available: libbmo runs the decode step on the GPU only");
    }
    device = cfg.device >= 0 ? cfg.device : env_int("BMO_DEVICE", -1);
    if (device < 0) ck(cudaGetDevice(&device), "cudaGetDevice");
    if (device >= n_dev) throw std::runtime_error("BMO device index out of range");
    ck(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    ck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major < 10) throw std::runtime_error("libbmo is built for sm_100a (B200); this device is sm_" +
                                                  std::to_string(prop.major * 10 + prop.minor));
    sm_count = prop.multiProcessorCount;
    ck(configure_kernels(), "configure kernels");
    ck(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    cfg_.graphs = cfg.graphs && env_int("BMO_GRAPHS", 1) != 0;
    cfg_.pdl = cfg.pdl && env_int("BMO_PDL", 1) != 0;
    n_ctx = cfg.n_ctx > 0 ? cfg.n_ctx : 2048;
    if (n_ctx > attn_max_ctx()) throw std::runtime_error("n_ctx exceeds the ring limit of " + std::to_string(attn_max_ctx()));
    if (cfg.kv_type >= 0) {
        kv_type = cfg.kv_type;
    } else {
        const char *kt = std::getenv("BMO_KV_TYPE");
        kv_type = (kt && (std::strcmp(kt, "q4_0") == 0 || std::strcmp(kt, "q4") == 0)) ? kKvQ4_0 : kKvF16;
    }
    if (cfg.tp_size >= 1) {
        tensor_parallel = true;
        tp_size = cfg.tp_size;
        tp_rank = cfg.tp_rank;
        if (tp_rank < 0 || tp_rank >= tp_size) throw std::runtime_error("tensor parallel: rank outside [0, size)");
    }
    load(gguf_path);
    int want = cfg.semantics;
    if (const char *sem = std::getenv("BMO_SEMANTICS")) {
        if (std::strcmp(sem, "exact") == 0) want = 0;
        else if (std::strcmp(sem, "ref") == 0) want = 1;
    }
    choose_semantics(want);
    if (tensor_parallel) tp_comm_.reset(new TpComm(cfg.tp_id, tp_rank, tp_size));
    alloc_state();
    setup_tp_exchange();
    setup_dep_cascade();
}

int Engine::frame_launches() const {
    int n = 1 + static_cast<int>(ops_temporal().size());  // embed + temporal ops + text head
    if (has_dep_tables && dep_dim > 0 && dep_q > 0) {
        if (dep_cluster_ || dep_grid_) {
            n += 1;
        } else {
            std::vector<FramePhase> v;
            ops_cascade(v, z_, TokenSrc{});
            n += static_cast<int>(v.size());
        }
    }
    return n;
}


// The greedy cascade as one launch when the depformer fits the kernels'
// design (reference order, one GPU, 64-dimension heads, the shared-memory
// and per-op tile limits) and the device can run it; otherwise the per-op
// chain.  Two forms: over every SM with epoch-tagged exchanges in global
// memory (BMO_DEP_GRID=1), or on one thread-block cluster of one CTA per head
// (BMO_FLAG_DEP_CLUSTER / BMO_DEP_CLUSTER=1; measured on B200 for the 7B
// depformer at 1.59-1.67 ms per cascade against 1.19 ms for the per-op
// chain -- on 16 SMs the reference-order dot products are compute- and
// latency-bound).
void Engine::setup_dep_cascade() {
    dep_cluster_ = dep_grid_ = false;
    const bool want_cluster = cfg_.dep_cluster || env_int("BMO_DEP_CLUSTER", 0) != 0;
    const bool want_grid = !want_cluster && env_int("BMO_DEP_GRID", 0) != 0;
    if (!want_cluster && !want_grid) return;
    if (!ref_order_ || tensor_parallel || !has_dep_tables || dep_q <= 0 || dep_q > kDepMaxSteps) return;
    if (dep_hd != dep_cascade_head_dim() || dep_heads < 1 || dep_heads * dep_hd != dep_dim || dep_n_ctx != dep_q)
        return;
    const int grid = want_cluster ? dep_heads : std::min(sm_count, dep_cascade_ll_max_grid());
    if (want_cluster && dep_heads > dep_cascade_max_cluster()) return;
    if (want_grid && dep_heads > grid) return;
    std::vector<DepOp> ops;
    auto add = [&](const QMatDesc &W, int kind, int layer, int step, const float *gamma) {
        DepOp o{};
        o.W = W;
        o.kind = kind;
        o.layer = layer;
        o.step = step;
        o.gamma = gamma;
        ops.push_back(o);
    };
    for (int cb = 0; cb < dep_q; ++cb) {
        if (!has_dep_head[cb]) return;
        add(dep_in_[cb], kDepIn, 0, cb, nullptr);
        for (int i = 0; i < kDepLayers; ++i) {
            add(D_[i].qkv[cb], kDepQKV, i, cb, D_[i].norm1);
            add(D_[i].wo[cb], kDepO, i, cb, nullptr);
            add(D_[i].ffn_in[cb], kDepFfnIn, i, cb, D_[i].norm2);
            add(D_[i].ffn_out[cb], kDepFfnOut, i, cb, nullptr);
        }
        add(dep_head_[cb], kDepHead, 0, cb, nullptr);
    }
    // shapes, tile limits and the RMSNorm-weight prefetch chain
    std::vector<int> norm_ops;
    for (size_t k = 0; k < ops.size(); ++k) {
        DepOp &o = ops[k];
        const QMatDesc &W = o.W;
        const int want_cols = o.kind == kDepIn ? n_embd : o.kind == kDepFfnOut ? dep_ffn : dep_dim;
        const int want_rows = o.kind == kDepQKV ? 3 * dep_dim : o.kind == kDepFfnIn ? 2 * dep_ffn
                            : o.kind == kDepHead ? audio_vocab : dep_dim;
        const int want_perm = o.kind == kDepFfnIn ? kPermSwiGLU : kPermIdentity;
        if (!W.tiles || W.cols != want_cols || W.rows != want_rows || W.perm != want_perm ||
            W.nbx != ((W.cols / 32 + 7) & ~7) || W.cpt * 8 != W.nbx)
            return;
        if (o.kind == kDepFfnIn && W.swiglu_f != dep_ffn) return;
        const int ng = KeyChains::of(W.cols / 32, W.cpt).groups();
        if (want_cluster) {
            const int max_loc = o.kind == kDepQKV ? 3 * dep_hd / kTileRows : (W.n_tiles + grid - 1) / grid;
            if (max_loc * ng > dep_cascade_part_slots() || max_loc > dep_cascade_max_local_tiles()) return;
        } else {
            const int max_loc = (W.n_tiles + grid - 1) / grid;
            if (max_loc * ng > dep_cascade_ll_items() || max_loc > dep_cascade_ll_max_local_tiles()) return;
            if (o.kind != kDepIn && W.cols > dep_cascade_ll_max_in()) return;
        }
        if (o.gamma) {
            if (reinterpret_cast<uintptr_t>(o.gamma) & 15) return;
            o.norm_idx = static_cast<int>(norm_ops.size());
            norm_ops.push_back(static_cast<int>(k));
        }
    }
    for (size_t n = 0; n + 2 < norm_ops.size(); ++n) ops[norm_ops[n]].gamma_ahead = ops[norm_ops[n + 2]].gamma;
    if (dep_dim % 4 || n_embd % 32 || dep_ffn % 32) return;
    const int n_phases = dep_q * (2 + 5 * kDepLayers);
    const int ll_stride = std::max(std::max(3 * dep_dim, dep_ffn), 2 * grid);
    size_t smem = 0;
    if (want_cluster) {
        smem = dep_cascade_smem_bytes(dep_dim, dep_ffn, n_embd, kDepLayers, dep_n_ctx);
        if (dep_cascade_configure(dep_heads, smem) < 1) return;
    } else {
        if (n_phases > dep_cascade_ll_phases() || 2 * grid > dep_cascade_ll_max_in() ||
            static_cast<int>(ops.size()) > dep_cascade_ll_max_ops())
            return;
        // the input projection's activation (n_embd) is quantised through the chain buffers
        const int rows = std::min((n_embd / 32 + 7) / 8, 32);
        if (static_cast<size_t>(8 * (rows * 33 + 32)) * 4 > static_cast<size_t>(dep_cascade_ll_items()) * 2048) return;
        smem = dep_cascade_ll_smem_bytes(dep_dim, dep_ffn, n_embd, kDepLayers, dep_n_ctx);
        if (dep_cascade_ll_configure(smem, sm_count) < grid) return;
    }

    auto dalloc = [&](size_t bytes) -> void * {
        void *q = nullptr;
        ck(cudaMalloc(&q, std::max<size_t>(bytes, 16)), "cudaMalloc depformer cascade");
        ck(cudaMemset(q, 0, std::max<size_t>(bytes, 16)), "cudaMemset depformer cascade");
        allocs_.push_back(q);
        device_bytes += bytes;
        return q;
    };
    dep_ops_d_ = static_cast<DepOp *>(dalloc(sizeof(DepOp) * ops.size()));
    ck(cudaMemcpy(dep_ops_d_, ops.data(), sizeof(DepOp) * ops.size(), cudaMemcpyHostToDevice), "depformer op table");
    DepCascadeArgs &a = dep_args_;
    a = DepCascadeArgs{};
    a.ops = dep_ops_d_;
    a.n_ops = static_cast<int>(ops.size());
    for (int b = 0; b < 2; ++b) a.gamma0[b] = b < static_cast<int>(norm_ops.size()) ? ops[norm_ops[b]].gamma : nullptr;
    for (int cb = 0; cb < dep_q; ++cb) a.emb[cb] = cb == 0 ? dep_text_emb_ : dep_emb_[cb - 1];
    a.n_embd = n_embd;
    a.tok_out = tok_out_;
    a.logits = dlogits_;
    a.logits_stride = audio_vocab;
    a.pairs = dpairs_;
    a.pairs_stride = dpairs_stride_;
    a.k_cache = dk_cache_;
    a.v_cache = dv_cache_;
    a.dep_q = dep_q;
    a.n_layers = kDepLayers;
    a.dim = dep_dim;
    a.ffn = dep_ffn;
    a.heads = dep_heads;
    a.hd = dep_hd;
    a.n_ctx = dep_n_ctx;
    a.argmax_limit = std::min(audio_vocab, 2048);
    a.eps = norm_eps;
    a.scale = 1.0f / std::sqrt(static_cast<float>(dep_hd));
    a.status = status_;
    if (want_grid) {
        a.ll = static_cast<unsigned long long *>(dalloc(sizeof(unsigned long long) * n_phases * ll_stride));
        a.ll_stride = ll_stride;
        a.seq = static_cast<unsigned *>(dalloc(sizeof(unsigned)));
        const unsigned one = 1;  // epoch 0 is what zeroed exchange words carry
        ck(cudaMemcpy(a.seq, &one, sizeof one, cudaMemcpyHostToDevice), "depformer launch counter");
        dep_grid_ctas_ = grid;
        dep_grid_ = true;
    } else {
        dep_cluster_ = true;
    }
    dep_smem_ = smem;
}

// The reference kernels' own fp32 order where everything on the path has a
// reference kernel to follow (fp16 rings, one GPU, shapes those kernels and
// the fused prologue take); otherwise the exact-reduction order.
void Engine::choose_semantics(int want) {
    std::string why;
    const bool dep = has_dep_tables && dep_dim > 0 && dep_q > 0;
    if (kv_type != kKvF16) why = "the KV ring is Q4_0 (the reference's rings are fp16)";
    else if (tensor_parallel) why = "tensor parallel sums partial projections over the ranks";
    else if (!attn_ref_supported(head_dim, n_ctx, true))
        why = "temporal head_dim must be 64 or 128 and n_ctx at most " + std::to_string(attn_ref_max_ctx());
    else if (dep && !attn_ref_supported(dep_hd, dep_n_ctx, dep_n_ctx > 64))
        why = "depformer head_dim must be 64 or 128";
    else if (n_embd > gemv_ref_max_norm_cols() || (dep && dep_dim > gemv_ref_max_norm_cols()))
        why = "normalised widths above " + std::to_string(gemv_ref_max_norm_cols());
    if (want == 1 && !why.empty()) throw std::runtime_error("reference-order semantics unavailable: " + why);
    ref_order_ = want != 0 && why.empty();
}

Engine::~Engine() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    batch_.reset();
    auto drop = [](cudaGraphExec_t &g) {
        if (g) cudaGraphExecDestroy(g);
        g = nullptr;
    };
    drop(g_temporal_);  // graphs holding NCCL calls go before the communicator
    drop(g_layers_);
    drop(g_cascade_z_);
    drop(g_cascade_);
    drop(g_frame_);
    drop(g_loop_);
    for (auto &g : g_depth_) drop(g);
    teardown_tp_exchange();
    tp_comm_.reset();
    for (void *p : allocs_) cudaFree(p);
    for (void *p : {(void *)fin_h_, (void *)z_h_, (void *)logits_h_, (void *)zin_h_, (void *)dlogits_h_,
                    (void *)tok_h_, (void *)status_h_, (void *)loop_in_h_, (void *)loop_out_h_})
        if (p) cudaFreeHost(p);
    if (stream) cudaStreamDestroy(stream);
}

void *Engine::arena(size_t bytes) {
    const size_t off = round_up(arena_used_, 256);
    if (off + bytes > arena_size_) throw std::runtime_error("internal: weight arena overflow");
    arena_used_ = off + bytes;
    return arena_ + off;
}

static size_t q4_tiled_bytes(int64_t rows, int64_t cols, int perm, int swiglu_f) {
    const int64_t nbx = round_up(static_cast<size_t>(cols / 32), kChunkBlocks);
    const int64_t tiles = perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows;
    return static_cast<size_t>(tiles * (nbx / kChunkBlocks) * kChunkBytes);
}

QMatDesc Engine::upload_q4(const GgufTensor *t, int perm, int swiglu_f, int64_t row0, int64_t rows) {
    if (!t) throw std::runtime_error("internal: null weight");
    if (t->type != kTQ4_0) throw std::runtime_error("weight " + t->name + " is not Q4_0 (only Q4_0 GEMV weights are supported)");
    const int64_t cols = t->ne[0];
    if (cols % 32) throw std::runtime_error("weight " + t->name + ": row length not a multiple of 32");
    if (rows < 0) rows = t->rows() - row0;
    if (row0 + rows > t->rows()) throw std::runtime_error("weight " + t->name + ": row slice out of range");
    // a repacked file's tiles, when the slice is whole row tiles of the stored form
    if (t->tiled && t->tiled_perm == perm) {
        const bool whole = row0 == 0 && rows == t->rows();
        const bool ok = perm == kPermSwiGLU
                            ? whole && t->tiled_f == swiglu_f
                            : row0 % kTileRows == 0 && (rows % kTileRows == 0 || row0 + rows == t->rows());
        if (ok) {
            const size_t tile_bytes = static_cast<size_t>(round_up(static_cast<size_t>(cols / 32), kChunkBlocks) /
                                                          kChunkBlocks) * kChunkBytes;
            return upload_q4_tiled(t->name, t->tiled + static_cast<size_t>(row0 / kTileRows) * tile_bytes, rows, cols,
                                   perm, swiglu_f);
        }
    }
    if (!t->data)
        throw std::runtime_error("weight " + t->name + ": this slice needs the raw Q4_0 rows, which the repacked file "
                                 "does not keep (repack with --keep-raw)");
    const size_t row_bytes = static_cast<size_t>(cols / 32) * 18;
    return upload_q4_raw(t->name, t->data + static_cast<size_t>(row0) * row_bytes, rows, cols, perm, swiglu_f);
}

QMatDesc Engine::upload_q4_sel(const GgufTensor *t, int perm, int swiglu_f,
                               const std::vector<std::pair<int64_t, int64_t>> &row_ranges, int64_t col0, int64_t ncols) {
    if (!t) throw std::runtime_error("internal: null weight");
    if (t->type != kTQ4_0) throw std::runtime_error("weight " + t->name + " is not Q4_0 (only Q4_0 GEMV weights are supported)");
    const int64_t cols = t->ne[0];
    if (cols % 32 || col0 % 32 || ncols % 32 || col0 < 0 || ncols <= 0 || col0 + ncols > cols)
        throw std::runtime_error("weight " + t->name + ": column slice not on 32-column blocks");
    if (!t->data)
        throw std::runtime_error("weight " + t->name + ": tensor-parallel shards need the raw Q4_0 rows, which the "
                                 "repacked file does not keep (repack with --keep-raw)");
    int64_t rows = 0;
    for (const auto &r : row_ranges) {
        if (r.first < 0 || r.second <= 0 || r.first + r.second > t->rows())
            throw std::runtime_error("weight " + t->name + ": row slice out of range");
        rows += r.second;
    }
    // gather the selected rows' blocks on the host, then the regular upload + repack
    const size_t src_row = static_cast<size_t>(cols / 32) * 18, dst_row = static_cast<size_t>(ncols / 32) * 18;
    std::vector<uint8_t> host(static_cast<size_t>(rows) * dst_row);
    size_t o = 0;
    for (const auto &r : row_ranges)
        for (int64_t i = 0; i < r.second; ++i, o += dst_row)
            std::memcpy(&host[o], t->data + static_cast<size_t>(r.first + i) * src_row + static_cast<size_t>(col0 / 32) * 18,
                        dst_row);
    return upload_q4_raw(t->name, host.data(), rows, ncols, perm, swiglu_f);
}

QMatDesc Engine::upload_q4_raw(const std::string &name, const uint8_t *src, int64_t rows, int64_t cols, int perm,
                               int swiglu_f) {
    QMatDesc m{};
    m.rows = static_cast<int>(perm == kPermSwiGLU ? 2 * swiglu_f : rows);
    m.cols = static_cast<int>(cols);
    m.nbx = static_cast<int>(round_up(static_cast<size_t>(cols / 32), kChunkBlocks));
    m.cpt = m.nbx / kChunkBlocks;
    m.perm = perm;
    m.swiglu_f = swiglu_f;
    m.n_tiles = static_cast<int>(perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows);
    if (m.nbx > gemv_max_nbx()) throw std::runtime_error("weight " + name + ": row length exceeds the GEMV limit");
    const size_t bytes = static_cast<size_t>(m.n_tiles) * m.cpt * kChunkBytes;
    void *dst = arena(bytes);
    m.tiles = static_cast<const uint8_t *>(dst);
    const size_t raw = static_cast<size_t>(cols / 32) * 18 * static_cast<size_t>(rows);
    if (raw > staging_bytes_) throw std::runtime_error("internal: staging buffer too small");
    ck(cudaMemcpyAsync(staging_d_, src, raw, cudaMemcpyHostToDevice, stream), "upload weight");
    ck(launch_repack_q4_0(staging_d_, dst, static_cast<int>(rows), static_cast<int>(cols), m, stream), "repack");
    ck(cudaStreamSynchronize(stream), "repack sync");
    return m;
}

// A matrix already in the row-tile layout (a repacked file): one copy.
QMatDesc Engine::upload_q4_tiled(const std::string &name, const uint8_t *tiles, int64_t rows, int64_t cols, int perm,
                                 int swiglu_f) {
    QMatDesc m{};
    m.rows = static_cast<int>(perm == kPermSwiGLU ? 2 * swiglu_f : rows);
    m.cols = static_cast<int>(cols);
    m.nbx = static_cast<int>(round_up(static_cast<size_t>(cols / 32), kChunkBlocks));
    m.cpt = m.nbx / kChunkBlocks;
    m.perm = perm;
    m.swiglu_f = swiglu_f;
    m.n_tiles = static_cast<int>(perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows);
    if (m.nbx > gemv_max_nbx()) throw std::runtime_error("weight " + name + ": row length exceeds the GEMV limit");
    const size_t bytes = static_cast<size_t>(m.n_tiles) * m.cpt * kChunkBytes;
    void *dst = arena(bytes);
    m.tiles = static_cast<const uint8_t *>(dst);
    ck(cudaMemcpy(dst, tiles, bytes, cudaMemcpyHostToDevice), "upload tiled weight");
    ++tiled_weights_;
    return m;
}

float *Engine::upload_f32(const GgufTensor *t, int64_t n) {
    if (!t) return nullptr;
    if (t->type != kTF32) throw std::runtime_error("tensor " + t->name + " must be F32");
    if (!t->data) throw std::runtime_error("tensor " + t->name + " has no data in the file");
    if (static_cast<int64_t>(t->nbytes / 4) < n) throw std::runtime_error("tensor " + t->name + " is too short");
    float *d = static_cast<float *>(arena(static_cast<size_t>(n) * 4));
    ck(cudaMemcpy(d, t->data, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice), "upload f32");
    return d;
}

EmbTable Engine::upload_table(const GgufTensor *t) {
    EmbTable e{};
    if (!t) return e;
    switch (t->type) {
    case kTF32: case kTF16: case kTBF16: case kTQ4_0: case kTQ8_0: break;
    default: throw std::runtime_error("embedding table " + t->name + " has an unsupported type");
    }
    if (!t->data) throw std::runtime_error("embedding table " + t->name + " has no raw rows in the file");
    void *d = arena(t->nbytes);
    ck(cudaMemcpy(d, t->data, t->nbytes, cudaMemcpyHostToDevice), "upload table");
    e.data = d;
    e.type = t->type;
    e.rows = static_cast<int>(t->rows());
    e.dim = static_cast<int>(t->ne[0]);
    e.row_bytes = ggml_row_bytes(t->type, t->ne[0]);
    return e;
}

// Tensor-name contract and hyperparameters of the reference loader
// (src/bmo.cpp:285-568).
void Engine::load(const std::string &path) {
    file_.open(path);
    const GgufFile &g = file_;
    auto any = [&](std::initializer_list<std::string> names) -> const GgufTensor * {
        for (const auto &n : names)
            if (const GgufTensor *t = g.find(n)) return t;
        return nullptr;
    };

    n_layers = g.scalar_i32("n_layers", 0);
    if (n_layers <= 0) n_layers = g.scalar_i32("n_layer", 32);
    n_heads = g.scalar_i32("n_heads", 0);
    if (n_heads <= 0) n_heads = g.scalar_i32("n_head", 0);
    n_embd = g.scalar_i32("n_embd", 0);
    if (n_embd <= 0) n_embd = g.scalar_i32("hidden_size", 0);
    head_dim = g.scalar_i32("head_dim", 0);
    if (head_dim <= 0) head_dim = g.scalar_i32("n_embd_head_k", 0);
    rope_theta = g.scalar_f32("rope_theta", 0.0f);
    if (rope_theta <= 0.0f) rope_theta = g.scalar_f32("rope_freq_base", 0.0f);
    if (rope_theta <= 0.0f) rope_theta = 10000.0f;
    norm_eps = g.scalar_f32("norm_eps", 0.0f);
    if (norm_eps <= 0.0f) norm_eps = g.scalar_f32("rms_norm_eps", 0.0f);
    if (norm_eps <= 0.0f) norm_eps = 1e-8f;
    if (n_heads <= 0) n_heads = 32;
    if (n_embd <= 0) n_embd = 4096;
    if (head_dim <= 0) head_dim = n_embd / n_heads;
    if (n_layers <= 0 || n_layers > 1024) throw std::runtime_error("implausible n_layers");

    struct Names { const GgufTensor *qkv, *wo, *fin, *fout, *n1, *n2; };
    std::vector<Names> ln(n_layers);
    for (int i = 0; i < n_layers; ++i) {
        const std::string b = "transformer_layers_" + std::to_string(i);
        ln[i].qkv = any({b + "_self_attn_in_proj_weight", b + "_self_attn_in_proj"});
        ln[i].wo = any({b + "_self_attn_out_proj_weight", b + "_self_attn_out_proj"});
        ln[i].fin = any({b + "_gating_linear_in_weight", b + "_gating_linear_in"});
        ln[i].fout = any({b + "_gating_linear_out_weight", b + "_gating_linear_out"});
        ln[i].n1 = any({b + "_norm1_weight", b + "_attn_norm.weight", b + "_norm1.weight"});
        ln[i].n2 = any({b + "_norm2_weight", b + "_ffn_norm.weight", b + "_norm2.weight"});
        if (!ln[i].qkv || !ln[i].wo || !ln[i].fin || !ln[i].fout)
            throw std::runtime_error("missing temporal weights for " + b);
        if (!ln[i].n1 || !ln[i].n2) throw std::runtime_error("missing per-layer norm weights for " + b);
    }
    const int q_dim = n_heads * head_dim;
    if (ln[0].qkv->ne[0] != n_embd) throw std::runtime_error("QKV width does not match n_embd");
    const int64_t qkv_w = ln[0].qkv->rows();
    if (qkv_w <= q_dim || (qkv_w - q_dim) % 2) throw std::runtime_error("invalid QKV width");
    n_kv_heads = static_cast<int>((qkv_w - q_dim) / 2 / head_dim);
    ffn = static_cast<int>(ln[0].fin->rows() / 2);
    if (n_kv_heads <= 0 || n_heads % n_kv_heads) throw std::runtime_error("invalid KV head count");
    if (head_dim != 64 && head_dim != 128) throw std::runtime_error("head_dim must be 64 or 128");
    if (n_embd % 32 || ffn % 32 || ffn % 16) throw std::runtime_error("n_embd and FFN width must be multiples of 32");

    // depformer (bmo.cpp:376-433)
    const GgufTensor *dep_in_t[kDepQMax] = {}, *dep_emb_t[kDepQMax] = {}, *dep_head_t[kDepQMax] = {};
    for (int k = 0; k < kDepQMax; ++k) {
        dep_in_t[k] = g.find(fmt("depformer_in.%d.weight", k));
        dep_emb_t[k] = g.find(fmt("depformer_emb.%d.weight", k));
        dep_head_t[k] = g.find(fmt("linears.%d.weight", k));
    }
    const GgufTensor *dep_text_t = g.find("depformer_text_emb.weight");
    const GgufTensor *tl = g.find("text_linear.weight");
    const GgufTensor *tb = g.find("text_linear.bias");
    const GgufTensor *on = g.find("out_norm_weight");

    // temporal embeddings (bmo.cpp:491-508): emb.{k} trimmed after the last present
    std::vector<const GgufTensor *> aemb(32, nullptr);
    int last = -1;
    for (int k = 0; k < 32; ++k) {
        aemb[k] = g.find(fmt("emb.%d.weight", k));
        if (aemb[k]) last = k;
    }
    aemb.resize(static_cast<size_t>(last + 1));
    const GgufTensor *temb = g.find("text_emb.weight");

    // geometry (bmo.cpp:510-568)
    int nq = 0, in_vocab = 0;
    for (auto *t : aemb)
        if (t) {
            ++nq;
            if (!in_vocab) in_vocab = static_cast<int>(t->rows());
        }
    if (nq == 0)
        for (auto *t : dep_emb_t)
            if (t) {
                ++nq;
                if (!in_vocab) in_vocab = static_cast<int>(t->rows());
            }
    int dq = 0, out_vocab = 0;
    for (int k = 0; k < kDepQMax; ++k) {
        if (dep_in_t[k]) ++dq;
        if (!out_vocab && dep_head_t[k]) out_vocab = static_cast<int>(dep_head_t[k]->rows());
    }
    n_q = nq;
    num_codebooks = nq > 0 ? nq + 1 : 0;
    dep_q = dq;
    audio_vocab = out_vocab > 0 ? out_vocab : in_vocab;
    text_vocab = tl ? static_cast<int>(tl->rows()) : temb ? static_cast<int>(temb->rows())
               : dep_text_t ? static_cast<int>(dep_text_t->rows()) : 0;
    if (num_codebooks > kMaxTokens) throw std::runtime_error("too many codebooks");

    // depformer geometry: heads from an optional scalar, else the reference's 16
    dep_heads = g.scalar_i32("depformer_num_heads", 16);
    dep_dim = dep_in_t[0] ? static_cast<int>(dep_in_t[0]->rows()) : 0;
    dep_hd = dep_heads > 0 ? dep_dim / dep_heads : 0;
    dep_n_ctx = std::min(dep_q, kDepQMax);
    struct DNames { const GgufTensor *in, *out, *n1, *n2, *gin[kDepQMax], *gout[kDepQMax]; };
    std::vector<DNames> dn(kDepLayers);
    bool dep_ok = dep_q > 0 && dep_dim > 0;
    for (int i = 0; i < kDepLayers && dep_ok; ++i) {
        const std::string dp = "depformer.layers." + std::to_string(i);
        const std::string ub = "depformer_layers_" + std::to_string(i);
        dn[i].n1 = any({dp + ".norm1.weight", ub + "_norm1_weight"});
        dn[i].n2 = any({dp + ".norm2.weight", ub + "_norm2_weight"});
        dn[i].in = any({dp + ".self_attn.in_proj_weight", ub + "_self_attn_in_proj_weight"});
        dn[i].out = any({dp + ".self_attn.out_proj.weight", ub + "_self_attn_out_proj_weight"});
        for (int s = 0; s < kDepQMax; ++s) {
            dn[i].gin[s] = any({fmt2("depformer_layers_%d_gating_%d_linear_in_weight", i, s),
                                fmt2("depformer_layers_%d_gating_%d_linear_in", i, s)});
            dn[i].gout[s] = any({fmt2("depformer_layers_%d_gating_%d_linear_out_weight", i, s),
                                 fmt2("depformer_layers_%d_gating_%d_linear_out", i, s)});
        }
        if (!dn[i].n1 || !dn[i].n2 || !dn[i].in || !dn[i].out) dep_ok = false;
        for (int s = 0; s < dep_q && dep_ok; ++s)
            if (!dn[i].gin[s] || !dn[i].gout[s]) dep_ok = false;
    }
    if (dep_ok) {
        if (dep_hd != 64 && dep_hd != 128) throw std::runtime_error("depformer head_dim must be 64 or 128");
        dep_ffn = static_cast<int>(dn[0].gin[0]->rows() / 2);
        if (dep_ffn % 32) throw std::runtime_error("depformer FFN width must be a multiple of 32");
    } else {
        dep_q = dq;  // geometry still reported; depth calls fail with a clear error
    }

    // ---- tensor parallel: this rank's heads and FFN columns ----
    const int T = tensor_parallel ? tp_size : 1, R = tensor_parallel ? tp_rank : 0;
    const int kv_dim_g = n_kv_heads * head_dim, ffn_g = ffn, dep_ffn_g = dep_ffn;
    if (tensor_parallel) {
        if (n_heads % T || n_kv_heads % T || ffn % (32 * T) || (dep_ok && (dep_heads % T || dep_ffn % (32 * T))))
            throw std::runtime_error("tensor parallel: heads and FFN widths must split into 32-column shards over " +
                                     std::to_string(T) + " ranks");
        n_heads /= T;
        n_kv_heads /= T;
        ffn /= T;
        if (dep_ok) {
            dep_heads /= T;
            dep_ffn /= T;
        }
    }
    const int q_l = n_heads * head_dim, kv_l = n_kv_heads * head_dim;  // this rank's q / kv widths
    const int dq_l = dep_heads * dep_hd;                                  // depformer q width per rank

    // ---- size the weight arena ----
    size_t total = 0, staging = 0;
    auto plan_q4c = [&](const GgufTensor *t, int perm, int f, int64_t rows, int64_t cols) {
        if (!t) return;
        const int64_t r = rows < 0 ? t->rows() : rows, c = cols < 0 ? t->ne[0] : cols;
        total += round_up(q4_tiled_bytes(r, c, perm, f), 256);
        staging = std::max(staging, static_cast<size_t>(r * (c / 32) * 18));
    };
    auto plan_q4 = [&](const GgufTensor *t, int perm, int f, int64_t rows) { plan_q4c(t, perm, f, rows, -1); };
    auto plan_bytes = [&](const GgufTensor *t) {
        if (t) total += round_up(t->nbytes, 256);
    };
    for (int i = 0; i < n_layers; ++i) {
        plan_q4(ln[i].qkv, kPermIdentity, 0, q_l + 2 * kv_l);
        plan_q4c(ln[i].wo, kPermIdentity, 0, -1, q_l);
        plan_q4(ln[i].fin, kPermSwiGLU, ffn, 2LL * ffn);
        plan_q4c(ln[i].fout, kPermIdentity, 0, -1, ffn);
        plan_bytes(ln[i].n1);
        plan_bytes(ln[i].n2);
    }
    plan_q4(tl, kPermIdentity, 0, -1);
    plan_bytes(tb);
    plan_bytes(on);
    plan_bytes(temb);
    for (auto *t : aemb) plan_bytes(t);
    if (dep_ok) {
        for (int k = 0; k < dep_q; ++k) {
            plan_q4(dep_in_t[k], kPermIdentity, 0, -1);
            plan_q4(dep_head_t[k], kPermIdentity, 0, -1);
            plan_bytes(dep_emb_t[k]);
        }
        plan_bytes(dep_text_t);
        for (int i = 0; i < kDepLayers; ++i) {
            for (int s = 0; s < dep_q; ++s) {
                plan_q4(dn[i].in, kPermIdentity, 0, 3LL * dq_l);
                plan_q4c(dn[i].out, kPermIdentity, 0, dep_dim, dq_l);
                plan_q4(dn[i].gin[s], kPermSwiGLU, dep_ffn, 2LL * dep_ffn);
                plan_q4c(dn[i].gout[s], kPermIdentity, 0, -1, dep_ffn);
            }
            plan_bytes(dn[i].n1);
            plan_bytes(dn[i].n2);
        }
    }
    arena_size_ = total + 4096;
    ck(cudaMalloc(&arena_, arena_size_), "cudaMalloc weights");
    allocs_.push_back(arena_);
    staging_bytes_ = std::max<size_t>(staging, 16);
    ck(cudaMalloc(&staging_d_, staging_bytes_), "cudaMalloc staging");

    // ---- upload ----
    L_.resize(n_layers);
    for (int i = 0; i < n_layers; ++i) {
        if (ln[i].fin->rows() != 2LL * ffn_g) throw std::runtime_error("FFN-in width differs between layers");
        if (ln[i].qkv->rows() != qkv_w || ln[i].wo->rows() != n_embd || ln[i].wo->ne[0] != q_dim ||
            ln[i].fout->ne[0] != ffn_g || ln[i].fout->rows() != n_embd)
            throw std::runtime_error("inconsistent temporal weight shapes in layer " + std::to_string(i));
        if (tensor_parallel) {
            // q rows of this rank's heads, then its k rows, then its v rows; O-proj and
            // FFN-out columns of the same heads / FFN slice; FFN-in gate and up rows
            L_[i].qkv = upload_q4_sel(ln[i].qkv, kPermIdentity, 0,
                                      {{static_cast<int64_t>(R) * q_l, q_l},
                                       {q_dim + static_cast<int64_t>(R) * kv_l, kv_l},
                                       {q_dim + kv_dim_g + static_cast<int64_t>(R) * kv_l, kv_l}},
                                      0, n_embd);
            L_[i].wo = upload_q4_sel(ln[i].wo, kPermIdentity, 0, {{0, n_embd}}, static_cast<int64_t>(R) * q_l, q_l);
            L_[i].ffn_in = upload_q4_sel(ln[i].fin, kPermSwiGLU, ffn,
                                         {{static_cast<int64_t>(R) * ffn, ffn}, {ffn_g + static_cast<int64_t>(R) * ffn, ffn}},
                                         0, n_embd);
            L_[i].ffn_out = upload_q4_sel(ln[i].fout, kPermIdentity, 0, {{0, n_embd}}, static_cast<int64_t>(R) * ffn, ffn);
        } else {
            L_[i].qkv = upload_q4(ln[i].qkv, kPermIdentity, 0, 0, -1);
            L_[i].wo = upload_q4(ln[i].wo, kPermIdentity, 0, 0, -1);
            L_[i].ffn_in = upload_q4(ln[i].fin, kPermSwiGLU, ffn, 0, -1);
            L_[i].ffn_out = upload_q4(ln[i].fout, kPermIdentity, 0, 0, -1);
        }
        L_[i].norm1 = upload_f32(ln[i].n1, n_embd);
        L_[i].norm2 = upload_f32(ln[i].n2, n_embd);
    }
    if (tl) {
        if (tl->ne[0] != n_embd) throw std::runtime_error("text_linear width does not match n_embd");
        text_head_ = upload_q4(tl, kPermIdentity, 0, 0, -1);
        has_text_head = true;
    }
    text_bias_ = (tb && tb->type == kTF32 && static_cast<int64_t>(tb->nbytes / 4) >= text_vocab) ? upload_f32(tb, text_vocab)
                                                                                                  : nullptr;
    out_norm_ = on ? upload_f32(on, n_embd) : nullptr;
    std::vector<EmbTable> tt(1 + aemb.size());
    tt[0] = upload_table(temb);
    for (size_t k = 0; k < aemb.size(); ++k) tt[1 + k] = upload_table(aemb[k]);
    n_ttables_ = static_cast<int>(tt.size());
    ttables_d_ = static_cast<EmbTable *>(arena(sizeof(EmbTable) * tt.size()));
    ck(cudaMemcpy(ttables_d_, tt.data(), sizeof(EmbTable) * tt.size(), cudaMemcpyHostToDevice), "upload tables");

    if (dep_ok) {
        for (int k = 0; k < dep_q; ++k) {
            if (dep_in_t[k]) dep_in_[k] = upload_q4(dep_in_t[k], kPermIdentity, 0, 0, -1);
            if (dep_head_t[k]) {
                dep_head_[k] = upload_q4(dep_head_t[k], kPermIdentity, 0, 0, -1);
                has_dep_head[k] = dep_head_[k].cols == dep_dim;
            }
            dep_emb_[k] = upload_table(dep_emb_t[k]);
        }
        dep_text_emb_ = upload_table(dep_text_t);
        has_dep_tables = dep_text_t != nullptr;
        for (int i = 0; i < kDepLayers; ++i) {
            for (int s = 0; s < dep_q; ++s) {
                // per-step row slices of the stacked projections (bmo_compute.cpp:2908-2932)
                if (tensor_parallel) {
                    const int64_t b = 3LL * dep_dim * s, hr = static_cast<int64_t>(R) * dq_l;
                    D_[i].qkv[s] = upload_q4_sel(dn[i].in, kPermIdentity, 0,
                                                 {{b + hr, dq_l}, {b + dep_dim + hr, dq_l}, {b + 2LL * dep_dim + hr, dq_l}},
                                                 0, dep_dim);
                    D_[i].wo[s] = upload_q4_sel(dn[i].out, kPermIdentity, 0, {{static_cast<int64_t>(dep_dim) * s, dep_dim}},
                                                hr, dq_l);
                    D_[i].ffn_in[s] = upload_q4_sel(dn[i].gin[s], kPermSwiGLU, dep_ffn,
                                                    {{static_cast<int64_t>(R) * dep_ffn, dep_ffn},
                                                     {dep_ffn_g + static_cast<int64_t>(R) * dep_ffn, dep_ffn}},
                                                    0, dep_dim);
                    D_[i].ffn_out[s] = upload_q4_sel(dn[i].gout[s], kPermIdentity, 0, {{0, dep_dim}},
                                                     static_cast<int64_t>(R) * dep_ffn, dep_ffn);
                } else {
                    D_[i].qkv[s] = upload_q4(dn[i].in, kPermIdentity, 0, 3LL * dep_dim * s, 3LL * dep_dim);
                    D_[i].wo[s] = upload_q4(dn[i].out, kPermIdentity, 0, static_cast<int64_t>(dep_dim) * s, dep_dim);
                    D_[i].ffn_in[s] = upload_q4(dn[i].gin[s], kPermSwiGLU, dep_ffn, 0, -1);
                    D_[i].ffn_out[s] = upload_q4(dn[i].gout[s], kPermIdentity, 0, 0, -1);
                }
            }
            D_[i].norm1 = upload_f32(dn[i].n1, dep_dim);
            D_[i].norm2 = upload_f32(dn[i].n2, dep_dim);
        }
    } else {
        dep_dim = 0;
    }
    cudaFree(staging_d_);
    staging_d_ = nullptr;
    device_bytes += arena_size_;
}

void Engine::alloc_state() {
    auto dalloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        ck(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc state");
        ck(cudaMemset(p, 0, std::max<size_t>(bytes, 16)), "cudaMemset state");
        allocs_.push_back(p);
        device_bytes += bytes;
        return p;
    };
    const size_t kv_elems = static_cast<size_t>(n_layers) * n_kv_heads * n_ctx * head_dim;
    if (kv_type == kKvF16) {
        kv_plane_bytes_ = kv_elems * 2;
        kv_scale_bytes_ = 0;
    } else {
        kv_plane_bytes_ = kv_elems / 2;
        kv_scale_bytes_ = kv_elems / 32 * 2;
        k_scale_ = static_cast<uint8_t *>(dalloc(kv_scale_bytes_));
        v_scale_ = static_cast<uint8_t *>(dalloc(kv_scale_bytes_));
    }
    k_cache_ = dalloc(kv_plane_bytes_);
    v_cache_ = dalloc(kv_plane_bytes_);

    const int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    resid_ = static_cast<float *>(dalloc(sizeof(float) * n_embd * (n_layers + 1)));
    xmid_ = static_cast<float *>(dalloc(sizeof(float) * n_embd));
    q_ = static_cast<float *>(dalloc(sizeof(float) * q_dim));
    vraw_ = static_cast<float *>(dalloc(sizeof(float) * kv_dim));
    attn_ = static_cast<float *>(dalloc(sizeof(float) * q_dim));
    act_ = static_cast<float *>(dalloc(sizeof(float) * ffn));
    z_ = static_cast<float *>(dalloc(sizeof(float) * n_embd));
    logits_ = static_cast<float *>(dalloc(sizeof(float) * std::max(text_vocab, 1)));
    rope_ = static_cast<float2 *>(dalloc(sizeof(float2) * head_dim / 2));
    tpairs_ = static_cast<float2 *>(dalloc(sizeof(float2) * std::max(text_head_.n_tiles, 1)));

    const int ddim = std::max(dep_dim, 32);
    dkv_bytes_ = static_cast<size_t>(kDepLayers) * dep_heads * std::max(dep_n_ctx, 1) * std::max(dep_hd, 1) * 2;
    dk_cache_ = static_cast<__half *>(dalloc(dkv_bytes_));
    dv_cache_ = static_cast<__half *>(dalloc(dkv_bytes_));
    dz_ = static_cast<float *>(dalloc(sizeof(float) * n_embd));
    dxa_ = static_cast<float *>(dalloc(sizeof(float) * ddim));
    dxb_ = static_cast<float *>(dalloc(sizeof(float) * ddim));
    dq_ = static_cast<float *>(dalloc(sizeof(float) * ddim));
    dvraw_ = static_cast<float *>(dalloc(sizeof(float) * ddim));
    dattn_ = static_cast<float *>(dalloc(sizeof(float) * ddim));
    dact_ = static_cast<float *>(dalloc(sizeof(float) * std::max(dep_ffn, 32)));
    dlogits_ = static_cast<float *>(dalloc(sizeof(float) * kDepQMax * std::max(audio_vocab, 1)));
    dpairs_stride_ = 1;
    for (int k = 0; k < kDepQMax; ++k) dpairs_stride_ = std::max(dpairs_stride_, dep_head_[k].n_tiles);
    dpairs_ = static_cast<float2 *>(dalloc(sizeof(float2) * kDepQMax * dpairs_stride_));
    dep_pos_ = static_cast<int *>(dalloc(sizeof(int) * kDepQMax));
    int dp[kDepQMax];
    for (int k = 0; k < kDepQMax; ++k) dp[k] = k;
    ck(cudaMemcpy(dep_pos_, dp, sizeof dp, cudaMemcpyHostToDevice), "dep pos");
    tok_out_ = static_cast<int *>(dalloc(sizeof(int) * (1 + kDepQMax)));

    // stream-K scratch sized for the largest matrix
    size_t gp = 0, gc = 0;
    auto acc = [&](const QMatDesc &m) {
        if (!m.tiles) return;
        gp = std::max(gp, static_cast<size_t>(m.n_tiles) * (m.cpt + 1) * 32 * sizeof(double));
        gc = std::max(gc, static_cast<size_t>(m.n_tiles) * sizeof(int));
    };
    for (auto &l : L_) { acc(l.qkv); acc(l.wo); acc(l.ffn_in); acc(l.ffn_out); }
    acc(text_head_);
    for (int k = 0; k < kDepQMax; ++k) { acc(dep_in_[k]); acc(dep_head_[k]); }
    for (auto &d : D_)
        for (int s = 0; s < kDepQMax; ++s) { acc(d.qkv[s]); acc(d.wo[s]); acc(d.ffn_in[s]); acc(d.ffn_out[s]); }
    gpart_bytes_ = gp;
    gcount_bytes_ = gc;
    gpart_ = static_cast<double *>(dalloc(gp));
    gcount_ = static_cast<int *>(dalloc(gc));

    tp_part_ = static_cast<double *>(dalloc(sizeof(double) * std::max(n_embd, std::max(dep_dim, 1))));
    attn_splits_ = attn_splits_for(n_ctx);
    status_ =static_cast<int *>(dalloc(sizeof(int)));
    fin_d_ = static_cast<FrameIn *>(dalloc(sizeof(FrameIn)));

    auto halloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        ck(cudaHostAlloc(&p, std::max<size_t>(bytes, 16), cudaHostAllocDefault), "cudaHostAlloc");
        std::memset(p, 0, std::max<size_t>(bytes, 16));
        return p;
    };
    fin_h_ = static_cast<FrameIn *>(halloc(sizeof(FrameIn)));
    z_h_ = static_cast<float *>(halloc(sizeof(float) * n_embd));
    zin_h_ = static_cast<float *>(halloc(sizeof(float) * n_embd));
    logits_h_ = static_cast<float *>(halloc(sizeof(float) * std::max(text_vocab, 1)));
    dlogits_h_ = static_cast<float *>(halloc(sizeof(float) * std::max(audio_vocab, 1)));
    tok_h_ = static_cast<int *>(halloc(sizeof(int) * (1 + kDepQMax)));
    status_h_ = static_cast<int *>(halloc(sizeof(int)));
    ck(cudaDeviceSynchronize(), "alloc sync");
}

// ---------------------------------------------------------------------------
// enqueue sequences
// ---------------------------------------------------------------------------
GemvArgs Engine::gemv_base(const QMatDesc &m) const {
    GemvArgs a{};
    a.W = m;
    a.gpart = gpart_;
    a.gcount = gcount_;
    a.status = status_;
    a.argmax_limit = INT_MAX;
    return a;
}

static FramePhase gemv_op(const GemvArgs &g, int pro, int epi) {
    FramePhase p{};
    p.kind = kPhGemv;
    p.pro = pro;
    p.epi = epi;
    p.g = g;
    return p;
}

// Maps every rank's exchange block into this process through CUDA IPC (the
// handles travel over the NCCL communicator).  All ranks agree: if any rank
// cannot export or map a block, every rank keeps the NCCL path
// (BMO_TP_P2P=0 forces it).
void Engine::setup_tp_exchange() {
    tp_p2p_ = false;
    if (!tensor_parallel || tp_size < 2) return;
    int ok = tp_size <= kTpMaxRanks && std::max(n_embd, dep_dim) <= kTpBufDoubles && env_int("BMO_TP_P2P", 1) != 0;
    cudaIpcMemHandle_t mine{};
    if (ok) {
        ok = cudaMalloc(&tp_block_, kTpBlockBytes) == cudaSuccess &&
             cudaMemset(tp_block_, 0, kTpBlockBytes) == cudaSuccess &&
             cudaIpcGetMemHandle(&mine, tp_block_) == cudaSuccess;
        if (!ok) cudaGetLastError();
    }
    if (!tp_comm_->all_min(ok)) {
        teardown_tp_exchange();
        return;
    }
    std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(tp_size));
    tp_comm_->all_gather_bytes(&mine, all.data(), sizeof mine);
    for (int r = 0; r < tp_size; ++r) {
        if (r == tp_rank) {
            tp_peer_[r] = tp_block_;
        } else if (ok && cudaIpcOpenMemHandle(&tp_peer_[r], all[static_cast<size_t>(r)],
                                              cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            tp_peer_[r] = nullptr;
            ok = 0;
        }
    }
    if (!tp_comm_->all_min(ok)) {  // every rank has mapped every block, or none uses them
        teardown_tp_exchange();
        return;
    }
    void *seq = nullptr;
    ck(cudaMalloc(&seq, sizeof(unsigned long long)), "cudaMalloc exchange count");
    allocs_.push_back(seq);
    ck(cudaMemset(seq, 0, sizeof(unsigned long long)), "cudaMemset exchange count");
    tp_seq_ = static_cast<unsigned long long *>(seq);
    tp_p2p_ = true;
}

// Unmaps the peers' blocks and frees this rank's once every rank is done with
// them (a barrier when the exchange was live).
void Engine::teardown_tp_exchange() {
    if (tp_p2p_ && tp_comm_) {
        try {
            tp_comm_->barrier();
        } catch (...) {
        }
    }
    for (int r = 0; r < kTpMaxRanks; ++r) {
        if (tp_peer_[r] && tp_peer_[r] != tp_block_) cudaIpcCloseMemHandle(tp_peer_[r]);
        tp_peer_[r] = nullptr;
    }
    if (tp_block_) cudaFree(tp_block_);
    tp_block_ = nullptr;
    tp_p2p_ = false;
}

// Tensor parallel: the split projection g (whose output rows are partial over
// the ranks) as a GEMV storing double partials, their sum over the ranks, and
// y = resid + the sum rounded once.  Over peer memory (default): the partials
// go to this rank's exchange buffer `buf` (a layer's two split projections use
// buffers 0 and 1) and one exchange kernel sums every rank's buffer and adds
// the residual; else an NCCL all-reduce and a residual kernel.
void Engine::ops_tp_reduce(std::vector<FramePhase> &v, const GemvArgs &g, const float *resid, float *y, int n,
                           int buf) const {
    GemvArgs p = g;
    if (tp_p2p_) {
        p.ypart = tp_buf(tp_rank, buf);
        v.push_back(gemv_op(p, kProPlain, kEpiPartial));
        FramePhase ex{};
        ex.kind = kPhTpExchange;
        ex.splits = buf;
        ex.g.resid = resid;
        ex.g.y = y;
        ex.count = n;
        v.push_back(ex);
        return;
    }
    p.ypart = tp_part_;
    v.push_back(gemv_op(p, kProPlain, kEpiPartial));
    FramePhase ar{};
    ar.kind = kPhAllReduce;
    ar.g.ypart = tp_part_;
    ar.count = n;
    v.push_back(ar);
    FramePhase ra{};
    ra.kind = kPhResidAdd;
    ra.g.ypart = tp_part_;
    ra.g.resid = resid;
    ra.g.y = y;
    ra.count = n;
    v.push_back(ra);
}

// One temporal layer (bmo_compute.cpp:2188-2640): reads resid[l], writes resid[l+1].
void Engine::ops_layer(std::vector<FramePhase> &v, int l) const {
    const int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    float *x_in = resid_ + static_cast<size_t>(l) * n_embd;
    float *x_out = x_in + n_embd;
    const long long layer_off = static_cast<long long>(l) * n_kv_heads * n_ctx * head_dim;

    GemvArgs a = gemv_base(L_[l].qkv);
    a.x = x_in;
    a.gamma = L_[l].norm1;
    a.eps = norm_eps;
    a.y = q_;
    a.q_dim = q_dim;
    a.kv_dim = kv_dim;
    a.head_dim = head_dim;
    a.rope_cs = rope_;
    a.k_cache = k_cache_;
    a.v_cache = v_cache_;
    a.k_scale = k_scale_;
    a.v_scale = v_scale_;
    a.kv_type = kv_type;
    a.n_ctx = n_ctx;
    a.pos = &fin_d_->pos;
    a.kv_layer_off = layer_off;
    a.v_out = vraw_;
    v.push_back(gemv_op(a, kProNorm, kEpiQKV));

    FramePhase at{};
    at.kind = kPhAttn;
    at.head_dim = head_dim;
    at.splits = ref_order_ ? 8 : attn_splits_;
    at.at.q = q_;
    at.at.v_raw = vraw_;
    at.at.k_cache = k_cache_;
    at.at.v_cache = v_cache_;
    at.at.k_scale = k_scale_;
    at.at.v_scale = v_scale_;
    at.at.kv_layer_off = layer_off;
    at.at.n_heads = n_heads;
    at.at.n_kv_heads = n_kv_heads;
    at.at.n_ctx = n_ctx;
    at.at.kv_type = kv_type;
    at.at.pos = &fin_d_->pos;
    at.at.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
    at.at.out = attn_;
    at.at.status = status_;
    v.push_back(at);

    GemvArgs o = gemv_base(L_[l].wo);
    o.x = attn_;
    o.y = xmid_;
    o.resid = x_in;
    if (tensor_parallel) ops_tp_reduce(v, o, x_in, xmid_, n_embd, 0);
    else v.push_back(gemv_op(o, kProPlain, kEpiResid));

    GemvArgs fi = gemv_base(L_[l].ffn_in);
    fi.x = xmid_;
    fi.gamma = L_[l].norm2;
    fi.eps = norm_eps;
    fi.y = act_;
    v.push_back(gemv_op(fi, kProNorm, kEpiSwiGLU));

    GemvArgs fo = gemv_base(L_[l].ffn_out);
    fo.x = act_;
    fo.y = x_out;
    fo.resid = xmid_;
    if (tensor_parallel) ops_tp_reduce(v, fo, xmid_, x_out, n_embd, 1);
    else v.push_back(gemv_op(fo, kProPlain, kEpiResid));
}

// Output norm, text logits and per-tile argmax (the greedy text token).
void Engine::ops_text_head(std::vector<FramePhase> &v) const {
    GemvArgs h = gemv_base(text_head_);
    h.x = resid_ + static_cast<size_t>(n_layers) * n_embd;
    h.gamma = out_norm_;
    h.eps = norm_eps;
    h.xn_out = z_;
    h.y = logits_;
    h.bias = text_bias_;
    h.argmax_pairs = tpairs_;
    h.argmax_limit = text_vocab;
    v.push_back(gemv_op(h, out_norm_ ? kProNorm : kProPlain, kEpiLogits));
}

std::vector<FramePhase> Engine::ops_temporal() const {
    std::vector<FramePhase> v;
    for (int l = 0; l < n_layers; ++l) ops_layer(v, l);
    if (has_text_head) ops_text_head(v);
    return v;
}

// One depformer codebook step (bmo_build_depth_graph, bmo_compute.cpp:2741-3340).
void Engine::ops_depth_step(std::vector<FramePhase> &v, int cb, const float *z, const TokenSrc &tok) const {
    GemvArgs w = gemv_base(dep_in_[cb]);
    w.x = z;
    w.y = dxa_;
    w.emb = cb == 0 ? dep_text_emb_ : dep_emb_[cb - 1];
    w.tok = tok;
    v.push_back(gemv_op(w, kProPlain, kEpiEmbAdd));
    for (int i = 0; i < kDepLayers; ++i) {
        const long long layer_off = static_cast<long long>(i) * dep_heads * dep_n_ctx * dep_hd;
        GemvArgs a = gemv_base(D_[i].qkv[cb]);
        a.x = dxa_;
        a.gamma = D_[i].norm1;
        a.eps = norm_eps;
        a.y = dq_;
        a.q_dim = dep_heads * dep_hd;  // this rank's heads (all of them without tensor parallelism)
        a.kv_dim = dep_heads * dep_hd;
        a.head_dim = dep_hd;
        a.rope_cs = nullptr;
        a.k_cache = dk_cache_;
        a.v_cache = dv_cache_;
        a.kv_type = kKvF16;
        a.n_ctx = dep_n_ctx;
        a.pos = dep_pos_ + cb;
        a.kv_layer_off = layer_off;
        a.v_out = dvraw_;
        v.push_back(gemv_op(a, kProNorm, kEpiQKV));

        AttnArgs at{};
        at.q = dq_;
        at.v_raw = dvraw_;
        at.k_cache = dk_cache_;
        at.v_cache = dv_cache_;
        at.kv_layer_off = layer_off;
        at.n_heads = dep_heads;
        at.n_kv_heads = dep_heads;
        at.n_ctx = dep_n_ctx;
        at.kv_type = kKvF16;
        at.pos = dep_pos_ + cb;
        at.scale = 1.0f / std::sqrt(static_cast<float>(dep_hd));
        at.out = dattn_;
        at.status = status_;

        GemvArgs o = gemv_base(D_[i].wo[cb]);
        o.x = dattn_;
        o.y = dxb_;
        o.resid = dxa_;
        FramePhase ap{};
        ap.kind = kPhAttn;
        ap.at = at;
        ap.head_dim = dep_hd;
        ap.splits = (ref_order_ && dep_n_ctx > 64) ? 8 : 1;
        v.push_back(ap);
        if (tensor_parallel) ops_tp_reduce(v, o, dxa_, dxb_, dep_dim, 0);
        else v.push_back(gemv_op(o, kProPlain, kEpiResid));

        GemvArgs fi = gemv_base(D_[i].ffn_in[cb]);
        fi.x = dxb_;
        fi.gamma = D_[i].norm2;
        fi.eps = norm_eps;
        fi.y = dact_;
        v.push_back(gemv_op(fi, kProNorm, kEpiSwiGLU));

        GemvArgs fo = gemv_base(D_[i].ffn_out[cb]);
        fo.x = dact_;
        fo.y = dxa_;
        fo.resid = dxb_;
        if (tensor_parallel) ops_tp_reduce(v, fo, dxb_, dxa_, dep_dim, 1);
        else v.push_back(gemv_op(fo, kProPlain, kEpiResid));
    }
    GemvArgs h = gemv_base(dep_head_[cb]);
    h.x = dxa_;
    h.y = dlogits_ + static_cast<size_t>(cb) * audio_vocab;
    h.argmax_pairs = dpairs_ + static_cast<size_t>(cb) * dpairs_stride_;
    h.argmax_limit = std::min(audio_vocab, 2048);
    v.push_back(gemv_op(h, kProPlain, kEpiLogits));
}

// dep_q greedy steps, each step's token the argmax of the previous head,
// then the last step's token.
void Engine::ops_cascade(std::vector<FramePhase> &v, const float *z, const TokenSrc &first) const {
    for (int cb = 0; cb < dep_q; ++cb) {
        TokenSrc t{};
        if (cb == 0) {
            t = first;
            t.tok_out = tok_out_;
        } else {
            t.pairs = dpairs_ + static_cast<size_t>(cb - 1) * dpairs_stride_;
            t.n_pairs = dep_head_[cb - 1].n_tiles;
            t.tok_out = tok_out_ + cb;
        }
        ops_depth_step(v, cb, z, t);
    }
    FramePhase f{};
    f.kind = kPhTokenOut;
    f.tok.pairs = dpairs_ + static_cast<size_t>(dep_q - 1) * dpairs_stride_;
    f.tok.n_pairs = dep_head_[dep_q - 1].n_tiles;
    f.tok.tok_out = tok_out_ + dep_q;
    v.push_back(f);
}

// Per-op path: one kernel per entry, chained by programmatic dependent launch.
void Engine::enqueue_ops(cudaStream_t s, const std::vector<FramePhase> &ops) {
    // The peer-memory exchange lets its dependent launch start early; that is
    // safe only when the next kernel is a GEMV, which waits (griddepcontrol)
    // before it reads the exchange's output or rewrites its partial buffer.
    for (size_t k = 0; k < ops.size(); ++k)
        if (ops[k].kind == kPhTpExchange && k + 1 < ops.size() && ops[k + 1].kind != kPhGemv)
            throw std::runtime_error("internal: a tensor-parallel exchange must be followed by a GEMV");
    for (const FramePhase &op : ops) {
        switch (op.kind) {
        case kPhGemv: {
            if (ref_order_) {
                ck(launch_gemv_ref(op.g, op.pro, op.epi, gemv_ref_grid(op.g.W, sm_count), s, cfg_.pdl), "launch gemv");
                break;
            }
            const GemvPlan p = plan_gemv(op.g.W, sm_count);
            GemvArgs b = op.g;
            b.tile_aligned = p.tile_aligned;
            ck(launch_gemv(b, op.pro, op.epi, p.grid, s, cfg_.pdl), "launch gemv");
            break;
        }
        case kPhAttn:
            if (ref_order_) ck(launch_attention_ref(op.at, op.head_dim, op.splits > 1, s, cfg_.pdl), "launch attention");
            else ck(launch_attention(op.at, op.head_dim, op.splits, s, cfg_.pdl), "launch attention");
            break;
        case kPhTokenOut:
            ck(launch_finalize_token(op.tok.pairs, op.tok.n_pairs, op.tok.tok_out, s, cfg_.pdl), "launch finalize");
            break;
        case kPhAllReduce: tp_comm_->all_reduce_sum(op.g.ypart, static_cast<size_t>(op.count), s); break;
        case kPhResidAdd: ck(launch_tp_resid(op.g.ypart, op.g.resid, op.g.y, op.count, s), "launch tp resid"); break;
        case kPhTpExchange: {
            TpExchangeArgs a{};
            for (int r = 0; r < tp_size; ++r) {
                a.part[r] = tp_buf(r, op.splits);
                a.flag_out[r] =
                    reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(tp_peer_[r]) + kTpFlagOffset) + tp_rank;
            }
            a.flag_in = reinterpret_cast<const unsigned long long *>(static_cast<uint8_t *>(tp_block_) + kTpFlagOffset);
            a.seq = tp_seq_;
            a.resid = op.g.resid;
            a.y = op.g.y;
            a.status = status_;
            a.rank = tp_rank;
            a.size = tp_size;
            a.n = op.count;
            ck(launch_tp_exchange(a, s, cfg_.pdl), "launch tp exchange");
            break;
        }
        default: throw std::runtime_error("internal: unknown op");
        }
    }
}

void Engine::enqueue_embed(cudaStream_t s) {
    ck(launch_embed(ttables_d_, n_ttables_, fin_d_->tokens, &fin_d_->n_tok, n_embd, resid_, &fin_d_->pos, rope_theta,
                    head_dim, rope_, ref_order_, s),
       "launch embed");
}

void Engine::enqueue_temporal(cudaStream_t s) {
    enqueue_embed(s);
    enqueue_ops(s, ops_temporal());
}

void Engine::enqueue_layer(cudaStream_t s, int l) {
    std::vector<FramePhase> v;
    ops_layer(v, l);
    enqueue_ops(s, v);
}

void Engine::enqueue_depth_step(cudaStream_t s, int cb, const float *z, const TokenSrc &tok) {
    std::vector<FramePhase> v;
    ops_depth_step(v, cb, z, tok);
    enqueue_ops(s, v);
}

void Engine::reset_depth_kv_async(cudaStream_t s) {
    ck(cudaMemsetAsync(dk_cache_, 0, dkv_bytes_, s), "reset depth kv");
    ck(cudaMemsetAsync(dv_cache_, 0, dkv_bytes_, s), "reset depth kv");
}

// One greedy frame: the depformer rings are emptied first, so that kernels
// alone run from the text head into the cascade (programmatic launches chain
// them), then the temporal step and the cascade on its hidden state.
void Engine::enqueue_frame_greedy(cudaStream_t s) {
    reset_depth_kv_async(s);
    enqueue_temporal(s);
    TokenSrc t{};
    t.pairs = tpairs_;
    t.n_pairs = text_head_.n_tiles;
    enqueue_cascade(s, z_, t, false);
}

void Engine::enqueue_cascade(cudaStream_t s, const float *z, const TokenSrc &first, bool reset_kv) {
    if (dep_cluster_ || dep_grid_) {
        DepCascadeArgs a = dep_args_;
        a.z = z;
        a.first = first;
        a.first.tok_out = nullptr;
        if (dep_grid_) ck(launch_dep_cascade_ll(a, dep_grid_ctas_, dep_smem_, s), "launch depformer cascade");
        else ck(launch_dep_cascade(a, dep_smem_, s, cfg_.pdl), "launch depformer cascade");
        return;
    }
    if (reset_kv) reset_depth_kv_async(s);
    std::vector<FramePhase> v;
    ops_cascade(v, z, first);
    enqueue_ops(s, v);
}

cudaGraphExec_t Engine::capture(const std::function<void(cudaStream_t)> &fn) {
    cudaGraph_t g = nullptr;
    ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
        fn(stream);
    } catch (...) {
        cudaStreamEndCapture(stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    ck(cudaStreamEndCapture(stream, &g), "end capture");
    cudaGraphExec_t e = nullptr;
    const cudaError_t err = cudaGraphInstantiate(&e, g, 0);
    cudaGraphDestroy(g);
    ck(err, "graph instantiate");
    return e;
}

void Engine::launch(cudaGraphExec_t &g, const std::function<void(cudaStream_t)> &fn) {
    if (!cfg_.graphs) {
        fn(stream);
        return;
    }
    if (!g) g = capture(fn);
    ck(cudaGraphLaunch(g, stream), "graph launch");
}

// Status word back to the host; a raised device error leaves the split
// counters undefined, so they are cleared before the error is reported.
void Engine::finish_call() {
    ck(cudaMemcpyAsync(status_h_, status_, sizeof(int), cudaMemcpyDeviceToHost, stream), "status copy");
    ck(cudaStreamSynchronize(stream), "stream sync");
    if (*status_h_ != 0) {
        const int st = *status_h_;
        cudaMemsetAsync(status_, 0, sizeof(int), stream);
        cudaMemsetAsync(gcount_, 0, gcount_bytes_, stream);
        batch_clear_counters(stream);
        cudaStreamSynchronize(stream);
        std::string what;
        if (st & (1 << 1)) what += " a bulk copy wait timed out;";
        if (st & (1 << 2)) what += " launch arguments inconsistent with the weight layout;";
        if (st & (1 << 4)) what += " a tensor-parallel peer's partial sums did not arrive;";
        throw std::runtime_error("device status " + std::to_string(st) + ":" + what);
    }
}

// ---------------------------------------------------------------------------
// operations
// ---------------------------------------------------------------------------
void Engine::run_temporal(const int32_t *tokens, int K, int pos) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    std::memset(fin_h_->tokens, 0, sizeof(fin_h_->tokens));
    std::memcpy(fin_h_->tokens, tokens, sizeof(int32_t) * static_cast<size_t>(K));
    fin_h_->n_tok = K;
    fin_h_->pos = pos;
    ck(cudaMemcpyAsync(fin_d_, fin_h_, sizeof(FrameIn), cudaMemcpyHostToDevice, stream), "input copy");
    launch(g_temporal_, [this](cudaStream_t s) { enqueue_temporal(s); });
    ck(cudaMemcpyAsync(z_h_, z_, sizeof(float) * n_embd, cudaMemcpyDeviceToHost, stream), "z copy");
    if (has_text_head)
        ck(cudaMemcpyAsync(logits_h_, logits_, sizeof(float) * text_vocab, cudaMemcpyDeviceToHost, stream), "logits copy");
    finish_call();
}

void Engine::copy_resid(int layer, float *out) {
    ck(cudaMemcpy(out, resid_ + static_cast<size_t>(layer + 1) * n_embd, sizeof(float) * n_embd,
                  cudaMemcpyDeviceToHost),
       "capture copy");
}

void Engine::run_layers(const float *x_in, int pos, int layer_begin, int layer_end, float *x_out) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    fin_h_->pos = pos;
    fin_h_->n_tok = 0;
    std::memcpy(zin_h_, x_in, sizeof(float) * n_embd);
    ck(cudaMemcpyAsync(fin_d_, fin_h_, sizeof(FrameIn), cudaMemcpyHostToDevice, stream), "input copy");
    ck(cudaMemcpyAsync(resid_ + static_cast<size_t>(layer_begin) * n_embd, zin_h_, sizeof(float) * n_embd,
                       cudaMemcpyHostToDevice, stream),
       "hidden copy");
    if (g_layers_ && (g_layers_range_[0] != layer_begin || g_layers_range_[1] != layer_end)) {
        cudaGraphExecDestroy(g_layers_);
        g_layers_ = nullptr;
    }
    g_layers_range_[0] = layer_begin;
    g_layers_range_[1] = layer_end;
    launch(g_layers_, [this, layer_begin, layer_end](cudaStream_t s) {
        // RoPE table only (no embedding output)
        ck(launch_embed(ttables_d_, 0, fin_d_->tokens, nullptr, n_embd, nullptr, &fin_d_->pos, rope_theta, head_dim,
                        rope_, ref_order_, s),
           "launch rope");
        for (int l = layer_begin; l < layer_end; ++l) enqueue_layer(s, l);
    });
    ck(cudaMemcpyAsync(z_h_, resid_ + static_cast<size_t>(layer_end) * n_embd, sizeof(float) * n_embd,
                       cudaMemcpyDeviceToHost, stream),
       "hidden out copy");
    finish_call();
    std::memcpy(x_out, z_h_, sizeof(float) * n_embd);
}

void Engine::run_depth(int cb, int32_t prev, const float *z) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    std::memcpy(zin_h_, z, sizeof(float) * n_embd);
    fin_h_->prev_token = prev;
    ck(cudaMemcpyAsync(dz_, zin_h_, sizeof(float) * n_embd, cudaMemcpyHostToDevice, stream), "z in copy");
    ck(cudaMemcpyAsync(fin_d_, fin_h_, sizeof(FrameIn), cudaMemcpyHostToDevice, stream), "input copy");
    launch(g_depth_[cb], [this, cb](cudaStream_t s) {
        if (cb == 0) reset_depth_kv_async(s);
        TokenSrc t{};
        t.tok = &fin_d_->prev_token;
        enqueue_depth_step(s, cb, dz_, t);
    });
    ck(cudaMemcpyAsync(dlogits_h_, dlogits_ + static_cast<size_t>(cb) * audio_vocab, sizeof(float) * audio_vocab,
                       cudaMemcpyDeviceToHost, stream),
       "audio logits copy");
    finish_call();
}

void Engine::run_cascade_greedy(int32_t text_tok, const float *z, int32_t *out_tokens) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    std::memcpy(zin_h_, z, sizeof(float) * n_embd);
    fin_h_->prev_token = text_tok;
    ck(cudaMemcpyAsync(dz_, zin_h_, sizeof(float) * n_embd, cudaMemcpyHostToDevice, stream), "z in copy");
    ck(cudaMemcpyAsync(fin_d_, fin_h_, sizeof(FrameIn), cudaMemcpyHostToDevice, stream), "input copy");
    launch(g_cascade_, [this](cudaStream_t s) {
        TokenSrc t{};
        t.tok = &fin_d_->prev_token;
        enqueue_cascade(s, dz_, t);
    });
    ck(cudaMemcpyAsync(tok_h_, tok_out_, sizeof(int) * (1 + kDepQMax), cudaMemcpyDeviceToHost, stream), "tokens copy");
    finish_call();
    for (int cb = 0; cb < dep_q; ++cb) out_tokens[cb] = tok_h_[1 + cb];
}

void Engine::run_frame_greedy(const int32_t *tokens, int K, int pos, int32_t *out_text_tok, int32_t *out_audio) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    std::memset(fin_h_->tokens, 0, sizeof(fin_h_->tokens));
    std::memcpy(fin_h_->tokens, tokens, sizeof(int32_t) * static_cast<size_t>(K));
    fin_h_->n_tok = K;
    fin_h_->pos = pos;
    ck(cudaMemcpyAsync(fin_d_, fin_h_, sizeof(FrameIn), cudaMemcpyHostToDevice, stream), "input copy");
    launch(g_frame_, [this](cudaStream_t s) { enqueue_frame_greedy(s); });
    ck(cudaMemcpyAsync(z_h_, z_, sizeof(float) * n_embd, cudaMemcpyDeviceToHost, stream), "z copy");
    ck(cudaMemcpyAsync(logits_h_, logits_, sizeof(float) * text_vocab, cudaMemcpyDeviceToHost, stream), "logits copy");
    ck(cudaMemcpyAsync(tok_h_, tok_out_, sizeof(int) * (1 + kDepQMax), cudaMemcpyDeviceToHost, stream), "tokens copy");
    finish_call();
    if (out_text_tok) *out_text_tok = tok_h_[0];
    if (out_audio)
        for (int cb = 0; cb < dep_q; ++cb) out_audio[cb] = tok_h_[1 + cb];
}

void Engine::enqueue_frame_device(const int32_t *tokens_dev, int K, int pos, int32_t *out_tokens_dev) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(launch_set_frame(fin_d_->tokens, &fin_d_->n_tok, &fin_d_->pos, tokens_dev, K, pos, stream), "set frame");
    launch(g_frame_, [this](cudaStream_t s) { enqueue_frame_greedy(s); });
    if (out_tokens_dev)
        ck(cudaMemcpyAsync(out_tokens_dev, tok_out_, sizeof(int) * (1 + dep_q), cudaMemcpyDeviceToDevice, stream),
           "tokens copy");
}

void Engine::enqueue_temporal_device(const int32_t *tokens_dev, int K, int pos) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(launch_set_frame(fin_d_->tokens, &fin_d_->n_tok, &fin_d_->pos, tokens_dev, K, pos, stream), "set frame");
    launch(g_temporal_, [this](cudaStream_t s) { enqueue_temporal(s); });
}

void Engine::enqueue_cascade_device(int32_t text_token) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(launch_set_int(&fin_d_->prev_token, text_token, stream), "set token");
    launch(g_cascade_z_, [this](cudaStream_t s) {
        TokenSrc t{};
        t.tok = &fin_d_->prev_token;
        enqueue_cascade(s, z_, t);
    });
}

// ---------------------------------------------------------------------------
// the caller's frame loop on the device
// ---------------------------------------------------------------------------
bool Engine::loop_supported() const {
    return has_text_head && has_dep_tables && dep_dim > 0 && dep_q == kLoopCb && !tensor_parallel &&
           (num_codebooks == 1 + kLoopCb || num_codebooks == 1 + 2 * kLoopCb);
}

// The daemon's start state (bmo_daemon.cpp:641-647): text pad, audio pads,
// codebook-0 token 1049, std::mt19937 seeded with `seed`.
void Engine::loop_reset(uint32_t seed) {
    if (!loop_supported())
        throw std::runtime_error("frame loop needs a text head, 8 depformer steps, 9 or 17 input channels, one GPU");
    ck(cudaSetDevice(device), "cudaSetDevice");
    if (!loop_st_) {
        void *p = nullptr;
        ck(cudaMalloc(&p, sizeof(LoopState)), "cudaMalloc loop state");
        allocs_.push_back(p);
        loop_st_ = static_cast<LoopState *>(p);
        ck(cudaMallocHost(&loop_in_h_, sizeof(LoopParams) * kLoopRing), "cudaMallocHost loop");
        ck(cudaMallocHost(&loop_out_h_, sizeof(int32_t) * kLoopRing * kLoopOut), "cudaMallocHost loop");
    }
    auto st = std::make_unique<LoopState>();
    std::memset(st.get(), 0, sizeof(LoopState));
    st->prev_text = text_vocab;
    for (int i = 0; i < kLoopCb; ++i) st->prev_audio[i] = st->prev_user[i] = audio_vocab;
    st->prev_cb0 = 1049;
    st->mt[0] = seed;
    for (int i = 1; i < 624; ++i) st->mt[i] = 1812433253u * (st->mt[i - 1] ^ (st->mt[i - 1] >> 30)) + static_cast<unsigned>(i);
    st->mti = 624;
    ck(cudaMemcpy(loop_st_, st.get(), sizeof(LoopState), cudaMemcpyHostToDevice), "loop state copy");
    loop_frame_ = 0;
    reset_kv();
}

bool Engine::loop_params_ok(const LoopParams &in) const {
    if (!in.sampling) return true;
    return std::min(in.top_k_text, std::min(text_vocab, 32000)) <= kLoopTopKMax &&
           std::min(in.top_k_audio, std::min(audio_vocab, 2048)) <= kLoopTopKMax;
}

void Engine::enqueue_loop_frame(cudaStream_t s) {
    LoopConfig c{};
    c.text_n = std::min(text_vocab, 32000);
    c.audio_n = std::min(audio_vocab, 2048);
    c.text_pad = text_vocab;
    c.audio_pad = audio_vocab;
    c.n_tok = num_codebooks;
    ck(launch_loop_begin(loop_st_, c, fin_d_->tokens, &fin_d_->n_tok, &fin_d_->pos, s), "launch loop begin");
    // the depformer rings are emptied here, so that kernels alone run from the
    // text head to the last audio draw (programmatic launches chain them)
    reset_depth_kv_async(s);
    enqueue_temporal(s);
    SampleArgs sa{};
    sa.st = loop_st_;
    sa.mt = loop_st_->mt;
    sa.mti = &loop_st_->mti;
    sa.logits = logits_;
    sa.n = c.text_n;
    sa.text = 1;
    sa.out = &loop_st_->next_text;
    ck(launch_sample(sa, s, cfg_.pdl), "launch text sample");
    for (int cb = 0; cb < dep_q; ++cb) {
        TokenSrc t{};
        t.tok = cb == 0 ? &loop_st_->next_text : &loop_st_->audio[cb - 1];
        enqueue_depth_step(s, cb, z_, t);
        sa.logits = dlogits_ + static_cast<size_t>(cb) * audio_vocab;
        sa.n = c.audio_n;
        sa.text = 0;
        sa.out = &loop_st_->audio[cb];
        ck(launch_sample(sa, s, cfg_.pdl), "launch audio sample");
    }
    ck(launch_loop_end(loop_st_, s), "launch loop end");
}

void Engine::loop_run(int n, const LoopParams *in, int32_t *out) {
    if (!loop_st_) throw std::runtime_error("frame loop not reset");
    if (n < 1 || n > kLoopRing) throw std::runtime_error("frame loop: 1 to 64 frames per call");
    for (int i = 0; i < n; ++i)
        if (!loop_params_ok(in[i])) throw std::runtime_error("frame loop: top-k above 2048");
    ck(cudaSetDevice(device), "cudaSetDevice");
    const int f0 = loop_frame_;
    // this call's inputs into their ring rows (one copy, two when the rows wrap)
    const int r0 = f0 % kLoopRing, first = std::min(n, kLoopRing - r0);
    std::memcpy(loop_in_h_ + r0, in, sizeof(LoopParams) * static_cast<size_t>(first));
    std::memcpy(loop_in_h_, in + first, sizeof(LoopParams) * static_cast<size_t>(n - first));
    ck(cudaMemcpyAsync(loop_st_->in + r0, loop_in_h_ + r0, sizeof(LoopParams) * static_cast<size_t>(first),
                       cudaMemcpyHostToDevice, stream),
       "loop input copy");
    if (n > first)
        ck(cudaMemcpyAsync(loop_st_->in, loop_in_h_, sizeof(LoopParams) * static_cast<size_t>(n - first),
                           cudaMemcpyHostToDevice, stream),
           "loop input copy");
    for (int i = 0; i < n; ++i) launch(g_loop_, [this](cudaStream_t s) { enqueue_loop_frame(s); });
    ck(cudaMemcpyAsync(loop_out_h_ + static_cast<size_t>(r0) * kLoopOut, loop_st_->out[r0],
                       sizeof(int32_t) * kLoopOut * static_cast<size_t>(first), cudaMemcpyDeviceToHost, stream),
       "loop output copy");
    if (n > first)
        ck(cudaMemcpyAsync(loop_out_h_, loop_st_->out[0], sizeof(int32_t) * kLoopOut * static_cast<size_t>(n - first),
                           cudaMemcpyDeviceToHost, stream),
           "loop output copy");
    finish_call();
    loop_frame_ = f0 + n;
    std::memcpy(out, loop_out_h_ + static_cast<size_t>(r0) * kLoopOut, sizeof(int32_t) * kLoopOut * static_cast<size_t>(first));
    std::memcpy(out + static_cast<size_t>(first) * kLoopOut, loop_out_h_,
                sizeof(int32_t) * kLoopOut * static_cast<size_t>(n - first));
}

int Engine::sync_status() {
    ck(cudaSetDevice(device), "cudaSetDevice");
    finish_call();
    return 0;
}

void Engine::capture_all() {
    ck(cudaSetDevice(device), "cudaSetDevice");
    if (!cfg_.graphs) {
        graphs_ready_ = false;
        return;
    }
    auto temporal = [this](cudaStream_t s) { enqueue_temporal(s); };
    if (!g_temporal_) g_temporal_ = capture(temporal);
    if (has_dep_tables && dep_dim > 0) {
        for (int cb = 0; cb < dep_q; ++cb) {
            if (g_depth_[cb]) continue;
            g_depth_[cb] = capture([this, cb](cudaStream_t s) {
                if (cb == 0) reset_depth_kv_async(s);
                TokenSrc t{};
                t.tok = &fin_d_->prev_token;
                enqueue_depth_step(s, cb, dz_, t);
            });
        }
        if (!g_cascade_)
            g_cascade_ = capture([this](cudaStream_t s) {
                TokenSrc t{};
                t.tok = &fin_d_->prev_token;
                enqueue_cascade(s, dz_, t);
            });
        if (!g_frame_ && has_text_head)
            g_frame_ = capture([this](cudaStream_t s) { enqueue_frame_greedy(s); });
    }
    graphs_ready_ = true;
}

void Engine::reset_kv() {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(cudaMemsetAsync(k_cache_, 0, kv_plane_bytes_, stream), "reset kv");
    ck(cudaMemsetAsync(v_cache_, 0, kv_plane_bytes_, stream), "reset kv");
    if (kv_scale_bytes_) {
        ck(cudaMemsetAsync(k_scale_, 0, kv_scale_bytes_, stream), "reset kv");
        ck(cudaMemsetAsync(v_scale_, 0, kv_scale_bytes_, stream), "reset kv");
    }
    ck(cudaStreamSynchronize(stream), "reset sync");
}

void Engine::reset_depth_kv() {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(cudaMemsetAsync(dk_cache_, 0, dkv_bytes_, stream), "reset depth kv");
    ck(cudaMemsetAsync(dv_cache_, 0, dkv_bytes_, stream), "reset depth kv");
    ck(cudaStreamSynchronize(stream), "reset sync");
}

// Host-side conversion of fp32 rows into the ring format, one contiguous
// run of slots per head.
int Engine::kv_import(int layer, int slot0, int n, const float *k_rows, const float *v_rows) {
    return kv_import_into(k_cache_, v_cache_, k_scale_, v_scale_, layer, slot0, n, k_rows, v_rows);
}

int Engine::kv_import_into(void *kc, void *vc, uint8_t *ks, uint8_t *vs, int layer, int slot0, int n,
                           const float *k_rows, const float *v_rows) {
    if (layer < 0 || layer >= n_layers || slot0 < 0 || n <= 0 || slot0 + n > n_ctx) return 2;
    ck(cudaSetDevice(device), "cudaSetDevice");
    const int hd = head_dim;
    std::vector<uint8_t> plane, scales;
    for (int which = 0; which < 2; ++which) {
        const float *src = which ? v_rows : k_rows;
        uint8_t *cache = static_cast<uint8_t *>(which ? vc : kc);
        uint8_t *scale = which ? vs : ks;
        for (int h = 0; h < n_kv_heads; ++h) {
            const size_t row0 = (static_cast<size_t>(layer) * n_kv_heads + h) * n_ctx + slot0;
            std::vector<float> rows(static_cast<size_t>(n) * hd);
            for (int i = 0; i < n; ++i)
                std::memcpy(&rows[static_cast<size_t>(i) * hd], src + (static_cast<size_t>(i) * n_kv_heads + h) * hd,
                            sizeof(float) * hd);
            if (kv_type == kKvF16) {
                std::vector<__half> hv(rows.size());
                for (size_t e = 0; e < rows.size(); ++e) hv[e] = __float2half_rn(rows[e]);
                ck(cudaMemcpy(cache + row0 * hd * 2, hv.data(), hv.size() * 2, cudaMemcpyHostToDevice), "kv import");
            } else {
                std::vector<uint8_t> blocks(rows.size() / 32 * 18);
                bmo_quantize_q4_0_ref(rows.data(), static_cast<long long>(rows.size()), blocks.data());
                plane.assign(rows.size() / 2, 0);
                scales.assign(rows.size() / 32 * 2, 0);
                for (size_t b = 0; b < rows.size() / 32; ++b) {
                    std::memcpy(&scales[b * 2], &blocks[b * 18], 2);
                    std::memcpy(&plane[b * 16], &blocks[b * 18 + 2], 16);
                }
                ck(cudaMemcpy(cache + row0 * hd / 2, plane.data(), plane.size(), cudaMemcpyHostToDevice), "kv import");
                ck(cudaMemcpy(scale + row0 * (hd / 32) * 2, scales.data(), scales.size(), cudaMemcpyHostToDevice),
                   "kv import");
            }
        }
    }
    return 0;
}

int Engine::copy_cache_f32(int which, int layer, int t_start, int n_positions, float *out) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(cudaStreamSynchronize(stream), "sync");
    const int hd = head_dim;
    const uint8_t *cache = static_cast<const uint8_t *>(which ? v_cache_ : k_cache_);
    const uint8_t *scale = which ? v_scale_ : k_scale_;
    int w = 0;
    for (int h = 0; h < n_kv_heads; ++h) {
        const size_t row0 = (static_cast<size_t>(layer) * n_kv_heads + h) * n_ctx + t_start;
        std::vector<float> rows(static_cast<size_t>(n_positions) * hd);
        if (kv_type == kKvF16) {
            std::vector<__half> hv(rows.size());
            ck(cudaMemcpy(hv.data(), cache + row0 * hd * 2, hv.size() * 2, cudaMemcpyDeviceToHost), "kv copy");
            for (size_t e = 0; e < rows.size(); ++e) rows[e] = __half2float(hv[e]);
        } else {
            std::vector<uint8_t> plane(rows.size() / 2);
            std::vector<__half> sc(rows.size() / 32);
            ck(cudaMemcpy(plane.data(), cache + row0 * hd / 2, plane.size(), cudaMemcpyDeviceToHost), "kv copy");
            ck(cudaMemcpy(sc.data(), scale + row0 * (hd / 32) * 2, sc.size() * 2, cudaMemcpyDeviceToHost), "kv copy");
            for (size_t b = 0; b < sc.size(); ++b) {
                const float d = __half2float(sc[b]);
                for (int j = 0; j < 16; ++j) {
                    rows[b * 32 + j] = static_cast<float>((plane[b * 16 + j] & 0x0F) - 8) * d;
                    rows[b * 32 + 16 + j] = static_cast<float>((plane[b * 16 + j] >> 4) - 8) * d;
                }
            }
        }
        for (int p = 0; p < n_positions; ++p)
            std::memcpy(out + (static_cast<size_t>(p) * n_kv_heads + h) * hd, &rows[static_cast<size_t>(p) * hd],
                        sizeof(float) * hd);
        w += n_positions * hd;
    }
    return w;
}

int Engine::debug_tap(int which, float *out, int max_floats) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(cudaStreamSynchronize(stream), "sync");
    const float *src = nullptr;
    int n = 0;
    switch (which) {
    case 0: src = q_; n = n_heads * head_dim; break;
    case 1: src = vraw_; n = n_kv_heads * head_dim; break;
    case 2: src = attn_; n = n_heads * head_dim; break;
    case 3: src = xmid_; n = n_embd; break;
    case 4: src = act_; n = ffn; break;
    case 5: src = z_; n = n_embd; break;
    case 6: src = reinterpret_cast<const float *>(rope_); n = head_dim; break;
    case 7: src = dlogits_; n = dep_q * audio_vocab; break;
    default: return -1;
    }
    if (n > max_floats) return -1;
    ck(cudaMemcpy(out, src, sizeof(float) * n, cudaMemcpyDeviceToHost), "debug tap");
    return n;
}

long long Engine::copy_kv_raw(int which, int part, int layer, void *out, long long max_bytes) {
    ck(cudaSetDevice(device), "cudaSetDevice");
    ck(cudaStreamSynchronize(stream), "sync");
    const size_t layer_elems = static_cast<size_t>(n_kv_heads) * n_ctx * head_dim;
    const uint8_t *src;
    size_t bytes;
    if (part == 0) {
        const size_t per = kv_type == kKvF16 ? layer_elems * 2 : layer_elems / 2;
        src = static_cast<const uint8_t *>(which ? v_cache_ : k_cache_) + per * layer;
        bytes = per;
    } else {
        if (kv_type == kKvF16) return 0;
        const size_t per = layer_elems / 32 * 2;
        src = (which ? v_scale_ : k_scale_) + per * layer;
        bytes = per;
    }
    if (static_cast<long long>(bytes) > max_bytes) return -2;
    ck(cudaMemcpy(out, src, bytes, cudaMemcpyDeviceToHost), "kv raw copy");
    return static_cast<long long>(bytes);
}

}  // namespace bmo
