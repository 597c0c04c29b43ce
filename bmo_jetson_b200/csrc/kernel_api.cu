// kernel_api.cu -- the device-pointer kernel layer (include/bmo_kernels.h).
#include <climits>

#include "../../include/bmo_kernels.h"
#include "kernels/common.cuh"
#include "launch.h"

namespace bmo {
namespace {

QMatDesc make_desc(const void *tiles, int rows, int cols, int perm, int swiglu_f) {
    QMatDesc m{};
    m.tiles = static_cast<const uint8_t *>(tiles);
    m.rows = perm == kPermSwiGLU ? 2 * swiglu_f : rows;
    m.cols = cols;
    m.nbx = ((cols / 32) + kChunkBlocks - 1) / kChunkBlocks * kChunkBlocks;
    m.cpt = m.nbx / kChunkBlocks;
    m.perm = perm;
    m.swiglu_f = swiglu_f;
    m.n_tiles = perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows;
    return m;
}

bool shape_ok(int rows, int cols, int perm, int swiglu_f) {
    if (cols <= 0 || cols % 32) return false;
    if (perm == kPermSwiGLU) return swiglu_f > 0 && swiglu_f % 16 == 0 && rows == 2 * swiglu_f;
    return perm == kPermIdentity && rows > 0;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Appends one token's K and V (fp32 [n_kv][hd]) at ring slot pos % n_ctx:
// one warp per 32-element block, fp16 rows or Q4_0 blocks (the same
// conversions as the QKV epilogue of the GEMV).
__global__ void kv_append_kernel(const float *k, const float *v, void *k_cache, void *v_cache, uint8_t *k_scale,
                                 uint8_t *v_scale, int n_kv, int hd, int n_ctx, const int *pos, long long layer_off,
                                 int kv_type) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int blocks = n_kv * hd / 32;
    if (warp >= 2 * blocks) return;
    const bool is_v = warp >= blocks;
    const int b = is_v ? warp - blocks : warp;
    const int kh = (b * 32) / hd, d = (b * 32) % hd + lane;
    const float x = (is_v ? v : k)[kh * hd + d];
    const int slot = *pos % n_ctx;
    const long long e = layer_off + (static_cast<long long>(kh) * n_ctx + slot) * hd + d;
    void *cache = is_v ? v_cache : k_cache;
    if (kv_type == kKvF16) {
        static_cast<__half *>(cache)[e] = __float2half_rn(x);
    } else {
        const long long e0 = e - lane;
        warp_store_q4_0(x, lane, static_cast<uint8_t *>(cache) + e0 / 2,
                        reinterpret_cast<__half *>(is_v ? v_scale : k_scale) + e0 / 32);
    }
}

}  // namespace
}  // namespace bmo

namespace bmo {
// The argument rules of bmo_k_gemv_q4_0 other than the scratch: pointers,
// shape, activation length and alignment (shared with the fixed-scratch entry
// point, which must reject a call before it touches its shared buffer).
bool gemv_kernel_args_ok(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f, const float *x_dev,
                         const float *gamma_dev, const float *y_dev, const float *xn_out_dev) {
    if (!tiled_dev || !x_dev || !y_dev || !shape_ok(rows, cols, perm, swiglu_f)) return false;
    const QMatDesc m = make_desc(nullptr, rows, cols, perm, swiglu_f);
    if (m.nbx > gemv_max_nbx() || (gamma_dev && cols > gemv_max_norm_cols())) return false;
    return !(reinterpret_cast<uintptr_t>(x_dev) & 15) && !(reinterpret_cast<uintptr_t>(xn_out_dev) & 15);
}
}  // namespace bmo

using namespace bmo;

extern "C" {

int bmo_k_quantize_q8_1(const float *x_dev, void *out_dev, int n, void *stream) {
    if (!x_dev || !out_dev || n < 0 || n % 32) return static_cast<int>(cudaErrorInvalidValue);
    return static_cast<int>(launch_quantize_q8_1(x_dev, out_dev, n, static_cast<cudaStream_t>(stream)));
}

size_t bmo_k_q4_0_tiled_bytes(int rows, int cols, int perm, int swiglu_f) {
    if (!shape_ok(rows, cols, perm, swiglu_f)) return 0;
    const QMatDesc m = make_desc(nullptr, rows, cols, perm, swiglu_f);
    return static_cast<size_t>(m.n_tiles) * m.cpt * kChunkBytes;
}

int bmo_k_repack_q4_0(const void *ggml_dev, void *tiled_dev, int rows, int cols, int perm, int swiglu_f,
                      void *stream) {
    if (!ggml_dev || !tiled_dev || !shape_ok(rows, cols, perm, swiglu_f)) return static_cast<int>(cudaErrorInvalidValue);
    const QMatDesc m = make_desc(tiled_dev, rows, cols, perm, swiglu_f);
    return static_cast<int>(launch_repack_q4_0(ggml_dev, tiled_dev, rows, cols, m, static_cast<cudaStream_t>(stream)));
}

size_t bmo_k_gemv_scratch_bytes(int rows, int cols, int perm, int swiglu_f) {
    if (!shape_ok(rows, cols, perm, swiglu_f)) return 0;
    const QMatDesc m = make_desc(nullptr, rows, cols, perm, swiglu_f);
    return align256(static_cast<size_t>(m.n_tiles) * (m.cpt + 1) * 32 * sizeof(double)) +
           align256(static_cast<size_t>(m.n_tiles) * sizeof(int)) + 256;
}


int bmo_k_gemv_q4_0(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f, const float *x_dev,
                    const float *gamma_dev, float eps, const float *resid_dev, float *y_dev, void *q8_out_dev,
                    float *xn_out_dev, void *scratch_dev, size_t scratch_bytes, int grid, void *stream) {
    if (!scratch_dev || !gemv_kernel_args_ok(tiled_dev, rows, cols, perm, swiglu_f, x_dev, gamma_dev, y_dev, xn_out_dev))
        return static_cast<int>(cudaErrorInvalidValue);
    if (scratch_bytes < bmo_k_gemv_scratch_bytes(rows, cols, perm, swiglu_f)) return static_cast<int>(cudaErrorInvalidValue);
    const QMatDesc m = make_desc(tiled_dev, rows, cols, perm, swiglu_f);
    GemvArgs a{};
    a.W = m;
    a.x = x_dev;
    a.gamma = gamma_dev;
    a.eps = eps;
    a.xn_out = xn_out_dev;
    a.q8_out = static_cast<uint8_t *>(q8_out_dev);
    a.y = y_dev;
    a.resid = resid_dev;
    a.argmax_limit = INT_MAX;
    uint8_t *s = static_cast<uint8_t *>(scratch_dev);
    a.gpart = reinterpret_cast<double *>(s);
    a.gcount = reinterpret_cast<int *>(s + align256(static_cast<size_t>(m.n_tiles) * (m.cpt + 1) * 32 * sizeof(double)));
    a.status = a.gcount + m.n_tiles;  // last word of the scratch block
    const long long nc = static_cast<long long>(m.n_tiles) * m.cpt;
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long g;
    if (grid > 0) {  // caller-chosen grid: even (stream-K) split
        g = grid;
        const long long need = (m.n_tiles + gemv_max_tiles_per_cta() - 3) / (gemv_max_tiles_per_cta() - 2);
        if (g < need) g = need < nc ? need : nc;
        if (g > nc) g = nc;
        a.tile_aligned = 0;
    } else {
        const GemvPlan p = plan_gemv(m, sms);
        g = p.grid;
        a.tile_aligned = p.tile_aligned;
    }
    const int pro = gamma_dev ? kProNorm : kProPlain;
    const int epi = perm == kPermSwiGLU ? kEpiSwiGLU : (resid_dev ? kEpiResid : kEpiStore);
    return static_cast<int>(launch_gemv(a, pro, epi, static_cast<int>(g), static_cast<cudaStream_t>(stream), false));
}

int bmo_k_gemv_q4_0_ref(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f, const float *x_dev,
                        const float *gamma_dev, float eps, const float *resid_dev, float *y_dev, void *q8_out_dev,
                        float *xn_out_dev, int *status_dev, void *stream) {
    if (!tiled_dev || !x_dev || !y_dev || !shape_ok(rows, cols, perm, swiglu_f))
        return static_cast<int>(cudaErrorInvalidValue);
    if (cols / 32 > gemv_max_nbx() * kChunkBlocks || (gamma_dev && cols > gemv_ref_max_norm_cols()))
        return static_cast<int>(cudaErrorInvalidValue);
    if ((reinterpret_cast<uintptr_t>(x_dev) & 15) || (reinterpret_cast<uintptr_t>(xn_out_dev) & 15))
        return static_cast<int>(cudaErrorInvalidValue);
    const QMatDesc m = make_desc(tiled_dev, rows, cols, perm, swiglu_f);
    GemvArgs a{};
    a.W = m;
    a.x = x_dev;
    a.gamma = gamma_dev;
    a.eps = eps;
    a.xn_out = xn_out_dev;
    a.q8_out = static_cast<uint8_t *>(q8_out_dev);
    a.y = y_dev;
    a.resid = resid_dev;
    a.argmax_limit = INT_MAX;
    a.status = status_dev;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int pro = gamma_dev ? kProNorm : kProPlain;
    const int epi = perm == kPermSwiGLU ? kEpiSwiGLU : (resid_dev ? kEpiResid : kEpiStore);
    return static_cast<int>(
        launch_gemv_ref(a, pro, epi, gemv_ref_grid(m, sms), static_cast<cudaStream_t>(stream), false));
}

namespace {
struct BatchScratch {
    size_t xq, xds, ws, cnt, status, total;
};
BatchScratch batch_scratch_layout(const QMatDesc &m, int n_sess, int sms) {
    BatchScratch b{};
    const size_t P = static_cast<size_t>(batch_pad(n_sess));
    b.xq = 0;
    b.xds = align256(static_cast<size_t>(m.nbx) * P * 64);
    b.ws = b.xds + align256(static_cast<size_t>(m.nbx) * P * 3 * sizeof(float));
    b.cnt = b.ws + align256(batch_mma_ws_floats(m, sms) * sizeof(float));
    b.status = b.cnt + align256(static_cast<size_t>(m.n_tiles) * sizeof(int));
    b.total = b.status + 256;
    return b;
}
int device_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}
}  // namespace

size_t bmo_k_batch_gemm_scratch_bytes(int rows, int cols, int perm, int swiglu_f, int n_sess) {
    if (!shape_ok(rows, cols, perm, swiglu_f) || n_sess < 1 || n_sess > kBatchMax) return 0;
    return batch_scratch_layout(make_desc(nullptr, rows, cols, perm, swiglu_f), n_sess, device_sms()).total;
}

int bmo_k_batch_gemm_q4_0(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f, const float *x_dev,
                          const float *gamma_dev, float eps, const float *resid_dev, float *y_dev, int n_sess,
                          int tensor_cores, void *scratch_dev, size_t scratch_bytes, void *stream) {
    if (!tiled_dev || !x_dev || !y_dev || !scratch_dev || !shape_ok(rows, cols, perm, swiglu_f) || n_sess < 1 ||
        n_sess > kBatchMax)
        return static_cast<int>(cudaErrorInvalidValue);
    const int sms = device_sms();
    const QMatDesc m = make_desc(tiled_dev, rows, cols, perm, swiglu_f);
    const BatchScratch L = batch_scratch_layout(m, n_sess, sms);
    if (scratch_bytes < L.total) return static_cast<int>(cudaErrorInvalidValue);
    uint8_t *sc = static_cast<uint8_t *>(scratch_dev);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    BatchStageArgs st{};
    st.x = x_dev;
    st.x_stride = cols;
    st.cols = cols;
    st.nbx = m.nbx;
    st.n_sess = n_sess;
    st.gamma = gamma_dev;
    st.eps = eps;
    st.xq = reinterpret_cast<int8_t *>(sc + L.xq);
    st.xds = reinterpret_cast<float *>(sc + L.xds);
    cudaError_t e = launch_batch_stage(st, s);
    if (e != cudaSuccess) return static_cast<int>(e);
    BatchGemmArgs a{};
    a.W = m;
    a.n_sess = n_sess;
    a.xq = st.xq;
    a.xds = st.xds;
    a.y = y_dev;
    a.y_stride = perm == kPermSwiGLU ? swiglu_f : rows;
    a.resid = resid_dev;
    a.resid_stride = rows;
    a.argmax_limit = INT_MAX;
    a.status = reinterpret_cast<int *>(sc + L.status);
    a.ws = reinterpret_cast<float *>(sc + L.ws);
    a.cnt = reinterpret_cast<int *>(sc + L.cnt);
    a.max_contrib = batch_mma_max_contrib(m, sms);
    const int epi = perm == kPermSwiGLU ? kEpiSwiGLU : (resid_dev ? kEpiResid : kEpiStore);
    e = tensor_cores ? launch_batch_mma(a, epi, sms, tensor_cores == 1, s)
                     : launch_batch_gemm(a, epi, batch_gemm_grid(m, sms), s);
    return static_cast<int>(e);
}

int bmo_k_decode_attention(const float *q_dev, const float *k_dev, const float *v_dev, void *k_cache_dev,
                           void *v_cache_dev, void *k_scale_dev, void *v_scale_dev, float *out_dev, int head_dim,
                           int n_heads, int n_kv_heads, int n_ctx, const int *pos_dev, int layer, int kv_type,
                           void *stream) {
    if (!q_dev || !k_dev || !v_dev || !k_cache_dev || !v_cache_dev || !out_dev || !pos_dev)
        return static_cast<int>(cudaErrorInvalidValue);
    if ((head_dim != 64 && head_dim != 128) || n_kv_heads <= 0 || n_heads % n_kv_heads || n_ctx <= 0 ||
        n_ctx > attn_max_ctx() || layer < 0)
        return static_cast<int>(cudaErrorInvalidValue);
    if (kv_type == kKvQ4_0 && (!k_scale_dev || !v_scale_dev)) return static_cast<int>(cudaErrorInvalidValue);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long layer_off = static_cast<long long>(layer) * n_kv_heads * n_ctx * head_dim;
    const int warps = 2 * n_kv_heads * head_dim / 32;
    kv_append_kernel<<<(warps * 32 + 127) / 128, 128, 0, s>>>(
        k_dev, v_dev, k_cache_dev, v_cache_dev, static_cast<uint8_t *>(k_scale_dev), static_cast<uint8_t *>(v_scale_dev),
        n_kv_heads, head_dim, n_ctx, pos_dev, layer_off, kv_type);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
    AttnArgs a{};
    a.q = q_dev;
    a.v_raw = v_dev;
    a.k_cache = k_cache_dev;
    a.v_cache = v_cache_dev;
    a.k_scale = static_cast<const uint8_t *>(k_scale_dev);
    a.v_scale = static_cast<const uint8_t *>(v_scale_dev);
    a.kv_layer_off = layer_off;
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    a.n_ctx = n_ctx;
    a.kv_type = kv_type;
    a.pos = pos_dev;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.out = out_dev;
    return static_cast<int>(launch_attention(a, head_dim, attn_splits_for(n_ctx), s, false));
}

int bmo_k_decode_attention_ref(const float *q_dev, const float *k_dev, const float *v_dev, void *k_cache_dev,
                               void *v_cache_dev, float *out_dev, int head_dim, int n_heads, int n_kv_heads, int n_ctx,
                               const int *pos_dev, int layer, void *stream) {
    if (!q_dev || !k_dev || !v_dev || !k_cache_dev || !v_cache_dev || !out_dev || !pos_dev)
        return static_cast<int>(cudaErrorInvalidValue);
    const bool split = n_ctx > 64;
    if (!attn_ref_supported(head_dim, n_ctx, split) || n_kv_heads <= 0 || n_heads % n_kv_heads || layer < 0)
        return static_cast<int>(cudaErrorInvalidValue);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long layer_off = static_cast<long long>(layer) * n_kv_heads * n_ctx * head_dim;
    const int warps = 2 * n_kv_heads * head_dim / 32;
    kv_append_kernel<<<(warps * 32 + 127) / 128, 128, 0, s>>>(k_dev, v_dev, k_cache_dev, v_cache_dev, nullptr, nullptr,
                                                             n_kv_heads, head_dim, n_ctx, pos_dev, layer_off, kKvF16);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
    AttnArgs a{};
    a.q = q_dev;
    a.v_raw = v_dev;
    a.k_cache = k_cache_dev;
    a.v_cache = v_cache_dev;
    a.kv_layer_off = layer_off;
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    a.n_ctx = n_ctx;
    a.kv_type = kKvF16;
    a.pos = pos_dev;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.out = out_dev;
    return static_cast<int>(launch_attention_ref(a, head_dim, split, s, false));
}

int bmo_k_tp_exchange(const double *const *parts, unsigned long long *const *flag_out,
                      const unsigned long long *flag_in_dev, unsigned long long *seq_dev, const float *resid_dev,
                      float *y_dev, int *status_dev, int rank, int size, int n, void *stream) {
    if (!parts || !flag_out || !flag_in_dev || !seq_dev || !resid_dev || !y_dev || !status_dev || size < 2 ||
        size > kTpMaxRanks || rank < 0 || rank >= size || n <= 0 || n > kTpBufDoubles)
        return static_cast<int>(cudaErrorInvalidValue);
    TpExchangeArgs a{};
    for (int r = 0; r < size; ++r) {
        if (!parts[r] || (r != rank && !flag_out[r])) return static_cast<int>(cudaErrorInvalidValue);
        a.part[r] = parts[r];
        a.flag_out[r] = flag_out[r];
    }
    a.flag_in = flag_in_dev;
    a.seq = seq_dev;
    a.resid = resid_dev;
    a.y = y_dev;
    a.status = status_dev;
    a.rank = rank;
    a.size = size;
    a.n = n;
    return static_cast<int>(launch_tp_exchange(a, static_cast<cudaStream_t>(stream), false));
}

int bmo_k_sample_token(const float *logits_dev, int n, float temp, int top_k, int pause_rule, uint32_t *rng_dev,
                       int32_t *out_dev, void *stream) {
    if (!logits_dev || !rng_dev || !out_dev || n <= 0 || n > kSampleMaxN || (top_k < n ? top_k : n) > kLoopTopKMax)
        return static_cast<int>(cudaErrorInvalidValue);
    SampleArgs a{};
    a.logits = logits_dev;
    a.n = n;
    a.text = pause_rule ? 1 : 0;
    a.sampling = 1;
    a.top_k = top_k;
    a.temp = temp;
    a.mt = rng_dev;
    a.mti = reinterpret_cast<int *>(rng_dev + 624);
    a.out = out_dev;
    return static_cast<int>(launch_sample(a, static_cast<cudaStream_t>(stream), false));
}

}  // extern "C"
