// attention.cu -- single-token decode attention over the circular KV ring.
//
// Semantics follow bmo_decode_attention_kernel (src/bmo_cuda_kernels.cu:713-848):
// total = pos+1 tokens, window = min(total, n_ctx), logical positions
// [total-window, pos] live at slots t % n_ctx (oldest first); scores are
// (q . k) * 1/sqrt(hd), softmax, out = sum p * v.  The current token's K/V
// were appended at slot pos % n_ctx by the QKV epilogue and are read back
// through the cache format like every other position; a window of one
// returns the raw fp32 v.
//
// B200 design: grid (heads, splits).  Each CTA owns a contiguous slice of the
// window (flash-decode split).  Everything except the newest slot was written
// by earlier frames, so those K/V rows are fetched by the TMA bulk-copy
// engine before griddepcontrol.wait and overlap the QKV GEMV still running;
// the newest row is read after the wait.  Split results (max, sum, o) are
// combined by the last split to finish (per-head counter, fixed order).
// The ring is either fp16 rows (the reference format) or Q4_0 blocks along
// head_dim (nibble plane + fp16 scale plane), dequantised on the fly.
#include "common.cuh"
#include "../launch.h"

namespace bmo {

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxPer = 64;  // window positions per split

template <int HD, bool Q4>
struct AttnSmem {
    static constexpr int kRowBytes = Q4 ? HD / 2 : HD * 2;
    static constexpr int kScales = Q4 ? HD / 32 : 1;
    uint64_t bar;
    alignas(128) uint8_t k[kAttnMaxPer][kRowBytes];
    alignas(128) uint8_t v[kAttnMaxPer][kRowBytes];
    __half kd[kAttnMaxPer][kScales];
    __half vd[kAttnMaxPer][kScales];
    float q[HD];
    float p[kAttnMaxPer];
    int last;
};

template <int HD, bool Q4>
__device__ __forceinline__ float kv_elem(const uint8_t *row, const __half *sc, int d) {
    if constexpr (Q4) {
        const uint8_t b = row[(d >> 5) * 16 + (d & 15)];
        const int nib = (d & 31) < 16 ? (b & 0x0F) : (b >> 4);
        return static_cast<float>(nib - 8) * __half2float(sc[d >> 5]);
    } else {
        return __half2float(reinterpret_cast<const __half *>(row)[d]);
    }
}

template <int HD, bool Q4>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const __grid_constant__ AttnArgs a) {
    using Smem = AttnSmem<HD, Q4>;
    constexpr int kRowBytes = Smem::kRowBytes;
    constexpr int kSc = Smem::kScales;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem &S = *reinterpret_cast<Smem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, sp = blockIdx.y, nsp = gridDim.y;

    // The position was copied to the device before this graph's first kernel.
    const int pos = *a.pos;
    const int total = pos + 1;
    const int window = total > a.n_ctx ? a.n_ctx : total;
    const int start = total - window;
    const int per = (window + nsp - 1) / nsp;
    const int i0 = sp * per;
    const int i1 = min(window, i0 + per);
    const int n = max(0, i1 - i0);
    const bool has_newest = n > 0 && i1 == window;
    const int n_pre = has_newest ? n - 1 : n;  // rows written by earlier frames
    const int kh = (a.n_kv_heads == a.n_heads) ? h : h / (a.n_heads / a.n_kv_heads);
    const long long head_row0 = a.kv_layer_off / HD + static_cast<long long>(kh) * a.n_ctx;  // row index
    const uint8_t *kc = static_cast<const uint8_t *>(a.k_cache) + head_row0 * kRowBytes;
    const uint8_t *vc = static_cast<const uint8_t *>(a.v_cache) + head_row0 * kRowBytes;
    const __half *kdc = Q4 ? reinterpret_cast<const __half *>(a.k_scale) + head_row0 * kSc : nullptr;
    const __half *vdc = Q4 ? reinterpret_cast<const __half *>(a.v_scale) + head_row0 * kSc : nullptr;
    const int s0 = (start + i0) % a.n_ctx;
    const int run_a = min(n_pre, a.n_ctx - s0);

    if (tid == 0) {
        mbar_init(&S.bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    // Older ring rows: bulk copies issued before waiting on the QKV kernel.
    if (tid == 0) {
        mbar_arrive_expect_tx(&S.bar, static_cast<uint32_t>(n_pre) * kRowBytes * 2);
        if (n_pre > 0) {
            const uint64_t pol = l2_evict_first_policy();
            bulk_load(S.k[0], kc + static_cast<long long>(s0) * kRowBytes, run_a * kRowBytes, &S.bar, pol);
            bulk_load(S.v[0], vc + static_cast<long long>(s0) * kRowBytes, run_a * kRowBytes, &S.bar, pol);
            if (n_pre > run_a) {
                bulk_load(S.k[run_a], kc, (n_pre - run_a) * kRowBytes, &S.bar, pol);
                bulk_load(S.v[run_a], vc, (n_pre - run_a) * kRowBytes, &S.bar, pol);
            }
        }
    }
    if constexpr (Q4) {
        for (int e = tid; e < n_pre * kSc; e += kAttnThreads) {
            const int j = e / kSc, b = e % kSc;
            const long long slot = (start + i0 + j) % a.n_ctx;
            S.kd[j][b] = kdc[slot * kSc + b];
            S.vd[j][b] = vdc[slot * kSc + b];
        }
    }

    pdl_wait();

    if (window == 1) {
        if (sp == 0)
            for (int d = tid; d < HD; d += kAttnThreads) a.out[h * HD + d] = a.v_raw[kh * HD + d];
        mbar_wait(&S.bar, 0);
        return;
    }

    for (int d = tid; d < HD; d += kAttnThreads) S.q[d] = a.q[h * HD + d];
    if (has_newest) {
        // newest row was written by this frame's QKV kernel: plain loads after the wait
        const long long cur_slot = pos % a.n_ctx;
        const uint32_t *kr = reinterpret_cast<const uint32_t *>(kc + cur_slot * kRowBytes);
        const uint32_t *vr = reinterpret_cast<const uint32_t *>(vc + cur_slot * kRowBytes);
        for (int b = tid; b < kRowBytes / 4; b += kAttnThreads) {
            reinterpret_cast<uint32_t *>(S.k[n - 1])[b] = __ldcg(kr + b);
            reinterpret_cast<uint32_t *>(S.v[n - 1])[b] = __ldcg(vr + b);
        }
        if constexpr (Q4) {
            for (int b = tid; b < kSc; b += kAttnThreads) {
                S.kd[n - 1][b] = __ldcg(kdc + cur_slot * kSc + b);
                S.vd[n - 1][b] = __ldcg(vdc + cur_slot * kSc + b);
            }
        }
    }
    if (!mbar_wait(&S.bar, 0)) raise_error(a.status, kErrTmaTimeout);
    __syncthreads();

    // scores: one warp per position, lanes split the head dimension
    for (int j = warp; j < n; j += kAttnThreads / 32) {
        float s = 0.0f;
#pragma unroll
        for (int d = lane; d < HD; d += 32) s = fmaf(S.q[d], kv_elem<HD, Q4>(S.k[j], S.kd[j], d), s);
        s = warp_sum(s);
        if (lane == 0) S.p[j] = s * a.scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = 0; j < n; ++j) m = fmaxf(m, S.p[j]);
    __syncthreads();
    if (tid < n) S.p[tid] = expf(S.p[tid] - m);
    __syncthreads();
    float l = 0.0f;
    for (int j = 0; j < n; ++j) l += S.p[j];

    float *part = a.part + (static_cast<size_t>(h) * nsp + sp) * (HD + 2);
    for (int d = tid; d < HD; d += kAttnThreads) {
        float o = 0.0f;
        for (int j = 0; j < n; ++j) o = fmaf(S.p[j], kv_elem<HD, Q4>(S.v[j], S.vd[j], d), o);
        part[d] = o;
    }
    if (tid == 0) {
        part[HD] = m;
        part[HD + 1] = l;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) S.last = (atomicAdd(&a.count[h], 1) == nsp - 1);
    __syncthreads();
    if (!S.last) return;
    __threadfence();
    const float *base = a.part + static_cast<size_t>(h) * nsp * (HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsp; ++s) M = fmaxf(M, __ldcg(base + s * (HD + 2) + HD));
    float L = 0.0f;
    for (int s = 0; s < nsp; ++s) {
        const float ms = __ldcg(base + s * (HD + 2) + HD);
        if (ms != -INFINITY) L += __ldcg(base + s * (HD + 2) + HD + 1) * expf(ms - M);
    }
    for (int d = tid; d < HD; d += kAttnThreads) {
        float o = 0.0f;
        for (int s = 0; s < nsp; ++s) {
            const float ms = __ldcg(base + s * (HD + 2) + HD);
            if (ms != -INFINITY) o += __ldcg(base + s * (HD + 2) + d) * expf(ms - M);
        }
        a.out[h * HD + d] = o / L;
    }
    if (tid == 0) a.count[h] = 0;
}

template <int HD, bool Q4>
static cudaError_t launch_attn_t(const AttnArgs &a, int splits, cudaStream_t s, bool pdl) {
    static unsigned long long configured = 0;
    const size_t smem = sizeof(AttnSmem<HD, Q4>);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(attn_kernel<HD, Q4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_heads, splits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_kernel<HD, Q4>, a);
}

int attn_max_per_split() { return kAttnMaxPer; }

cudaError_t configure_attention() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(attn_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sizeof(AttnSmem<128, false>)))) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(attn_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sizeof(AttnSmem<128, true>)))) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(attn_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sizeof(AttnSmem<64, false>)))) != cudaSuccess)
        return e;
    return cudaFuncSetAttribute(attn_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(AttnSmem<64, true>)));
}

cudaError_t launch_attention(const AttnArgs &a, int head_dim, int splits, cudaStream_t s, bool pdl) {
    if (splits <= 0 || (a.n_ctx + splits - 1) / splits > kAttnMaxPer) return cudaErrorInvalidValue;
    const bool q4 = a.kv_type == kKvQ4_0;
    if (head_dim == 128)
        return q4 ? launch_attn_t<128, true>(a, splits, s, pdl) : launch_attn_t<128, false>(a, splits, s, pdl);
    if (head_dim == 64)
        return q4 ? launch_attn_t<64, true>(a, splits, s, pdl) : launch_attn_t<64, false>(a, splits, s, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace bmo
