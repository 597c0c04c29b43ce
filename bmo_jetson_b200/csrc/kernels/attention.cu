// attention.cu -- single-token decode attention over the circular KV ring.
//
// Semantics follow bmo_decode_attention_kernel (src/bmo_cuda_kernels.cu:713-848):
// total = pos+1 tokens, window = min(total, n_ctx), logical positions
// [total-window, pos] live at slots t % n_ctx (oldest first); scores are
// (q . k) * 1/sqrt(hd), softmax over the window, out = sum p * v.  The
// current token's K/V were appended at slot pos % n_ctx by the QKV epilogue
// and are read back through the cache format like every other position; a
// window of one returns the raw fp32 v.  Exact-reduction semantics: q . k
// in double rounded once, p = exp(s - max) in double rounded once, the
// weighted sum and its normaliser in double, one rounding per output.
//
// B200 design: one thread-block cluster per head, its CTAs splitting the
// window (flash-decode split).  Rows written by earlier frames are fetched
// by the TMA bulk-copy engine before griddepcontrol.wait, overlapping the
// QKV GEMV still running; the newest row is read after the wait.  The
// window maximum and the partial sums travel through distributed shared
// memory and cluster barriers, so the softmax is the exact two-pass one
// and no global scratch or atomics are needed.  The ring is either fp16
// rows (the reference format) or Q4_0 blocks along head_dim (nibble plane +
// fp16 scale plane), dequantised on the fly.
#include <cooperative_groups.h>

#include "common.cuh"
#include "../launch.h"

namespace cg = cooperative_groups;

namespace bmo {

constexpr int kAttnThreads = 128;
constexpr int kAttnSub = 64;          // rows per staged sub-chunk
constexpr int kAttnMaxSplits = 8;     // portable cluster size
constexpr int kAttnMaxPos = 1024;     // window positions per split
constexpr int kAttnMaxCtx = kAttnMaxSplits * kAttnMaxPos;

template <int HD, bool Q4>
struct AttnSmem {
    static constexpr int kRowBytes = Q4 ? HD / 2 : HD * 2;
    static constexpr int kScales = Q4 ? HD / 32 : 1;
    uint64_t kbar, vbar;
    alignas(128) uint8_t k[kAttnSub][kRowBytes];
    alignas(128) uint8_t v[kAttnSub][kRowBytes];
    __half kd[kAttnSub][kScales];
    __half vd[kAttnSub][kScales];
    float q[HD];
    float s[kAttnMaxPos];  // scores, then p
    double o_part[HD];
    double l_part;
    float m_local;
};

template <int HD, bool Q4>
__device__ __forceinline__ float kv_elem(const uint8_t *row, const __half *sc, int d) {
    if constexpr (Q4) {
        const uint8_t b = row[(d >> 5) * 16 + (d & 15)];
        const int nib = (d & 31) < 16 ? (b & 0x0F) : (b >> 4);
        return __fmul_rn(static_cast<float>(nib - 8), __half2float(sc[d >> 5]));
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
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sp = blockIdx.x, nsp = gridDim.x, h = blockIdx.y;

    // The position was copied to the device before this graph's first kernel.
    const int pos = *a.pos;
    const int total = pos + 1;
    const int window = total > a.n_ctx ? a.n_ctx : total;
    const int start = total - window;
    const int per = (window + nsp - 1) / nsp;
    const int i0 = min(window, sp * per);
    const int n = max(0, min(window, i0 + per) - i0);
    const int nsub = (n + kAttnSub - 1) / kAttnSub;
    const int kh = (a.n_kv_heads == a.n_heads) ? h : h / (a.n_heads / a.n_kv_heads);
    const long long head_row0 = a.kv_layer_off / HD + static_cast<long long>(kh) * a.n_ctx;  // ring row index
    const uint8_t *kc = static_cast<const uint8_t *>(a.k_cache) + head_row0 * kRowBytes;
    const uint8_t *vc = static_cast<const uint8_t *>(a.v_cache) + head_row0 * kRowBytes;
    const __half *kdc = Q4 ? reinterpret_cast<const __half *>(a.k_scale) + head_row0 * kSc : nullptr;
    const __half *vdc = Q4 ? reinterpret_cast<const __half *>(a.v_scale) + head_row0 * kSc : nullptr;
    const uint64_t pol = l2_evict_first_policy();

    // Stages rows [j0, j0+nj) of this split (minus the newest, which the QKV
    // kernel of this frame writes) into buf via bulk copies completing on bar.
    auto stage = [&](uint8_t (*buf)[kRowBytes], __half (*sc)[kSc], const uint8_t *ring, const __half *scales,
                     uint64_t *bar, int j0, int nj) {
        const bool newest = (i0 + j0 + nj == window);
        const int m = newest ? nj - 1 : nj;
        if (tid == 0) {
            fence_proxy_async();  // earlier generic reads of buf before the async-proxy writes
            mbar_arrive_expect_tx(bar, static_cast<uint32_t>(m) * kRowBytes);
            if (m > 0) {
                const int s0 = (start + i0 + j0) % a.n_ctx;
                const int run_a = min(m, a.n_ctx - s0);
                bulk_load(buf[0], ring + static_cast<long long>(s0) * kRowBytes, run_a * kRowBytes, bar, pol);
                if (m > run_a) bulk_load(buf[run_a], ring, (m - run_a) * kRowBytes, bar, pol);
            }
        }
        if constexpr (Q4) {
            for (int e = tid; e < m * kSc; e += kAttnThreads) {
                const int j = e / kSc, b = e % kSc;
                const long long slot = (start + i0 + j0 + j) % a.n_ctx;
                sc[j][b] = scales[slot * kSc + b];
            }
        }
    };
    // Newest row (this frame's K/V): plain loads after the wait.
    auto load_newest = [&](uint8_t (*buf)[kRowBytes], __half (*sc)[kSc], const uint8_t *ring, const __half *scales,
                           int j) {
        const long long slot = pos % a.n_ctx;
        const uint32_t *src = reinterpret_cast<const uint32_t *>(ring + slot * kRowBytes);
        for (int b = tid; b < kRowBytes / 4; b += kAttnThreads) reinterpret_cast<uint32_t *>(buf[j])[b] = __ldcg(src + b);
        if constexpr (Q4)
            for (int b = tid; b < kSc; b += kAttnThreads) sc[j][b] = __ldcg(scales + slot * kSc + b);
    };

    if (tid == 0) {
        mbar_init(&S.kbar, 1);
        mbar_init(&S.vbar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    uint32_t kphase = 0, vphase = 0;
    const bool prefetched = (nsub == 1);
    if (prefetched) {  // common case: the whole split fits one sub-chunk
        stage(S.k, S.kd, kc, kdc, &S.kbar, 0, n);
        stage(S.v, S.vd, vc, vdc, &S.vbar, 0, n);
    }

    pdl_wait();

    if (window == 1) {  // uniform over the cluster: no cluster barrier is reached
        if (sp == 0)
            for (int d = tid; d < HD; d += kAttnThreads) a.out[h * HD + d] = a.v_raw[kh * HD + d];
        if (prefetched) {
            mbar_wait(&S.kbar, 0);
            mbar_wait(&S.vbar, 0);
        }
        return;
    }
    bool ok = true;
    for (int d = tid; d < HD; d += kAttnThreads) S.q[d] = a.q[h * HD + d];

    // ---- pass 1: scores of this split ----
    for (int sub = 0; sub < nsub; ++sub) {
        const int j0 = sub * kAttnSub, nj = min(kAttnSub, n - j0);
        if (!prefetched) stage(S.k, S.kd, kc, kdc, &S.kbar, j0, nj);
        if (i0 + j0 + nj == window) load_newest(S.k, S.kd, kc, kdc, nj - 1);
        ok &= mbar_wait(&S.kbar, kphase);
        kphase ^= 1u;
        __syncthreads();
        for (int j = warp; j < nj; j += kAttnThreads / 32) {
            double dot = 0.0;
#pragma unroll
            for (int d = lane; d < HD; d += 32)
                dot = fma(static_cast<double>(S.q[d]), static_cast<double>(kv_elem<HD, Q4>(S.k[j], S.kd[j], d)), dot);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0) S.s[j0 + j] = __fmul_rn(__double2float_rn(dot), a.scale);
        }
        __syncthreads();
    }
    float m = -INFINITY;
    for (int j = 0; j < n; ++j) m = fmaxf(m, S.s[j]);
    if (tid == 0) S.m_local = m;
    cluster.sync();
    float M = -INFINITY;
    for (int r = 0; r < nsp; ++r) M = fmaxf(M, *cluster.map_shared_rank(&S.m_local, r));

    // ---- pass 2: p = exp(s - M), partial sums in double ----
    for (int j = tid; j < n; j += kAttnThreads)
        S.s[j] = __double2float_rn(exp(static_cast<double>(__fsub_rn(S.s[j], M))));
    __syncthreads();
    static_assert(HD <= kAttnThreads, "one thread per output dimension");
    double o = 0.0, l = 0.0;
    for (int sub = 0; sub < nsub; ++sub) {
        const int j0 = sub * kAttnSub, nj = min(kAttnSub, n - j0);
        if (!prefetched) stage(S.v, S.vd, vc, vdc, &S.vbar, j0, nj);
        if (i0 + j0 + nj == window) load_newest(S.v, S.vd, vc, vdc, nj - 1);
        ok &= mbar_wait(&S.vbar, vphase);
        vphase ^= 1u;
        __syncthreads();
        if (tid < HD) {
            for (int j = 0; j < nj; ++j) {
                const double p = static_cast<double>(S.s[j0 + j]);
                o = fma(p, static_cast<double>(kv_elem<HD, Q4>(S.v[j], S.vd[j], tid)), o);
                if (tid == 0) l += p;
            }
        }
        __syncthreads();
    }
    if (tid < HD) S.o_part[tid] = o;
    if (tid == 0) S.l_part = l;
    if (!ok && tid == 0) raise_error(a.status, kErrTmaTimeout);
    cluster.sync();
    if (sp == 0 && tid < HD) {
        double ot = 0.0, lt = 0.0;
        for (int r = 0; r < nsp; ++r) {
            ot += cluster.map_shared_rank(S.o_part, r)[tid];
            lt += *cluster.map_shared_rank(&S.l_part, r);
        }
        a.out[h * HD + tid] = __double2float_rn(__ddiv_rn(ot, lt));
    }
    cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
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
    cfg.gridDim = dim3(splits, a.n_heads);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = splits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attn_kernel<HD, Q4>, a);
}

int attn_splits_for(int n_ctx) {
    int s = (n_ctx + kAttnSub - 1) / kAttnSub;
    return s < 1 ? 1 : (s > kAttnMaxSplits ? kAttnMaxSplits : s);
}

int attn_max_ctx() { return kAttnMaxCtx; }

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
    if (splits <= 0 || splits > kAttnMaxSplits || a.n_ctx <= 0 || a.n_ctx > kAttnMaxCtx) return cudaErrorInvalidValue;
    if ((a.n_ctx + splits - 1) / splits > kAttnMaxPos) return cudaErrorInvalidValue;
    const bool q4 = a.kv_type == kKvQ4_0;
    if (head_dim == 128)
        return q4 ? launch_attn_t<128, true>(a, splits, s, pdl) : launch_attn_t<128, false>(a, splits, s, pdl);
    if (head_dim == 64)
        return q4 ? launch_attn_t<64, true>(a, splits, s, pdl) : launch_attn_t<64, false>(a, splits, s, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace bmo
