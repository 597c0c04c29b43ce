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

constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnPosPerWarp = 4;  // positions one warp scores at a time (independent accumulators)

template <int HD, bool Q4>
struct AttnSmem {
    static constexpr int kRowBytes = Q4 ? HD / 2 : HD * 2;
    static constexpr int kScales = Q4 ? HD / 32 : 1;
    // position groups of the weighted sum: fp16 rows one dimension per thread,
    // Q4_0 rows one 32-bit word (8 dimensions) per thread
    static constexpr int kGroups = Q4 ? kAttnThreads / (HD / 8) : kAttnThreads / HD;
    uint64_t kbar, vbar;
    alignas(128) uint8_t k[kAttnSub][kRowBytes];
    alignas(128) uint8_t v[kAttnSub][kRowBytes];
    __half kd[kAttnSub][kScales];
    __half vd[kAttnSub][kScales];
    float q[HD];
    float s[kAttnMaxPos];                // scores, then p
    float wmax[kAttnWarps];
    float m_rank[kAttnMaxSplits];        // every split's local maximum (pushed by the owner)
    double o_grp[kGroups][HD];
    double l_warp;
    double o_rank[kAttnMaxSplits][HD];   // rank 0: every split's partial output (pushed)
    double l_rank[kAttnMaxSplits];
    // Q4_0 rings: (n - 8) as doubles, and per staged row the block scales (pass 1)
    // or p times the block scales (pass 2) as doubles -- every K/V element then
    // enters the double sums through one table read and one fma, with no
    // per-element conversion
    alignas(128) double tbl[16];
    double kdd[Q4 ? kAttnSub : 1][kScales];
    double pd[Q4 ? kAttnSub : 1][kScales];
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

// (n - 8) as a double for the Q4_0 nibble at bit SH of x, read from the
// 16-entry table: the nibble shifted to a byte offset (n * 8) in one step.
template <int SH>
__device__ __forceinline__ double nib_val(const double *tbl, uint32_t x) {
    const uint32_t off = SH >= 3 ? (x >> (SH - 3)) & 0x78u : (x << (3 - SH)) & 0x78u;
    return *reinterpret_cast<const double *>(reinterpret_cast<const char *>(tbl) + off);
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
    const int sp = blockIdx.x, nsp = gridDim.x, h = blockIdx.y, sess = blockIdx.z;
    // batched sessions: this session's q / raw v / output / ring / position
    const float *qv = a.q + static_cast<long long>(sess) * a.qo_stride;
    const float *vraw = a.v_raw + static_cast<long long>(sess) * a.vraw_stride;
    float *outv = a.out + static_cast<long long>(sess) * a.qo_stride;

    // The position was copied to the device before this graph's first kernel.
    const int pos = a.pos[sess * a.pos_stride];
    const int total = pos + 1;
    const int window = total > a.n_ctx ? a.n_ctx : total;
    const int start = total - window;
    const int per = (window + nsp - 1) / nsp;
    const int i0 = min(window, sp * per);
    const int n = max(0, min(window, i0 + per) - i0);
    const int nsub = (n + kAttnSub - 1) / kAttnSub;
    const int kh = (a.n_kv_heads == a.n_heads) ? h : h / (a.n_heads / a.n_kv_heads);
    const long long head_row0 =
        (a.kv_layer_off + (a.ring_of ? a.ring_of[sess] : sess) * a.kv_sess_stride) / HD +
        static_cast<long long>(kh) * a.n_ctx;  // ring row index
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
    if (Q4 && tid < 16) S.tbl[tid] = static_cast<double>(tid - 8);
    __syncthreads();
    // Every CTA of the cluster must be running before any writes into its
    // shared memory: arrive now, wait just before the first remote store.
    cluster_arrive_relaxed();
    uint32_t kphase = 0, vphase = 0;
    const bool prefetched = (nsub == 1);
    if (prefetched) {  // common case: the whole split fits one sub-chunk
        stage(S.k, S.kd, kc, kdc, &S.kbar, 0, n);
        stage(S.v, S.vd, vc, vdc, &S.vbar, 0, n);
    }

    pdl_wait();

    if (window == 1) {  // uniform over the cluster: no cluster barrier is reached
        if (sp == 0)
            for (int d = tid; d < HD; d += kAttnThreads) outv[h * HD + d] = vraw[kh * HD + d];
        if (prefetched) {
            mbar_wait(&S.kbar, 0);
            mbar_wait(&S.vbar, 0);
        }
        cluster_wait();
        return;
    }
    bool ok = true;
    // q and (single-sub splits) the newest K/V rows: one memory round trip
    for (int d = tid; d < HD; d += kAttnThreads) S.q[d] = __ldcg(qv + h * HD + d);
    const bool newest_here = n > 0 && i0 + n == window;
    if (prefetched && newest_here) {
        load_newest(S.k, S.kd, kc, kdc, n - 1);
        load_newest(S.v, S.vd, vc, vdc, n - 1);
    }
    __syncthreads();
    float qr[HD / 32];
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) qr[i] = S.q[lane + 32 * i];
    // Q4_0: kLP lanes per position, lane pb holding q's block pb as doubles
    constexpr int kLP = HD / 32, kPP = 32 / kLP;
    const int pb = lane % kLP, pl = lane / kLP;
    double qd[Q4 ? 32 : 1];
    if constexpr (Q4) {
#pragma unroll
        for (int i = 0; i < 32; ++i) qd[i] = static_cast<double>(S.q[32 * pb + i]);
    }

    // ---- pass 1: scores of this split, kAttnPosPerWarp positions per warp at a time ----
    for (int sub = 0; sub < nsub; ++sub) {
        const int j0 = sub * kAttnSub, nj = min(kAttnSub, n - j0);
        if (!prefetched) {
            stage(S.k, S.kd, kc, kdc, &S.kbar, j0, nj);
            if (i0 + j0 + nj == window) load_newest(S.k, S.kd, kc, kdc, nj - 1);
        }
        ok &= mbar_wait(&S.kbar, kphase);
        kphase ^= 1u;
        __syncthreads();
        if constexpr (Q4) {
            for (int e = tid; e < nj * kSc; e += kAttnThreads)
                S.kdd[e / kSc][e % kSc] = static_cast<double>(__half2float(S.kd[e / kSc][e % kSc]));
            __syncthreads();
        }
        if constexpr (Q4) {
            // kPP positions per warp step; per lane the 32 products of one block,
            // sum_i q_i (n_i - 8) in double, times the block scale, then the
            // kLP blocks of the position added across lanes
            for (int jb = warp * kPP; jb < nj; jb += kAttnWarps * kPP) {
                const int j = jb + pl;
                double dot = 0.0;
                if (j < nj) {
                    const uint4 x = *reinterpret_cast<const uint4 *>(&S.k[j][16 * pb]);
                    const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
                    double c[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        // byte 4w + k: element 4w + k (low nibble), 4w + k + 16 (high nibble)
                        c[0] = fma(qd[4 * w + 0], nib_val<0>(S.tbl, xw[w]), c[0]);
                        c[1] = fma(qd[4 * w + 1], nib_val<8>(S.tbl, xw[w]), c[1]);
                        c[2] = fma(qd[4 * w + 2], nib_val<16>(S.tbl, xw[w]), c[2]);
                        c[3] = fma(qd[4 * w + 3], nib_val<24>(S.tbl, xw[w]), c[3]);
                        c[0] = fma(qd[16 + 4 * w + 0], nib_val<4>(S.tbl, xw[w]), c[0]);
                        c[1] = fma(qd[16 + 4 * w + 1], nib_val<12>(S.tbl, xw[w]), c[1]);
                        c[2] = fma(qd[16 + 4 * w + 2], nib_val<20>(S.tbl, xw[w]), c[2]);
                        c[3] = fma(qd[16 + 4 * w + 3], nib_val<28>(S.tbl, xw[w]), c[3]);
                    }
                    dot = ((c[0] + c[1]) + (c[2] + c[3])) * S.kdd[j][pb];
                }
#pragma unroll
                for (int o = 1; o < kLP; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
                if (pb == 0 && j < nj) S.s[j0 + j] = __fmul_rn(__double2float_rn(dot), a.scale);
            }
            __syncthreads();
            continue;
        }
        for (int jb = warp * kAttnPosPerWarp; jb < nj; jb += kAttnThreads / 32 * kAttnPosPerWarp) {
            double dot[kAttnPosPerWarp];
#pragma unroll
            for (int u = 0; u < kAttnPosPerWarp; ++u) {
                const int j = min(jb + u, nj - 1);
                dot[u] = 0.0;
#pragma unroll
                for (int i = 0; i < HD / 32; ++i)
                    dot[u] = fma(static_cast<double>(qr[i]),
                                 static_cast<double>(kv_elem<HD, Q4>(S.k[j], S.kd[j], lane + 32 * i)), dot[u]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < kAttnPosPerWarp; ++u) dot[u] += __shfl_xor_sync(0xffffffffu, dot[u], o);
            if (lane < kAttnPosPerWarp && jb + lane < nj) {
                double mine = dot[0];
#pragma unroll
                for (int u = 1; u < kAttnPosPerWarp; ++u) mine = lane == u ? dot[u] : mine;
                S.s[j0 + jb + lane] = __fmul_rn(__double2float_rn(mine), a.scale);
            }
        }
        __syncthreads();
    }
    pdl_launch_dependents();  // the next kernel prefetches during the softmax and weighted sum
    // local maximum, pushed into every split's shared memory
    float m = -INFINITY;
    for (int j = tid; j < n; j += kAttnThreads) m = fmaxf(m, S.s[j]);
    m = warp_max(m);
    if (lane == 0) S.wmax[warp] = m;
    __syncthreads();
    cluster_wait();
    if (tid < nsp) {
        float mm = S.wmax[0];
#pragma unroll
        for (int w = 1; w < kAttnWarps; ++w) mm = fmaxf(mm, S.wmax[w]);
        cluster.map_shared_rank(S.m_rank, tid)[sp] = mm;
    }
    cluster.sync();
    float M = S.m_rank[0];
    for (int r = 1; r < nsp; ++r) M = fmaxf(M, S.m_rank[r]);

    // ---- pass 2: p = exp(s - M), weighted sums in double ----
    for (int j = tid; j < n; j += kAttnThreads)
        S.s[j] = __double2float_rn(exp(static_cast<double>(__fsub_rn(S.s[j], M))));
    __syncthreads();
    static_assert(kAttnThreads % HD == 0, "threads cover the output dimensions");
    constexpr int kG = Smem::kGroups;
    const int dim = tid % HD, grp = tid / HD;
    double o4[4] = {0.0, 0.0, 0.0, 0.0};
    // Q4_0: thread = (32-bit word wd of the row, position group g2); the word
    // holds dimensions 32 b2 + 4 (wd % 4) + k (low nibbles) and + 16 (high)
    constexpr int kWPR = HD / 8;
    const int wd = tid % kWPR, g2 = tid / kWPR, b2 = wd / 4;
    double o8[Q4 ? 8 : 1];
#pragma unroll
    for (int k = 0; k < (Q4 ? 8 : 1); ++k) o8[k] = 0.0;
    double l = 0.0;
    for (int sub = 0; sub < nsub; ++sub) {
        const int j0 = sub * kAttnSub, nj = min(kAttnSub, n - j0);
        if (!prefetched) {
            stage(S.v, S.vd, vc, vdc, &S.vbar, j0, nj);
            if (i0 + j0 + nj == window) load_newest(S.v, S.vd, vc, vdc, nj - 1);
        }
        ok &= mbar_wait(&S.vbar, vphase);
        vphase ^= 1u;
        __syncthreads();
        if constexpr (Q4) {
            // p times the block scale, exact in double (fp32 x fp16)
            for (int e = tid; e < nj * kSc; e += kAttnThreads)
                S.pd[e / kSc][e % kSc] = static_cast<double>(S.s[j0 + e / kSc]) *
                                         static_cast<double>(__half2float(S.vd[e / kSc][e % kSc]));
            __syncthreads();
        }
        if constexpr (Q4) {
            // p v = (p d) (n - 8), both factors exact in double
            for (int j = g2; j < nj; j += kG) {
                const uint32_t x = reinterpret_cast<const uint32_t *>(S.v[j])[wd];
                const double pdj = S.pd[j][b2];
                o8[0] = fma(pdj, nib_val<0>(S.tbl, x), o8[0]);
                o8[1] = fma(pdj, nib_val<8>(S.tbl, x), o8[1]);
                o8[2] = fma(pdj, nib_val<16>(S.tbl, x), o8[2]);
                o8[3] = fma(pdj, nib_val<24>(S.tbl, x), o8[3]);
                o8[4] = fma(pdj, nib_val<4>(S.tbl, x), o8[4]);
                o8[5] = fma(pdj, nib_val<12>(S.tbl, x), o8[5]);
                o8[6] = fma(pdj, nib_val<20>(S.tbl, x), o8[6]);
                o8[7] = fma(pdj, nib_val<28>(S.tbl, x), o8[7]);
            }
        } else {
            // one weighted term: p v in double
            auto term = [&](int j, double o) {
                return fma(static_cast<double>(S.s[j0 + j]), static_cast<double>(kv_elem<HD, Q4>(S.v[j], S.vd[j], dim)), o);
            };
            int j = grp;
            for (; j + 3 * kG < nj; j += 4 * kG) {
#pragma unroll
                for (int u = 0; u < 4; ++u) o4[u] = term(j + u * kG, o4[u]);
            }
            for (; j < nj; j += kG) o4[0] = term(j, o4[0]);
        }
        if (warp == kAttnWarps - 1)
            for (int j = lane; j < nj; j += 32) l += static_cast<double>(S.s[j0 + j]);
        __syncthreads();
    }
    if constexpr (Q4) {
        const int d0 = 32 * b2 + 4 * (wd % 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            S.o_grp[g2][d0 + k] = o8[k];
            S.o_grp[g2][d0 + 16 + k] = o8[4 + k];
        }
    } else {
        S.o_grp[grp][dim] = (o4[0] + o4[1]) + (o4[2] + o4[3]);
    }
    if (warp == kAttnWarps - 1) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) S.l_warp = l;
    }
    if (!ok && tid == 0) raise_error(a.status, kErrTmaTimeout);
    __syncthreads();
    // push this split's partials into rank 0's shared memory
    if (tid < HD) {
        double ot = S.o_grp[0][tid];
#pragma unroll
        for (int g = 1; g < kG; ++g) ot += S.o_grp[g][tid];
        cluster.map_shared_rank(&S.o_rank[0][0], 0)[sp * HD + tid] = ot;
    }
    if (tid == 0) cluster.map_shared_rank(S.l_rank, 0)[sp] = S.l_warp;
    cluster.sync();
    if (sp == 0 && tid < HD) {
        double ot = 0.0, lt = 0.0;
        for (int r = 0; r < nsp; ++r) {
            ot += S.o_rank[r][tid];
            lt += S.l_rank[r];
        }
        outv[h * HD + tid] = __double2float_rn(__ddiv_rn(ot, lt));
    }
}

template <int HD, bool Q4>
static cudaError_t launch_attn_t(const AttnArgs &a, int splits, int n_sess, cudaStream_t s, bool pdl) {
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
    cfg.gridDim = dim3(splits, a.n_heads, n_sess);
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

cudaError_t launch_attention(const AttnArgs &a, int head_dim, int splits, cudaStream_t s, bool pdl, int n_sess) {
    if (splits <= 0 || splits > kAttnMaxSplits || a.n_ctx <= 0 || a.n_ctx > kAttnMaxCtx) return cudaErrorInvalidValue;
    if ((a.n_ctx + splits - 1) / splits > kAttnMaxPos) return cudaErrorInvalidValue;
    if (n_sess < 1 || n_sess > 65535 || (n_sess > 1 && a.qo_stride <= 0) ||
        ((n_sess > 1 || a.ring_of) && a.kv_sess_stride <= 0) || a.kv_sess_stride % head_dim)
        return cudaErrorInvalidValue;
    const bool q4 = a.kv_type == kKvQ4_0;
    if (head_dim == 128)
        return q4 ? launch_attn_t<128, true>(a, splits, n_sess, s, pdl) : launch_attn_t<128, false>(a, splits, n_sess, s, pdl);
    if (head_dim == 64)
        return q4 ? launch_attn_t<64, true>(a, splits, n_sess, s, pdl) : launch_attn_t<64, false>(a, splits, n_sess, s, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace bmo
