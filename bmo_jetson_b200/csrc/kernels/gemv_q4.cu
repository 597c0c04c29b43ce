// gemv_q4.cu -- batch-1 Q4_0 x Q8_1 GEMV for sm_100a with fused prologues
// and epilogues.
//
// Computes, per output row r, the reference dot product
// (bmo_gemv_q4_0_q8_1_kernel, src/bmo_cuda_kernels.cu:560-683): each half
// block h (elements {0..7,16..23} and {8..15,24..31}) contributes the fp32
// term  d4 * ((float)sumi_h * d8 - 4 * s8),  and the terms are summed.  The
// activation is quantised to Q8_1 in shared memory by the rule of
// bmo_quantize_row_q8_1_kernel (:529-558).  Exact-reduction semantics: the
// terms are formed with separately rounded fp32 operations as the reference
// writes them and summed in double, rounded once to fp32 -- the same value
// the CPU oracle computes, whatever the split of the work.
//
// Design (B200): one CTA of 8 warps per SM, sized (registers <= 128, shared
// memory < half an SM) so that the NEXT kernel's CTA is resident beside it.
// The weight stream is the only HBM traffic that matters, so each warp keeps
// kRing 4.6 KB chunks in flight through the TMA bulk-copy engine into a
// private shared-memory ring.  The first chunks (and the RMSNorm weight) are
// issued before griddepcontrol.wait, so under programmatic dependent launch
// they stream while the previous kernel finishes its epilogue (the dependent
// launch is triggered after the weight loop); after the wait the activation
// costs a single memory round trip.
// Work split: normally each CTA owns whole row tiles (no cross-CTA traffic);
// where that balances badly, CTA c owns an even range of (row tile, chunk)
// units ("stream-K") and tiles that straddle CTAs are finished by the last
// owner to arrive (per-tile counter, fixed summation order, deterministic).
// Epilogues fuse RoPE + KV-ring append, SwiGLU, residual adds, logits +
// argmax and the depformer embedding add.
#include <algorithm>

#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

#ifndef BMO_GEMV_RING
#define BMO_GEMV_RING 2
#endif
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRing = BMO_GEMV_RING;  // chunks in flight per warp
constexpr int kMaxNbx = 384;  // activations up to 12288 elements (at most two blocks per thread)
constexpr int kMaxTilesPerCta = 10;
constexpr int kMaxNormCols = kMaxTilesPerCta * kWarps * 32 * 2;  // RMSNorm weight staged in `part`'s space
// A cross-CTA combine (partial store, release, acquire, reload) costs about as
// long as one SM streaming this many chunks.
constexpr int kCombineChunks = 12;

// Kept under half of an SM's shared memory so that the next kernel's CTA fits
// beside this one under programmatic dependent launch and prefetches its weights.
struct GemvSmem {
    uint64_t bar[kWarps][kRing];
    uint64_t gbar;  // RMSNorm weight bulk copy
    alignas(128) uint8_t ring[kWarps][kRing][kChunkBytes];
    alignas(16) int8_t xq[kMaxNbx * 32];
    float2 xds[kMaxNbx];  // (d8, 4 * s8) of each Q8_1 block
    union {
        alignas(16) double part[kMaxTilesPerCta][kWarps][32];  // main loop and epilogue
        float gamma[kMaxNormCols];                               // prologue only
    };
    double red[kWarps];
    float tok_v[kWarps];
    int tok_i[kWarps];
    int err;
};

size_t gemv_smem_bytes() { return sizeof(GemvSmem); }
int gemv_max_tiles_per_cta() { return kMaxTilesPerCta; }
int gemv_max_nbx() { return kMaxNbx; }
int gemv_max_norm_cols() { return kMaxNormCols; }

__device__ __forceinline__ int cta_of_chunk(long long k, long long nc, int g) {
    return static_cast<int>(((k + 1) * g - 1) / nc);
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_q4_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    GemvSmem &S = *reinterpret_cast<GemvSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int cpt = a.W.cpt;
    const long long NC = static_cast<long long>(a.W.n_tiles) * cpt;
    int c0, c1;
    if (a.tile_aligned) {
        c0 = static_cast<int>(static_cast<long long>(a.W.n_tiles) * c / G) * cpt;
        c1 = static_cast<int>(static_cast<long long>(a.W.n_tiles) * (c + 1) / G) * cpt;
    } else {
        c0 = static_cast<int>(NC * c / G);
        c1 = static_cast<int>(NC * (c + 1) / G);
    }
    const int n_mine = (c1 - c0 > warp) ? (c1 - c0 - warp + kWarps - 1) / kWarps : 0;
    const int nb = a.W.cols / 32, nbx = a.W.nbx;
    // the RMSNorm weight comes through the bulk-copy engine when it is 16-byte aligned
    const bool gbulk = PRO == kProNorm && (reinterpret_cast<uintptr_t>(a.gamma) & 15) == 0;

    if (tid < kWarps * kRing) mbar_init(&S.bar[tid / kRing][tid % kRing], 1);
    if (tid == kWarps * kRing) mbar_init(&S.gbar, 1);
    if (tid == 0) S.err = 0;
    fence_barrier_init();
    __syncthreads();

    // Weights never depend on earlier kernels: start streaming them now.
    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](int i) {
        const long long k = c0 + warp + static_cast<long long>(kWarps) * i;
        uint64_t *bar = &S.bar[warp][i % kRing];
        mbar_arrive_expect_tx(bar, kChunkBytes);
        bulk_load(S.ring[warp][i % kRing], a.W.tiles + k * kChunkBytes, kChunkBytes, bar, pol);
    };
    if (lane == 0)
        for (int i = 0; i < kRing && i < n_mine; ++i) issue(i);
    if (gbulk && tid == 0) {
        const uint32_t gb = static_cast<uint32_t>(a.W.cols) * 4u;
        mbar_arrive_expect_tx(&S.gbar, gb);
        bulk_load(S.gamma, a.gamma, gb, &S.gbar, l2_evict_last_policy());
    }

    pdl_wait();

    // ---- prologue: activation -> Q8_1 blocks in shared memory ----
    // Thread t converts blocks t and t + kThreads.  Both are loaded before any
    // other memory access so that the activation costs one round trip.
    float v0[32], v1[32];
    const bool h0 = tid < nb, h1 = tid + kThreads < nb;
    if (h0) load_block32(a.x + tid * 32, v0);
    if (h1) load_block32(a.x + (tid + kThreads) * 32, v1);
    int tok = -1;
    if constexpr (EPI == kEpiEmbAdd) {
        tok = resolve_token<kThreads>(a.tok, S.tok_v, S.tok_i, [] { __syncthreads(); });
        if (c == 0 && tid == 0 && a.tok.tok_out) *a.tok.tok_out = tok;
    }
    float scale = 1.0f;
    const float *gam = a.gamma;
    if constexpr (PRO == kProNorm) {
        // rmsnorm_kernel (bmo_cuda_kernels.cu:244-295): scale = 1/sqrt(mean(x^2)+eps),
        // the sum of squares in double, the root and reciprocal in double
        double ss = (h0 ? sum_sq_double(v0) : 0.0) + (h1 ? sum_sq_double(v1) : 0.0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) S.red[warp] = ss;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += S.red[w];
        const float total = __double2float_rn(tot);
        const float mean_eps = __fadd_rn(__fdiv_rn(total, static_cast<float>(a.W.cols)), a.eps);
        scale = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(static_cast<double>(mean_eps))));
        if (gbulk) {
            if (!mbar_wait(&S.gbar, 0)) atomicOr(&S.err, 1);
            gam = S.gamma;
        }
    }
    if (tid < nbx) quantize_x_block<PRO>(a, S.xq, S.xds, tid, h0, v0, scale, gam, c == 0);
    if (tid + kThreads < nbx) quantize_x_block<PRO>(a, S.xq, S.xds, tid + kThreads, h1, v1, scale, gam, c == 0);
    __syncthreads();

    // ---- main loop: stream chunks through the ring ----
    // part[t][w] receives warp w's sum over tile t; every warp writes each
    // tile of the CTA's range once (0 for tiles it had no chunk of).
    const int t_first = c0 / cpt;
    const int t_last = c1 > c0 ? (c1 - 1) / cpt : t_first - 1;
    int next_unwritten = t_first, cur = -1;
    double acc = 0.0;
    auto flush = [&](int upto) {  // write tiles [next_unwritten, upto], cur's sum at cur
        for (int t = next_unwritten; t <= upto; ++t) S.part[t - t_first][warp][lane] = t == cur ? acc : 0.0;
        next_unwritten = upto + 1;
    };
    for (int i = 0; i < n_mine; ++i) {
        const int k = c0 + warp + kWarps * i;
        const int tile = k / cpt, kc = k - tile * cpt;
        if (tile != cur) {
            if (cur >= 0) flush(cur);
            acc = 0.0;
            cur = tile;
        }
        if (!mbar_wait(&S.bar[warp][i % kRing], (i / kRing) & 1)) {
            if (lane == 0) atomicOr(&S.err, 1);
            for (int j = i + 1; j < n_mine && j < i + kRing; ++j) mbar_wait(&S.bar[warp][j % kRing], (j / kRing) & 1);
            break;
        }
        acc += chunk_dot(S.ring[warp][i % kRing], S.xq + kc * kChunkBlocks * 32, S.xds + kc * kChunkBlocks, lane);
        __syncwarp();
        if (lane == 0 && i + kRing < n_mine) {
            fence_proxy_async();
            issue(i + kRing);
        }
    }
    if (cur >= 0) flush(cur);
    flush(t_last);
    // The next kernel may start now: its weight prefetch then overlaps this
    // kernel's epilogue instead of competing with its weight stream (measured:
    // triggering at kernel start costs ~10% of the frame rate).
    pdl_launch_dependents();
    __syncthreads();
    if (S.err) {
        if (tid == 0) raise_error(a.status, kErrTmaTimeout);
        return;
    }
    if (c1 <= c0) return;

    // ---- per-tile reduction (fixed order, double) and epilogue ----
    for (int tl = warp; tl <= t_last - t_first; tl += kWarps) {
        const int t = t_first + tl;
        double v = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += S.part[tl][w][lane];
        const int f = a.tile_aligned ? 0 : cta_of_chunk(static_cast<long long>(t) * cpt, NC, G);
        const int l = a.tile_aligned ? 0 : cta_of_chunk(static_cast<long long>(t) * cpt + cpt - 1, NC, G);
        if (f != l) {
            double *gp = a.gpart + (static_cast<size_t>(t) * (cpt + 1)) * 32;
            gp[(c - f) * 32 + lane] = v;
            __threadfence();
            __syncwarp();
            int old = 0;
            if (lane == 0) old = atomicAdd(&a.gcount[t], 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old != l - f) continue;
            __threadfence();
            v = 0.0;
            for (int o = 0; o <= l - f; ++o) v += __ldcg(gp + o * 32 + lane);
            if (lane == 0) a.gcount[t] = 0;
        }
        if constexpr (EPI == kEpiPartial) {
            const int r = t * kTileRows + lane;
            if (r < a.W.rows) a.ypart[r] = v;  // rounded once, after the sum over ranks
        } else {
            tile_epilogue<EPI>(a, t, lane, __double2float_rn(v), tok, a.rope_cs);
        }
    }
}

// ---------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------
template <int PRO, int EPI>
static cudaError_t launch_t(const GemvArgs &a, int grid, cudaStream_t s, bool pdl) {
    // The shared-memory opt-in is per device; remember which devices have it.
    static unsigned long long configured = 0;
    const size_t smem = sizeof(GemvSmem);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(gemv_q4_kernel<PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_q4_kernel<PRO, EPI>, a);
}

template <int P, int E>
static cudaError_t configure_one() {
    return cudaFuncSetAttribute(gemv_q4_kernel<P, E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(GemvSmem)));
}

#define BMO_GEMV_VARIANTS(X)  \
    X(kProNorm, kEpiQKV)      \
    X(kProPlain, kEpiResid)   \
    X(kProNorm, kEpiSwiGLU)   \
    X(kProNorm, kEpiLogits)   \
    X(kProPlain, kEpiLogits)  \
    X(kProPlain, kEpiEmbAdd)  \
    X(kProPlain, kEpiStore)   \
    X(kProNorm, kEpiStore)    \
    X(kProPlain, kEpiSwiGLU)  \
    X(kProNorm, kEpiResid)    \
    X(kProPlain, kEpiPartial)

cudaError_t configure_gemv() {
    cudaError_t e = cudaSuccess;
#define BMO_GEMV_CFG(P, E) \
    if ((e = configure_one<P, E>()) != cudaSuccess) return e;
    BMO_GEMV_VARIANTS(BMO_GEMV_CFG)
#undef BMO_GEMV_CFG
    return e;
}

static long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }

// Smallest stream-K grid whose CTAs stay within the partial table.
static long long streamk_min_grid(const QMatDesc &m) {
    return ceil_div(m.n_tiles, kMaxTilesPerCta - 2);
}

GemvPlan plan_gemv(const QMatDesc &m, int sms) {
    const long long nc = static_cast<long long>(m.n_tiles) * m.cpt;
    long long gs = std::min<long long>(sms, nc);
    gs = std::max(gs, std::min(streamk_min_grid(m), nc));
    long long ga = std::min<long long>(sms, m.n_tiles);
    ga = std::max(ga, ceil_div(m.n_tiles, kMaxTilesPerCta));
    const long long busiest_aligned = ceil_div(m.n_tiles, ga) * m.cpt;
    const long long busiest_streamk = ceil_div(nc, gs);
    if (busiest_aligned <= busiest_streamk + kCombineChunks) return GemvPlan{static_cast<int>(ga), 1};
    return GemvPlan{static_cast<int>(std::max<long long>(gs, 1)), 0};
}

cudaError_t launch_gemv(const GemvArgs &a, int prologue, int epilogue, int grid, cudaStream_t s, bool pdl) {
    if (a.W.nbx > kMaxNbx || grid <= 0 || a.W.cpt <= 0 || a.W.n_tiles <= 0) return cudaErrorInvalidValue;
    if (prologue == kProNorm && a.W.cols > kMaxNormCols) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(a.x) & 15) return cudaErrorInvalidValue;
    // every CTA's tile range must fit the shared partial table
    const long long nc = static_cast<long long>(a.W.n_tiles) * a.W.cpt;
    if (a.tile_aligned) {
        if (grid > a.W.n_tiles || ceil_div(a.W.n_tiles, grid) > kMaxTilesPerCta) return cudaErrorInvalidValue;
    } else {
        if (grid > nc) return cudaErrorInvalidValue;
        const long long per_cta = ceil_div(nc, grid);
        if (ceil_div(per_cta, a.W.cpt) + 1 > kMaxTilesPerCta) return cudaErrorInvalidValue;
    }
#define BMO_GEMV_CASE(P, E) \
    if (prologue == P && epilogue == E) return launch_t<P, E>(a, grid, s, pdl);
    BMO_GEMV_VARIANTS(BMO_GEMV_CASE)
#undef BMO_GEMV_CASE
    return cudaErrorInvalidValue;
}

}  // namespace bmo
