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
// Design (B200): one CTA per SM, 8 warps.  The weight stream is the only
// HBM traffic that matters, so each warp keeps kRing 4.6 KB chunks in flight
// through the TMA bulk-copy engine into a private shared-memory ring.  The
// first chunks are issued before griddepcontrol.wait, so under programmatic
// dependent launch the stream starts while the previous kernel finishes.
// Work is split "stream-K" style: CTA c owns a contiguous range of
// (row tile, chunk) units, tiles that straddle CTAs are finished by the last
// owner to arrive (per-tile counter, fixed summation order, deterministic).
// Epilogues fuse RoPE + KV-ring append, SwiGLU, residual adds, logits +
// argmax and the depformer embedding add.
#include "common.cuh"
#include "../launch.h"

namespace bmo {

#ifndef BMO_GEMV_RING
#define BMO_GEMV_RING 2
#endif
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRing = BMO_GEMV_RING;  // chunks in flight per warp
constexpr int kMaxNbx = 384;  // activations up to 12288 elements
constexpr int kMaxTilesPerCta = 10;

struct GemvSmem {
    uint64_t bar[kWarps][kRing];
    alignas(128) uint8_t ring[kWarps][kRing][kChunkBytes];
    alignas(16) int8_t xq[kMaxNbx * 32];
    float2 xds[kMaxNbx];  // (d8, 4 * s8) of each Q8_1 block
    double part[kMaxTilesPerCta][kWarps][32];
    double red[kWarps];
    float tok_v[kWarps];
    int tok_i[kWarps];
    int err;
};

size_t gemv_smem_bytes() { return sizeof(GemvSmem); }
int gemv_max_tiles_per_cta() { return kMaxTilesPerCta; }
int gemv_max_nbx() { return kMaxNbx; }

__device__ __forceinline__ int cta_of_chunk(long long k, long long nc, int g) {
    return static_cast<int>(((k + 1) * g - 1) / nc);
}

// One half-block term of the reference: d4 * ((float)sumi * d8 - 4 * s8).
__device__ __forceinline__ float half_term(int sumi, float d4, float2 ds) {
    return __fmul_rn(d4, __fsub_rn(__fmul_rn(static_cast<float>(sumi), ds.x), ds.y));
}

// Dot product of one 8-block chunk (32 rows, lane = row) with the activation.
__device__ __forceinline__ double chunk_dot(const uint8_t *ch, const int8_t *xq, const float2 *xds, int lane) {
    double acc = 0.0;
#pragma unroll
    for (int blk = 0; blk < kChunkBlocks; ++blk) {
        const uint4 w = *reinterpret_cast<const uint4 *>(ch + blk * 512 + lane * 16);
        const float d4 = __half2float(*reinterpret_cast<const __half *>(ch + kChunkQsBytes + blk * 64 + lane * 2));
        const int4 xa = *reinterpret_cast<const int4 *>(xq + blk * 32);
        const int4 xb = *reinterpret_cast<const int4 *>(xq + blk * 32 + 16);
        const float2 ds = xds[blk];
        // byte j holds element j (low nibble) and element j+16 (high nibble);
        // bytes 0-7 form the first half block, bytes 8-15 the second
        int lo = __dp4a(static_cast<int>(w.x & 0x0F0F0F0Fu), xa.x, 0);
        lo = __dp4a(static_cast<int>((w.x >> 4) & 0x0F0F0F0Fu), xb.x, lo);
        lo = __dp4a(static_cast<int>(w.y & 0x0F0F0F0Fu), xa.y, lo);
        lo = __dp4a(static_cast<int>((w.y >> 4) & 0x0F0F0F0Fu), xb.y, lo);
        int hi = __dp4a(static_cast<int>(w.z & 0x0F0F0F0Fu), xa.z, 0);
        hi = __dp4a(static_cast<int>((w.z >> 4) & 0x0F0F0F0Fu), xb.z, hi);
        hi = __dp4a(static_cast<int>(w.w & 0x0F0F0F0Fu), xa.w, hi);
        hi = __dp4a(static_cast<int>((w.w >> 4) & 0x0F0F0F0Fu), xb.w, hi);
        acc += static_cast<double>(half_term(lo, d4, ds));
        acc += static_cast<double>(half_term(hi, d4, ds));
    }
    return acc;
}

// ---- embedding element fetch (ggml to_float for the supported types) ----
__device__ __forceinline__ float emb_elem(const EmbTable &e, int tok, int i) {
    const uint8_t *row = static_cast<const uint8_t *>(e.data) + static_cast<size_t>(tok) * e.row_bytes;
    switch (e.type) {
    case kTF32: return reinterpret_cast<const float *>(row)[i];
    case kTF16: return __half2float(reinterpret_cast<const __half *>(row)[i]);
    case kTBF16: return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t *>(row)[i]) << 16);
    case kTQ4_0: {
        const uint8_t *b = row + (i >> 5) * 18;
        const float d = __half2float(*reinterpret_cast<const __half *>(b));
        const int j = i & 31;
        const int nib = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
        return __fmul_rn(static_cast<float>(nib - 8), d);
    }
    case kTQ8_0: {
        const uint8_t *b = row + (i >> 5) * 34;
        const float d = __half2float(*reinterpret_cast<const __half *>(b));
        return __fmul_rn(static_cast<float>(static_cast<int8_t>(b[2 + (i & 31)])), d);
    }
    default: return 0.0f;
    }
}

// (value, index) max with the lowest index winning ties (first maximum).
__device__ __forceinline__ void argmax_merge(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}

// Resolves the token of an embedding lookup (whole CTA participates).
__device__ int resolve_token(const TokenSrc &src, float *red_v, int *red_i) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (!src.pairs) return src.tok ? *src.tok : -1;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = tid; p < src.n_pairs; p += blockDim.x) {
        const float2 pr = __ldcg(&src.pairs[p]);
        argmax_merge(bv, bi, pr.x, __float_as_int(pr.y));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
    __syncthreads();
    float fv = red_v[0];
    int fi = red_i[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) argmax_merge(fv, fi, red_v[w], red_i[w]);
    __syncthreads();
    return fi;
}

template <int EPI>
__device__ __forceinline__ void tile_epilogue(const GemvArgs &a, int t, int lane, float v, int tok) {
    const int r = t * kTileRows + lane;
    if constexpr (EPI == kEpiStore) {
        if (r < a.W.rows) a.y[r] = a.bias ? __fadd_rn(v, a.bias[r]) : v;
    } else if constexpr (EPI == kEpiResid) {
        if (r < a.W.rows) a.y[r] = __fadd_rn(a.resid[r], v);
    } else if constexpr (EPI == kEpiSwiGLU) {
        // silu(gate) * up (swiglu_split_kernel, bmo_cuda_kernels.cu:370-387),
        // exp evaluated in double and rounded once
        const float up = __shfl_down_sync(0xffffffffu, v, 16);
        const int h = t * 16 + lane;
        if (lane < 16 && h < a.W.swiglu_f) {
            const float e = __double2float_rn(exp(-static_cast<double>(v)));
            const float silu = __fdiv_rn(v, __fadd_rn(1.0f, e));
            a.y[h] = __fmul_rn(silu, up);
        }
    } else if constexpr (EPI == kEpiLogits) {
        float val = -INFINITY;
        if (r < a.W.rows) {
            val = a.bias ? __fadd_rn(v, a.bias[r]) : v;
            a.y[r] = val;
        }
        float bv = (r < a.W.rows && r < a.argmax_limit) ? val : -INFINITY;
        int bi = r;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, ov, oi);
        }
        if (lane == 0 && a.argmax_pairs) a.argmax_pairs[t] = make_float2(bv, __int_as_float(bi));
    } else if constexpr (EPI == kEpiEmbAdd) {
        if (r < a.W.rows) {
            const bool ok = tok >= 0 && tok < a.emb.rows && a.emb.dim == a.W.rows;
            a.y[r] = ok ? __fadd_rn(v, emb_elem(a.emb, tok, r)) : __fadd_rn(v, 0.0f);
        }
    } else if constexpr (EPI == kEpiQKV) {
        // whole tile lies inside one head of q, k or v (head_dim % 32 == 0)
        const int hd = a.head_dim;
        float out = v;
        const bool is_q = r < a.q_dim;
        const bool is_k = !is_q && r < a.q_dim + a.kv_dim;
        if ((is_q || is_k) && a.rope_cs) {
            // interleaved RoPE (rope_interleaved_kernel, :317-368), separately rounded
            const int d = (is_q ? r : r - a.q_dim) % hd;
            const float2 cs = a.rope_cs[d >> 1];
            const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
            out = (lane & 1) ? __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(v, cs.x))
                             : __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(partner, cs.y));
        }
        if (is_q) {
            a.y[r] = out;
            return;
        }
        const int rr = is_k ? r - a.q_dim : r - a.q_dim - a.kv_dim;
        if (!is_k && a.v_out) a.v_out[rr] = v;
        const int kh = rr / hd, d = rr % hd;
        const int slot = *a.pos % a.n_ctx;
        const long long e = a.kv_layer_off + (static_cast<long long>(kh) * a.n_ctx + slot) * hd + d;
        void *cache = is_k ? a.k_cache : a.v_cache;
        if (a.kv_type == kKvF16) {
            static_cast<__half *>(cache)[e] = __float2half_rn(out);
        } else {
            const long long e0 = e - lane;  // first element of this 32-block
            uint8_t *qs = static_cast<uint8_t *>(cache) + e0 / 2;
            __half *dp = reinterpret_cast<__half *>(is_k ? a.k_scale : a.v_scale) + e0 / 32;
            warp_store_q4_0(out, lane, qs, dp);
        }
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_q4_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    GemvSmem &S = *reinterpret_cast<GemvSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int cpt = a.W.cpt;
    const long long NC = static_cast<long long>(a.W.n_tiles) * cpt;
    const int c0 = static_cast<int>(NC * c / G), c1 = static_cast<int>(NC * (c + 1) / G);
    const int n_mine = (c1 - c0 > warp) ? (c1 - c0 - warp + kWarps - 1) / kWarps : 0;

    if (tid < kWarps * kRing) mbar_init(&S.bar[tid / kRing][tid % kRing], 1);
    if (tid == 0) S.err = 0;
    fence_barrier_init();
    __syncthreads();
    pdl_launch_dependents();

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

    pdl_wait();

    // ---- prologue: activation -> Q8_1 blocks in shared memory ----
    const int nb = a.W.cols / 32, nbx = a.W.nbx;
    float scale = 1.0f;
    if constexpr (PRO == kProNorm) {
        // rmsnorm_kernel (bmo_cuda_kernels.cu:244-295): scale = 1/sqrt(mean(x^2)+eps),
        // the sum of squares in double, the root and reciprocal in double
        double ss = 0.0;
        for (int i = tid; i < a.W.cols; i += kThreads) {
            const double xv = static_cast<double>(a.x[i]);
            ss = fma(xv, xv, ss);
        }
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
    }
    for (int b = tid; b < nbx; b += kThreads) {
        int4 *qd = reinterpret_cast<int4 *>(S.xq + b * 32);
        if (b < nb) {
            float v[32];
            int8_t q[32];
            const float4 *xp = reinterpret_cast<const float4 *>(a.x + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 t4 = xp[j];
                v[4 * j] = t4.x; v[4 * j + 1] = t4.y; v[4 * j + 2] = t4.z; v[4 * j + 3] = t4.w;
            }
            if constexpr (PRO == kProNorm) {
                const float4 *gp = reinterpret_cast<const float4 *>(a.gamma + b * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 g4 = gp[j];
                    v[4 * j] = __fmul_rn(__fmul_rn(v[4 * j], scale), g4.x);
                    v[4 * j + 1] = __fmul_rn(__fmul_rn(v[4 * j + 1], scale), g4.y);
                    v[4 * j + 2] = __fmul_rn(__fmul_rn(v[4 * j + 2], scale), g4.z);
                    v[4 * j + 3] = __fmul_rn(__fmul_rn(v[4 * j + 3], scale), g4.w);
                }
            }
            const __half2 ds = quant_block_q8_1(v, q);
            const int *qi = reinterpret_cast<const int *>(q);
            qd[0] = make_int4(qi[0], qi[1], qi[2], qi[3]);
            qd[1] = make_int4(qi[4], qi[5], qi[6], qi[7]);
            S.xds[b] = make_float2(__low2float(ds), 4.0f * __high2float(ds));
            if (c == 0 && a.q8_out) {
                int *o = reinterpret_cast<int *>(a.q8_out + static_cast<size_t>(b) * 36);
                o[0] = *reinterpret_cast<const int *>(&ds);
#pragma unroll
                for (int j = 0; j < 8; ++j) o[1 + j] = qi[j];
            }
            if (c == 0 && a.xn_out) {
                float4 *xo = reinterpret_cast<float4 *>(a.xn_out + b * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) xo[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        } else {
            qd[0] = make_int4(0, 0, 0, 0);
            qd[1] = make_int4(0, 0, 0, 0);
            S.xds[b] = make_float2(0.0f, 0.0f);
        }
    }
    for (int i = tid; i < kMaxTilesPerCta * kWarps * 32; i += kThreads) (&S.part[0][0][0])[i] = 0.0;
    int tok = -1;
    if constexpr (EPI == kEpiEmbAdd) {
        tok = resolve_token(a.tok, S.tok_v, S.tok_i);
        if (c == 0 && tid == 0 && a.tok.tok_out) *a.tok.tok_out = tok;
    }
    __syncthreads();

    // ---- main loop: stream chunks through the ring ----
    const int t_first = c0 / cpt;
    int cur = -1;
    double acc = 0.0;
    for (int i = 0; i < n_mine; ++i) {
        const int k = c0 + warp + kWarps * i;
        const int tile = k / cpt, kc = k - tile * cpt;
        if (tile != cur) {
            if (cur >= 0) S.part[cur - t_first][warp][lane] = acc;
            acc = 0.0;
            cur = tile;
        }
        if (!mbar_wait(&S.bar[warp][i % kRing], (i / kRing) & 1)) {
            if (lane == 0) atomicOr(&S.err, 1);
            for (int j = i + 1; j < n_mine && j < i + kRing; ++j) mbar_wait(&S.bar[warp][j % kRing], (j / kRing) & 1);
            cur = -1;
            break;
        }
        acc += chunk_dot(S.ring[warp][i % kRing], S.xq + kc * kChunkBlocks * 32, S.xds + kc * kChunkBlocks, lane);
        __syncwarp();
        if (lane == 0 && i + kRing < n_mine) {
            fence_proxy_async();
            issue(i + kRing);
        }
    }
    if (cur >= 0) S.part[cur - t_first][warp][lane] = acc;
    __syncthreads();
    if (S.err) {
        if (tid == 0) raise_error(a.status, kErrTmaTimeout);
        return;
    }
    if (c1 <= c0) return;

    // ---- per-tile reduction (fixed order, double) and epilogue ----
    const int t_last = (c1 - 1) / cpt;
    for (int tl = warp; tl <= t_last - t_first; tl += kWarps) {
        const int t = t_first + tl;
        double v = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += S.part[tl][w][lane];
        const int f = cta_of_chunk(static_cast<long long>(t) * cpt, NC, G);
        const int l = cta_of_chunk(static_cast<long long>(t) * cpt + cpt - 1, NC, G);
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
        tile_epilogue<EPI>(a, t, lane, __double2float_rn(v), tok);
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
    X(kProNorm, kEpiResid)

cudaError_t configure_gemv() {
    cudaError_t e = cudaSuccess;
#define BMO_GEMV_CFG(P, E) \
    if ((e = configure_one<P, E>()) != cudaSuccess) return e;
    BMO_GEMV_VARIANTS(BMO_GEMV_CFG)
#undef BMO_GEMV_CFG
    return e;
}

cudaError_t launch_gemv(const GemvArgs &a, int prologue, int epilogue, int grid, cudaStream_t s, bool pdl) {
    if (a.W.nbx > kMaxNbx || grid <= 0 || a.W.cpt <= 0 || a.W.n_tiles <= 0) return cudaErrorInvalidValue;
    // every CTA's tile range must fit the shared partial table
    const long long nc = static_cast<long long>(a.W.n_tiles) * a.W.cpt;
    if (grid > nc) return cudaErrorInvalidValue;
    const long long per_cta = (nc + grid - 1) / grid;
    if ((per_cta + a.W.cpt - 1) / a.W.cpt + 1 > kMaxTilesPerCta) return cudaErrorInvalidValue;
#define BMO_GEMV_CASE(P, E) \
    if (prologue == P && epilogue == E) return launch_t<P, E>(a, grid, s, pdl);
    BMO_GEMV_VARIANTS(BMO_GEMV_CASE)
#undef BMO_GEMV_CASE
    return cudaErrorInvalidValue;
}

}  // namespace bmo
