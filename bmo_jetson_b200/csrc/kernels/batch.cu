// batch.cu -- batched decode (config 4 of the reference's benchmark plan):
// up to 64 independent sessions per GPU, each with its own KV ring and
// position, stepped in lockstep so that every weight byte is streamed once
// per frame for all of them.
//
// Each GEMV becomes two kernels:
//  * batch_stage_kernel: one CTA per session -- RMSNorm (optional) and the
//    Q8_1 quantiser of bmo_quantize_row_q8_1_kernel (bmo_cuda_kernels.cu:
//    529-558), written in the block-major layout of layout.h; for the
//    depformer input it also resolves the session's token from the previous
//    head's per-tile argmax pairs;
//  * batch_gemm_kernel: the CUDA-core form of the skinny GEMM
//    Y[S][rows] = X[S][cols] . W^T (the tensor-core form is batch_mma.cu)
//    with the reference's Q4_0 x Q8_1 arithmetic per (session, row): the same
//    half-block fp32 terms as the batch-1 GEMV (gemv_dev.cuh), summed in
//    double and rounded once.  A CTA owns whole row tiles; its 4 warps form 2
//    teams of 2, a team working on one row tile at a time, warp g of a team
//    serving sessions [32g, 32g + 32) with one lane per session.  Per 8-block
//    chunk a team's 2-slot ring receives, through the TMA bulk-copy engine,
//    the weight chunk (4.6 KB) and the sessions' Q8_1 codes and scales for it
//    (P x 608 B, L2-resident).  Weight rows are shared-memory broadcasts; each
//    lane keeps its session's 32 row sums in registers, so the fused epilogue
//    (RoPE + KV append into the session's ring, SwiGLU, residual, logits +
//    argmax, embedding add) runs per lane with no cross-warp reduction.
// Every mbarrier wait is bounded; a timeout raises the status word.
#include <atomic>

#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

constexpr int kBtTeams = 2;
constexpr int kBtWarps = 2 * kBtTeams;
constexpr int kBtThreads = kBtWarps * 32;
constexpr int kBtSlots = 2;
constexpr int kBtXqBytes = kBatchMax * 8 * 64;   // Q8_1 codes of one chunk, all sessions (half-split rows)
constexpr int kBtXdsBytes = kBatchMax * 8 * 12;  // their scales
constexpr int kBtSlotBytes = kChunkBytes + kBtXqBytes + kBtXdsBytes;
static_assert(kBtSlotBytes % 16 == 0, "bulk-copy destinations stay 16-byte aligned");
static_assert(kBatchMax <= 2 * 32, "two warps of a team cover the sessions");

struct BatchSmem {
    uint64_t full[kBtTeams][kBtSlots];
    uint64_t empty[kBtTeams][kBtSlots];
    int err;
    alignas(128) uint8_t slot[kBtTeams][kBtSlots][kBtSlotBytes];
};

size_t batch_gemm_smem_bytes() { return sizeof(BatchSmem); }

// Tiles per CTA: whole row tiles, at most one per team per pass.
int batch_gemm_grid(const QMatDesc &m, int sms) { return m.n_tiles < sms ? m.n_tiles : sms; }

// ---------------------------------------------------------------------------
// staging: x -> (RMSNorm) -> Q8_1, one CTA per session
// ---------------------------------------------------------------------------
template <bool NORM>
__global__ void __launch_bounds__(256) batch_stage_kernel(const __grid_constant__ BatchStageArgs a) {
    __shared__ double red[8];
    __shared__ float tok_v[8];
    __shared__ int tok_i[8];
    const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *x = a.x + static_cast<long long>(s) * a.x_stride;
    const int nb = a.cols / 32, P = batch_pad(a.n_sess);
    if (a.tok) {
        TokenSrc src{};
        src.pairs = a.pairs ? a.pairs + static_cast<long long>(s) * a.pairs_stride : nullptr;
        src.n_pairs = a.n_pairs;
        src.tok = a.tok_in ? a.tok_in + s : nullptr;
        const int t = resolve_token<256>(src, tok_v, tok_i, [] { __syncthreads(); });
        if (tid == 0) {
            a.tok[s] = t;
            if (a.tok_out) a.tok_out[static_cast<long long>(s) * a.tok_out_stride] = t;
        }
    }
    float scale = 1.0f;
    if constexpr (NORM) {
        double ss = 0.0;
        for (int i = tid; i < a.cols; i += 256) {
            const double xv = static_cast<double>(__ldcg(x + i));
            ss = fma(xv, xv, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < 8; ++w) tot += red[w];
        const float total = __double2float_rn(tot);
        const float mean_eps = __fadd_rn(__fdiv_rn(total, static_cast<float>(a.cols)), a.eps);
        scale = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(static_cast<double>(mean_eps))));
    }
    for (int b = tid; b < a.nbx; b += 256) {
        // rows 2s (codes 0-7, 16-23) and 2s + 1 (codes 8-15, 24-31) of the block's B operand,
        // 16-byte K slices k = 0 (elements 0-15) and k = 1 (elements 16-31)
        int8_t *blk = a.xq + static_cast<long long>(b) * P * 64;
        const int r0 = 2 * s, r1 = 2 * s + 1;
        int4 *lo0 = reinterpret_cast<int4 *>(blk + (r0 >> 3) * 256 + (r0 & 7) * 16);
        int4 *lo1 = reinterpret_cast<int4 *>(blk + (r0 >> 3) * 256 + 128 + (r0 & 7) * 16);
        int4 *hi0 = reinterpret_cast<int4 *>(blk + (r1 >> 3) * 256 + (r1 & 7) * 16);
        int4 *hi1 = reinterpret_cast<int4 *>(blk + (r1 >> 3) * 256 + 128 + (r1 & 7) * 16);
        float *sc = a.xds + static_cast<long long>(b) * P * 3;
        float *d4p = sc + (s >> 1) * 4 + (s & 1);      // d8 at [0], -M d8 at [2]
        float *s4p = sc + 2 * P + (s >> 1) * 2 + (s & 1);
        if (b >= nb) {
            *lo0 = *lo1 = *hi0 = *hi1 = make_int4(0, 0, 0, 0);
            d4p[0] = 0.0f;
            d4p[2] = 0.0f;
            *s4p = 0.0f;
            continue;
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __ldcg(x + b * 32 + j);
        if constexpr (NORM) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), a.gamma[b * 32 + j]);
        }
        if (a.xn_out) {
            float *xo = a.xn_out + static_cast<long long>(s) * a.xn_stride + b * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) xo[j] = v[j];
        }
        int8_t q[32];
        const __half2 ds = quant_block_q8_1(v, q);
        const int *qi = reinterpret_cast<const int *>(q);
        *lo0 = make_int4(qi[0], qi[1], 0, 0);
        *lo1 = make_int4(qi[4], qi[5], 0, 0);
        *hi0 = make_int4(0, 0, qi[2], qi[3]);
        *hi1 = make_int4(0, 0, qi[6], qi[7]);
        const float d8 = __low2float(ds);
        d4p[0] = d8;
        d4p[2] = -12582912.0f * d8;  // exact: 1.5 * 2^23 times an 11-bit significand
        *s4p = -4.0f * __high2float(ds);
    }
}

// ---------------------------------------------------------------------------
// per-lane epilogue helpers
// ---------------------------------------------------------------------------
// Q4_0 block of 32 values held by one thread (ggml quantize_row_q4_0_ref, the
// rule of warp_store_q4_0): signed max by magnitude, first occurrence.
__device__ __forceinline__ void thread_store_q4_0(const float (&x)[32], uint8_t *qs_dst, __half *d_dst) {
    float amax = 0.0f, mx = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(x[j]);
        if (a > amax) { amax = a; mx = x[j]; }
    }
    const float d = __fdiv_rn(mx, -8.0f);
    const float id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;
    uint8_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) q[j] = static_cast<uint8_t>(min(15, __float2int_rz(__fadd_rn(__fmul_rn(x[j], id), 8.5f))));
#pragma unroll
    for (int j = 0; j < 16; ++j) qs_dst[j] = static_cast<uint8_t>(q[j] | (q[j + 16] << 4));
    *d_dst = __float2half_rn(d);
}

template <int EPI>
__device__ __forceinline__ void batch_tile_epilogue(const BatchGemmArgs &a, int t, int s, const double (&acc)[32]) {
    float v[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) v[r] = __double2float_rn(acc[r]);
    const long long ys = static_cast<long long>(s) * a.y_stride;
    const int r0 = t * kTileRows;
    if constexpr (EPI == kEpiStore) {
#pragma unroll
        for (int r = 0; r < 32; ++r)
            if (r0 + r < a.W.rows) a.y[ys + r0 + r] = a.bias ? __fadd_rn(v[r], a.bias[r0 + r]) : v[r];
    } else if constexpr (EPI == kEpiResid) {
        const float *res = a.resid + static_cast<long long>(s) * a.resid_stride;
#pragma unroll
        for (int r = 0; r < 32; ++r)
            if (r0 + r < a.W.rows) a.y[ys + r0 + r] = __fadd_rn(__ldcg(res + r0 + r), v[r]);
    } else if constexpr (EPI == kEpiSwiGLU) {
        // rows 0-15 of the tile are gate rows 16t + r, rows 16-31 the matching up rows
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int h = t * 16 + r;
            if (h < a.W.swiglu_f) {
                const float e = __double2float_rn(exp(-static_cast<double>(v[r])));
                const float silu = __fdiv_rn(v[r], __fadd_rn(1.0f, e));
                a.y[ys + h] = __fmul_rn(silu, v[r + 16]);
            }
        }
    } else if constexpr (EPI == kEpiLogits) {
        // first maximum of the tile; an all -inf (or fully excluded) tile
        // reports its first row, as the batch-1 epilogue
        float bv = -INFINITY;
        int bi = r0;
#pragma unroll
        for (int r = 0; r < 32; ++r) {
            const int row = r0 + r;
            if (row < a.W.rows) {
                const float val = a.bias ? __fadd_rn(v[r], a.bias[row]) : v[r];
                a.y[ys + row] = val;
                if (row < a.argmax_limit && val > bv) { bv = val; bi = row; }
            }
        }
        a.pairs[static_cast<long long>(s) * a.pairs_stride + t] = make_float2(bv, __int_as_float(bi));
    } else if constexpr (EPI == kEpiEmbAdd) {
        const int tok = a.tok[s];
        const bool ok = tok >= 0 && tok < a.emb.rows && a.emb.dim == a.W.rows;
#pragma unroll
        for (int r = 0; r < 32; ++r)
            if (r0 + r < a.W.rows) a.y[ys + r0 + r] = ok ? __fadd_rn(v[r], emb_elem(a.emb, tok, r0 + r)) : __fadd_rn(v[r], 0.0f);
    } else if constexpr (EPI == kEpiQKV) {
        // the tile lies inside one head of q, k or v (head_dim % 32 == 0)
        const int hd = a.head_dim;
        const bool is_q = r0 < a.q_dim;
        const bool is_k = !is_q && r0 < a.q_dim + a.kv_dim;
        float out[32];
#pragma unroll
        for (int r = 0; r < 32; ++r) out[r] = v[r];
        if ((is_q || is_k) && a.rope) {
            const float2 *cs = a.rope + static_cast<long long>(s) * (hd / 2);
            const int d0 = (is_q ? r0 : r0 - a.q_dim) % hd;
#pragma unroll
            for (int r = 0; r < 32; r += 2) {
                const float2 c = cs[(d0 + r) >> 1];
                out[r] = __fsub_rn(__fmul_rn(v[r], c.x), __fmul_rn(v[r + 1], c.y));
                out[r + 1] = __fadd_rn(__fmul_rn(v[r], c.y), __fmul_rn(v[r + 1], c.x));
            }
        }
        if (is_q) {
#pragma unroll
            for (int r = 0; r < 32; ++r) a.y[ys + r0 + r] = out[r];
            return;
        }
        const int rr0 = is_k ? r0 - a.q_dim : r0 - a.q_dim - a.kv_dim;
        if (!is_k && a.v_out) {
            float *vo = a.v_out + static_cast<long long>(s) * a.v_out_stride;
#pragma unroll
            for (int r = 0; r < 32; ++r) vo[rr0 + r] = v[r];
        }
        const int kh = rr0 / hd, d0 = rr0 % hd;
        const int slot = a.pos[s * a.pos_stride] % a.n_ctx;
        const long long ring = a.ring_of ? a.ring_of[s] : s;
        const long long e0 = ring * a.kv_sess_stride + a.kv_layer_off + (static_cast<long long>(kh) * a.n_ctx + slot) * hd + d0;
        void *cache = is_k ? a.k_cache : a.v_cache;
        if (a.kv_type == kKvF16) {
            __half *c = static_cast<__half *>(cache) + e0;
#pragma unroll
            for (int r = 0; r < 32; ++r) c[r] = __float2half_rn(out[r]);
        } else {
            uint8_t *qs = static_cast<uint8_t *>(cache) + e0 / 2;
            __half *dp = reinterpret_cast<__half *>(is_k ? a.k_scale : a.v_scale) + e0 / 32;
            thread_store_q4_0(out, qs, dp);
        }
    }
}

// ---------------------------------------------------------------------------
// skinny GEMM
// ---------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(kBtThreads, 1) batch_gemm_kernel(const __grid_constant__ BatchGemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    BatchSmem &S = *reinterpret_cast<BatchSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int team = warp >> 1, g = warp & 1;
    const int G = gridDim.x, c = blockIdx.x;
    const int cpt = a.W.cpt, ns = a.n_sess, P = batch_pad(ns);
    const int t0 = static_cast<int>(static_cast<long long>(a.W.n_tiles) * c / G);
    const int t1 = static_cast<int>(static_cast<long long>(a.W.n_tiles) * (c + 1) / G);
    const int n_tiles_team = t1 - t0 > team ? (t1 - t0 - team + kBtTeams - 1) / kBtTeams : 0;
    const int units = n_tiles_team * cpt;
    const uint32_t xqb = static_cast<uint32_t>(P) * 512u, xdsb = static_cast<uint32_t>(P) * 96u;

    if (tid < kBtTeams * kBtSlots) {
        mbar_init(&S.full[tid / kBtSlots][tid % kBtSlots], 1);
        mbar_init(&S.empty[tid / kBtSlots][tid % kBtSlots], 2);
    }
    if (tid == 0) S.err = 0;
    fence_barrier_init();
    __syncthreads();

    const bool issuer = g == 0 && lane == 0;
    const uint64_t pol_w = l2_evict_first_policy(), pol_x = l2_evict_last_policy();
    auto issue = [&](int u) {
        const int i = u / cpt, kc = u - i * cpt;
        const int t = t0 + team + kBtTeams * i;
        const int sl = u % kBtSlots;
        uint8_t *dst = S.slot[team][sl];
        uint64_t *bar = &S.full[team][sl];
        mbar_arrive_expect_tx(bar, kChunkBytes + xqb + xdsb);
        bulk_load(dst, a.W.tiles + (static_cast<size_t>(t) * cpt + kc) * kChunkBytes, kChunkBytes, bar, pol_w);
        bulk_load(dst + kChunkBytes, a.xq + static_cast<size_t>(kc) * 8 * P * 64, xqb, bar, pol_x);
        bulk_load(dst + kChunkBytes + kBtXqBytes, a.xds + static_cast<size_t>(kc) * 8 * P * 3, xdsb, bar, pol_x);
    };
    int issued = 0;  // meaningful in the issuing thread only
    if (issuer)
        for (; issued < kBtSlots && issued < units; ++issued) issue(issued);

    const int sess = 32 * g + lane;
    const bool act = sess < ns;
    double acc[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) acc[r] = 0.0;
    bool ok = true;
    int consumed = 0;  // units whose copies have landed
    for (int u = 0; u < units; ++u) {
        const int sl = u % kBtSlots;
        const uint32_t par = (u / kBtSlots) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&S.full[team][sl], par))) {
            ok = false;
            break;
        }
        consumed = u + 1;
        const uint8_t *w = S.slot[team][sl];
        const int8_t *xq = reinterpret_cast<const int8_t *>(w + kChunkBytes);
        const float *xds = reinterpret_cast<const float *>(w + kChunkBytes + kBtXqBytes);
#pragma unroll 1
        for (int blk = 0; blk < kChunkBlocks; ++blk) {
            int4 xa = make_int4(0, 0, 0, 0), xb = make_int4(0, 0, 0, 0);
            float2 ds = make_float2(0.0f, 0.0f);
            if (act) {
                // codes 0-15 and 16-31 from the two half-block rows
                const int8_t *xp = xq + blk * P * 64;
                const int r0 = 2 * sess, r1 = 2 * sess + 1;
                const int2 l0 = *reinterpret_cast<const int2 *>(xp + (r0 >> 3) * 256 + (r0 & 7) * 16);
                const int2 h0 = *reinterpret_cast<const int2 *>(xp + (r1 >> 3) * 256 + (r1 & 7) * 16 + 8);
                const int2 l1 = *reinterpret_cast<const int2 *>(xp + (r0 >> 3) * 256 + 128 + (r0 & 7) * 16);
                const int2 h1 = *reinterpret_cast<const int2 *>(xp + (r1 >> 3) * 256 + 128 + (r1 & 7) * 16 + 8);
                xa = make_int4(l0.x, l0.y, h0.x, h0.y);
                xb = make_int4(l1.x, l1.y, h1.x, h1.y);
                const float *sp = xds + blk * P * 3;
                ds = make_float2(sp[(sess >> 1) * 4 + (sess & 1)], -sp[2 * P + (sess >> 1) * 2 + (sess & 1)]);  // (d8, 4 s8)
            }
            const uint8_t *wb = w + blk * 512;
            const __half *db = reinterpret_cast<const __half *>(w + kChunkQsBytes + blk * 64);
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                const uint4 wv = *reinterpret_cast<const uint4 *>(wb + r * 16);  // broadcast
                const float d4 = __half2float(db[r]);
                int lo = __dp4a(static_cast<int>(wv.x & 0x0F0F0F0Fu), xa.x, 0);
                lo = __dp4a(static_cast<int>((wv.x >> 4) & 0x0F0F0F0Fu), xb.x, lo);
                lo = __dp4a(static_cast<int>(wv.y & 0x0F0F0F0Fu), xa.y, lo);
                lo = __dp4a(static_cast<int>((wv.y >> 4) & 0x0F0F0F0Fu), xb.y, lo);
                int hi = __dp4a(static_cast<int>(wv.z & 0x0F0F0F0Fu), xa.z, 0);
                hi = __dp4a(static_cast<int>((wv.z >> 4) & 0x0F0F0F0Fu), xb.z, hi);
                hi = __dp4a(static_cast<int>(wv.w & 0x0F0F0F0Fu), xa.w, hi);
                hi = __dp4a(static_cast<int>((wv.w >> 4) & 0x0F0F0F0Fu), xb.w, hi);
                acc[r] += static_cast<double>(half_term(lo, d4, ds));
                acc[r] += static_cast<double>(half_term(hi, d4, ds));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[team][sl]);
        if (issuer && issued < units) {
            // both warps of the team are done with the slot
            if (!mbar_wait(&S.empty[team][sl], par)) {
                ok = false;
            } else {
                fence_proxy_async();
                issue(issued);
                ++issued;
            }
        }
        const int i = u / cpt, kc = u - i * cpt;
        if (kc == cpt - 1) {
            if (act) batch_tile_epilogue<EPI>(a, t0 + team + kBtTeams * i, sess, acc);
#pragma unroll
            for (int r = 0; r < 32; ++r) acc[r] = 0.0;
        }
        if (!__all_sync(0xffffffffu, ok)) break;
    }
    if (!ok && lane == 0) atomicOr(&S.err, 1);
    __syncthreads();
    if (S.err) {
        if (tid == 0) raise_error(a.status, kErrTmaTimeout);
        // copies still in flight land before the CTA exits (bounded waits)
        if (issuer)
            for (int v = consumed; v < issued; ++v) mbar_wait(&S.full[team][v % kBtSlots], (v / kBtSlots) & 1);
    }
}

// ---------------------------------------------------------------------------
// embedding sum and RoPE tables of all sessions; last greedy token
// ---------------------------------------------------------------------------
__global__ void batch_embed_kernel(const EmbTable *tables, int n_tables, const BatchIn *in, int n_embd, float *out,
                                   float theta, int head_dim, float2 *rope) {
    const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    const int *tk = in->tokens + s * kBatchMaxTokens;
    const int n_tok = in->n_tok;
    if (i < n_embd) {
        // bmo_embed_input_tokens_into (bmo_compute.cpp:1867-1912), as embed_kernel
        float acc = 0.0f;
        for (int ch = 0; ch < n_tok && ch < n_tables; ++ch) {
            const EmbTable t = tables[ch];
            const int tok = tk[ch];
            if (!t.data || tok < 0 || tok >= t.rows || t.dim != n_embd) continue;
            acc = __fadd_rn(acc, emb_elem(t, tok, i));
        }
        out[static_cast<long long>(s) * n_embd + i] = acc;
    }
    if (blockIdx.x == 0 && rope && threadIdx.x < head_dim / 2) {
        // exponent and angle in fp32 as the reference; power and trig in double, rounded once
        const int k = threadIdx.x;
        const float exponent = __fdiv_rn(static_cast<float>(2 * k), static_cast<float>(head_dim));
        const float inv_freq = __double2float_rn(pow(static_cast<double>(theta), -static_cast<double>(exponent)));
        const float angle = __fmul_rn(static_cast<float>(in->pos[s]), inv_freq);
        double sn, cs;
        sincos(static_cast<double>(angle), &sn, &cs);
        rope[static_cast<long long>(s) * (head_dim / 2) + k] = make_float2(__double2float_rn(cs), __double2float_rn(sn));
    }
}

// Device-resident inputs of a batched frame from device arrays.
__global__ void batch_set_inputs_kernel(BatchIn *in, const int *sess, const int *tokens, int K, const int *pos, int n) {
    const int s = blockIdx.x;
    if (s >= n) return;
    for (int k = threadIdx.x; k < kBatchMaxTokens; k += blockDim.x)
        in->tokens[s * kBatchMaxTokens + k] = k < K ? tokens[s * K + k] : 0;
    if (threadIdx.x == 0) {
        in->sess[s] = sess ? sess[s] : s;
        in->pos[s] = pos[s];
        if (s == 0) in->n_tok = K;
    }
}

__global__ void batch_finalize_kernel(const float2 *pairs, int pairs_stride, int n_pairs, int *out, int out_stride) {
    __shared__ float v[8];
    __shared__ int ix[8];
    const int s = blockIdx.x;
    TokenSrc src{};
    src.pairs = pairs + static_cast<long long>(s) * pairs_stride;
    src.n_pairs = n_pairs;
    const int t = resolve_token<256>(src, v, ix, [] { __syncthreads(); });
    if (threadIdx.x == 0) out[static_cast<long long>(s) * out_stride] = t;
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
cudaError_t launch_batch_stage(const BatchStageArgs &a, cudaStream_t s) {
    if (a.n_sess < 1 || a.n_sess > kBatchMax || a.cols <= 0 || a.cols % 32 || a.nbx < a.cols / 32 || a.nbx % 8)
        return cudaErrorInvalidValue;
    if (a.gamma) batch_stage_kernel<true><<<a.n_sess, 256, 0, s>>>(a);
    else batch_stage_kernel<false><<<a.n_sess, 256, 0, s>>>(a);
    return cudaGetLastError();
}

template <int EPI>
static cudaError_t launch_bg(const BatchGemmArgs &a, int grid, cudaStream_t s) {
    batch_gemm_kernel<EPI><<<grid, kBtThreads, sizeof(BatchSmem), s>>>(a);
    return cudaGetLastError();
}

template <int EPI>
static cudaError_t configure_bg() {
    return cudaFuncSetAttribute(batch_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(BatchSmem)));
}

static std::atomic<unsigned long long> g_bg_configured{0};  // bit per device

cudaError_t configure_batch() {
    const cudaError_t es[] = {configure_bg<kEpiStore>(), configure_bg<kEpiResid>(), configure_bg<kEpiSwiGLU>(),
                              configure_bg<kEpiQKV>(),   configure_bg<kEpiLogits>(), configure_bg<kEpiEmbAdd>()};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return e;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev < 64) g_bg_configured.fetch_or(1ull << dev);
    return cudaSuccess;
}

static cudaError_t ensure_bg_configured() {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev < 64 && (g_bg_configured.load() & (1ull << dev))) return cudaSuccess;
    return configure_batch();
}

cudaError_t launch_batch_gemm(const BatchGemmArgs &a, int epi, int grid, cudaStream_t s) {
    if (a.n_sess < 1 || a.n_sess > kBatchMax || grid <= 0 || grid > a.W.n_tiles || a.W.cpt <= 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a.xq) & 15) || (reinterpret_cast<uintptr_t>(a.xds) & 15)) return cudaErrorInvalidValue;
    const cudaError_t ce = ensure_bg_configured();
    if (ce != cudaSuccess) return ce;
    switch (epi) {
    case kEpiStore: return launch_bg<kEpiStore>(a, grid, s);
    case kEpiResid: return launch_bg<kEpiResid>(a, grid, s);
    case kEpiSwiGLU: return launch_bg<kEpiSwiGLU>(a, grid, s);
    case kEpiQKV:
        if (a.head_dim % 32 || a.q_dim % 32 || a.kv_dim % 32) return cudaErrorInvalidValue;
        return launch_bg<kEpiQKV>(a, grid, s);
    case kEpiLogits: return launch_bg<kEpiLogits>(a, grid, s);
    case kEpiEmbAdd: return launch_bg<kEpiEmbAdd>(a, grid, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_batch_embed(const EmbTable *tables, int n_tables, const BatchIn *in, int n_embd, float *out,
                               int n_sess, float theta, int head_dim, float2 *rope, cudaStream_t s) {
    if (n_sess < 1 || n_sess > kBatchMax || head_dim / 2 > 256) return cudaErrorInvalidValue;
    const int threads = 256;
    dim3 grid((n_embd + threads - 1) / threads, n_sess);
    batch_embed_kernel<<<grid, threads, 0, s>>>(tables, n_tables, in, n_embd, out, theta, head_dim, rope);
    return cudaGetLastError();
}

cudaError_t launch_batch_set_inputs(BatchIn *in, const int *sess, const int *tokens, int K, const int *pos, int n,
                                    cudaStream_t s) {
    if (n < 1 || n > kBatchMax || K < 0 || K > kBatchMaxTokens) return cudaErrorInvalidValue;
    batch_set_inputs_kernel<<<n, 64, 0, s>>>(in, sess, tokens, K, pos, n);
    return cudaGetLastError();
}

cudaError_t launch_batch_finalize(const float2 *pairs, int pairs_stride, int n_pairs, int *out, int out_stride,
                                  int n_sess, cudaStream_t s) {
    if (n_sess < 1 || n_sess > 65535) return cudaErrorInvalidValue;
    batch_finalize_kernel<<<n_sess, 256, 0, s>>>(pairs, pairs_stride, n_pairs, out, out_stride);
    return cudaGetLastError();
}

}  // namespace bmo
