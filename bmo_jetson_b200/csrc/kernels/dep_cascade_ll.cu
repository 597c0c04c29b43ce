// dep_cascade_ll.cu -- the depformer's greedy cascade (dep_q codebook steps,
// each the input projection + embedding of the previous token, the 6 layers
// and the audio head of bmo_build_depth_graph, src/bmo_compute.cpp:2741-3340)
// as ONE cooperative launch over every SM, every value in the reference
// kernels' fp32 order: the same bits as the per-op chain of gemv_ref_kernel /
// attn_ref_kernel.
//
// Why.  The per-op chain pays ~4.6 us per kernel -- the predecessor's
// completion and memory flush, the activation's round trip, the tail -- for
// ops whose weights stream in well under a microsecond across the GPU.
// Here one CTA per SM stays resident for the whole cascade:
//  * weights never depend on activations, so each warp streams its share of
//    every matrix of the cascade, op after op, through a private two-chunk TMA
//    ring that never stops at op boundaries;
//  * an op's output rows go to an exchange region in global memory as 64-bit
//    words (epoch << 32 | value): a consumer polls the words it needs until
//    they carry the op's epoch, so the data and its readiness arrive in one
//    L2 round trip -- no grid barrier, no atomics.  Every phase of a launch
//    has its own region (no CTA can overwrite words another still has to
//    read: the attention phase's writers depend on a few CTAs only), and
//    epochs are unique per launch (a device launch counter), so nothing is
//    reset between launches;
//  * every CTA keeps the residual stream and the op inputs it reads in shared
//    memory, and runs the RMSNorm and Q8_1 quantiser of each op itself;
//  * CTA h runs head h's attention, the head's K/V ring kept in its shared
//    memory;
//  * the input projection's dot products (its input z is fixed for the
//    cascade) run before it waits for the previous head's argmax.
//
// Per-row arithmetic is gemv_ref_kernel's: 32-row tiles, one chain per key
// group (KeyChains) accumulated by chunk_acc_ref, the groups combined in the
// reference's lane order and the 32-leaf shfl_down tree; the RMSNorm, the
// Q8_1 quantiser and the epilogues use the same fp32 operations, the
// attention the shared phases of attention_ref_dev.cuh.  An op's tiles are
// split evenly over the CTAs; a CTA's (tile, key group) items are dealt
// round-robin to its warps, and one warp per tile combines the groups.
//
// Waits: every ring wait is bounded (kWaitPolls); every exchange wait is
// bounded by %globaltimer (2 s) -- a CTA that gives up sets the status bit,
// fills the missing values with zeros and waits no more in this launch, so
// every CTA finishes.  The launch is cooperative: the CTAs that poll each
// other are guaranteed to be resident together.
#include "attention_ref_dev.cuh"
#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

namespace {

constexpr int kLW = 8;                   // warps per CTA
constexpr int kLT = kLW * 32;            // the reference RMSNorm's 256 threads
constexpr int kLRing = 2;                // chunks in flight per warp
constexpr int kLItems = 16;              // (tile, key group) chain buffers of one op per CTA
constexpr int kLMaxLocalTiles = 32;
constexpr int kLMaxIn = 4096;            // exchange entries one CTA reads (16 per thread)
constexpr int kLMaxGrid = 160;           // CTAs (each publishes one argmax pair per head)
constexpr int kLPer = kLMaxIn / kLT;
constexpr int kLHD = 64;                 // depformer head size
constexpr int kLAttnThreads = 128;       // warps 0-3 run the head's attention
constexpr int kLBarAttn = 1;
constexpr unsigned long long kLWaitNs = 2000000000ull;
constexpr unsigned kLPollNs = 100;       // back-off between polls of exchange words
constexpr int kPhasesPerLaunch = 1024;   // epoch stride of one launch (>= the cascade's phases)
constexpr int kLMaxOps = 8 * 26;         // weight ops of a cascade (dep_q <= 8, 6 layers)

__host__ __device__ inline int lnbx(int cols) { return ((cols / 32) + 7) & ~7; }

struct LLLayout {
    uint32_t vec, off_ring, off_part, off_xa, off_xb, off_attn, off_act, off_xq, off_xds, off_zq, off_zds, off_gamma,
        off_kk, off_kv, off_q, off_vraw, off_ss, off_red, off_tpair, off_pairs, off_ops, off_rng, off_misc, bytes;
    __host__ __device__ static uint32_t up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
    __host__ __device__ LLLayout(int dim, int ffn, int n_embd, int n_layers, int n_ctx) {
        const uint32_t nbx_max = lnbx(dim) > lnbx(ffn) ? lnbx(dim) : lnbx(ffn);
        const uint32_t z_nbx = lnbx(n_embd);
        vec = up(dim, 32);
        uint32_t o = (kLW * kLRing + 2) * 8;
        off_ring = o = up(o, 128);
        o += kLW * kLRing * kChunkBytes;
        off_part = o;  // also the prologue's per-warp scratch
        o += kLItems * 2 * kChunkBlocks * 32 * 4;
        off_xa = o;
        o += vec * 4;
        off_xb = o;
        o += vec * 4;
        off_attn = o;
        o += vec * 4;
        off_act = o;
        o += up(ffn, 32) * 4;
        off_xq = o;
        o += nbx_max * 32;
        off_xds = o;
        o += nbx_max * 8;
        off_zq = o;
        o += z_nbx * 32;
        off_zds = o;
        o += z_nbx * 8;
        off_gamma = o = up(o, 16);
        o += 2 * vec * 4;
        const uint32_t kv = up(static_cast<uint32_t>(n_layers) * n_ctx * kLHD * 2, 16);
        off_kk = o;
        o += kv;
        off_kv = o;
        o += kv;
        off_q = o;
        o += kLHD * 4;
        off_vraw = o;
        o += kLHD * 4;
        off_ss = o;
        o += up(n_ctx, 32) * 4;
        off_red = o;
        o += 16 * 4;
        off_tpair = o;
        o += kLMaxLocalTiles * 8;
        off_pairs = o;  // the CTAs' published (max, argmax) pairs
        o += kLMaxGrid * 8;
        off_ops = o = up(o, 16);  // the op table
        o += kLMaxOps * static_cast<uint32_t>(sizeof(DepOp));
        off_rng = o;  // this CTA's first tile and tile count of every op
        o += kLMaxOps * 4;
        off_misc = o;  // tok_v[kLW], tok_i[kLW], err
        o += (2 * kLW + 4) * 4;
        bytes = o;
    }
};

struct LGeo {
    const uint8_t *tiles;
    KeyChains kc;
    int cpt, ng, n_loc, t0;
    __device__ int items() const { return n_loc * ng; }
};

// The CTA's share of op o, from the shared-memory tables filled at kernel
// start (rng[o] = first tile | tile count << 16).
__device__ __forceinline__ LGeo lgeo(const DepOp *ops, const int *rng, int o) {
    LGeo g;
    const DepOp &op = ops[o];
    g.tiles = op.W.tiles;
    g.cpt = op.W.cpt;
    g.kc = KeyChains::of(op.W.cols / 32, op.W.cpt);
    g.ng = g.kc.groups();
    g.t0 = rng[o] & 0xffff;
    g.n_loc = rng[o] >> 16;
    return g;
}

struct LCursor {
    int o, k, p, len;
    LGeo g;
};

__device__ __forceinline__ void lcur_seek(LCursor &u, const DepOp *ops, const int *rng, int n_ops, int w) {
    for (; u.o < n_ops; ++u.o) {
        u.g = lgeo(ops, rng, u.o);
        if (w < u.g.items()) {
            u.k = w;
            u.p = 0;
            u.len = u.g.kc.len(w % u.g.ng);
            return;
        }
    }
}

__device__ __forceinline__ void lcur_next(LCursor &u, const DepOp *ops, const int *rng, int n_ops, int w) {
    if (++u.p < u.len) return;
    u.p = 0;
    u.k += kLW;
    if (u.k < u.g.items()) {
        u.len = u.g.kc.len(u.k % u.g.ng);
        return;
    }
    ++u.o;
    lcur_seek(u, ops, rng, n_ops, w);
}

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long ll_load(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void ll_store(unsigned long long *p, float v, unsigned epoch) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// Entries [0, n) of src once they carry `epoch`, into dst (shared memory).
// All threads call it; it ends with __syncthreads.  On a timeout the CTA's
// error word gets bit 1, the missing values read as 0, and later calls of the
// CTA wait no more.
__device__ __noinline__ void ll_gather(const unsigned long long *src, int n, unsigned epoch, float *dst, int tid, int *err) {
    unsigned pending = 0;
#pragma unroll
    for (int k = 0; k < kLPer; ++k)
        if (tid + kLT * k < n) pending |= 1u << k;
    const unsigned long long t0 = gtime();
    while (pending) {
        unsigned long long w[kLPer];
#pragma unroll
        for (int k = 0; k < kLPer; ++k)
            if (pending & (1u << k)) w[k] = ll_load(src + tid + kLT * k);
#pragma unroll
        for (int k = 0; k < kLPer; ++k)
            if ((pending & (1u << k)) && static_cast<unsigned>(w[k] >> 32) == epoch) {
                dst[tid + kLT * k] = __uint_as_float(static_cast<unsigned>(w[k]));
                pending &= ~(1u << k);
            }
        if (pending && (*reinterpret_cast<volatile int *>(err) || gtime() - t0 > kLWaitNs)) {
            atomicOr(err, 1);
#pragma unroll
            for (int k = 0; k < kLPer; ++k)
                if (pending & (1u << k)) dst[tid + kLT * k] = 0.0f;
            pending = 0;
        }
        if (pending) __nanosleep(kLPollNs);  // keep the polled L2 lines free for the writers
    }
    __syncthreads();
}

// One exchange word once it carries `epoch` (bounded like ll_gather).
__device__ __forceinline__ float ll_fetch(const unsigned long long *src, unsigned epoch, int *err) {
    const unsigned long long t0 = gtime();
    for (;;) {
        const unsigned long long w = ll_load(src);
        if (static_cast<unsigned>(w >> 32) == epoch) return __uint_as_float(static_cast<unsigned>(w));
        if (*reinterpret_cast<volatile int *>(err) || gtime() - t0 > kLWaitNs) {
            atomicOr(err, 1);
            return 0.0f;
        }
        __nanosleep(kLPollNs);
    }
}

// x (n values in shared memory) -> Q8_1 blocks, optionally RMS-normalised
// first (the reference RMSNorm: thread t of 256 sums x[t + 256 k]^2 with fma,
// a shfl_down tree per warp, ((w0+w4)+(w2+w6))+((w1+w5)+(w3+w7)), scale =
// rsqrtf(total / n + eps), v = (x * scale) * gamma).  Warp w takes blocks w +
// 8 m into its padded scratch; lane m takes the amax, d, 1/d and in-order sum
// of block m (quant_block_q8_1's operations); every lane quantises its
// element of each block.  All threads call it; it ends with __syncthreads.
__device__ __noinline__ void ll_quantise(const float *x, bool x_global, int n, int nbx, const float *gamma, float eps, int8_t *xq,
                            float2 *xds, float *red, float *scratch, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    float scale = 1.0f;
    if (gamma) {
        float ss = 0.0f;
        for (int i = tid; i < n; i += kLT) ss = __fmaf_rn(x[i], x[i], ss);
        ss = shfl_down_tree(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        const float total = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[4]), __fadd_rn(red[2], red[6])),
                                      __fadd_rn(__fadd_rn(red[1], red[5]), __fadd_rn(red[3], red[7])));
        scale = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(n)), eps));
    }
    const int nb = n / 32;
    const int nbw = nb > warp ? (nb - warp + kLW - 1) / kLW : 0;
    const int rows = (nb + kLW - 1) / kLW < 32 ? (nb + kLW - 1) / kLW : 32;  // scratch blocks per warp
    float *scr = scratch + warp * (rows * 33 + 32);
    float *sid = scr + rows * 33;
    for (int m0 = 0; m0 < nbw; m0 += 32) {
        const int nr = nbw - m0 < 32 ? nbw - m0 : 32;
#pragma unroll 4
        for (int mm = 0; mm < nr; ++mm) {
            const int e = (warp + kLW * (m0 + mm)) * 32 + lane;
            const float xv = x_global ? __ldcg(x + e) : x[e];
            scr[mm * 33 + lane] = gamma ? __fmul_rn(__fmul_rn(xv, scale), gamma[e]) : xv;
        }
        __syncwarp();
        if (lane < nr) {
            const float *e = scr + lane * 33;
            float amax = 0.0f, sum = 0.0f;
#pragma unroll 8
            for (int k = 0; k < 32; ++k) {
                amax = fmaxf(amax, fabsf(e[k]));
                sum = __fadd_rn(sum, e[k]);
            }
            const float d = __fdiv_rn(amax, 127.0f);
            sid[lane] = (d != 0.0f) ? __frcp_rn(d) : 0.0f;
            const __half2 ds = __halves2half2(__float2half_rn(d), __float2half_rn(sum));
            xds[warp + kLW * (m0 + lane)] = make_float2(__low2float(ds), 4.0f * __high2float(ds));
        }
        __syncwarp();
#pragma unroll 4
        for (int mm = 0; mm < nr; ++mm) {
            int qi = __float2int_rz(roundf(__fmul_rn(scr[mm * 33 + lane], sid[mm])));
            qi = max(-128, min(127, qi));
            xq[(warp + kLW * (m0 + mm)) * 32 + lane] = static_cast<int8_t>(qi);
        }
        __syncwarp();
    }
    for (int b = nb + warp; b < nbx; b += kLW) {  // padding blocks
        xq[b * 32 + lane] = 0;
        if (lane == 0) xds[b] = make_float2(0.0f, 0.0f);
    }
    __syncthreads();
}

}  // namespace

__global__ void __launch_bounds__(kLT, 1) dep_cascade_ll_kernel(const __grid_constant__ DepCascadeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int c = blockIdx.x, G = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const LLLayout Ly(a.dim, a.ffn, a.n_embd, a.n_layers, a.n_ctx);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);  // [kLW][kLRing]
    uint64_t *gbars = bars + kLW * kLRing;                // [2]
    uint8_t *ring = smem + Ly.off_ring;
    float *part = reinterpret_cast<float *>(smem + Ly.off_part);
    float *xa = reinterpret_cast<float *>(smem + Ly.off_xa);
    float *xb = reinterpret_cast<float *>(smem + Ly.off_xb);
    float *attn = reinterpret_cast<float *>(smem + Ly.off_attn);
    float *act = reinterpret_cast<float *>(smem + Ly.off_act);
    int8_t *xq = reinterpret_cast<int8_t *>(smem + Ly.off_xq);
    float2 *xds = reinterpret_cast<float2 *>(smem + Ly.off_xds);
    int8_t *zq = reinterpret_cast<int8_t *>(smem + Ly.off_zq);
    float2 *zds = reinterpret_cast<float2 *>(smem + Ly.off_zds);
    float *gam = reinterpret_cast<float *>(smem + Ly.off_gamma);
    __half *kk = reinterpret_cast<__half *>(smem + Ly.off_kk);
    __half *kv = reinterpret_cast<__half *>(smem + Ly.off_kv);
    float *qv = reinterpret_cast<float *>(smem + Ly.off_q);
    float *vraw = reinterpret_cast<float *>(smem + Ly.off_vraw);
    float *ss = reinterpret_cast<float *>(smem + Ly.off_ss);
    float *red = reinterpret_cast<float *>(smem + Ly.off_red);
    float2 *tpair = reinterpret_cast<float2 *>(smem + Ly.off_tpair);
    float *pairs = reinterpret_cast<float *>(smem + Ly.off_pairs);
    DepOp *ops = reinterpret_cast<DepOp *>(smem + Ly.off_ops);
    int *rng = reinterpret_cast<int *>(smem + Ly.off_rng);
    float *tok_v = reinterpret_cast<float *>(smem + Ly.off_misc);
    int *tok_i = reinterpret_cast<int *>(tok_v + kLW);
    int *err = tok_i + kLW;
    const uint32_t gbytes = static_cast<uint32_t>(a.dim) * 4u;

    if (tid < kLW * kLRing + 2) mbar_init(bars + tid, 1);
    if (tid == 0) *err = 0;
    {  // the op table and this CTA's tile range of every op (no divisions later)
        const int words = a.n_ops * static_cast<int>(sizeof(DepOp) / 4);
        for (int i = tid; i < words; i += kLT) reinterpret_cast<int *>(ops)[i] = reinterpret_cast<const int *>(a.ops)[i];
        for (int o = tid; o < a.n_ops; o += kLT) {
            const int nt = a.ops[o].W.n_tiles;
            const int t0 = nt * c / G, t1 = nt * (c + 1) / G;
            rng[o] = t0 | ((t1 - t0) << 16);
        }
    }
    fence_barrier_init();
    __syncthreads();

    // Weights and RMSNorm weights never depend on earlier kernels: start now.
    const uint64_t pol = l2_evict_first_policy();
    LCursor pc;
    int issued = 0;
    auto issue = [&]() {
        const int slot = issued % kLRing;
        uint64_t *bar = bars + warp * kLRing + slot;
        const int j = pc.k / pc.g.ng, grp = pc.k % pc.g.ng;
        const long long ch = static_cast<long long>(pc.g.t0 + j) * pc.g.cpt + pc.g.kc.chunk(grp, pc.p);
        mbar_arrive_expect_tx(bar, kChunkBytes);
        bulk_load(ring + (warp * kLRing + slot) * kChunkBytes, pc.g.tiles + ch * kChunkBytes, kChunkBytes, bar, pol);
        ++issued;
        lcur_next(pc, ops, rng, a.n_ops, warp);
    };
    if (lane == 0) {
        pc.o = 0;
        lcur_seek(pc, ops, rng, a.n_ops, warp);
        while (issued < kLRing && pc.o < a.n_ops) issue();
    }
    if (tid == 0)
        for (int b = 0; b < 2; ++b)
            if (a.gamma0[b]) {
                mbar_arrive_expect_tx(gbars + b, gbytes);
                bulk_load(gam + b * Ly.vec, a.gamma0[b], gbytes, gbars + b, l2_evict_last_policy());
            }

    pdl_wait();
    const unsigned base = (*reinterpret_cast<volatile unsigned *>(a.seq)) * kPhasesPerLaunch;

    // z -> Q8_1 once: every step's input projection reads it
    ll_quantise(a.z, true, a.n_embd, lnbx(a.n_embd), nullptr, a.eps, zq, zds, red, part, tid);
    int tok = resolve_token<kLT>(a.first, tok_v, tok_i, [] { __syncthreads(); });
    if (c == 0 && tid == 0 && a.tok_out) a.tok_out[0] = tok;
    __syncthreads();

    int gi = 0, first_bad = 0, p = 0;
    int p_xa = -1, p_xb = -1;  // phases that produced the residual stream's current values
    bool bad = false;
    for (int o = 0; o < a.n_ops; ++o) {
        const DepOp &op = ops[o];
        const LGeo g = lgeo(ops, rng, o);
        const int kind = op.kind;
        const unsigned ep_in = base + p - 1, ep_out = base + p;
        const unsigned long long *lin = a.ll + static_cast<long long>(p - 1) * a.ll_stride;  // (p >= 1 when read)
        unsigned long long *lout = a.ll + static_cast<long long>(p) * a.ll_stride;

        // ---- input: the previous phase's output, then RMSNorm / Q8_1 ----
        const int8_t *xqo = xq;
        const float2 *xdso = xds;
        if (kind == kDepIn) {
            xqo = zq;
            xdso = zds;
        } else {
            float *dst = (kind == kDepQKV || kind == kDepHead) ? xa
                       : kind == kDepO                          ? attn
                       : kind == kDepFfnIn                      ? xb
                                                                : act;
            if (g.n_loc > 0) ll_gather(lin, op.W.cols, ep_in, dst, tid, err);  // only CTAs with rows need it
            const float *gm = nullptr;
            if (op.gamma) {
                const int bsel = op.norm_idx & 1;
                if (!mbar_wait(gbars + bsel, (op.norm_idx >> 1) & 1)) atomicOr(err, 2);
                gm = gam + bsel * Ly.vec;
            }
            if (g.n_loc > 0) ll_quantise(dst, false, op.W.cols, op.W.nbx, gm, a.eps, xq, xds, red, part, tid);
            else __syncthreads();  // (the RMSNorm weight buffer is released below all the same)
            if (op.gamma && op.gamma_ahead && tid == 0) {  // its buffer is free again: the weight two norms ahead
                const int bsel = op.norm_idx & 1;
                fence_proxy_async();
                mbar_arrive_expect_tx(gbars + bsel, gbytes);
                bulk_load(gam + bsel * Ly.vec, op.gamma_ahead, gbytes, gbars + bsel, l2_evict_last_policy());
            }
        }

        // ---- items: this warp's (tile, key group) chains ----
        const int n_items = g.items();
        for (int k = warp; k < n_items; k += kLW) {
            const int j = k / g.ng, grp = k % g.ng, len = g.kc.len(grp);
            float acc[kChunkBlocks][2];
#pragma unroll
            for (int b = 0; b < kChunkBlocks; ++b) acc[b][0] = acc[b][1] = 0.0f;
            for (int q = 0; q < len; ++q, ++gi) {
                const int slot = gi % kLRing;
                if (!bad && !mbar_wait(bars + warp * kLRing + slot, (gi / kLRing) & 1)) {
                    bad = true;
                    first_bad = gi;
                    if (lane == 0) atomicOr(err, 2);
                }
                if (!bad) {
                    const int ch = g.kc.chunk(grp, q);
                    chunk_acc_ref(ring + (warp * kLRing + slot) * kChunkBytes, xqo + ch * kChunkBlocks * 32,
                                  xdso + ch * kChunkBlocks, lane, acc);
                }
                __syncwarp();
                if (lane == 0 && !bad && pc.o < a.n_ops) {  // refill the slot just read
                    fence_proxy_async();
                    issue();
                }
            }
            float *pp = part + (j * g.ng + grp) * (2 * kChunkBlocks * 32);
#pragma unroll
            for (int b = 0; b < kChunkBlocks; ++b) {
                pp[(2 * b) * 32 + lane] = acc[b][0];
                pp[(2 * b + 1) * 32 + lane] = acc[b][1];
            }
        }
        if (kind == kDepIn && op.step > 0 && (g.n_loc > 0 || c == 0)) {  // the previous head's first maximum
            ll_gather(lin, 2 * G, ep_in, pairs, tid, err);  // (value, index bits) per CTA
            if (warp == 0) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int r = lane; r < G; r += 32) argmax_merge(bv, bi, pairs[2 * r], __float_as_int(pairs[2 * r + 1]));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    argmax_merge(bv, bi, ov, oi);
                }
                if (lane == 0) tok_i[0] = bi;
            }
            __syncthreads();
            tok = tok_i[0];
            if (c == 0 && tid == 0 && a.tok_out) a.tok_out[op.step] = tok;
        }
        __syncthreads();

        // ---- combine (one warp per tile) and epilogue ----
        for (int j = warp; j < g.n_loc; j += kLW) {
            const float *P = part + j * g.ng * (2 * kChunkBlocks * 32);
            auto pv = [&](int grp, int kk2) { return grp < g.ng ? P[(grp * 2 * kChunkBlocks + kk2) * 32 + lane] : 0.0f; };
            float L[32];
#pragma unroll
            for (int m = 0; m < 16; ++m) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int kk2 = 2 * (m & 7) + h, mh = m >> 3;
                    float s = __fadd_rn(pv(mh, kk2), pv(2 + mh, kk2));
                    s = __fadd_rn(s, pv(4 + mh, kk2));
                    L[2 * m + h] = __fadd_rn(s, pv(6 + mh, kk2));
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int q = 0; q < off; ++q) L[q] = __fadd_rn(L[q], L[q + off]);
            const float v = L[0];
            const int t = g.t0 + j;
            const int r = t * kTileRows + lane;
            const bool in = r < op.W.rows;
            switch (kind) {
            case kDepIn: {
                if (in) {
                    const EmbTable &e = a.emb[op.step];
                    const bool ok = tok >= 0 && tok < e.rows && e.dim == op.W.rows;
                    ll_store(lout + r, ok ? __fadd_rn(v, emb_elem(e, tok, r)) : __fadd_rn(v, 0.0f), ep_out);
                }
                break;
            }
            case kDepQKV: {  // raw q, k, v out; k and v also into the depformer ring (fp16)
                if (in) {
                    ll_store(lout + r, v, ep_out);
                    if (r >= a.dim) {
                        const int rr = r - a.dim, which = rr / a.dim, head = (rr % a.dim) / kLHD, d = rr % kLHD;
                        const long long ge =
                            ((static_cast<long long>(op.layer) * a.heads + head) * a.n_ctx + op.step % a.n_ctx) * kLHD + d;
                        (which == 0 ? a.k_cache : a.v_cache)[ge] = __float2half_rn(v);
                    }
                }
                break;
            }
            case kDepO:  // residual: the layer input, from the phase that produced it
                if (in) {
                    const float res = ll_fetch(a.ll + static_cast<long long>(p_xa) * a.ll_stride + r, base + p_xa, err);
                    ll_store(lout + r, __fadd_rn(res, v), ep_out);
                }
                break;
            case kDepFfnIn: {
                const float up = __shfl_down_sync(0xffffffffu, v, 16);
                const int hh = t * 16 + lane;
                if (lane < 16 && hh < a.ffn) {
                    const float silu = __fdiv_rn(v, __fadd_rn(1.0f, __expf(-v)));
                    ll_store(lout + hh, __fmul_rn(silu, up), ep_out);
                }
                break;
            }
            case kDepFfnOut:
                if (in) {
                    const float res = ll_fetch(a.ll + static_cast<long long>(p_xb) * a.ll_stride + r, base + p_xb, err);
                    ll_store(lout + r, __fadd_rn(res, v), ep_out);
                }
                break;
            default: {  // kDepHead: logits and the tile's first maximum
                float val = -INFINITY;
                if (in) {
                    val = v;
                    a.logits[static_cast<long long>(op.step) * a.logits_stride + r] = val;
                }
                float bv = (in && r < a.argmax_limit) ? val : -INFINITY;
                int bi = r;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    argmax_merge(bv, bi, ov, oi);
                }
                if (lane == 0) {
                    tpair[j] = make_float2(bv, __int_as_float(bi));
                    if (a.pairs) a.pairs[static_cast<long long>(op.step) * a.pairs_stride + t] = tpair[j];
                }
                break;
            }
            }
        }
        if (kind == kDepIn || kind == kDepFfnOut) p_xa = p;
        if (kind == kDepO) p_xb = p;
        ++p;

        if (kind == kDepHead) {  // the CTA's first maximum (every CTA publishes one, tiles or not)
            __syncthreads();
            if (warp == 0) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int j = lane; j < g.n_loc; j += 32) argmax_merge(bv, bi, tpair[j].x, __float_as_int(tpair[j].y));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    argmax_merge(bv, bi, ov, oi);
                }
                if (lane == 0) {
                    ll_store(lout + 2 * c, bv, ep_out);
                    ll_store(lout + 2 * c + 1, __int_as_float(bi), ep_out);
                }
            }
        }

        if (kind == kDepQKV) {  // attention phase: CTA h runs head h
            const unsigned ep_att = base + p;
            unsigned long long *latt = a.ll + static_cast<long long>(p) * a.ll_stride;
            if (c < a.heads) {
                // q, k, v of head c from the QKV phase's buffer (lout, epoch ep_out)
                float *qkv = part;  // staging: q[64], k[64], v[64]
                {
                    const int n3 = 3 * kLHD;
                    unsigned pending = tid < n3 ? 1u : 0u;
                    const int src = tid < n3 ? (tid / kLHD) * a.dim + c * kLHD + tid % kLHD : 0;
                    const unsigned long long t0 = gtime();
                    while (pending) {
                        const unsigned long long w = ll_load(lout + src);
                        if (static_cast<unsigned>(w >> 32) == ep_out) {
                            qkv[tid] = __uint_as_float(static_cast<unsigned>(w));
                            pending = 0;
                        } else if (*reinterpret_cast<volatile int *>(err) || gtime() - t0 > kLWaitNs) {
                            atomicOr(err, 1);
                            qkv[tid] = 0.0f;
                            pending = 0;
                        }
                    }
                    __syncthreads();
                }
                const int slot = op.step % a.n_ctx;
                if (tid < kLHD) {
                    qv[tid] = qkv[tid];
                    const int e = (op.layer * a.n_ctx + slot) * kLHD + tid;
                    kk[e] = __float2half_rn(qkv[kLHD + tid]);
                    kv[e] = __float2half_rn(qkv[2 * kLHD + tid]);
                    vraw[tid] = qkv[2 * kLHD + tid];
                }
                __syncthreads();
                if (warp < kLAttnThreads / 32) {
                    const int W = op.step + 1 < a.n_ctx ? op.step + 1 : a.n_ctx;
                    unsigned long long *dst = latt + c * kLHD;
                    if (W == 1) {  // the reference's window of one: the raw fp32 v
                        for (int d = tid; d < kLHD; d += kLAttnThreads) ll_store(dst + d, vraw[d], ep_att);
                    } else {  // positions 0..W-1 sit at slots 0..W-1 (the ring never wraps in a cascade)
                        const __half *kb = kk + op.layer * a.n_ctx * kLHD;
                        const __half *vb = kv + op.layer * a.n_ctx * kLHD;
                        attn_ref_scores<kLHD, kLAttnThreads, kLHD>(qv, kb, 0, W, a.scale, tid,
                                                             [&](int i, float s) { ss[i] = s; });
                        named_sync(kLBarAttn, kLAttnThreads);
                        attn_ref_softmax<kLHD, kLAttnThreads>(ss, W, red, tid,
                                                              [] { named_sync(kLBarAttn, kLAttnThreads); });
                        if (tid < kLHD) ll_store(dst + tid, attn_ref_vchain(ss, vb + tid, W, kLHD), ep_att);
                    }
                }
            }
            ++p;
            __syncthreads();
        }
    }

    // the last head's token
    if (c == 0) {
        const unsigned long long *lin = a.ll + static_cast<long long>(p - 1) * a.ll_stride;
        ll_gather(lin, 2 * G, base + p - 1, pairs, tid, err);
        if (warp == 0) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int r = lane; r < G; r += 32) argmax_merge(bv, bi, pairs[2 * r], __float_as_int(pairs[2 * r + 1]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                argmax_merge(bv, bi, ov, oi);
            }
            if (lane == 0 && a.tok_out) a.tok_out[a.dep_q] = bi;
            if (lane == 0) *reinterpret_cast<volatile unsigned *>(a.seq) = base / kPhasesPerLaunch + 1;
        }
    }
    pdl_launch_dependents();
    if (lane == 0 && bad)  // let this warp's copies in flight land before the CTA exits
        for (int j = first_bad; j < issued; ++j) mbar_wait(bars + warp * kLRing + j % kLRing, (j / kLRing) & 1);
    __syncthreads();
    if (*err && tid == 0) raise_error(a.status, (*err & 2) ? kErrTmaTimeout : kErrPeerTimeout);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t dep_cascade_ll_smem_bytes(int dim, int ffn, int n_embd, int n_layers, int n_ctx) {
    return LLLayout(dim, ffn, n_embd, n_layers, n_ctx).bytes;
}
int dep_cascade_ll_items() { return kLItems; }
int dep_cascade_ll_max_local_tiles() { return kLMaxLocalTiles; }
int dep_cascade_ll_max_in() { return kLMaxIn; }
int dep_cascade_ll_head_dim() { return kLHD; }
int dep_cascade_ll_phases() { return kPhasesPerLaunch; }
int dep_cascade_ll_max_grid() { return kLMaxGrid; }
int dep_cascade_ll_max_ops() { return kLMaxOps; }

// Opt-ins on the current device; returns how many CTAs can run co-resident
// (one per SM at most), 0 if the kernel cannot run here.
int dep_cascade_ll_configure(size_t smem_bytes, int sms) {
    if (cudaFuncSetAttribute(dep_cascade_ll_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem_bytes)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dep_cascade_ll_kernel, kLT, smem_bytes) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm >= 1 ? sms : 0;
}

cudaError_t launch_dep_cascade_ll(const DepCascadeArgs &a, int grid, size_t smem_bytes, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLT);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dep_cascade_ll_kernel, a);
}

}  // namespace bmo
