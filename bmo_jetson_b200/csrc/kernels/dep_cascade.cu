// dep_cascade.cu -- the depformer's greedy cascade (dep_q codebook steps,
// each the input projection + embedding of the previous token, the 6 layers
// and the audio head of bmo_build_depth_graph, src/bmo_compute.cpp:2741-3340,
// with the greedy token of each head feeding the next step) as ONE launch on
// one thread-block cluster, every value in the reference kernels' fp32 order:
// the same bits as the per-op chain of gemv_ref_kernel / attn_ref_kernel.
//
// Why one launch.  The per-op chain runs 256 small kernels per cascade at
// ~4.5 us each -- launch, the activation's round trip, the norm and the
// quantiser, the tail -- for 375 MB of weights that take 57 us at the copy
// peak.  Here the cascade runs on a cluster of `heads` CTAs (16 for the 7B
// depformer, one per SM):
//  * weights never depend on activations, so each warp streams its share of
//    every matrix of the cascade, op after op, through a private two-chunk TMA
//    ring: the next op's first chunks are in flight while the cluster waits
//    for the current op's output;
//  * every activation vector (the residual stream, the attention output, the
//    SwiGLU output) is replicated in every CTA's shared memory: a CTA stores
//    each row it computes into every CTA's copy (distributed shared memory)
//    and one hardware cluster barrier separates an op from the next -- no
//    global-memory round trip, no grid-wide barrier;
//  * CTA c owns head c: its QKV rows are that head's q, k and v, so the
//    attention (the head's K/V ring kept in shared memory) is local.
//
// Measured on B200 (7B depformer, 16 CTAs): 1.59-1.67 ms per cascade against
// 1.19 ms for the per-op chain, so the engine runs it only on request.  A
// per-op timeline of this kernel: the dot products of the 16 SMs take ~700
// us (~1.2 us per 4.6 KB chunk per warp: instruction issue, shared-memory
// wavefronts and too few bytes in flight per SM), the in-order Q8_1 sums of
// the prologues ~400 us, the combines ~180 us, the cluster barriers and the
// attention ~270 us.
//
// Per-row arithmetic is gemv_ref_kernel's: 32-row tiles, one chain per key
// group (KeyChains) accumulated by chunk_acc_ref, the groups combined in the
// reference's lane order and the 32-leaf shfl_down tree; the RMSNorm, the
// Q8_1 quantiser (one warp per block, the same operations) and the
// epilogues use the same fp32 operations, the attention the shared phases of
// attention_ref_dev.cuh.  Work split: the CTA's tiles of an op x the key
// groups that hold chunks are "items", dealt round-robin to the warps; a
// warp's items, op after op, are the chunk sequence its ring streams.  After
// an op's items, one warp per tile combines the groups and runs the epilogue.
//
// Waits: every ring and RMSNorm-weight wait is bounded (kWaitPolls); a copy
// that does not land sets the status bit, the warp stops reading weights but
// passes every barrier, so all CTAs finish.  Cluster barriers cannot time
// out; every thread of every CTA passes the same sequence of them.
#include <cooperative_groups.h>

#include "attention_ref_dev.cuh"
#include "gemv_dev.cuh"
#include "../launch.h"

namespace cg = cooperative_groups;

namespace bmo {

namespace {

constexpr int kCW = 12;                  // warps per CTA
constexpr int kCT = kCW * 32;
constexpr int kCRing = 2;                // chunks in flight per warp
constexpr int kPartSlots = 24;           // (tile, key group) chain buffers of one op
constexpr int kMaxCluster = 16;
constexpr int kMaxLocalTiles = 64;       // tiles of one op per CTA
constexpr int kHD = 64;                  // depformer head size
constexpr int kAttnThreads = 128;        // warps 0-3 run the head's attention
constexpr int kBarAttn = 1;              // their named barrier
constexpr int kNormThreads = 256;        // the reference RMSNorm's thread count

__host__ __device__ inline int nbx_of(int cols) { return ((cols / 32) + 7) & ~7; }

struct DepLayout {
    uint32_t vec, off_ring, off_part, off_xa, off_xb, off_attn, off_act, off_xq, off_xds, off_zq, off_zds, off_gamma,
        off_kk, off_kv, off_q, off_vraw, off_ss, off_red, off_tpair, off_cpair, off_misc, bytes;
    __host__ __device__ static uint32_t up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
    __host__ __device__ DepLayout(int dim, int ffn, int n_embd, int n_layers, int n_ctx) {
        const uint32_t nbx_max = nbx_of(dim) > nbx_of(ffn) ? nbx_of(dim) : nbx_of(ffn);
        const uint32_t z_nbx = nbx_of(n_embd);
        vec = up(dim, 32);
        uint32_t o = (kCW * kCRing + 2) * 8;  // mbarriers: rings, then the two RMSNorm-weight buffers
        off_ring = o = up(o, 128);
        o += kCW * kCRing * kChunkBytes;
        off_part = o;
        o += kPartSlots * 2 * kChunkBlocks * 32 * 4;
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
        const uint32_t kv = up(static_cast<uint32_t>(n_layers) * n_ctx * kHD * 2, 16);
        off_kk = o;
        o += kv;
        off_kv = o;
        o += kv;
        off_q = o;
        o += kHD * 4;
        off_vraw = o;
        o += kHD * 4;
        off_ss = o;
        o += up(n_ctx, 32) * 4;
        off_red = o;
        o += 16 * 4;
        off_tpair = o;
        o += kMaxLocalTiles * 8;
        off_cpair = o;
        o += kMaxCluster * 8;
        off_misc = o;  // tok_v[kCW], tok_i[kCW], err
        o += (2 * kCW + 4) * 4;
        bytes = o;
    }
};

// The CTA's share of one op: its row tiles and the key groups that hold chunks.
struct OpGeo {
    const uint8_t *tiles;
    KeyChains kc;
    int cpt, ng, n_loc, t0, tph;  // tph > 0: QKV, the head-aligned tiles of CTA c
    __device__ int items() const { return n_loc * ng; }
    __device__ int tile(int j, int c, int heads) const {
        return tph ? (j / tph) * heads * tph + c * tph + j % tph : t0 + j;
    }
};

__device__ __forceinline__ OpGeo op_geo(const DepOp &op, int c, int cs) {
    OpGeo g;
    g.tiles = op.W.tiles;
    g.cpt = op.W.cpt;
    g.kc = KeyChains::of(op.W.cols / 32, op.W.cpt);
    g.ng = g.kc.groups();
    if (op.kind == kDepQKV) {  // q, k and v rows of head c
        g.tph = kHD / kTileRows;
        g.t0 = 0;
        g.n_loc = 3 * g.tph;
    } else {
        g.tph = 0;
        g.t0 = static_cast<int>(static_cast<long long>(op.W.n_tiles) * c / cs);
        g.n_loc = static_cast<int>(static_cast<long long>(op.W.n_tiles) * (c + 1) / cs) - g.t0;
    }
    return g;
}

// A warp's position in its chunk sequence (op, item, chain position); the
// producer lane walks it ahead of the consumer by the ring depth.
struct Cursor {
    int o, k, p, len;
    OpGeo g;
};

__device__ __forceinline__ void cur_seek(Cursor &u, const DepCascadeArgs &a, int c, int cs, int w) {
    for (; u.o < a.n_ops; ++u.o) {
        u.g = op_geo(a.ops[u.o], c, cs);
        if (w < u.g.items()) {
            u.k = w;
            u.p = 0;
            u.len = u.g.kc.len(w % u.g.ng);
            return;
        }
    }
}

__device__ __forceinline__ void cur_next(Cursor &u, const DepCascadeArgs &a, int c, int cs, int w) {
    if (++u.p < u.len) return;
    u.p = 0;
    u.k += kCW;
    if (u.k < u.g.items()) {
        u.len = u.g.kc.len(u.k % u.g.ng);
        return;
    }
    ++u.o;
    cur_seek(u, a, c, cs, w);
}

__device__ __forceinline__ const uint8_t *cur_src(const Cursor &u, int c, int heads) {
    const int j = u.k / u.g.ng, grp = u.k % u.g.ng;
    const long long ch = static_cast<long long>(u.g.tile(j, c, heads)) * u.g.cpt + u.g.kc.chunk(grp, u.p);
    return u.g.tiles + ch * kChunkBytes;
}

// One Q8_1 block, lane j holding element j: quant_block_q8_1's operations
// (amax; d = amax / 127; id = 1 / d; q = round(v id) clamped; s = v0 + v1 +
// ... + v31 in order) spread over the warp.
__device__ __forceinline__ void quant_block_q8_1_warp(float v, int lane, int8_t *q_dst, float2 *ds_dst) {
    const float amax = warp_max(fabsf(v));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;
    int qi = __float2int_rz(roundf(__fmul_rn(v, id)));
    qi = max(-128, min(127, qi));
    q_dst[lane] = static_cast<int8_t>(qi);
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, v, j));
    if (lane == 0) *ds_dst = make_float2(__half2float(__float2half_rn(d)), 4.0f * __half2float(__float2half_rn(s)));
}

// The op's input (n values in shared memory) -> Q8_1 blocks; with gamma the
// reference RMSNorm first: thread t of 256 sums x[t + 256 k]^2 with fma, a
// shfl_down tree per warp, ((w0+w4)+(w2+w6))+((w1+w5)+(w3+w7)), scale =
// rsqrtf(total / n + eps), v = (x * scale) * gamma.  All threads call it.
__device__ __forceinline__ void dep_prologue(const float *x, int n, int nbx, const float *gamma, float eps,
                                             int8_t *xq, float2 *xds, float *red, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    float scale = 1.0f;
    if (gamma) {
        if (tid < kNormThreads) {
            float ss = 0.0f;
            for (int i = tid; i < n; i += kNormThreads) ss = __fmaf_rn(x[i], x[i], ss);
            ss = shfl_down_tree(ss);
            if (lane == 0) red[warp] = ss;
        }
        __syncthreads();
        const float total = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[4]), __fadd_rn(red[2], red[6])),
                                      __fadd_rn(__fadd_rn(red[1], red[5]), __fadd_rn(red[3], red[7])));
        scale = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(n)), eps));
    }
    const int nb = n / 32;
    for (int b = warp; b < nbx; b += kCW) {
        if (b < nb) {
            float v = x[32 * b + lane];
            if (gamma) v = __fmul_rn(__fmul_rn(v, scale), gamma[32 * b + lane]);
            quant_block_q8_1_warp(v, lane, xq + 32 * b, xds + b);
        } else {  // padding block
            xq[32 * b + lane] = 0;
            if (lane == 0) xds[b] = make_float2(0.0f, 0.0f);
        }
    }
}

__device__ __forceinline__ void bcast(const cg::cluster_group &cl, float *p, float v, int cs) {
    for (int rk = 0; rk < cs; ++rk) *cl.map_shared_rank(p, rk) = v;
}

}  // namespace

__global__ void __launch_bounds__(kCT, 1) dep_cascade_kernel(const __grid_constant__ DepCascadeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const cg::cluster_group cl = cg::this_cluster();
    const int c = static_cast<int>(cl.block_rank()), cs = static_cast<int>(cl.num_blocks());
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const DepLayout Ly(a.dim, a.ffn, a.n_embd, a.n_layers, a.n_ctx);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);  // [kCW][kCRing]
    uint64_t *gbars = bars + kCW * kCRing;                // [2]
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
    float2 *cpair = reinterpret_cast<float2 *>(smem + Ly.off_cpair);
    float *tok_v = reinterpret_cast<float *>(smem + Ly.off_misc);
    int *tok_i = reinterpret_cast<int *>(tok_v + kCW);
    int *err = tok_i + kCW;
    const uint32_t gbytes = static_cast<uint32_t>(a.dim) * 4u;

    if (tid < kCW * kCRing + 2) mbar_init(bars + tid, 1);
    if (tid == 0) *err = 0;
    fence_barrier_init();
    // every CTA of the cluster has started before any distributed-shared-memory store
    cl.sync();

    // Weights and RMSNorm weights never depend on earlier kernels: start now.
    const uint64_t pol = l2_evict_first_policy();
    Cursor pc;
    int issued = 0;
    auto issue = [&]() {
        const int slot = issued % kCRing;
        uint64_t *bar = bars + warp * kCRing + slot;
        mbar_arrive_expect_tx(bar, kChunkBytes);
        bulk_load(ring + (warp * kCRing + slot) * kChunkBytes, cur_src(pc, c, a.heads), kChunkBytes, bar, pol);
        ++issued;
        cur_next(pc, a, c, cs, warp);
    };
    if (lane == 0) {
        pc.o = 0;
        cur_seek(pc, a, c, cs, warp);
        while (issued < kCRing && pc.o < a.n_ops) issue();
    }
    if (tid == 0)
        for (int b = 0; b < 2; ++b)
            if (a.gamma0[b]) {
                mbar_arrive_expect_tx(gbars + b, gbytes);
                bulk_load(gam + b * Ly.vec, a.gamma0[b], gbytes, gbars + b, l2_evict_last_policy());
            }

    pdl_wait();

    // z -> Q8_1 once: every step's input projection reads it (plain prologue)
    const int z_nb = a.n_embd / 32, z_nbx = nbx_of(a.n_embd);
    for (int b = warp; b < z_nbx; b += kCW) {
        if (b < z_nb) {
            quant_block_q8_1_warp(__ldcg(a.z + 32 * b + lane), lane, zq + 32 * b, zds + b);
        } else {
            zq[32 * b + lane] = 0;
            if (lane == 0) zds[b] = make_float2(0.0f, 0.0f);
        }
    }
    int tok = resolve_token<kCT>(a.first, tok_v, tok_i, [] { __syncthreads(); });
    if (c == 0 && tid == 0 && a.tok_out) a.tok_out[0] = tok;
    __syncthreads();

    int gi = 0;  // chunks this warp has consumed
    int first_bad = 0;
    bool bad = false;
    for (int o = 0; o < a.n_ops; ++o) {
        const DepOp op = a.ops[o];
        const OpGeo g = op_geo(op, c, cs);
        const int kind = op.kind;

        // ---- prologue: the op's input as Q8_1 blocks ----
        const int8_t *xqo = xq;
        const float2 *xdso = xds;
        if (kind == kDepIn) {
            xqo = zq;
            xdso = zds;
        } else {
            const float *src = (kind == kDepQKV || kind == kDepHead) ? xa
                             : kind == kDepO                          ? attn
                             : kind == kDepFfnIn                      ? xb
                                                                      : act;
            const float *gm = nullptr;
            if (op.gamma) {
                const int bsel = op.norm_idx & 1;
                if (!mbar_wait(gbars + bsel, (op.norm_idx >> 1) & 1)) atomicOr(err, 1);
                gm = gam + bsel * Ly.vec;
            }
            dep_prologue(src, op.W.cols, op.W.nbx, gm, a.eps, xq, xds, red, tid);
            __syncthreads();
            if (op.gamma && op.gamma_ahead && tid == 0) {  // its buffer is free again: the weight two norms ahead
                const int bsel = op.norm_idx & 1;
                fence_proxy_async();
                mbar_arrive_expect_tx(gbars + bsel, gbytes);
                bulk_load(gam + bsel * Ly.vec, op.gamma_ahead, gbytes, gbars + bsel, l2_evict_last_policy());
            }
        }

        // ---- items: this warp's (tile, key group) chains ----
        const int n_items = g.items();
        for (int k = warp; k < n_items; k += kCW) {
            const int j = k / g.ng, grp = k % g.ng, len = g.kc.len(grp);
            float acc[kChunkBlocks][2];
#pragma unroll
            for (int b = 0; b < kChunkBlocks; ++b) acc[b][0] = acc[b][1] = 0.0f;
            for (int p = 0; p < len; ++p, ++gi) {
                const int slot = gi % kCRing;
                if (!bad && !mbar_wait(bars + warp * kCRing + slot, (gi / kCRing) & 1)) {
                    bad = true;
                    first_bad = gi;
                    if (lane == 0) atomicOr(err, 1);
                }
                if (!bad) {
                    const int ch = g.kc.chunk(grp, p);
                    chunk_acc_ref(ring + (warp * kCRing + slot) * kChunkBytes, xqo + ch * kChunkBlocks * 32,
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
        __syncthreads();

        // ---- combine (one warp per tile) and epilogue ----
        for (int j = warp; j < g.n_loc; j += kCW) {
            const float *P = part + j * g.ng * (2 * kChunkBlocks * 32);
            auto pv = [&](int grp, int kk2) { return grp < g.ng ? P[(grp * 2 * kChunkBlocks + kk2) * 32 + lane] : 0.0f; };
            // lane value L[2m + h] = ((A0 + A1) + A2) + A3, A_j from key group 2j + m/8
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
            const int t = g.tile(j, c, a.heads);
            const int r = t * kTileRows + lane;
            const bool in = r < op.W.rows;
            switch (kind) {
            case kDepIn: {  // y = W z + embedding row of the step's input token
                if (in) {
                    const EmbTable &e = a.emb[op.step];
                    const bool ok = tok >= 0 && tok < e.rows && e.dim == op.W.rows;
                    bcast(cl, xa + r, ok ? __fadd_rn(v, emb_elem(e, tok, r)) : __fadd_rn(v, 0.0f), cs);
                }
                break;
            }
            case kDepQKV: {  // head c's q, and its k, v appended at slot `step` (no RoPE in the depformer)
                const int which = j / g.tph, d = (j % g.tph) * kTileRows + lane;
                const int slot = op.step % a.n_ctx;
                if (which == 0) {
                    qv[d] = v;
                } else {
                    const __half hv = __float2half_rn(v);
                    const int e = (op.layer * a.n_ctx + slot) * kHD + d;
                    const long long ge = ((static_cast<long long>(op.layer) * a.heads + c) * a.n_ctx + slot) * kHD + d;
                    if (which == 1) {
                        kk[e] = hv;
                        a.k_cache[ge] = hv;
                    } else {
                        kv[e] = hv;
                        a.v_cache[ge] = hv;
                        vraw[d] = v;
                    }
                }
                break;
            }
            case kDepO:
                if (in) bcast(cl, xb + r, __fadd_rn(xa[r], v), cs);
                break;
            case kDepFfnIn: {  // silu(gate) * up; lanes 0-15 gate rows, 16-31 up rows
                const float up = __shfl_down_sync(0xffffffffu, v, 16);
                const int hh = t * 16 + lane;
                if (lane < 16 && hh < a.ffn) {
                    const float silu = __fdiv_rn(v, __fadd_rn(1.0f, __expf(-v)));
                    bcast(cl, act + hh, __fmul_rn(silu, up), cs);
                }
                break;
            }
            case kDepFfnOut:
                if (in) bcast(cl, xa + r, __fadd_rn(xb[r], v), cs);
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

        // ---- hand-off to the next op ----
        if (kind == kDepQKV) {
            __syncthreads();  // head c's q, k, v are in shared memory
            if (warp < kAttnThreads / 32) {
                const int W = op.step + 1 < a.n_ctx ? op.step + 1 : a.n_ctx;
                float *dst = attn + c * kHD;
                if (W == 1) {  // the reference's window of one: the raw fp32 v
                    for (int d = tid; d < kHD; d += kAttnThreads) bcast(cl, dst + d, vraw[d], cs);
                } else {
                    // positions 0..W-1 sit at slots 0..W-1 (the ring never wraps in a cascade)
                    const __half *kb = kk + op.layer * a.n_ctx * kHD;
                    const __half *vb = kv + op.layer * a.n_ctx * kHD;
                    attn_ref_scores<kHD, kAttnThreads, kHD>(qv, kb, 0, W, a.scale, tid, [&](int i, float s) { ss[i] = s; });
                    named_sync(kBarAttn, kAttnThreads);
                    attn_ref_softmax<kHD, kAttnThreads>(ss, W, red, tid, [] { named_sync(kBarAttn, kAttnThreads); });
                    if (tid < kHD) bcast(cl, dst + tid, attn_ref_vchain(ss, vb + tid, W, kHD), cs);
                }
            }
            cl.sync();
        } else if (kind == kDepHead) {
            __syncthreads();
            if (warp == 0) {  // the CTA's first maximum, into every CTA's slot c
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int j = lane; j < g.n_loc; j += 32) argmax_merge(bv, bi, tpair[j].x, __float_as_int(tpair[j].y));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    argmax_merge(bv, bi, ov, oi);
                }
                if (lane < cs) *cl.map_shared_rank(cpair + c, lane) = make_float2(bv, __int_as_float(bi));
            }
            cl.sync();
            float bv = cpair[0].x;
            int bi = __float_as_int(cpair[0].y);
            for (int rk = 1; rk < cs; ++rk) argmax_merge(bv, bi, cpair[rk].x, __float_as_int(cpair[rk].y));
            tok = bi;
            if (c == 0 && tid == 0 && a.tok_out) a.tok_out[op.step + 1] = tok;
        } else {
            cl.sync();  // the op's rows are in every CTA's copy
        }
    }

    pdl_launch_dependents();
    if (lane == 0 && bad)  // let this warp's copies in flight land before the CTA exits
        for (int j = first_bad; j < issued; ++j) mbar_wait(bars + warp * kCRing + j % kCRing, (j / kCRing) & 1);
    __syncthreads();
    if (*err && tid == 0) raise_error(a.status, kErrTmaTimeout);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t dep_cascade_smem_bytes(int dim, int ffn, int n_embd, int n_layers, int n_ctx) {
    return DepLayout(dim, ffn, n_embd, n_layers, n_ctx).bytes;
}

int dep_cascade_part_slots() { return kPartSlots; }
int dep_cascade_max_cluster() { return kMaxCluster; }
int dep_cascade_max_local_tiles() { return kMaxLocalTiles; }
int dep_cascade_head_dim() { return kHD; }

// Sets the kernel's shared-memory and cluster-size opt-ins on the current
// device and returns how many clusters of `heads` CTAs can be resident (0:
// the cascade kernel cannot run here).
int dep_cascade_configure(int heads, size_t smem_bytes) {
    if (heads < 1 || heads > kMaxCluster) return 0;
    if (cudaFuncSetAttribute(dep_cascade_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem_bytes)) != cudaSuccess ||
        cudaFuncSetAttribute(dep_cascade_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(heads);
    cfg.blockDim = dim3(kCT);
    cfg.dynamicSmemBytes = smem_bytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = heads;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, dep_cascade_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

cudaError_t launch_dep_cascade(const DepCascadeArgs &a, size_t smem_bytes, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.heads);
    cfg.blockDim = dim3(kCT);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.heads;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, dep_cascade_kernel, a);
}

}  // namespace bmo
