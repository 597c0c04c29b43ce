// attention_ref_dev.cuh -- the three phases of the reference decode
// attention (bmo_decode_attention_kernel, src/bmo_cuda_kernels.cu:713-848) in
// the reference's own fp32 order, over K/V rows already in shared memory:
// the scores, the softmax in place, and the weighted sum of V.  Used by the
// per-op attention kernel (attention_ref.cu) and by the depformer cascade
// (dep_cascade.cu), so both compute the same bits.
//
//   s_i  = fl(T_i * scale), T_i = ((0 + G_0) + G_1) + ... over the head's
//          32-dimension groups, G_g the __shfl_down_sync tree of fl(q_d k_d)
//   M    = max(-1e20, max_i s_i)
//   e_i  = expf(s_i - M); thread t < head_dim sums e_{t + head_dim k} in
//          order, each warp reduces by a shfl_down tree, the warp sums are
//          added in order starting from 0; inv = 1 / sum; p_i = fl(e_i inv)
//   out_d = fma chain over i of p_i v_{i,d}
#pragma once

#include "common.cuh"

namespace bmo {

// Scores of positions [i0, i1): kb holds their K rows (row i - i0 at kb +
// (i - i0) * KS, HD fp16 values each; KS * 2 a multiple of 16 bytes), sq the
// query (16-byte aligned).  Each of the NT threads takes (position,
// 32-dimension group) tasks; all NT threads (whole warps) must call it.
// emit(i, s) receives each score once.  With KS = HD + 8 the rows a warp
// reads at once fall on distinct shared-memory banks (KS = HD puts every
// row of a warp on the same banks).
template <int HD, int NT, int KS, typename Emit>
__device__ __forceinline__ void attn_ref_scores(const float *sq, const __half *kb, int i0, int i1, float scale,
                                                int tid, Emit emit) {
    static_assert(KS >= HD && KS % 8 == 0, "K rows: whole 16-byte pieces");
    constexpr int kGroups = HD / 32;
    const int lane = tid & 31;
    const int g = tid % kGroups;  // kGroups divides 32: a position's groups are adjacent lanes
    float qg[32];
    const float4 *q4 = reinterpret_cast<const float4 *>(sq + 32 * g);
#pragma unroll
    for (int d = 0; d < 8; ++d) {
        const float4 t = q4[d];
        qg[4 * d] = t.x;
        qg[4 * d + 1] = t.y;
        qg[4 * d + 2] = t.z;
        qg[4 * d + 3] = t.w;
    }
    const int tasks = (i1 - i0) * kGroups;
    for (int u0 = 0; u0 < tasks; u0 += NT) {
        const int u = u0 + tid;
        const int i = i0 + u / kGroups;
        const bool on = u < tasks;
        float p[32];
        const uint4 *kr = reinterpret_cast<const uint4 *>(kb + (on ? (i - i0) : 0) * KS + 32 * g);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 w = kr[j];
            const __half2 *hp = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(hp[e]);
                p[8 * j + 2 * e] = __fmul_rn(qg[8 * j + 2 * e], kf.x);
                p[8 * j + 2 * e + 1] = __fmul_rn(qg[8 * j + 2 * e + 1], kf.y);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int d = 0; d < o; ++d) p[d] = __fadd_rn(p[d], p[d + o]);
        // ((0 + G0) + G1) + ... over the groups, in group order
        const int base = lane & ~(kGroups - 1);
        float tot = 0.0f;
#pragma unroll
        for (int k = 0; k < kGroups; ++k) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, p[0], base + k));
        if (on && g == 0) emit(i, __fmul_rn(tot, scale));
    }
}

// Softmax of ss[0, W) in place (ss ends as p_i), the reference's thread
// pattern.  NT threads (whole warps, NT >= HD) call it; red holds at least 16
// floats; sync() is their barrier.  Returns after a final sync().
template <int HD, int NT, typename Sync>
__device__ __forceinline__ void attn_ref_softmax(float *ss, int W, float *red, int tid, Sync sync) {
    static_assert(NT / 32 <= 8 && HD / 32 <= 8, "reduction slots");
    const int lane = tid & 31, warp = tid >> 5;
    float m = -1e20f;
    for (int i = tid; i < W; i += NT) m = ss[i] > m ? ss[i] : m;
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    sync();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) M = red[w] > M ? red[w] : M;
    sync();
    if (tid < HD) {  // the reference runs head_dim threads
        float ls = 0.0f;
        for (int i = tid; i < W; i += HD) {
            const float e = expf(__fsub_rn(ss[i], M));
            ss[i] = e;
            ls = __fadd_rn(ls, e);
        }
        ls = shfl_down_tree(ls);
        if (lane == 0) red[8 + warp] = ls;
    }
    sync();
    float se = 0.0f;
#pragma unroll
    for (int w = 0; w < HD / 32; ++w) se = __fadd_rn(se, red[8 + w]);
    const float inv = se > 0.0f ? __fdiv_rn(1.0f, se) : 0.0f;
    for (int i = tid; i < W; i += NT) ss[i] = __fmul_rn(ss[i], inv);
    sync();
}

// out_d for one dimension: the sequential fma chain over positions 0..W-1 of
// p_i * v_{i,d}; vcol points at v_{0,d} and consecutive positions are `stride`
// halves apart.
__device__ __forceinline__ float attn_ref_vchain(const float *ss, const __half *vcol, int W, int stride) {
    float acc = 0.0f;
    int i = 0;
    for (; i + 8 <= W; i += 8) {
        float pv[8], vv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            pv[j] = ss[i + j];
            vv[j] = __half2float(vcol[(i + j) * stride]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = __fmaf_rn(pv[j], vv[j], acc);
    }
    for (; i < W; ++i) acc = __fmaf_rn(ss[i], __half2float(vcol[i * stride]), acc);
    return acc;
}

}  // namespace bmo
