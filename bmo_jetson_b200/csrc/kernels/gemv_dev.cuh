// gemv_dev.cuh -- device pieces of the Q4_0 x Q8_1 GEMV shared by its two
// summation orders (gemv_q4.cu: exact double sums; gemv_ref.cu: the
// reference kernel's own fp32 order): the reference's per-half-block term,
// the 8-block chunk dot products, the activation quantiser and the fused tile
// epilogues.  Activations and residuals written earlier in the same launch by
// other CTAs are read with L2-only loads (ld.global.cg).
#pragma once

#include "common.cuh"

namespace bmo {

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

// The reference's accumulation of one 8-block chunk (32 rows, lane = row):
// for each block and half block h, with sumi the half block's integer dot
// product, acc[blk][h] = fma(d4, fma((float)sumi, d8, -4 s8), acc[blk][h]) --
// bmo_gemv_q4_0_q8_1_kernel's `acc += d4 * ((float) sumi * ds8.x - 4.0f *
// ds8.y)` (src/bmo_cuda_kernels.cu:648-651) as nvcc contracts it (measured
// bit-exact against the reference kernel on B200).  xds holds (d8, 4 s8).
__device__ __forceinline__ void chunk_acc_ref(const uint8_t *ch, const int8_t *xq, const float2 *xds, int lane,
                                              float (&acc)[kChunkBlocks][2]) {
#pragma unroll
    for (int blk = 0; blk < kChunkBlocks; ++blk) {
        const uint4 w = *reinterpret_cast<const uint4 *>(ch + blk * 512 + lane * 16);
        const float d4 = __half2float(*reinterpret_cast<const __half *>(ch + kChunkQsBytes + blk * 64 + lane * 2));
        const int4 xa = *reinterpret_cast<const int4 *>(xq + blk * 32);
        const int4 xb = *reinterpret_cast<const int4 *>(xq + blk * 32 + 16);
        const float2 ds = xds[blk];
        int lo = __dp4a(static_cast<int>(w.x & 0x0F0F0F0Fu), xa.x, 0);
        lo = __dp4a(static_cast<int>((w.x >> 4) & 0x0F0F0F0Fu), xb.x, lo);
        lo = __dp4a(static_cast<int>(w.y & 0x0F0F0F0Fu), xa.y, lo);
        lo = __dp4a(static_cast<int>((w.y >> 4) & 0x0F0F0F0Fu), xb.y, lo);
        int hi = __dp4a(static_cast<int>(w.z & 0x0F0F0F0Fu), xa.z, 0);
        hi = __dp4a(static_cast<int>((w.z >> 4) & 0x0F0F0F0Fu), xb.z, hi);
        hi = __dp4a(static_cast<int>(w.w & 0x0F0F0F0Fu), xa.w, hi);
        hi = __dp4a(static_cast<int>((w.w >> 4) & 0x0F0F0F0Fu), xb.w, hi);
        acc[blk][0] = __fmaf_rn(d4, __fmaf_rn(static_cast<float>(lo), ds.x, -ds.y), acc[blk][0]);
        acc[blk][1] = __fmaf_rn(d4, __fmaf_rn(static_cast<float>(hi), ds.x, -ds.y), acc[blk][1]);
    }
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

// Resolves the token of an embedding lookup: the device int, or the first
// maximum over per-tile (max, argmax) pairs.  Threads [0, NT) take part and
// `sync` is their barrier.
template <int NT, typename Sync>
__device__ int resolve_token(const TokenSrc &src, float *red_v, int *red_i, Sync sync) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (!src.pairs) return src.tok ? __ldcg(src.tok) : -1;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = tid; p < src.n_pairs; p += NT) {
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
    sync();
    float fv = red_v[0];
    int fi = red_i[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) argmax_merge(fv, fi, red_v[w], red_i[w]);
    sync();
    return fi;
}

// 32 consecutive fp32 activations (16-byte aligned) into registers.
__device__ __forceinline__ void load_block32(const float *p, float (&v)[32]) {
    const float4 *xp = reinterpret_cast<const float4 *>(p);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 t4 = __ldcg(xp + j);
        v[4 * j] = t4.x; v[4 * j + 1] = t4.y; v[4 * j + 2] = t4.z; v[4 * j + 3] = t4.w;
    }
}

__device__ __forceinline__ double sum_sq_double(const float (&v)[32]) {
    double s[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const double d = static_cast<double>(v[j]);
        s[j & 3] = fma(d, d, s[j & 3]);
    }
    return (s[0] + s[1]) + (s[2] + s[3]);
}

// Block b of the activation -> Q8_1 in shared memory (zeros for padding
// blocks).  NORM: v = (x * scale) * gamma, rounded per product as rmsnorm_kernel.
template <int PRO>
__device__ __forceinline__ void quantize_x_block(const GemvArgs &a, int8_t *xq, float2 *xds, int b, bool has,
                                                 float (&v)[32], float scale, const float *gam, bool cta0) {
    int4 *qd = reinterpret_cast<int4 *>(xq + b * 32);
    if (!has) {
        qd[0] = make_int4(0, 0, 0, 0);
        qd[1] = make_int4(0, 0, 0, 0);
        xds[b] = make_float2(0.0f, 0.0f);
        return;
    }
    if constexpr (PRO == kProNorm) {
        const float *gp = gam + b * 32;
        if ((reinterpret_cast<uintptr_t>(gp) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 g4 = reinterpret_cast<const float4 *>(gp)[j];
                v[4 * j] = __fmul_rn(__fmul_rn(v[4 * j], scale), g4.x);
                v[4 * j + 1] = __fmul_rn(__fmul_rn(v[4 * j + 1], scale), g4.y);
                v[4 * j + 2] = __fmul_rn(__fmul_rn(v[4 * j + 2], scale), g4.z);
                v[4 * j + 3] = __fmul_rn(__fmul_rn(v[4 * j + 3], scale), g4.w);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), gp[j]);
        }
    }
    int8_t q[32];
    const __half2 ds = quant_block_q8_1(v, q);
    const int *qi = reinterpret_cast<const int *>(q);
    qd[0] = make_int4(qi[0], qi[1], qi[2], qi[3]);
    qd[1] = make_int4(qi[4], qi[5], qi[6], qi[7]);
    xds[b] = make_float2(__low2float(ds), 4.0f * __high2float(ds));
    if (cta0 && a.q8_out) {
        int *o = reinterpret_cast<int *>(a.q8_out + static_cast<size_t>(b) * 36);
        o[0] = *reinterpret_cast<const int *>(&ds);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[1 + j] = qi[j];
    }
    if (cta0 && a.xn_out) {
        float4 *xo = reinterpret_cast<float4 *>(a.xn_out + b * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) xo[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
}

// REF: the reference's own fp32 forms (SwiGLU with __expf, RoPE with the
// products fused as nvcc fuses rope_interleaved_kernel's); otherwise the
// exact-reduction forms (transcendentals in double, every product rounded).
template <int EPI, bool REF = false>
__device__ __forceinline__ void tile_epilogue(const GemvArgs &a, int t, int lane, float v, int tok,
                                              const float2 *rope_cs) {
    const int r = t * kTileRows + lane;
    if constexpr (EPI == kEpiStore) {
        if (r < a.W.rows) a.y[r] = a.bias ? __fadd_rn(v, a.bias[r]) : v;
    } else if constexpr (EPI == kEpiResid) {
        if (r < a.W.rows) a.y[r] = __fadd_rn(__ldcg(a.resid + r), v);
    } else if constexpr (EPI == kEpiSwiGLU) {
        // silu(gate) * up (swiglu_split_kernel, bmo_cuda_kernels.cu:370-387);
        // exact form: exp evaluated in double and rounded once
        const float up = __shfl_down_sync(0xffffffffu, v, 16);
        const int h = t * 16 + lane;
        if (lane < 16 && h < a.W.swiglu_f) {
            const float e = REF ? __expf(-v) : __double2float_rn(exp(-static_cast<double>(v)));
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
        if ((is_q || is_k) && rope_cs) {
            // interleaved RoPE (rope_interleaved_kernel, :317-368): even lane
            // real part xr, odd lane imaginary part xi.  REF: y_r = fma(xr, c,
            // -(xi s)), y_i = fma(xr, s, xi c) (the reference's contraction);
            // exact form: every product rounded
            const int d = (is_q ? r : r - a.q_dim) % hd;
            const float2 cs = rope_cs[d >> 1];
            const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
            if constexpr (REF)
                out = (lane & 1) ? __fmaf_rn(partner, cs.y, __fmul_rn(v, cs.x))
                                 : __fmaf_rn(v, cs.x, -__fmul_rn(partner, cs.y));
            else
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

}  // namespace bmo
