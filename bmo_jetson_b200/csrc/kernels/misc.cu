// misc.cu -- frame-start embedding gather, RoPE table, Q4_0 repack and the
// standalone Q8_1 quantiser.
#include "common.cuh"
#include "../launch.h"

namespace bmo {

// Input embedding of one decode step (bmo_embed_input_tokens_into,
// src/bmo_compute.cpp:1867-1912): acc = text_emb[t0] + sum_k emb[k-1][t_k],
// channels added in order, a channel skipped when its token is negative or
// out of range or its table has the wrong width.  Block 0 also builds the
// RoPE (cos, sin) table of this position, inv_freq = theta^(-2i/hd) and
// angle = pos * inv_freq in fp32 as in rope_interleaved_kernel (:317-368);
// ref: the power and the trigonometry by the reference's own intrinsics
// (__powf, __sincosf), else evaluated in double and rounded once.
__global__ void embed_kernel(const EmbTable *tables, int n_tables, const int *tokens, const int *n_tok_dev,
                             int n_embd, float *out, const int *pos, float theta, int head_dim, float2 *rope_cs,
                             int ref) {
    pdl_launch_dependents();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int n_tok = n_tok_dev ? *n_tok_dev : 0;
    if (out && i < n_embd) {
        float acc = 0.0f;
        for (int ch = 0; ch < n_tok && ch < n_tables; ++ch) {
            const EmbTable t = tables[ch];
            const int tok = tokens[ch];
            if (!t.data || tok < 0 || tok >= t.rows || t.dim != n_embd) continue;
            const uint8_t *row = static_cast<const uint8_t *>(t.data) + static_cast<size_t>(tok) * t.row_bytes;
            float v = 0.0f;
            switch (t.type) {
            case kTF32: v = reinterpret_cast<const float *>(row)[i]; break;
            case kTF16: v = __half2float(reinterpret_cast<const __half *>(row)[i]); break;
            case kTBF16: v = __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t *>(row)[i]) << 16); break;
            case kTQ4_0: {
                const uint8_t *b = row + (i >> 5) * 18;
                const float d = __half2float(*reinterpret_cast<const __half *>(b));
                const int j = i & 31;
                const int nib = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
                v = static_cast<float>(nib - 8) * d;
                break;
            }
            case kTQ8_0: {
                const uint8_t *b = row + (i >> 5) * 34;
                v = static_cast<float>(static_cast<int8_t>(b[2 + (i & 31)])) * __half2float(*reinterpret_cast<const __half *>(b));
                break;
            }
            default: continue;
            }
            acc = __fadd_rn(acc, v);
        }
        out[i] = acc;
    }
    if (blockIdx.x == 0 && rope_cs && threadIdx.x < head_dim / 2) {
        const int k = threadIdx.x;
        const float exponent = __fdiv_rn(static_cast<float>(2 * k), static_cast<float>(head_dim));
        if (ref) {
            const float inv_freq = __powf(theta, -exponent);
            const float angle = __fmul_rn(static_cast<float>(*pos), inv_freq);
            float sn, cs;
            __sincosf(angle, &sn, &cs);
            rope_cs[k] = make_float2(cs, sn);
        } else {
            const float inv_freq = __double2float_rn(pow(static_cast<double>(theta), -static_cast<double>(exponent)));
            const float angle = __fmul_rn(static_cast<float>(*pos), inv_freq);
            double sn, cs;
            sincos(static_cast<double>(angle), &sn, &cs);
            rope_cs[k] = make_float2(__double2float_rn(cs), __double2float_rn(sn));
        }
    }
}

cudaError_t launch_embed(const EmbTable *tables, int n_tables, const int *tokens, const int *n_tok_dev, int n_embd,
                         float *out, const int *pos, float theta, int head_dim, float2 *rope_cs, bool ref,
                         cudaStream_t s) {
    const int threads = 256;
    const int blocks = (n_embd + threads - 1) / threads;
    embed_kernel<<<blocks, threads, 0, s>>>(tables, n_tables, tokens, n_tok_dev, n_embd, out, pos, theta, head_dim,
                                            rope_cs, ref ? 1 : 0);
    return cudaGetLastError();
}

// Device-resident frame inputs: copies K token ids and sets the position.
__global__ void set_frame_kernel(int *fin_tokens, int *fin_n_tok, int *fin_pos, const int *tokens, int K, int pos) {
    const int i = threadIdx.x;
    if (i < K) fin_tokens[i] = tokens[i];
    if (i == 0) {
        *fin_n_tok = K;
        *fin_pos = pos;
    }
}

cudaError_t launch_set_frame(int *fin_tokens, int *fin_n_tok, int *fin_pos, const int *tokens, int K, int pos,
                             cudaStream_t s) {
    set_frame_kernel<<<1, 64, 0, s>>>(fin_tokens, fin_n_tok, fin_pos, tokens, K, pos);
    return cudaGetLastError();
}

__global__ void set_int_kernel(int *dst, int v) { *dst = v; }

cudaError_t launch_set_int(int *dst, int v, cudaStream_t s) {
    set_int_kernel<<<1, 1, 0, s>>>(dst, v);
    return cudaGetLastError();
}

// Greedy token from per-tile (max, argmax) pairs: highest value, lowest
// index among equals (std::max_element's first maximum).
__global__ void finalize_token_kernel(const float2 *pairs, int n, int *out) {
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        const float2 pr = pairs[p];
        const int pi = __float_as_int(pr.y);
        if (pr.x > bv || (pr.x == bv && pi < bi)) { bv = pr.x; bi = pi; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        *out = bi;
    }
}

// Tensor-parallel residual add: y = resid + fl(sum of the ranks' double
// partials), the single rounding of the batch-1 GEMV's residual epilogue.
__global__ void tp_resid_kernel(const double *part, const float *resid, float *y, int n) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(resid[i], __double2float_rn(part[i]));
}

cudaError_t launch_tp_resid(const double *part, const float *resid, float *y, int n, cudaStream_t s) {
    tp_resid_kernel<<<(n + 255) / 256, 256, 0, s>>>(part, resid, y, n);
    return cudaGetLastError();
}

cudaError_t configure_gemv();
cudaError_t configure_gemv_ref();
cudaError_t configure_attention();
cudaError_t configure_attention_ref();
cudaError_t configure_batch();
cudaError_t configure_batch_mma();

cudaError_t configure_kernels() {
    cudaError_t e = configure_gemv();
    if (e == cudaSuccess) e = configure_gemv_ref();
    if (e == cudaSuccess) e = configure_attention();
    if (e == cudaSuccess) e = configure_attention_ref();
    if (e == cudaSuccess) e = configure_batch();
    return e != cudaSuccess ? e : configure_batch_mma();
}

cudaError_t launch_finalize_token(const float2 *pairs, int n, int *out, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, finalize_token_kernel, pairs, n, out);
}

// ggml Q4_0 row-major blocks -> row tiles (see layout.h).  One thread copies
// one (row, block): 16 nibble bytes and the fp16 scale.
__global__ void repack_q4_0_kernel(const uint8_t *src, uint8_t *dst, int rows, int nb, int nbx, int n_tiles, int perm,
                                   int swiglu_f) {
    const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long total = static_cast<long long>(n_tiles) * kTileRows * nbx;
    if (gid >= total) return;
    const int lane = static_cast<int>(gid % kTileRows);
    const long long rest = gid / kTileRows;
    const int b = static_cast<int>(rest % nbx);
    const int t = static_cast<int>(rest / nbx);
    int r;
    if (perm == kPermSwiGLU) r = lane < 16 ? t * 16 + lane : swiglu_f + t * 16 + (lane - 16);
    else r = t * kTileRows + lane;
    const bool live = r < rows && b < nb && (perm != kPermSwiGLU || t * 16 + (lane & 15) < swiglu_f);
    const int cpt = nbx / kChunkBlocks;
    uint8_t *chunk = dst + (static_cast<long long>(t) * cpt + b / kChunkBlocks) * kChunkBytes;
    const int blk = b % kChunkBlocks;
    uint8_t *qs = chunk + blk * 512 + lane * 16;
    uint16_t *dd = reinterpret_cast<uint16_t *>(chunk + kChunkQsBytes + blk * 64 + lane * 2);
    if (live) {
        const uint8_t *blkp = src + (static_cast<long long>(r) * nb + b) * 18;
        uint16_t d;
        memcpy(&d, blkp, 2);
        *dd = d;
        for (int j = 0; j < 16; ++j) qs[j] = blkp[2 + j];
    } else {
        *dd = 0;
        for (int j = 0; j < 16; ++j) qs[j] = 0x88;  // nibble 8 = weight 0 (scale 0 anyway)
    }
}

cudaError_t launch_repack_q4_0(const void *src, void *dst, int rows, int cols, const QMatDesc &m, cudaStream_t s) {
    const long long total = static_cast<long long>(m.n_tiles) * kTileRows * m.nbx;
    const int threads = 256;
    const long long blocks = (total + threads - 1) / threads;
    repack_q4_0_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), rows, cols / 32, m.nbx, m.n_tiles, m.perm,
        m.swiglu_f);
    return cudaGetLastError();
}

// Standalone Q8_1 quantiser (one thread per block), the same device routine
// the GEMV prologue runs; output in the reference's 36-byte block format.
__global__ void quantize_q8_1_kernel(const float *x, uint8_t *out, int nb) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    float v[32];
    int8_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = x[b * 32 + j];
    const __half2 ds = quant_block_q8_1(v, q);
    int *o = reinterpret_cast<int *>(out + static_cast<size_t>(b) * 36);
    o[0] = *reinterpret_cast<const int *>(&ds);
    const int *qi = reinterpret_cast<const int *>(q);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[1 + j] = qi[j];
}

cudaError_t launch_quantize_q8_1(const float *x, void *out, int n, cudaStream_t s) {
    const int nb = n / 32;
    if (nb <= 0) return cudaSuccess;
    quantize_q8_1_kernel<<<(nb + 127) / 128, 128, 0, s>>>(x, static_cast<uint8_t *>(out), nb);
    return cudaGetLastError();
}

}  // namespace bmo
