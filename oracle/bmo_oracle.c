/*
 * bmo_oracle.c -- CPU oracle for the Moshi decode step. TEST INFRASTRUCTURE:
 * the checker for the CUDA path and the timed CPU baseline, never the product.
 *
 * Restates the reference (utkarshyadav009/bmo_jetson) GPU arithmetic:
 *   Q8_1 quantisation      src/bmo_cuda_kernels.cu:529-558
 *   Q4_0 x Q8_1 GEMV       src/bmo_cuda_kernels.cu:560-683
 *   RMSNorm                src/bmo_cuda_kernels.cu:244-295
 *   interleaved RoPE       src/bmo_cuda_kernels.cu:317-368
 *   SwiGLU split           src/bmo_cuda_kernels.cu:370-387
 *   ring decode attention  src/bmo_cuda_kernels.cu:713-848
 *   embedding sum          src/bmo_compute.cpp:1867-1912
 *   temporal graph order   src/bmo_compute.cpp:2124-2739
 *   depformer graph order  src/bmo_compute.cpp:2741-3340
 *   greedy sampling        src/bmo_api.cpp:638-666 (+ cascade :668-743)
 *   tensor-name contract   src/bmo.cpp:285-568
 * and ggml's published Q4_0 reference quantiser (quantize_row_q4_0_ref, as
 * restated by gguf-py's quants.Q4_0) for weights and the Q4_0 KV mode.
 *
 * Build with -ffp-contract=off: the quantisers depend on separately rounded
 * multiplies and adds.
 *
 * Exact-reduction semantics.  Where the reference leaves a result to its
 * thread layout (the order of fp32 reductions) or to a fast approximation
 * (__expf, __powf, __sincosf, rsqrtf), this restatement fixes one value:
 * reductions are carried in double and rounded once, transcendentals are
 * evaluated in double and rounded once to fp32.  Every other operation is
 * the reference's fp32 operation in the reference's order.  The CUDA kernels
 * implement the same semantics, so the two agree bit for bit (up to rare
 * double-rounding ties) instead of drifting apart through the Q8_1
 * requantisation of every activation, which turns last-bit differences into
 * whole-code flips.
 */
#include "bmo_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* IEEE binary16 conversions (round to nearest even), written from the       */
/* format definition.                                                        */
/* ------------------------------------------------------------------------ */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    float f;
    if (e == 0) {
        f = (float)m * 5.9604644775390625e-08f; /* m * 2^-24, exact */
        memcpy(&x, &f, 4);
        x |= sign;
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    memcpy(&f, &x, 4);
    return f;
}

uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? (0x200u | ((a >> 13) & 0x3ffu)) : 0u));
    if (a >= 0x477ff000u) /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) { /* below 2^-14: subnormal or zero */
        if (a < 0x33000000u) return (uint16_t)sign; /* <= 2^-25 -> 0 */
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        uint32_t sh = 126u - e; /* 14..24 */
        uint32_t r = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t v = a - (112u << 23);
    uint32_t r = v >> 13, rem = v & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------------ */
/* Kernel-level restatements                                                 */
/* ------------------------------------------------------------------------ */

/* bmo_quantize_row_q8_1_kernel, bmo_cuda_kernels.cu:529-558: amax, d=amax/127,
 * id = d ? 1/d : 0, q = clamp(roundf(v*id)), ds = (half(d), half(sequential sum)). */
void orc_quantize_row_q8_1(const float *x, orc_block_q8_1 *y, int n) {
    const int nb = n / 32;
    for (int i = 0; i < nb; ++i) {
        const float *src = x + (size_t)i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = fabsf(src[j]);
            if (v > amax) amax = v;
        }
        const float d = amax / 127.0f;
        const float id = (d != 0.0f) ? (1.0f / d) : 0.0f;
        float sum = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = src[j];
            int q0 = (int)roundf(v * id);
            if (q0 < -128) q0 = -128;
            if (q0 > 127) q0 = 127;
            y[i].qs[j] = (int8_t)q0;
            sum += v;
        }
        y[i].d = orc_fp32_to_fp16(d);
        y[i].s = orc_fp32_to_fp16(sum);
    }
}

/* ggml quantize_row_q4_0_ref (as in gguf-py quants.Q4_0.quantize_blocks):
 * signed max-by-magnitude (first occurrence), d = max/-8, id = d ? 1/d : 0,
 * q = min(15, trunc(x*id + 8.5)); byte j = q[j] | q[j+16] << 4. */
void orc_quantize_row_q4_0(const float *x, orc_block_q4_0 *y, int n) {
    const int nb = n / 32;
    for (int i = 0; i < nb; ++i) {
        const float *src = x + (size_t)i * 32;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = src[j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8.0f;
        const float id = (d != 0.0f) ? (1.0f / d) : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < 16; ++j) {
            const float x0 = src[j] * id;
            const float x1 = src[16 + j] * id;
            int q0 = (int)(int8_t)(x0 + 8.5f);
            int q1 = (int)(int8_t)(x1 + 8.5f);
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            y[i].qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void orc_dequantize_row_q4_0(const orc_block_q4_0 *x, float *y, int n) {
    const int nb = n / 32;
    for (int i = 0; i < nb; ++i) {
        const float d = orc_fp16_to_fp32(x[i].d);
        for (int j = 0; j < 16; ++j) {
            y[(size_t)i * 32 + j] = (float)((int)(x[i].qs[j] & 0x0f) - 8) * d;
            y[(size_t)i * 32 + j + 16] = (float)((int)(x[i].qs[j] >> 4) - 8) * d;
        }
    }
}

static void dequantize_row_q8_0(const uint8_t *row, float *y, int n) {
    /* ggml block_q8_0: fp16 d + 32 int8 (34 bytes). */
    for (int i = 0; i < n / 32; ++i) {
        const uint8_t *b = row + (size_t)i * 34;
        uint16_t dh;
        memcpy(&dh, b, 2);
        const float d = orc_fp16_to_fp32(dh);
        for (int j = 0; j < 32; ++j) y[i * 32 + j] = (float)(int8_t)b[2 + j] * d;
    }
}

/* bmo_gemv_q4_0_q8_1_kernel, bmo_cuda_kernels.cu:560-683: each half block
 * (elements {0..7,16..23} and {8..15,24..31}) contributes
 * d4 * ((float)sumi * d8 - 4 * s8).  Terms are fp32 as in the kernel; the
 * cross-term sum is taken in double (the kernel's order is a thread-layout
 * detail). */
static float gemv_row(const orc_block_q4_0 *row, const orc_block_q8_1 *x, int nb) {
    double acc = 0.0;
    for (int b = 0; b < nb; ++b) {
        const float d4 = orc_fp16_to_fp32(row[b].d);
        const float d8 = orc_fp16_to_fp32(x[b].d);
        const float s8 = orc_fp16_to_fp32(x[b].s);
        for (int half = 0; half < 2; ++half) {
            int sumi = 0;
            for (int j = 8 * half; j < 8 * half + 8; ++j) {
                sumi += (int)(row[b].qs[j] & 0x0f) * (int)x[b].qs[j];
                sumi += (int)(row[b].qs[j] >> 4) * (int)x[b].qs[j + 16];
            }
            const float t = d4 * ((float)sumi * d8 - 4.0f * s8);
            acc += (double)t;
        }
    }
    return (float)acc;
}

void orc_gemv_q4_0_q8_1(const orc_block_q4_0 *W, const orc_block_q8_1 *x,
                        float *y, int rows, int cols) {
    const int nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) y[r] = gemv_row(W + (size_t)r * nb, x, nb);
}

/* ---- the reference kernels' own fp32 order ------------------------------
 * bmo_gemv_q4_0_q8_1_kernel (bmo_cuda_kernels.cu:560-683) exactly: a warp per
 * row, lane l takes half block l % 2 of blocks m = l / 2 (mod 16); its
 * accumulator j chains blocks 64 i + 16 j + m in order, the tail (blocks past
 * the last whole 64) continues accumulator 0 in steps of 16; each block adds
 * acc = fmaf(d4, fmaf((float)sumi, d8, -4 s8), acc) (the kernel's
 * `acc += d4 * ((float) sumi * ds8.x - 4.0f * ds8.y)` as nvcc contracts it);
 * lane value ((acc0 + acc1) + acc2) + acc3; row = the __shfl_down_sync tree
 * (offsets 16, 8, 4, 2, 1) of the 32 lane values.  Pure fp32 arithmetic, so
 * this restatement is bit-exact against the kernel (pinned to its outputs on
 * B200 in tests/golden/ref_kernels.npz). */
static float ref_half_term(const orc_block_q4_0 *b4, const orc_block_q8_1 *b8, int half, float acc) {
    const float d4 = orc_fp16_to_fp32(b4->d);
    const float d8 = orc_fp16_to_fp32(b8->d);
    const float s8 = orc_fp16_to_fp32(b8->s);
    int sumi = 0;
    for (int j = 8 * half; j < 8 * half + 8; ++j) {
        sumi += (int)(b4->qs[j] & 0x0f) * (int)b8->qs[j];
        sumi += (int)(b4->qs[j] >> 4) * (int)b8->qs[j + 16];
    }
    return fmaf(d4, fmaf((float)sumi, d8, -4.0f * s8), acc);
}

static float gemv_row_reforder(const orc_block_q4_0 *row, const orc_block_q8_1 *x, int nb) {
    float lane_val[32];
    for (int l = 0; l < 32; ++l) {
        const int m = l / 2, half = l % 2;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int base = 0;
        for (; base + 64 <= nb; base += 64)
            for (int j = 0; j < 4; ++j) acc[j] = ref_half_term(row + base + 16 * j + m, x + base + 16 * j + m, half, acc[j]);
        for (; base < nb; base += 16)
            if (base + m < nb) acc[0] = ref_half_term(row + base + m, x + base + m, half, acc[0]);
        lane_val[l] = ((acc[0] + acc[1]) + acc[2]) + acc[3];
    }
    for (int o = 16; o > 0; o >>= 1)
        for (int i = 0; i < o; ++i) lane_val[i] = lane_val[i] + lane_val[i + o];
    return lane_val[0];
}

void orc_gemv_q4_0_q8_1_reforder(const orc_block_q4_0 *W, const orc_block_q8_1 *x, float *y, int rows, int cols) {
    const int nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) y[r] = gemv_row_reforder(W + (size_t)r * nb, x, nb);
}

/* rmsnorm_kernel (bmo_cuda_kernels.cu:244-295) in its own order: thread t of
 * 256 sums x[t + 256 k]^2 with fmaf; each warp's shfl_down tree; the 8 warp
 * sums as ((w0+w4)+(w2+w6))+((w1+w5)+(w3+w7)); y = (x * scale) * w.  The
 * kernel's scale is rsqrtf (an approximate instruction); here it is the
 * correctly rounded 1/sqrt, so results agree to about an ulp of the scale. */
void orc_rmsnorm_reforder(const float *x, const float *w, float eps, int n, float *y) {
    float t[256], ws[8];
    for (int i = 0; i < 256; ++i) {
        t[i] = 0.0f;
        for (int k = i; k < n; k += 256) t[i] = fmaf(x[k], x[k], t[i]);
    }
    for (int wp = 0; wp < 8; ++wp) {
        float *v = t + 32 * wp;
        for (int o = 16; o > 0; o >>= 1)
            for (int i = 0; i < o; ++i) v[i] = v[i] + v[i + o];
        ws[wp] = v[0];
    }
    const float total = ((ws[0] + ws[4]) + (ws[2] + ws[6])) + ((ws[1] + ws[5]) + (ws[3] + ws[7]));
    const float scale = (float)(1.0 / sqrt((double)(total / (float)n + eps)));
    for (int i = 0; i < n; ++i) y[i] = (x[i] * scale) * w[i];
}

/* bmo_decode_attention_kernel (bmo_cuda_kernels.cu:713-848) in its own order
 * over an fp16 ring [layer][head][slot][hd] (head_dim threads, thread = dim):
 * s_i = fl(T_i * scale), T_i = in warp order from 0, the shfl_down tree of
 * each 32-dim group's products fl(q_d k_d); M = max(-1e20, s_i);
 * e_i = expf(s_i - M); thread t sums e_{t + hd k} in order, warp trees, warp
 * sums in order; inv = 1 / sum; p_i = fl(e_i inv); out_d = fmaf chain over i
 * of p_i v_{i,d}.  expf here is libm's, the kernel's is CUDA's (both within a
 * couple of ulp of exp), so results agree to a few ulp. */
void orc_decode_attention_f16_reforder(const float *q, const float *k, const float *v, uint16_t *k_cache,
                                       uint16_t *v_cache, float *out, int head_dim, int n_heads, int n_kv_heads,
                                       int n_ctx, int pos, int layer) {
    const int total = pos + 1, W = total > n_ctx ? n_ctx : total, start = total - W, cur = pos % n_ctx;
    const size_t per_layer = (size_t)head_dim * n_ctx * n_heads, per_head = (size_t)head_dim * n_ctx;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *s = (float *)malloc(sizeof(float) * (size_t)(W > 0 ? W : 1));
    float p[1024], tsum[1024], red[32];
    for (int h = 0; h < n_kv_heads; ++h)
        for (int d = 0; d < head_dim; ++d) {
            const size_t off = (size_t)layer * per_layer + (size_t)h * per_head + (size_t)cur * head_dim + d;
            k_cache[off] = orc_fp32_to_fp16(k[h * head_dim + d]);
            v_cache[off] = orc_fp32_to_fp16(v[h * head_dim + d]);
        }
    const int q_per_kv = n_heads / n_kv_heads, nw = (head_dim + 31) / 32;
    for (int h = 0; h < n_heads; ++h) {
        const int kh = (n_kv_heads == n_heads) ? h : h / q_per_kv;
        const size_t base = (size_t)layer * per_layer + (size_t)kh * per_head;
        if (W == 1) {
            for (int d = 0; d < head_dim; ++d) out[h * head_dim + d] = v[kh * head_dim + d];
            continue;
        }
        for (int i = 0; i < W; ++i) {
            const uint16_t *kr = k_cache + base + (size_t)((start + i) % n_ctx) * head_dim;
            float tot = 0.0f;
            for (int w = 0; w < nw; ++w) {
                for (int d = 0; d < 32; ++d) p[d] = q[h * head_dim + 32 * w + d] * orc_fp16_to_fp32(kr[32 * w + d]);
                for (int o = 16; o > 0; o >>= 1)
                    for (int d = 0; d < o; ++d) p[d] = p[d] + p[d + o];
                tot = tot + p[0];
            }
            s[i] = tot * scale;
        }
        float M = -1e20f;
        for (int i = 0; i < W; ++i) M = s[i] > M ? s[i] : M;
        for (int t = 0; t < head_dim; ++t) {
            tsum[t] = 0.0f;
            for (int i = t; i < W; i += head_dim) {
                s[i] = expf(s[i] - M);
                tsum[t] = tsum[t] + s[i];
            }
        }
        for (int w = 0; w < nw; ++w) {
            float *tv = tsum + 32 * w;
            for (int o = 16; o > 0; o >>= 1)
                for (int d = 0; d < o; ++d) tv[d] = tv[d] + tv[d + o];
            red[w] = tv[0];
        }
        float se = 0.0f;
        for (int w = 0; w < nw; ++w) se = se + red[w];
        const float inv = se > 0.0f ? 1.0f / se : 0.0f;
        for (int i = 0; i < W; ++i) s[i] = s[i] * inv;
        for (int d = 0; d < head_dim; ++d) {
            float acc = 0.0f;
            for (int i = 0; i < W; ++i)
                acc = fmaf(s[i], orc_fp16_to_fp32(v_cache[base + (size_t)((start + i) % n_ctx) * head_dim + d]), acc);
            out[h * head_dim + d] = acc;
        }
    }
    free(s);
}

/* apply_dense_q4_0_linear_gpu (bmo_compute.cpp:674-755) = launch_gemv_q4_0_q8_1:
 * quantise the activation to Q8_1, then the integer GEMV. */
static void linear_q4_0(const orc_block_q4_0 *W, const float *x, float *y,
                        int rows, int cols) {
    orc_block_q8_1 *xq = (orc_block_q8_1 *)malloc(sizeof(orc_block_q8_1) * (size_t)(cols / 32));
    orc_quantize_row_q8_1(x, xq, cols);
    orc_gemv_q4_0_q8_1(W, xq, y, rows, cols);
    free(xq);
}

/* rmsnorm_kernel, bmo_cuda_kernels.cu:244-295: y = x * rsqrt(mean(x^2) + eps) * w. */
void orc_rmsnorm(const float *x, const float *w, float eps, int n, float *y) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    const float total = (float)ss;
    const float scale = (float)(1.0 / sqrt((double)(total / (float)n + eps)));
    for (int i = 0; i < n; ++i) y[i] = x[i] * scale * w[i];
}

/* rope_interleaved_kernel, bmo_cuda_kernels.cu:317-368: pair (2i, 2i+1),
 * exponent 2i/hd and angle = pos*inv_freq in fp32 as in the kernel; the
 * power and the trig are evaluated in double and rounded once to fp32
 * (the kernel's __powf/__sincosf are approximations of the same values). */
void orc_rope_interleaved(const float *x, int n_heads, int head_dim, int pos,
                          float theta, float *y) {
    const int half = head_dim / 2;
    for (int h = 0; h < n_heads; ++h) {
        for (int i = 0; i < half; ++i) {
            const float exponent = (float)(2 * i) / (float)head_dim;
            const float inv_freq = (float)pow((double)theta, -(double)exponent);
            const float angle = (float)pos * inv_freq;
            const float cs = (float)cos((double)angle), sn = (float)sin((double)angle);
            const float xr = x[h * head_dim + 2 * i], xi = x[h * head_dim + 2 * i + 1];
            y[h * head_dim + 2 * i] = xr * cs - xi * sn;
            y[h * head_dim + 2 * i + 1] = xr * sn + xi * cs;
        }
    }
}

/* swiglu_split_kernel, bmo_cuda_kernels.cu:370-387: silu(gate) * up with
 * exp(-gate) evaluated in double and rounded once (the kernel's __expf is an
 * approximation of it); the divide and multiply are fp32. */
void orc_swiglu(const float *h, int d_ff, float *y) {
    for (int i = 0; i < d_ff; ++i) {
        const float gate = h[i], up = h[i + d_ff];
        const float e = (float)exp(-(double)gate);
        const float silu = gate / (1.0f + e);
        y[i] = silu * up;
    }
}

int orc_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i; /* first maximum wins, as std::max_element */
    return best;
}

/* bmo_decode_attention_kernel, bmo_cuda_kernels.cu:713-848.  Ring geometry:
 * total = pos+1, window = min(total, n_ctx), oldest-first logical positions
 * [total-window, pos] at slots t % n_ctx; the current K/V are appended at
 * slot pos % n_ctx first, so they are read back through the cache format.
 * A window of one returns v itself. */
typedef struct {
    int kind; /* ORC_KV_F16 or ORC_KV_Q4_0 */
    uint16_t *k16, *v16;
    orc_block_q4_0 *k4, *v4;
} kv_view;

static void kv_store(const kv_view *kv, int which, size_t row_elem_off, const float *src, int hd) {
    if (kv->kind == ORC_KV_F16) {
        uint16_t *dst = (which ? kv->v16 : kv->k16) + row_elem_off;
        for (int d = 0; d < hd; ++d) dst[d] = orc_fp32_to_fp16(src[d]);
    } else {
        orc_block_q4_0 *dst = (which ? kv->v4 : kv->k4) + row_elem_off / 32;
        orc_quantize_row_q4_0(src, dst, hd);
    }
}

static void kv_load(const kv_view *kv, int which, size_t row_elem_off, float *dst, int hd) {
    if (kv->kind == ORC_KV_F16) {
        const uint16_t *src = (which ? kv->v16 : kv->k16) + row_elem_off;
        for (int d = 0; d < hd; ++d) dst[d] = orc_fp16_to_fp32(src[d]);
    } else {
        const orc_block_q4_0 *src = (which ? kv->v4 : kv->k4) + row_elem_off / 32;
        orc_dequantize_row_q4_0(src, dst, hd);
    }
}

static void decode_attention(const float *q, const float *k, const float *v,
                             const kv_view *kv, float *out, int hd, int n_heads,
                             int n_kv_heads, int n_ctx, int pos, int layer) {
    const int total = pos + 1;
    const int window = total > n_ctx ? n_ctx : total;
    const int start = total - window;
    const int cur = pos % n_ctx;
    const size_t per_head = (size_t)hd * (size_t)n_ctx;
    const size_t per_layer = per_head * (size_t)n_kv_heads;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int h = 0; h < n_kv_heads; ++h) {
        const size_t off = (size_t)layer * per_layer + (size_t)h * per_head + (size_t)cur * hd;
        kv_store(kv, 0, off, k + (size_t)h * hd, hd);
        kv_store(kv, 1, off, v + (size_t)h * hd, hd);
    }
    const int q_per_kv = n_kv_heads > 0 ? n_heads / n_kv_heads : 1;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; ++h) {
        const int kv_h = (n_kv_heads == n_heads) ? h : h / q_per_kv;
        if (window == 1) {
            for (int d = 0; d < hd; ++d) out[(size_t)h * hd + d] = v[(size_t)kv_h * hd + d];
            continue;
        }
        float *scores = (float *)malloc(sizeof(float) * (size_t)window);
        float *row = (float *)malloc(sizeof(float) * (size_t)hd);
        double *acc = (double *)calloc((size_t)hd, sizeof(double));
        const size_t base = (size_t)layer * per_layer + (size_t)kv_h * per_head;
        float mx = -1e20f;
        for (int i = 0; i < window; ++i) {
            const int slot = (start + i) % n_ctx;
            kv_load(kv, 0, base + (size_t)slot * hd, row, hd);
            double dot = 0.0;
            for (int d = 0; d < hd; ++d) dot += (double)q[(size_t)h * hd + d] * (double)row[d];
            scores[i] = (float)dot * scale;
            if (scores[i] > mx) mx = scores[i];
        }
        /* p_i = exp(s_i - max) rounded once to fp32; the normalisation and the
         * weighted sum are carried in double and rounded once per output. */
        double sum = 0.0;
        for (int i = 0; i < window; ++i) {
            scores[i] = (float)exp((double)(scores[i] - mx));
            sum += (double)scores[i];
        }
        for (int i = 0; i < window; ++i) {
            const int slot = (start + i) % n_ctx;
            kv_load(kv, 1, base + (size_t)slot * hd, row, hd);
            for (int d = 0; d < hd; ++d) acc[d] += (double)scores[i] * (double)row[d];
        }
        for (int d = 0; d < hd; ++d) out[(size_t)h * hd + d] = (float)(acc[d] / sum);
        free(scores);
        free(row);
        free(acc);
    }
}

void orc_decode_attention_f16(const float *q, const float *k, const float *v,
                              uint16_t *k_cache, uint16_t *v_cache, float *out,
                              int head_dim, int n_heads, int n_kv_heads,
                              int n_ctx, int pos, int layer) {
    kv_view kv = {ORC_KV_F16, k_cache, v_cache, NULL, NULL};
    decode_attention(q, k, v, &kv, out, head_dim, n_heads, n_kv_heads, n_ctx, pos, layer);
}

void orc_decode_attention_q4(const float *q, const float *k, const float *v,
                             orc_block_q4_0 *k_cache, orc_block_q4_0 *v_cache,
                             float *out, int head_dim, int n_heads,
                             int n_kv_heads, int n_ctx, int pos, int layer) {
    kv_view kv = {ORC_KV_Q4_0, NULL, NULL, k_cache, v_cache};
    decode_attention(q, k, v, &kv, out, head_dim, n_heads, n_kv_heads, n_ctx, pos, layer);
}

/* ------------------------------------------------------------------------ */
/* Minimal GGUF reader (format: magic, version, tensor/kv counts, kv pairs,  */
/* tensor infos, aligned data section).                                      */
/* ------------------------------------------------------------------------ */
enum { GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_I32 = 26, GT_BF16 = 30 };

typedef struct {
    char name[128];
    int n_dims;
    int64_t ne[4];
    int type;
    uint64_t offset;
    const uint8_t *data;
} gg_tensor;

typedef struct {
    uint8_t *map;
    size_t size;
    gg_tensor *t;
    int64_t n_t;
} gg_file;

typedef struct { const uint8_t *p, *end; int ok; } rd;

static uint64_t rd_u(rd *r, int n) {
    uint64_t v = 0;
    if (r->p + n > r->end) { r->ok = 0; return 0; }
    memcpy(&v, r->p, (size_t)n);
    r->p += n;
    return v;
}
static void rd_skip(rd *r, uint64_t n) {
    if ((uint64_t)(r->end - r->p) < n) { r->ok = 0; return; }
    r->p += n;
}
static void rd_skip_val(rd *r, uint32_t type) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) { uint64_t n = rd_u(r, 8); rd_skip(r, n); return; }
    if (type == 9) {
        uint32_t et = (uint32_t)rd_u(r, 4);
        uint64_t cnt = rd_u(r, 8);
        for (uint64_t i = 0; i < cnt && r->ok; ++i) rd_skip_val(r, et);
        return;
    }
    if (type > 12) { r->ok = 0; return; }
    rd_skip(r, (uint64_t)sz[type]);
}

static int64_t type_row_bytes(int type, int64_t ne0) {
    switch (type) {
    case GT_F32: case GT_I32: return ne0 * 4;
    case GT_F16: case GT_BF16: return ne0 * 2;
    case GT_Q4_0: return ne0 / 32 * 18;
    case GT_Q8_0: return ne0 / 32 * 34;
    default: return -1;
    }
}

static int gg_open(const char *path, gg_file *g) {
    memset(g, 0, sizeof(*g));
    int fd = open(path, O_RDONLY);
    if (fd < 0) return -1;
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return -1; }
    g->size = (size_t)st.st_size;
    g->map = (uint8_t *)mmap(NULL, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (g->map == MAP_FAILED) { g->map = NULL; return -1; }
    rd r = {g->map, g->map + g->size, 1};
    if (rd_u(&r, 4) != 0x46554747u) return -2; /* "GGUF" */
    uint32_t ver = (uint32_t)rd_u(&r, 4);
    if (ver < 2) return -2;
    g->n_t = (int64_t)rd_u(&r, 8);
    int64_t n_kv = (int64_t)rd_u(&r, 8);
    uint64_t alignment = 32;
    for (int64_t i = 0; i < n_kv && r.ok; ++i) {
        uint64_t klen = rd_u(&r, 8);
        const char *key = (const char *)r.p;
        rd_skip(&r, klen);
        uint32_t vt = (uint32_t)rd_u(&r, 4);
        if (klen == 17 && memcmp(key, "general.alignment", 17) == 0 && vt == 4) alignment = rd_u(&r, 4);
        else rd_skip_val(&r, vt);
    }
    if (!r.ok || g->n_t < 0 || g->n_t > 1000000) return -2;
    g->t = (gg_tensor *)calloc((size_t)g->n_t + 1, sizeof(gg_tensor));
    for (int64_t i = 0; i < g->n_t && r.ok; ++i) {
        uint64_t nlen = rd_u(&r, 8);
        if (nlen >= sizeof(g->t[i].name)) { r.ok = 0; break; }
        memcpy(g->t[i].name, r.p, nlen);
        rd_skip(&r, nlen);
        g->t[i].n_dims = (int)rd_u(&r, 4);
        if (g->t[i].n_dims < 1 || g->t[i].n_dims > 4) { r.ok = 0; break; }
        for (int d = 0; d < 4; ++d) g->t[i].ne[d] = 1;
        for (int d = 0; d < g->t[i].n_dims; ++d) g->t[i].ne[d] = (int64_t)rd_u(&r, 8);
        g->t[i].type = (int)rd_u(&r, 4);
        g->t[i].offset = rd_u(&r, 8);
    }
    if (!r.ok) return -2;
    size_t hdr = (size_t)(r.p - g->map);
    size_t data0 = (hdr + alignment - 1) / alignment * alignment;
    for (int64_t i = 0; i < g->n_t; ++i) {
        gg_tensor *t = &g->t[i];
        int64_t rb = type_row_bytes(t->type, t->ne[0]);
        int64_t nbytes = rb < 0 ? 0 : rb * t->ne[1] * t->ne[2] * t->ne[3];
        if (data0 + t->offset + (uint64_t)nbytes > g->size) return -3;
        t->data = g->map + data0 + t->offset;
    }
    return 0;
}

static void gg_close(gg_file *g) {
    if (g->map) munmap(g->map, g->size);
    free(g->t);
    memset(g, 0, sizeof(*g));
}

static const gg_tensor *gg_find(const gg_file *g, const char *name) {
    for (int64_t i = 0; i < g->n_t; ++i)
        if (strcmp(g->t[i].name, name) == 0) return &g->t[i];
    return NULL;
}

static const gg_tensor *gg_find_any(const gg_file *g, const char *a, const char *b, const char *c) {
    const gg_tensor *t = gg_find(g, a);
    if (!t && b) t = gg_find(g, b);
    if (!t && c) t = gg_find(g, c);
    return t;
}

/* Scalar hyperparameters live in 1-element tensors (bmo.cpp:62-80). */
static int32_t scalar_i32(const gg_file *g, const char *name, int32_t fb) {
    const gg_tensor *t = gg_find(g, name);
    if (!t || !t->data) return fb;
    int32_t v;
    memcpy(&v, t->data, 4);
    return v;
}
static float scalar_f32(const gg_file *g, const char *name, float fb) {
    const gg_tensor *t = gg_find(g, name);
    if (!t || !t->data) return fb;
    float v;
    memcpy(&v, t->data, 4);
    return v;
}

/* One embedding row as fp32 (the to_float branch of unpack_emb_row,
 * bmo_api.cpp:80-100); returns 0 when the row is skipped. */
static int emb_row(const gg_tensor *t, int32_t tok, float *dst, int64_t dim) {
    if (!t || tok < 0 || tok >= t->ne[1] || t->ne[0] != dim) return 0;
    const int64_t rb = type_row_bytes(t->type, t->ne[0]);
    const uint8_t *row = t->data + (size_t)tok * (size_t)rb;
    switch (t->type) {
    case GT_F32: memcpy(dst, row, (size_t)dim * 4); return 1;
    case GT_F16:
        for (int64_t i = 0; i < dim; ++i) { uint16_t h; memcpy(&h, row + 2 * i, 2); dst[i] = orc_fp16_to_fp32(h); }
        return 1;
    case GT_BF16:
        for (int64_t i = 0; i < dim; ++i) { uint16_t h; memcpy(&h, row + 2 * i, 2); uint32_t u = (uint32_t)h << 16; memcpy(&dst[i], &u, 4); }
        return 1;
    case GT_Q4_0: orc_dequantize_row_q4_0((const orc_block_q4_0 *)row, dst, (int)dim); return 1;
    case GT_Q8_0: dequantize_row_q8_0(row, dst, (int)dim); return 1;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* Model                                                                     */
/* ------------------------------------------------------------------------ */
#define ORC_MAX_LAYERS 128
#define ORC_DEP_Q 8
#define ORC_DEP_LAYERS 6
#define ORC_MAX_EMBS 32

typedef struct {
    const gg_tensor *qkv, *wo, *ffn_in, *ffn_out, *norm1, *norm2;
} orc_layer;

struct orc_model {
    gg_file g;
    int n_layers, n_embd, n_heads, head_dim, n_kv_heads, ffn_hidden;
    int n_ctx, kv_type, n_q, num_codebooks, dep_q, text_vocab, audio_vocab;
    float rope_theta, norm_eps;
    orc_layer L[ORC_MAX_LAYERS];
    const gg_tensor *text_emb_t, *audio_emb_t[ORC_MAX_EMBS];
    int n_audio_emb_slots;
    const gg_tensor *out_norm, *text_linear, *text_bias;
    /* depformer */
    int dep_dim, dep_heads, dep_hd, dep_ffn, dep_n_ctx;
    const gg_tensor *dep_in[ORC_DEP_Q], *dep_emb[ORC_DEP_Q], *dep_text_emb, *dep_head[ORC_DEP_Q];
    const gg_tensor *dep_in_proj[ORC_DEP_LAYERS], *dep_out_proj[ORC_DEP_LAYERS];
    const gg_tensor *dep_norm1[ORC_DEP_LAYERS], *dep_norm2[ORC_DEP_LAYERS];
    const gg_tensor *dep_gin[ORC_DEP_LAYERS][ORC_DEP_Q], *dep_gout[ORC_DEP_LAYERS][ORC_DEP_Q];
    /* state */
    void *k_cache, *v_cache;           /* [layer][kv_head][slot][hd] */
    uint16_t *dk_cache, *dv_cache;     /* depth fp16 [layer][head][slot][hd] */
    /* independent temporal rings of batched sessions; k_cache/v_cache point
     * at ring `cur` (ring 0 is the one kv_alloc made) */
    void **sk, **sv;
    int n_sess, cur;
};

static const orc_block_q4_0 *q4(const gg_tensor *t) { return (const orc_block_q4_0 *)t->data; }
static const float *f32(const gg_tensor *t) { return (const float *)t->data; }

static size_t kv_elems(const orc_model *m) {
    return (size_t)m->n_layers * m->n_kv_heads * m->n_ctx * m->head_dim;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    gg_close(&m->g);
    if (m->sk) {
        for (int i = 0; i < m->n_sess; ++i) {
            free(m->sk[i]);
            free(m->sv[i]);
        }
        free(m->sk);
        free(m->sv);
    } else {
        free(m->k_cache);
        free(m->v_cache);
    }
    free(m->dk_cache);
    free(m->dv_cache);
    free(m);
}

static void kv_alloc(orc_model *m) {
    const size_t n = kv_elems(m);
    const size_t bytes = m->kv_type == ORC_KV_F16 ? n * 2 : n / 32 * sizeof(orc_block_q4_0);
    m->k_cache = calloc(1, bytes);
    m->v_cache = calloc(1, bytes);
    const size_t dn = (size_t)ORC_DEP_LAYERS * m->dep_heads * m->dep_n_ctx * m->dep_hd;
    m->dk_cache = (uint16_t *)calloc(dn > 0 ? dn : 1, 2);
    m->dv_cache = (uint16_t *)calloc(dn > 0 ? dn : 1, 2);
}

void orc_reset(orc_model *m) {
    const size_t n = kv_elems(m);
    const size_t bytes = m->kv_type == ORC_KV_F16 ? n * 2 : n / 32 * sizeof(orc_block_q4_0);
    memset(m->k_cache, 0, bytes);
    memset(m->v_cache, 0, bytes);
}

/* Batched sessions (the session-batched frame of the build's ABI extension):
 * n independent temporal rings over the same weights. */
int orc_sessions(orc_model *m, int n) {
    if (!m || n < 1 || m->sk) return 1;
    const size_t e = kv_elems(m);
    const size_t bytes = m->kv_type == ORC_KV_F16 ? e * 2 : e / 32 * sizeof(orc_block_q4_0);
    m->sk = (void **)calloc((size_t)n, sizeof(void *));
    m->sv = (void **)calloc((size_t)n, sizeof(void *));
    if (!m->sk || !m->sv) return 2;
    m->sk[0] = m->k_cache;
    m->sv[0] = m->v_cache;
    m->n_sess = n;
    for (int i = 1; i < n; ++i) {
        m->sk[i] = calloc(1, bytes);
        m->sv[i] = calloc(1, bytes);
        if (!m->sk[i] || !m->sv[i]) return 2;
    }
    m->cur = 0;
    return 0;
}

int orc_select_session(orc_model *m, int s) {
    if (!m || !m->sk || s < 0 || s >= m->n_sess) return 1;
    m->cur = s;
    m->k_cache = m->sk[s];
    m->v_cache = m->sv[s];
    return 0;
}

void orc_reset_depth_kv(orc_model *m) {
    const size_t dn = (size_t)ORC_DEP_LAYERS * m->dep_heads * m->dep_n_ctx * m->dep_hd;
    memset(m->dk_cache, 0, dn * 2);
    memset(m->dv_cache, 0, dn * 2);
}

void orc_model_set_threads(orc_model *m, int n_threads) {
    (void)m;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
}

orc_model *orc_model_load(const char *path, int n_ctx, int kv_type) {
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    if (!m) return NULL;
    if (gg_open(path, &m->g) != 0) { orc_model_free(m); return NULL; }
    const gg_file *g = &m->g;
    char a[160], b[160], c[160];

    /* hyperparameters, bmo.cpp:285-334 */
    m->n_layers = scalar_i32(g, "n_layers", 0);
    if (m->n_layers <= 0) m->n_layers = scalar_i32(g, "n_layer", 32);
    m->n_heads = scalar_i32(g, "n_heads", 0);
    if (m->n_heads <= 0) m->n_heads = scalar_i32(g, "n_head", 0);
    m->n_embd = scalar_i32(g, "n_embd", 0);
    if (m->n_embd <= 0) m->n_embd = scalar_i32(g, "hidden_size", 0);
    m->head_dim = scalar_i32(g, "head_dim", 0);
    if (m->head_dim <= 0) m->head_dim = scalar_i32(g, "n_embd_head_k", 0);
    m->rope_theta = scalar_f32(g, "rope_theta", 0.0f);
    if (m->rope_theta <= 0.0f) m->rope_theta = scalar_f32(g, "rope_freq_base", 0.0f);
    if (m->rope_theta <= 0.0f) m->rope_theta = 10000.0f;
    m->norm_eps = scalar_f32(g, "norm_eps", 0.0f);
    if (m->norm_eps <= 0.0f) m->norm_eps = scalar_f32(g, "rms_norm_eps", 0.0f);
    if (m->norm_eps <= 0.0f) m->norm_eps = 1e-8f;
    if (m->n_heads <= 0) m->n_heads = 32;
    if (m->n_embd <= 0) m->n_embd = 4096;
    if (m->head_dim <= 0) m->head_dim = m->n_embd / m->n_heads;
    if (m->n_layers > ORC_MAX_LAYERS) { orc_model_free(m); return NULL; }

    /* temporal layers, bmo.cpp:336-374 */
    for (int i = 0; i < m->n_layers; ++i) {
        orc_layer *L = &m->L[i];
        snprintf(a, sizeof a, "transformer_layers_%d_self_attn_in_proj_weight", i);
        snprintf(b, sizeof b, "transformer_layers_%d_self_attn_in_proj", i);
        L->qkv = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "transformer_layers_%d_self_attn_out_proj_weight", i);
        snprintf(b, sizeof b, "transformer_layers_%d_self_attn_out_proj", i);
        L->wo = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "transformer_layers_%d_gating_linear_in_weight", i);
        snprintf(b, sizeof b, "transformer_layers_%d_gating_linear_in", i);
        L->ffn_in = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "transformer_layers_%d_gating_linear_out_weight", i);
        snprintf(b, sizeof b, "transformer_layers_%d_gating_linear_out", i);
        L->ffn_out = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "transformer_layers_%d_norm1_weight", i);
        snprintf(b, sizeof b, "transformer_layers_%d_attn_norm.weight", i);
        snprintf(c, sizeof c, "transformer_layers_%d_norm1.weight", i);
        L->norm1 = gg_find_any(g, a, b, c);
        snprintf(a, sizeof a, "transformer_layers_%d_norm2_weight", i);
        snprintf(b, sizeof b, "transformer_layers_%d_ffn_norm.weight", i);
        snprintf(c, sizeof c, "transformer_layers_%d_norm2.weight", i);
        L->norm2 = gg_find_any(g, a, b, c);
        if (!L->qkv || !L->wo || !L->ffn_in || !L->ffn_out || !L->norm1 || !L->norm2 ||
            L->qkv->type != GT_Q4_0 || L->wo->type != GT_Q4_0 || L->ffn_in->type != GT_Q4_0 ||
            L->ffn_out->type != GT_Q4_0 || L->norm1->type != GT_F32 || L->norm2->type != GT_F32) {
            orc_model_free(m);
            return NULL;
        }
    }
    const int q_dim = m->n_heads * m->head_dim;
    m->n_kv_heads = (int)((m->L[0].qkv->ne[1] - q_dim) / 2 / m->head_dim);
    m->ffn_hidden = (int)(m->L[0].ffn_in->ne[1] / 2);

    /* depformer, bmo.cpp:376-410 */
    for (int i = 0; i < ORC_DEP_LAYERS; ++i) {
        snprintf(a, sizeof a, "depformer.layers.%d.norm1.weight", i);
        snprintf(b, sizeof b, "depformer_layers_%d_norm1_weight", i);
        m->dep_norm1[i] = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "depformer.layers.%d.norm2.weight", i);
        snprintf(b, sizeof b, "depformer_layers_%d_norm2_weight", i);
        m->dep_norm2[i] = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "depformer.layers.%d.self_attn.in_proj_weight", i);
        snprintf(b, sizeof b, "depformer_layers_%d_self_attn_in_proj_weight", i);
        m->dep_in_proj[i] = gg_find_any(g, a, b, NULL);
        snprintf(a, sizeof a, "depformer.layers.%d.self_attn.out_proj.weight", i);
        snprintf(b, sizeof b, "depformer_layers_%d_self_attn_out_proj_weight", i);
        m->dep_out_proj[i] = gg_find_any(g, a, b, NULL);
        for (int s = 0; s < ORC_DEP_Q; ++s) {
            snprintf(a, sizeof a, "depformer_layers_%d_gating_%d_linear_in_weight", i, s);
            snprintf(b, sizeof b, "depformer_layers_%d_gating_%d_linear_in", i, s);
            m->dep_gin[i][s] = gg_find_any(g, a, b, NULL);
            snprintf(a, sizeof a, "depformer_layers_%d_gating_%d_linear_out_weight", i, s);
            snprintf(b, sizeof b, "depformer_layers_%d_gating_%d_linear_out", i, s);
            m->dep_gout[i][s] = gg_find_any(g, a, b, NULL);
        }
    }
    for (int k = 0; k < ORC_DEP_Q; ++k) {
        snprintf(a, sizeof a, "depformer_emb.%d.weight", k);
        m->dep_emb[k] = gg_find(g, a);
        snprintf(a, sizeof a, "depformer_in.%d.weight", k);
        m->dep_in[k] = gg_find(g, a);
        snprintf(a, sizeof a, "linears.%d.weight", k);
        m->dep_head[k] = gg_find(g, a);
    }
    m->dep_text_emb = gg_find(g, "depformer_text_emb.weight");
    m->text_linear = gg_find(g, "text_linear.weight");
    m->text_bias = gg_find(g, "text_linear.bias");
    m->out_norm = gg_find(g, "out_norm_weight");

    /* temporal embeddings, bmo.cpp:491-508 */
    int last = -1;
    for (int k = 0; k < ORC_MAX_EMBS; ++k) {
        snprintf(a, sizeof a, "emb.%d.weight", k);
        m->audio_emb_t[k] = gg_find(g, a);
        if (m->audio_emb_t[k]) last = k;
    }
    m->n_audio_emb_slots = last + 1;
    m->text_emb_t = gg_find(g, "text_emb.weight");

    /* geometry, bmo.cpp:510-568 */
    int n_q = 0, in_vocab = 0;
    for (int k = 0; k < m->n_audio_emb_slots; ++k) {
        if (!m->audio_emb_t[k]) continue;
        ++n_q;
        if (!in_vocab) in_vocab = (int)m->audio_emb_t[k]->ne[1];
    }
    if (n_q == 0) {
        for (int k = 0; k < ORC_DEP_Q; ++k) {
            if (!m->dep_emb[k]) continue;
            ++n_q;
            if (!in_vocab) in_vocab = (int)m->dep_emb[k]->ne[1];
        }
    }
    int dq = 0, out_vocab = 0;
    for (int k = 0; k < ORC_DEP_Q; ++k) {
        if (m->dep_in[k]) ++dq;
        if (!out_vocab && m->dep_head[k]) out_vocab = (int)m->dep_head[k]->ne[1];
    }
    m->n_q = n_q;
    m->num_codebooks = n_q > 0 ? n_q + 1 : 0;
    m->dep_q = dq;
    m->audio_vocab = out_vocab > 0 ? out_vocab : in_vocab;
    m->text_vocab = m->text_linear ? (int)m->text_linear->ne[1]
                  : m->text_emb_t ? (int)m->text_emb_t->ne[1]
                  : m->dep_text_emb ? (int)m->dep_text_emb->ne[1] : 0;

    /* depth geometry: 16 heads, head_dim = dim/16, context min(dep_q, 8)
     * (bmo.cpp:1447-1452; the reference fixes dim=1024 and 16 heads).  A
     * "depformer_num_heads" scalar, absent from reference files, overrides
     * the head count for the small synthetic test models. */
    m->dep_dim = m->dep_in[0] ? (int)m->dep_in[0]->ne[1] : 0;
    m->dep_heads = scalar_i32(g, "depformer_num_heads", 16);
    if (m->dep_heads <= 0) m->dep_heads = 16;
    m->dep_hd = m->dep_dim / m->dep_heads;
    m->dep_ffn = m->dep_gin[0][0] ? (int)(m->dep_gin[0][0]->ne[1] / 2) : 0;
    m->dep_n_ctx = dq > ORC_DEP_Q ? ORC_DEP_Q : dq;

    m->n_ctx = n_ctx > 0 ? n_ctx : 2048;
    m->kv_type = kv_type;
    kv_alloc(m);
    if (!m->k_cache || !m->v_cache) { orc_model_free(m); return NULL; }
    return m;
}

int orc_model_geometry(const orc_model *m, int32_t *out, int n_out) {
    const int32_t v[12] = {m->n_layers, m->n_embd, m->n_heads, m->head_dim,
                           m->num_codebooks, m->dep_q, m->text_vocab, m->audio_vocab,
                           m->n_ctx, m->n_kv_heads, m->ffn_hidden, m->dep_dim};
    int n = n_out < 12 ? n_out : 12;
    for (int i = 0; i < n; ++i) out[i] = v[i];
    return n;
}

/* bmo_embed_input_tokens_into, bmo_compute.cpp:1867-1912. */
int orc_embed(orc_model *m, const int32_t *tokens, int K, float *acc) {
    const int n = m->n_embd;
    float *tmp = (float *)malloc(sizeof(float) * (size_t)n);
    memset(acc, 0, sizeof(float) * (size_t)n);
    if (emb_row(m->text_emb_t, tokens[0], tmp, n))
        for (int i = 0; i < n; ++i) acc[i] += tmp[i];
    for (int k = 1; k < K; ++k) {
        if (k - 1 >= m->n_audio_emb_slots) break;
        if (emb_row(m->audio_emb_t[k - 1], tokens[k], tmp, n))
            for (int i = 0; i < n; ++i) acc[i] += tmp[i];
    }
    free(tmp);
    return 0;
}

static kv_view temporal_kv(orc_model *m) {
    kv_view kv;
    kv.kind = m->kv_type;
    kv.k16 = (uint16_t *)m->k_cache;
    kv.v16 = (uint16_t *)m->v_cache;
    kv.k4 = (orc_block_q4_0 *)m->k_cache;
    kv.v4 = (orc_block_q4_0 *)m->v_cache;
    return kv;
}

/* One temporal layer, bmo_compute.cpp:2188-2640. */
static void temporal_layer(orc_model *m, int layer, float *x, int pos) {
    const int n = m->n_embd, hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv_heads * hd;
    const int F = m->ffn_hidden;
    const orc_layer *L = &m->L[layer];
    float *xn = (float *)malloc(sizeof(float) * (size_t)n);
    float *qkv = (float *)malloc(sizeof(float) * (size_t)(qd + 2 * kvd));
    float *q = (float *)malloc(sizeof(float) * (size_t)qd);
    float *k = (float *)malloc(sizeof(float) * (size_t)kvd);
    float *att = (float *)malloc(sizeof(float) * (size_t)qd);
    float *o = (float *)malloc(sizeof(float) * (size_t)n);
    float *h = (float *)malloc(sizeof(float) * (size_t)(2 * F));
    float *act = (float *)malloc(sizeof(float) * (size_t)F);

    orc_rmsnorm(x, f32(L->norm1), m->norm_eps, n, xn);
    linear_q4_0(q4(L->qkv), xn, qkv, qd + 2 * kvd, n);
    orc_rope_interleaved(qkv, m->n_heads, hd, pos, m->rope_theta, q);
    orc_rope_interleaved(qkv + qd, m->n_kv_heads, hd, pos, m->rope_theta, k);
    kv_view kv = temporal_kv(m);
    decode_attention(q, k, qkv + qd + kvd, &kv, att, hd, m->n_heads, m->n_kv_heads, m->n_ctx, pos, layer);
    linear_q4_0(q4(L->wo), att, o, n, qd);
    for (int i = 0; i < n; ++i) x[i] = x[i] + o[i];
    orc_rmsnorm(x, f32(L->norm2), m->norm_eps, n, xn);
    linear_q4_0(q4(L->ffn_in), xn, h, 2 * F, n);
    orc_swiglu(h, F, act);
    linear_q4_0(q4(L->ffn_out), act, o, n, F);
    for (int i = 0; i < n; ++i) x[i] = x[i] + o[i];

    free(xn); free(qkv); free(q); free(k); free(att); free(o); free(h); free(act);
}

int orc_forward_layers(orc_model *m, const float *x_in, int pos, int layer_begin,
                       int layer_end, float *x_out) {
    if (layer_begin < 0 || layer_end > m->n_layers || layer_begin >= layer_end) return 2;
    memcpy(x_out, x_in, sizeof(float) * (size_t)m->n_embd);
    for (int l = layer_begin; l < layer_end; ++l) temporal_layer(m, l, x_out, pos);
    return 0;
}

/* bmo_forward_temporal2, bmo_api.cpp:384-511. */
int orc_forward_temporal(orc_model *m, const int32_t *tokens, int K, int pos,
                         float *out_z, float *out_logits,
                         const int32_t *capture, int n_capture, float *capture_out) {
    if (!tokens || !out_z || !out_logits) return 1;
    if (K <= 0 || K > m->num_codebooks || pos < 0) return 2;
    const int n = m->n_embd;
    float *x = (float *)malloc(sizeof(float) * (size_t)n);
    orc_embed(m, tokens, K, x);
    for (int l = 0; l < m->n_layers; ++l) {
        temporal_layer(m, l, x, pos);
        for (int c = 0; c < n_capture; ++c)
            if (capture[c] == l) memcpy(capture_out + (size_t)c * n, x, sizeof(float) * (size_t)n);
    }
    float *fin = (float *)malloc(sizeof(float) * (size_t)n);
    if (m->out_norm) orc_rmsnorm(x, f32(m->out_norm), m->norm_eps, n, fin);
    else memcpy(fin, x, sizeof(float) * (size_t)n);
    memcpy(out_z, fin, sizeof(float) * (size_t)n);
    if (m->text_linear) {
        linear_q4_0(q4(m->text_linear), fin, out_logits, m->text_vocab, n);
        if (m->text_bias)
            for (int i = 0; i < m->text_vocab; ++i) out_logits[i] = out_logits[i] + f32(m->text_bias)[i];
    }
    free(x);
    free(fin);
    for (int c = 0; c < n_capture; ++c)
        if (capture[c] < 0 || capture[c] >= m->n_layers) return 6;
    return 0;
}

/* out_norm + text head on a given final residual (bmo_compute.cpp:2660-2735). */
int orc_text_head(orc_model *m, const float *x_final, float *out_z, float *out_logits) {
    const int n = m->n_embd;
    if (m->out_norm) orc_rmsnorm(x_final, f32(m->out_norm), m->norm_eps, n, out_z);
    else memcpy(out_z, x_final, sizeof(float) * (size_t)n);
    if (!m->text_linear) return 3;
    linear_q4_0(q4(m->text_linear), out_z, out_logits, m->text_vocab, n);
    if (m->text_bias)
        for (int i = 0; i < m->text_vocab; ++i) out_logits[i] = out_logits[i] + f32(m->text_bias)[i];
    return 0;
}

/* bmo_build_depth_graph, bmo_compute.cpp:2741-3340 (one codebook step). */
int orc_forward_depth(orc_model *m, int cb, int32_t prev_token, const float *z, float *out_logits) {
    if (!z || !out_logits) return 1;
    if (cb < 0 || cb >= m->dep_q || cb >= m->dep_n_ctx) return 2;
    const int D = m->dep_dim, hd = m->dep_hd, H = m->dep_heads, F = m->dep_ffn;
    if (cb == 0) orc_reset_depth_kv(m);
    float *x = (float *)malloc(sizeof(float) * (size_t)D);
    float *e = (float *)calloc((size_t)D, sizeof(float));
    float *xn = (float *)malloc(sizeof(float) * (size_t)D);
    float *qkv = (float *)malloc(sizeof(float) * (size_t)3 * D);
    float *att = (float *)malloc(sizeof(float) * (size_t)D);
    float *o = (float *)malloc(sizeof(float) * (size_t)D);
    float *h = (float *)malloc(sizeof(float) * (size_t)2 * F);
    float *act = (float *)malloc(sizeof(float) * (size_t)F);

    linear_q4_0(q4(m->dep_in[cb]), z, x, D, m->n_embd);
    const gg_tensor *et = cb == 0 ? m->dep_text_emb : m->dep_emb[cb - 1];
    if (!emb_row(et, prev_token, e, D)) memset(e, 0, sizeof(float) * (size_t)D);
    for (int i = 0; i < D; ++i) x[i] = x[i] + e[i];

    kv_view kv = {ORC_KV_F16, m->dk_cache, m->dv_cache, NULL, NULL};
    for (int i = 0; i < ORC_DEP_LAYERS; ++i) {
        const orc_block_q4_0 *w_in = q4(m->dep_in_proj[i]) + (size_t)cb * 3 * D * (D / 32);
        const orc_block_q4_0 *w_out = q4(m->dep_out_proj[i]) + (size_t)cb * D * (D / 32);
        orc_rmsnorm(x, f32(m->dep_norm1[i]), m->norm_eps, D, xn);
        linear_q4_0(w_in, xn, qkv, 3 * D, D);
        decode_attention(qkv, qkv + D, qkv + 2 * D, &kv, att, hd, H, H, m->dep_n_ctx, cb, i);
        linear_q4_0(w_out, att, o, D, D);
        for (int j = 0; j < D; ++j) x[j] = x[j] + o[j];
        orc_rmsnorm(x, f32(m->dep_norm2[i]), m->norm_eps, D, xn);
        linear_q4_0(q4(m->dep_gin[i][cb]), xn, h, 2 * F, D);
        orc_swiglu(h, F, act);
        linear_q4_0(q4(m->dep_gout[i][cb]), act, o, D, F);
        for (int j = 0; j < D; ++j) x[j] = x[j] + o[j];
    }
    linear_q4_0(q4(m->dep_head[cb]), x, out_logits, m->audio_vocab, D);
    free(x); free(e); free(xn); free(qkv); free(att); free(o); free(h); free(act);
    return 0;
}

/* bmo_forward_depth_cascade greedy branch, bmo_api.cpp:668-743. */
int orc_forward_depth_cascade_greedy(orc_model *m, int32_t text_token, const float *z,
                                     int32_t *out_tokens) {
    float *logits = (float *)malloc(sizeof(float) * (size_t)(m->audio_vocab > 2049 ? m->audio_vocab : 2049));
    int32_t prev = text_token;
    orc_reset_depth_kv(m);
    for (int cb = 0; cb < m->dep_q; ++cb) {
        int rc = orc_forward_depth(m, cb, prev, z, logits);
        if (rc) { free(logits); return rc; }
        if (m->audio_vocab > 2048) logits[2048] = -1e9f;
        const int nv = m->audio_vocab < 2048 ? m->audio_vocab : 2048;
        prev = orc_argmax(logits, nv);
        out_tokens[cb] = prev;
    }
    free(logits);
    return 0;
}

int orc_kv_import(orc_model *m, int layer, int slot0, int n, const float *k_rows, const float *v_rows) {
    if (layer < 0 || layer >= m->n_layers || slot0 < 0 || slot0 + n > m->n_ctx) return 2;
    kv_view kv = temporal_kv(m);
    const int hd = m->head_dim;
    const size_t per_head = (size_t)hd * m->n_ctx, per_layer = per_head * m->n_kv_heads;
    for (int i = 0; i < n; ++i)
        for (int h = 0; h < m->n_kv_heads; ++h) {
            const size_t off = (size_t)layer * per_layer + (size_t)h * per_head + (size_t)(slot0 + i) * hd;
            const size_t src = ((size_t)i * m->n_kv_heads + h) * hd;
            kv_store(&kv, 0, off, k_rows + src, hd);
            kv_store(&kv, 1, off, v_rows + src, hd);
        }
    return 0;
}

int orc_kv_export(orc_model *m, int which, int layer, int slot0, int n, float *out) {
    if (layer < 0 || layer >= m->n_layers || slot0 < 0 || slot0 + n > m->n_ctx) return 2;
    kv_view kv = temporal_kv(m);
    const int hd = m->head_dim;
    const size_t per_head = (size_t)hd * m->n_ctx, per_layer = per_head * m->n_kv_heads;
    for (int i = 0; i < n; ++i)
        for (int h = 0; h < m->n_kv_heads; ++h) {
            const size_t off = (size_t)layer * per_layer + (size_t)h * per_head + (size_t)(slot0 + i) * hd;
            kv_load(&kv, which, off, out + ((size_t)i * m->n_kv_heads + h) * hd, hd);
        }
    return 0;
}

/* ---- synthetic model data ------------------------------------------------
 * The counter-based generator of the benchmark models (splitmix64 finaliser
 * over (seed, stream, index), Box-Muller pairs), restated here so that the
 * CPU-only benchmark arm can write the same GGUF bit for bit without loading
 * the CUDA engine library.  Element i of a (seed, stream) tensor is the
 * cosine (even i) or sine (odd i) branch of pair i / 2. */
static uint64_t syn_mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static uint64_t syn_key(uint64_t seed, uint64_t stream) {
    return syn_mix64(seed) ^ syn_mix64(stream + 0x632be59bd9b4e019ull);
}

static double syn_uniform(uint64_t key, uint64_t i) {
    return ((double)(syn_mix64(key ^ syn_mix64(i)) >> 11) + 1.0) * 0x1.0p-53;
}

static void syn_pair(uint64_t key, uint64_t p, double *z0, double *z1) {
    const double r = sqrt(-2.0 * log(syn_uniform(key, 2 * p)));
    const double t = 6.283185307179586 * syn_uniform(key, 2 * p + 1);
    *z0 = r * cos(t);
    *z1 = r * sin(t);
}

void orc_synth_normal_f32(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, float *out) {
    const uint64_t key = syn_key(seed, stream);
#pragma omp parallel for schedule(static)
    for (long long p = 0; p < (n + 1) / 2; ++p) {
        double z[2];
        syn_pair(key, (uint64_t)p, &z[0], &z[1]);
        for (int k = 0; k < 2 && 2 * p + k < n; ++k) out[2 * p + k] = (float)((double)mean + (double)sigma * z[k]);
    }
}

void orc_synth_f16(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, uint16_t *out) {
    const uint64_t key = syn_key(seed, stream);
#pragma omp parallel for schedule(static)
    for (long long p = 0; p < (n + 1) / 2; ++p) {
        double z[2];
        syn_pair(key, (uint64_t)p, &z[0], &z[1]);
        for (int k = 0; k < 2 && 2 * p + k < n; ++k)
            out[2 * p + k] = orc_fp32_to_fp16((float)((double)mean + (double)sigma * z[k]));
    }
}

void orc_synth_q4_0(uint64_t seed, uint64_t stream, long long rows, long long cols, float sigma, uint8_t *out) {
    const uint64_t key = syn_key(seed, stream);
    const long long nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < rows; ++r) {
        float blk[32];
        for (long long b = 0; b < nb; ++b) {
            const uint64_t base = (uint64_t)(r * cols + b * 32);
            for (int j = 0; j < 32; j += 2) {
                double z0, z1;
                syn_pair(key, (base + (uint64_t)j) >> 1, &z0, &z1);
                blk[j] = (float)((double)sigma * z0);
                blk[j + 1] = (float)((double)sigma * z1);
            }
            orc_quantize_row_q4_0(blk, (orc_block_q4_0 *)(out + (size_t)(r * nb + b) * 18), 32);
        }
    }
}
