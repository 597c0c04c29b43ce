// batch_mma.cu -- the batched skinny GEMM Y[S][rows] = X[S][cols] . W^T on
// the 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Arithmetic per block b of 32 columns, row r, session s: the reference's
// Q4_0 x Q8_1 half-block terms (vec_dot_q4_0_q8_1, bmo_cuda_kernels.cu:
// 560-683)
//     t = d4[r][b] * (sumi_h[r][s][b] * d8[s][b] - 4 s8[s][b]),  h = low, high half
// with sumi_h the integer dot of 16 unsigned nibbles and 16 int8 codes (the
// reference's halves: elements 0-7 + 16-23 and 8-15 + 24-31).  The tensor
// core computes every sumi_h exactly: the activation rows are split into one
// row per half (layout.h), so one kind::i8 MMA of
// M = 128 rows x N = 2P rows x K = 32 per block (unsigned nibbles x signed
// codes, int32 accumulators) yields both half sums of every session, each
// block into its own TMEM slot.  The CUDA cores then form each term with the
// reference's fp32 roundings, two sessions per packed f32x2 instruction
// (sumi -> float exactly through the 2^23 + 2^22 bias, one fma against
// -M d8 = fl(sumi d8), one add of -4 s8, one multiply by d4), and
//   EXACT: sum the terms in double, rounded to fp32 once at the end -- the
//          double-sum semantics of the batch-1 GEMV and the oracle (equal up
//          to rare rounding ties from the summation order).  Each fp32 term
//          becomes a double times 2^-896 by moving its bit pattern with three
//          integer operations (exact for every finite float), which keeps the
//          conversion off the slow fp32-to-fp64 conversion unit; one multiply
//          by 2^896 restores each sum;
//   !EXACT: one full-block term d4 (sumi d8 - 8 s8) per block, summed in
//          fp32 (fp32-accurate, not reproducible bit for bit).
//
// CTA (one per SM, 20 warps; registers moved from the fifth warpgroup to the
// four epilogue warpgroups with setmaxnreg):
//   warp 17      TMEM owner; lane 0 the bulk-copy producer (per 8-block chunk
//                the four 32-row tiles' Q4_0 chunks of a 128-row block, 4 x
//                4608 B from HBM, the sessions' split Q8_1 codes, 512 P B, and
//                scales, 96 P B, from L2), lane 1 the MMA issuer
//   warp 16      unpacks nibbles into the MMA's K-major int8 layout (A)
//   warps 0-15   read the int32 half-block sums from TMEM (warp w: TMEM lanes
//                32(w%4).., sessions 16(w/4)..), release the slot, form and
//                sum the terms, then run the fused epilogue of layout.h's
//                Epilogue; four such warps per SM sub-partition hide each
//                other's TMEM-read and arithmetic latencies
// Work is split stream-K: the (128-row block, chunk) units are cut evenly
// over the CTAs; a row block shared by several CTAs is combined by the last
// one to finish, adding the partial float pairs in contributor order (the
// result does not depend on timing).  Every wait is bounded and any timeout
// makes all roles stop, drain the copies and MMAs in flight, free TMEM and
// raise the status word.
#include <atomic>

#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

constexpr int kMmaTiles = 4;                     // row tiles per 128-row block
constexpr int kMmaRows = kMmaTiles * kTileRows;  // MMA M
constexpr int kMmaStages = 2;
constexpr int kMmaABufs = 2;
constexpr int kMmaSlots = 4;                     // TMEM slots, one block each
constexpr int kMmaSlotCols = 128;                // >= N = 2P
constexpr int kMmaTmemCols = kMmaSlots * kMmaSlotCols;  // 512: all of TMEM
constexpr int kRawW = kMmaTiles * kChunkBytes;   // 18432
constexpr int kRawB = kBatchMax * 8 * 64;        // 32768: split codes of one chunk
constexpr int kRawS = kBatchMax * 8 * 12;        // 6144: their scales
constexpr int kRawBytes = kRawW + kRawB + kRawS;
constexpr int kABlockBytes = kMmaRows * 32;      // one block of A: 128 rows x 32 int8
constexpr int kABytes = kChunkBlocks * kABlockBytes;
constexpr int kGrpSess = 16;                       // sessions per epilogue warp
constexpr int kEpiGroups = kBatchMax / kGrpSess;   // epilogue warpgroups
constexpr int kEpiWarps = 4 * kEpiGroups, kUnpackWarps = 1;
constexpr int kCtlWarp = kEpiWarps + kUnpackWarps;  // lane 0: bulk-copy producer, lane 1: MMA issuer; owns TMEM
constexpr int kMmaThreads = (kEpiWarps + 4) * 32;   // five warpgroups; the last two warps only complete the fifth
// Register split (setmaxnreg, inside each role's branch): the launch gives
// every thread 96 registers (20 warps x 32 x 96 = 61440); the fifth
// warpgroup drops to 56 and the four epilogue warpgroups rise to 104:
// 4 x 128 x 104 + 128 x 56 = 60416 of the launch's 61440.
constexpr int kLaunchRegs = 96, kEpiRegs = 104, kCtlRegs = 56;
static_assert(kEpiGroups * 128 * kEpiRegs + 128 * kCtlRegs <= kMmaThreads * kLaunchRegs,
              "register split exceeds the launch");
static_assert(kGrpSess == 16, "an epilogue warp reads its sessions' half sums as four 8-column loads");
static_assert(kRawBytes % 1024 == 0 && kABytes % 1024 == 0, "stage buffers stay 1 KB aligned");
static_assert(2 * kBatchMax <= kMmaSlotCols, "a slot holds both halves of every session");

struct MmaSmem {
    uint8_t raw[kMmaStages][kRawBytes];
    uint8_t a[kMmaABufs][kABytes];
    uint64_t raw_full[kMmaStages], raw_empty[kMmaStages];
    uint64_t a_full[kMmaABufs], a_empty[kMmaABufs];
    uint64_t tm_full[kMmaSlots], tm_empty[kMmaSlots];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort;
    int last;
};

// ---- tcgen05 wrappers ----
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] = A . B^T (no accumulate): M=128 rows of unsigned 8-bit A, N
// columns of signed 8-bit B, K = 32, int32 accumulators.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0u)
        : "memory");
}
// Arrives on `bar` once every tcgen05 operation this thread issued before it has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
// 8 consecutive TMEM columns of this warp's 32 lanes (no wait).
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major without swizzle: 8-row x 16-byte
// core matrices stored as 128 contiguous bytes, the K-neighbour core matrix
// 128 bytes on (leading byte offset), the next 8 rows 256 bytes on (stride
// byte offset); bits 46-47 = 1 (sm_100 descriptor version).
__device__ __forceinline__ uint64_t kmajor_desc(const void *p) {
    return static_cast<uint64_t>((smem_addr(p) >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
           (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::i8: D s32 (bits 4-5 = 2), A u8 (bits 7-9 =
// 0), B s8 (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t idesc_i8(int n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(kMmaRows >> 4) << 24);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes (it wakes then, not at the end of the hint) or kSuspendNs
// pass, so a waiting role takes no issue slots from the epilogue warps.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// mbarrier wait for the pipeline hand-offs: repeated suspending try_waits, no
// sleep in between (a sleep would add its latency to every stage of every
// unit); gives up after 2 s, or as soon as another role has aborted.
constexpr uint64_t kWaitNs = 2000000000ull;
__device__ __forceinline__ bool wait_ab(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_hint(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort) return false;
            if (global_ns() - t0 > kWaitNs) break;
        }
    }
    *abort = 1;
    return false;
}

// Stream-K split: CTA c owns units [U c / G, U (c+1) / G); cta_of(u) is the owner of unit u.
__device__ __forceinline__ long long unit_lo(long long U, int G, int c) { return U * c / G; }
__device__ __forceinline__ int cta_of(long long u, long long U, int G) {
    return static_cast<int>(((u + 1) * G + U - 1) / U) - 1;
}

// ---------------------------------------------------------------------------
// per (row, session) epilogue; lane = row of tile t, all lanes take part
// ---------------------------------------------------------------------------
// QKV rows with the session's position and ring already in hand.
__device__ __forceinline__ void mma_qkv_row(const BatchGemmArgs &a, int t, int lane, int s, float v, int pos, int ring,
                                            float2 cs) {
    const int r = t * kTileRows + lane;
    const int hd = a.head_dim;
    float out = v;
    const bool is_q = r < a.q_dim;
    const bool is_k = !is_q && r < a.q_dim + a.kv_dim;
    if ((is_q || is_k) && a.rope) {
        const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
        out = (lane & 1) ? __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(v, cs.x))
                         : __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(partner, cs.y));
    }
    const long long ys = static_cast<long long>(s) * a.y_stride;
    if (is_q) {
        a.y[ys + r] = out;
        return;
    }
    const int rr = is_k ? r - a.q_dim : r - a.q_dim - a.kv_dim;
    if (!is_k && a.v_out) a.v_out[static_cast<long long>(s) * a.v_out_stride + rr] = v;
    const int kh = rr / hd, d = rr % hd;
    const int slot = pos % a.n_ctx;
    const long long e = static_cast<long long>(ring) * a.kv_sess_stride + a.kv_layer_off +
                        (static_cast<long long>(kh) * a.n_ctx + slot) * hd + d;
    void *cache = is_k ? a.k_cache : a.v_cache;
    if (a.kv_type == kKvF16) {
        static_cast<__half *>(cache)[e] = __float2half_rn(out);
    } else {
        const long long e0 = e - lane;
        warp_store_q4_0(out, lane, static_cast<uint8_t *>(cache) + e0 / 2,
                        reinterpret_cast<__half *>(is_k ? a.k_scale : a.v_scale) + e0 / 32);
    }
}

template <int EPI>
__device__ __forceinline__ void mma_row_epilogue(const BatchGemmArgs &a, int t, int lane, int s, float v) {
    const int r = t * kTileRows + lane;
    const long long ys = static_cast<long long>(s) * a.y_stride;
    if constexpr (EPI == kEpiStore) {
        if (r < a.W.rows) a.y[ys + r] = a.bias ? __fadd_rn(v, a.bias[r]) : v;
    } else if constexpr (EPI == kEpiResid) {
        if (r < a.W.rows) a.y[ys + r] = __fadd_rn(__ldcg(a.resid + static_cast<long long>(s) * a.resid_stride + r), v);
    } else if constexpr (EPI == kEpiSwiGLU) {
        const float up = __shfl_down_sync(0xffffffffu, v, 16);
        const int h = t * 16 + lane;
        if (lane < 16 && h < a.W.swiglu_f) {
            const float e = __double2float_rn(exp(-static_cast<double>(v)));
            a.y[ys + h] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, e)), up);
        }
    } else if constexpr (EPI == kEpiLogits) {
        float val = -INFINITY;
        if (r < a.W.rows) {
            val = a.bias ? __fadd_rn(v, a.bias[r]) : v;
            a.y[ys + r] = val;
        }
        float bv = (r < a.W.rows && r < a.argmax_limit) ? val : -INFINITY;
        int bi = r;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, ov, oi);
        }
        if (lane == 0) a.pairs[static_cast<long long>(s) * a.pairs_stride + t] = make_float2(bv, __int_as_float(bi));
    } else if constexpr (EPI == kEpiEmbAdd) {
        if (r < a.W.rows) {
            const int tok = a.tok[s];
            const bool ok = tok >= 0 && tok < a.emb.rows && a.emb.dim == a.W.rows;
            a.y[ys + r] = ok ? __fadd_rn(v, emb_elem(a.emb, tok, r)) : __fadd_rn(v, 0.0f);
        }
    } else if constexpr (EPI == kEpiQKV) {
        // the tile lies inside one head of q, k or v (head_dim % 32 == 0)
        const int hd = a.head_dim;
        float out = v;
        const bool is_q = r < a.q_dim;
        const bool is_k = !is_q && r < a.q_dim + a.kv_dim;
        if ((is_q || is_k) && a.rope) {
            const int d = (is_q ? r : r - a.q_dim) % hd;
            const float2 cs = a.rope[static_cast<long long>(s) * (hd / 2) + (d >> 1)];
            const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
            out = (lane & 1) ? __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(v, cs.x))
                             : __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(partner, cs.y));
        }
        if (is_q) {
            a.y[ys + r] = out;
            return;
        }
        const int rr = is_k ? r - a.q_dim : r - a.q_dim - a.kv_dim;
        if (!is_k && a.v_out) a.v_out[static_cast<long long>(s) * a.v_out_stride + rr] = v;
        const int kh = rr / hd, d = rr % hd;
        const int slot = a.pos[s * a.pos_stride] % a.n_ctx;
        const long long ring = a.ring_of ? a.ring_of[s] : s;
        const long long e = ring * a.kv_sess_stride + a.kv_layer_off + (static_cast<long long>(kh) * a.n_ctx + slot) * hd + d;
        void *cache = is_k ? a.k_cache : a.v_cache;
        if (a.kv_type == kKvF16) {
            static_cast<__half *>(cache)[e] = __float2half_rn(out);
        } else {
            const long long e0 = e - lane;
            warp_store_q4_0(out, lane, static_cast<uint8_t *>(cache) + e0 / 2,
                            reinterpret_cast<__half *>(is_k ? a.k_scale : a.v_scale) + e0 / 32);
        }
    }
}

// The kGrpSess sessions [kGrpSess h, kGrpSess (h + 1)) of tile t, one row per lane.  Every
// per-session operand (residual, token, position, ring, RoPE pair) is loaded
// for all 32 sessions before the first store, so the loads overlap instead of
// queueing behind stores they might alias.
template <int EPI>
__device__ __forceinline__ void mma_block_epilogue(const BatchGemmArgs &a, int t, int lane, int h,
                                                   const float2 (&v)[kGrpSess / 2]) {
    if (t >= a.W.n_tiles) return;
    const int r = t * kTileRows + lane;
    const int s0 = kGrpSess * h;
    const int ns = a.n_sess - s0;      // sessions of this warp (may exceed kGrpSess)
    float op[kGrpSess];                // per-session operand of this lane's row
    int tok = 0, pos = 0, ring = 0;    // lane i < kGrpSess: session s0 + i
    const int sl = s0 + lane;
    const bool mine = lane < kGrpSess && sl < a.n_sess;
    if constexpr (EPI == kEpiResid) {
#pragma unroll
        for (int j = 0; j < kGrpSess; ++j)
            op[j] = (j < ns && r < a.W.rows) ? __ldcg(a.resid + static_cast<long long>(s0 + j) * a.resid_stride + r) : 0.0f;
    } else if constexpr (EPI == kEpiEmbAdd) {
        tok = mine ? __ldcg(a.tok + sl) : -1;
#pragma unroll
        for (int j = 0; j < kGrpSess; ++j) {
            const int tj = __shfl_sync(0xffffffffu, tok, j);
            const bool ok = j < ns && r < a.W.rows && tj >= 0 && tj < a.emb.rows && a.emb.dim == a.W.rows;
            op[j] = ok ? emb_elem(a.emb, tj, r) : 0.0f;
        }
    }
    if constexpr (EPI == kEpiQKV) {
        if (mine) {
            pos = __ldcg(a.pos + sl * a.pos_stride);
            ring = a.ring_of ? __ldcg(a.ring_of + sl) : sl;
        }
        const bool rot = r < a.q_dim + a.kv_dim && a.rope;
        const int d = (r < a.q_dim ? r : r - a.q_dim) % a.head_dim;
        // eight sessions at a time: their RoPE pairs (cos, sin) of this row's frequency, then their stores
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float2 rp[kGrpSess / 2];
#pragma unroll
            for (int j = 0; j < kGrpSess / 2; ++j) {
                const int jj = hf * (kGrpSess / 2) + j;
                rp[j] = (rot && jj < ns) ? __ldcg(a.rope + static_cast<long long>(s0 + jj) * (a.head_dim / 2) + (d >> 1))
                                         : make_float2(1.0f, 0.0f);
            }
#pragma unroll
            for (int j = 0; j < kGrpSess / 2; ++j) {
                const int jj = hf * (kGrpSess / 2) + j;
                if (jj >= ns) continue;
                const float val = (jj & 1) ? v[jj >> 1].y : v[jj >> 1].x;
                mma_qkv_row(a, t, lane, s0 + jj, val, __shfl_sync(0xffffffffu, pos, jj), __shfl_sync(0xffffffffu, ring, jj),
                            rp[j]);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < kGrpSess / 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int jj = 2 * j + e, s = s0 + jj;
            if (s >= a.n_sess) continue;
            const float val = e ? v[j].y : v[j].x;
            if constexpr (EPI == kEpiResid) {
                if (r < a.W.rows) a.y[static_cast<long long>(s) * a.y_stride + r] = __fadd_rn(op[jj], val);
            } else if constexpr (EPI == kEpiEmbAdd) {
                if (r < a.W.rows) a.y[static_cast<long long>(s) * a.y_stride + r] = __fadd_rn(val, op[jj]);
            } else {
                mma_row_epilogue<EPI>(a, t, lane, s, val);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// fp32 -> fp64 times 2^-896, from the bit pattern alone: the sign stays in
// bit 63, the 8-bit exponent lands in the low bits of the 11-bit field and the
// mantissa at the top of the 52-bit field, so the double's value is exactly
// x * 2^(127 - 1023) for every finite x -- zero and subnormal floats included
// (a subnormal float becomes a subnormal double).  Sums of these scaled terms
// round exactly like the unscaled double sums: every fp32 value is a multiple
// of 2^-149, so scaled partial sums below the double normal range are multiples
// of 2^-1045 and add exactly, and above it double addition commutes with the
// power-of-two scale.  kUnscale restores the value before the fp32 rounding.
__device__ __forceinline__ double f2d_scaled(float x) {
    const int f = __float_as_int(x);
    const unsigned hi = static_cast<unsigned>(f >> 3) & 0x8FFFFFFFu;  // sign, then exponent and mantissa bits 30..3
    return __hiloint2double(static_cast<int>(hi), f << 29);
}
constexpr double kUnscale = 0x1p896;

// Terms of one 4-session register buffer r (r[2i] low-half sum, r[2i + 1]
// high-half sum of session i) into the accumulators of pairs [2k, 2k + 2).
template <bool EXACT>
__device__ __forceinline__ void mma_terms(const uint32_t (&r)[8], const float4 *sc4, const float2 *sc2, float d4,
                                          float2 (&S)[kGrpSess / 2], double (&D)[kGrpSess], int k) {
    const float2 d44 = make_float2(d4, d4);
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        const float4 p = sc4[2 * k + jj];   // d8, d8', -M d8, -M d8'
        const float2 m4 = sc2[2 * k + jj];  // -4 s8, -4 s8'
        const float2 d8 = make_float2(p.x, p.y), nm = make_float2(p.z, p.w);
        const int J = 2 * k + jj;
        if constexpr (EXACT) {
            // bits of 2^23 + 2^22 + sumi; the fma against -M d8 leaves fl(sumi d8)
            const float2 flo = make_float2(__int_as_float(static_cast<int>(r[4 * jj]) + 0x4B400000),
                                           __int_as_float(static_cast<int>(r[4 * jj + 2]) + 0x4B400000));
            const float2 fhi = make_float2(__int_as_float(static_cast<int>(r[4 * jj + 1]) + 0x4B400000),
                                           __int_as_float(static_cast<int>(r[4 * jj + 3]) + 0x4B400000));
            const float2 tl = __fmul2_rn(d44, __fadd2_rn(__ffma2_rn(flo, d8, nm), m4));
            const float2 th = __fmul2_rn(d44, __fadd2_rn(__ffma2_rn(fhi, d8, nm), m4));
            D[2 * J] += f2d_scaled(tl.x);
            D[2 * J + 1] += f2d_scaled(tl.y);
            D[2 * J] += f2d_scaled(th.x);
            D[2 * J + 1] += f2d_scaled(th.y);
        } else {
            const float2 f = make_float2(
                __int_as_float(static_cast<int>(r[4 * jj] + r[4 * jj + 1]) + 0x4B400000),
                __int_as_float(static_cast<int>(r[4 * jj + 2] + r[4 * jj + 3]) + 0x4B400000));
            const float2 u = __ffma2_rn(m4, make_float2(2.0f, 2.0f), __ffma2_rn(f, d8, nm));  // sumi d8 - 8 s8
            S[J] = __ffma2_rn(d44, u, S[J]);
        }
    }
}

template <int EPI, bool EXACT>
__global__ void __launch_bounds__(kMmaThreads, 1) batch_mma_kernel(const __grid_constant__ BatchGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    MmaSmem &S = *reinterpret_cast<MmaSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int cpt = a.W.cpt, ns = a.n_sess, P = batch_pad(ns);
    const int n_super = (a.W.n_tiles + kMmaTiles - 1) / kMmaTiles;
    const long long U = static_cast<long long>(n_super) * cpt;
    const long long u0 = unit_lo(U, G, c), u1 = unit_lo(U, G, c + 1);
    const int n_units = static_cast<int>(u1 - u0);
    const int groups = (ns + kGrpSess - 1) / kGrpSess;  // epilogue warpgroups (kGrpSess sessions a warp) with sessions
    volatile int *abort = &S.abort;

    if (tid == 0) {
        for (int i = 0; i < kMmaStages; ++i) {
            mbar_init(&S.raw_full[i], 1);
            mbar_init(&S.raw_empty[i], kUnpackWarps + 4 * groups + 1);
        }
        for (int i = 0; i < kMmaABufs; ++i) {
            mbar_init(&S.a_full[i], kUnpackWarps);
            mbar_init(&S.a_empty[i], 1);
        }
        for (int i = 0; i < kMmaSlots; ++i) {
            mbar_init(&S.tm_full[i], 1);
            mbar_init(&S.tm_empty[i], 4 * groups);
        }
        mbar_init(&S.mma_done, 1);
        S.abort = 0;
        S.last = 0;
        fence_barrier_init();
    }
    if (warp == kCtlWarp) {
        tmem_alloc(&S.tmem_base, kMmaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;

    if (warp >= kEpiWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtlRegs));
    if (warp == kCtlWarp) {
        // ---------------- bulk-copy producer (lane 0) ----------------
        int issued = 0;
        if (lane == 0) {
            const uint64_t pol_w = l2_evict_first_policy(), pol_x = l2_evict_last_policy();
            for (int g = 0; g < n_units; ++g) {
                const long long u = u0 + g;
                const int st = static_cast<int>(u / cpt), kc = static_cast<int>(u % cpt);
                const int sg = g % kMmaStages;
                if (g >= kMmaStages && !wait_ab(&S.raw_empty[sg], ((g / kMmaStages) + 1) & 1, abort)) break;
                uint8_t *dst = S.raw[sg];
                const int n_t = min(kMmaTiles, a.W.n_tiles - st * kMmaTiles);
                mbar_arrive_expect_tx(&S.raw_full[sg], static_cast<uint32_t>(n_t * kChunkBytes + P * 512 + P * 96));
                for (int q = 0; q < n_t; ++q)
                    bulk_load(dst + q * kChunkBytes,
                              a.W.tiles + (static_cast<size_t>(st * kMmaTiles + q) * cpt + kc) * kChunkBytes,
                              kChunkBytes, &S.raw_full[sg], pol_w);
                bulk_load(dst + kRawW, a.xq + static_cast<size_t>(kc) * 8 * P * 64, P * 512, &S.raw_full[sg], pol_x);
                bulk_load(dst + kRawW + kRawB, a.xds + static_cast<size_t>(kc) * 8 * P * 3, P * 96, &S.raw_full[sg],
                          pol_x);
                ++issued;
            }
            // copies in flight land before the CTA can exit (bounded)
            for (int g = max(0, issued - kMmaStages); g < issued; ++g)
                mbar_wait(&S.raw_full[g % kMmaStages], (g / kMmaStages) & 1);
        } else if (lane == 1) {
            // ---------------- MMA issuer (lane 1) ----------------
            const uint32_t idesc = idesc_i8(2 * P);
            for (int g = 0; g < n_units; ++g) {
                const int sg = g % kMmaStages, ab = g % kMmaABufs;
                if (!wait_ab(&S.a_full[ab], (g / kMmaABufs) & 1, abort)) break;
                tc_fence_after();
                bool ok = true;
                for (int b = 0; b < kChunkBlocks; ++b) {
                    const int gb = g * kChunkBlocks + b, slot = gb % kMmaSlots, use = gb / kMmaSlots;
                    if (use >= 1 && !wait_ab(&S.tm_empty[slot], (use + 1) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_i8(tmem + slot * kMmaSlotCols, kmajor_desc(S.a[ab] + b * kABlockBytes),
                           kmajor_desc(S.raw[sg] + kRawW + b * P * 64), idesc);
                    mma_commit(&S.tm_full[slot]);
                }
                if (!ok) break;
                mma_commit(&S.a_empty[ab]);
                mma_commit(&S.raw_empty[sg]);
            }
            // every MMA issued has completed before TMEM is freed (bounded)
            mma_commit(&S.mma_done);
            mbar_wait(&S.mma_done, 0);
        }
        __syncwarp();
    } else if (warp >= kEpiWarps && warp < kEpiWarps + kUnpackWarps) {
        // ---------------- unpack: Q4_0 nibbles -> K-major unsigned int8 ----------------
        const int ut = tid - kEpiWarps * 32;  // rows ut, ut + 32, ut + 64, ut + 96 of the 128-row block
        for (int g = 0; g < n_units; ++g) {
            const long long u = u0 + g;
            const int st = static_cast<int>(u / cpt);
            const int sg = g % kMmaStages, ab = g % kMmaABufs;
            bool ok = wait_ab(&S.raw_full[sg], (g / kMmaStages) & 1, abort);
            if (ok && g >= kMmaABufs) ok = wait_ab(&S.a_empty[ab], ((g / kMmaABufs) + 1) & 1, abort);
            if (!__all_sync(0xffffffffu, ok)) break;
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int m = ut + 32 * rr;
                const int q = m >> 5;
                const bool present = st * kMmaTiles + q < a.W.n_tiles;
                const uint8_t *src = S.raw[sg] + q * kChunkBytes + (m & 31) * 16;
                uint8_t *dst = S.a[ab] + (m >> 3) * 256 + (m & 7) * 16;
#pragma unroll
                for (int b = 0; b < kChunkBlocks; ++b) {
                    const uint4 w = present ? *reinterpret_cast<const uint4 *>(src + b * 512) : make_uint4(0, 0, 0, 0);
                    // byte j holds element j (low nibble) and element j + 16 (high nibble)
                    *reinterpret_cast<uint4 *>(dst + b * kABlockBytes) =
                        make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
                    *reinterpret_cast<uint4 *>(dst + b * kABlockBytes + 128) =
                        make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                   (w.w >> 4) & 0x0F0F0F0Fu);
                }
            }
            fence_proxy_async();  // generic-proxy writes -> the tensor core's reads
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&S.a_full[ab]);
                mbar_arrive(&S.raw_empty[sg]);
            }
        }
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kEpiRegs));
        // ---------------- epilogue warps ----------------
        const int q = warp & 3, h = warp >> 2;
        const bool active = h < groups;
        float2 Sacc[kGrpSess / 2];  // fast: fp32 sums of session pairs
        double Dacc[kGrpSess];      // exact: double sums of each session, scaled by 2^-896
#pragma unroll
        for (int j = 0; j < kGrpSess / 2; ++j) Sacc[j] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < kGrpSess; ++j) Dacc[j] = 0.0;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * q) << 16) + 2 * kGrpSess * h;
        uint32_t rA[8], rB[8];
        bool ok = true;
        for (int g = 0; active && g < n_units; ++g) {
            const long long u = u0 + g;
            const int st = static_cast<int>(u / cpt), kc = static_cast<int>(u % cpt);
            const int sg = g % kMmaStages;
            ok = wait_ab(&S.raw_full[sg], (g / kMmaStages) & 1, abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            const uint8_t *raw = S.raw[sg];
            const __half *d4p = reinterpret_cast<const __half *>(raw + q * kChunkBytes + kChunkQsBytes) + lane;
            for (int b = 0; b < kChunkBlocks; ++b) {
                const int gb = g * kChunkBlocks + b, slot = gb % kMmaSlots, use = gb / kMmaSlots;
                ok = wait_ab(&S.tm_full[slot], use & 1, abort);
                if (!__all_sync(0xffffffffu, ok)) break;
                tc_fence_after();
                // four reads of 4 sessions (8 columns); each read overlaps the previous one's arithmetic
                const uint32_t ta = lane_base + slot * kMmaSlotCols;
                tmem_ld8_nowait(ta, rA);
                const float d4 = __half2float(d4p[b * 32]);
                const uint8_t *scb = raw + kRawW + kRawB + b * P * 12;
                const float4 *sc4 = reinterpret_cast<const float4 *>(scb) + (kGrpSess / 2) * h;
                const float2 *sc2 = reinterpret_cast<const float2 *>(scb + P * 8) + (kGrpSess / 2) * h;
                tmem_wait_ld();
                tmem_ld8_nowait(ta + 8, rB);
                mma_terms<EXACT>(rA, sc4, sc2, d4, Sacc, Dacc, 0);
                tmem_wait_ld();
                tmem_ld8_nowait(ta + 16, rA);
                mma_terms<EXACT>(rB, sc4, sc2, d4, Sacc, Dacc, 1);
                tmem_wait_ld();
                tmem_ld8_nowait(ta + 24, rB);
                mma_terms<EXACT>(rA, sc4, sc2, d4, Sacc, Dacc, 2);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.tm_empty[slot]);  // every read of the slot has completed
                mma_terms<EXACT>(rB, sc4, sc2, d4, Sacc, Dacc, 3);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.raw_empty[sg]);
            const bool seg_end = kc == cpt - 1 || g == n_units - 1;
            if (!seg_end) continue;
            // ---- a 128-row block is complete in this CTA: epilogue or split combine ----
            const int t = st * kMmaTiles + q;
            const long long first = static_cast<long long>(st) * cpt, lastu = first + cpt - 1;
            if (first >= u0 && lastu < u1) {
                if constexpr (EXACT) {
#pragma unroll
                    for (int j = 0; j < kGrpSess / 2; ++j)
                        Sacc[j] = make_float2(__double2float_rn(Dacc[2 * j] * kUnscale),
                                           __double2float_rn(Dacc[2 * j + 1] * kUnscale));
                }
                mma_block_epilogue<EPI>(a, t, lane, h, Sacc);
            } else {
                const int cf = cta_of(first, U, G), cl = cta_of(lastu, U, G);
                const int n_c = cl - cf + 1;
                const size_t slab = static_cast<size_t>(P) * kMmaRows;  // one double (exact) or float per (session, row)
                double *part_d = reinterpret_cast<double *>(a.ws) + (static_cast<size_t>(st) * a.max_contrib + (c - cf)) * slab;
                float *part_f = reinterpret_cast<float *>(part_d);
                // the partial holds P sessions: padding sessions beyond P are not stored
#pragma unroll
                for (int j = 0; j < kGrpSess / 2; ++j) {
                    if (kGrpSess * h + 2 * j < P) {
                        const size_t i0 = static_cast<size_t>(kGrpSess * h + 2 * j) * kMmaRows + 32 * q + lane;
                        if constexpr (EXACT) {
                            part_d[i0] = Dacc[2 * j];
                            part_d[i0 + kMmaRows] = Dacc[2 * j + 1];
                        } else {
                            part_f[i0] = Sacc[j].x;
                            part_f[i0 + kMmaRows] = Sacc[j].y;
                        }
                    }
                }
                __threadfence();
                named_sync(1, 128 * groups);
                if (tid == 0) {
                    const int old = atomicAdd(&a.cnt[st], 1);
                    S.last = old == n_c - 1;
                    if (S.last) a.cnt[st] = 0;  // every contributor has counted: ready for the next launch
                    __threadfence();
                }
                named_sync(1, 128 * groups);
                if (S.last) {
                    // partials added in contributor order: the result does not depend on timing
                    const double *base = reinterpret_cast<const double *>(a.ws) + static_cast<size_t>(st) * a.max_contrib * slab;
                    // contributor by contributor, all of a contributor's loads in flight together
                    const int s0 = kGrpSess * h;
                    const size_t r0 = static_cast<size_t>(s0) * kMmaRows + 32 * q + lane;
#pragma unroll
                    for (int j = 0; j < kGrpSess; ++j) Dacc[j] = 0.0;
#pragma unroll
                    for (int j = 0; j < kGrpSess / 2; ++j) Sacc[j] = make_float2(0.0f, 0.0f);
                    for (int k = 0; k < n_c; ++k) {
                        const double *pk = base + k * slab + r0;
                        if constexpr (EXACT) {
                            double v[kGrpSess];
#pragma unroll
                            for (int j = 0; j < kGrpSess; ++j) v[j] = s0 + j < P ? __ldcg(pk + j * kMmaRows) : 0.0;
#pragma unroll
                            for (int j = 0; j < kGrpSess; ++j) Dacc[j] += v[j];
                        } else {
                            const float *pf = reinterpret_cast<const float *>(base + k * slab) + r0;
                            float v[kGrpSess];
#pragma unroll
                            for (int j = 0; j < kGrpSess; ++j) v[j] = s0 + j < P ? __ldcg(pf + j * kMmaRows) : 0.0f;
#pragma unroll
                            for (int j = 0; j < kGrpSess / 2; ++j)
                                Sacc[j] = make_float2(__fadd_rn(Sacc[j].x, v[2 * j]), __fadd_rn(Sacc[j].y, v[2 * j + 1]));
                        }
                    }
                    if constexpr (EXACT) {
#pragma unroll
                        for (int j = 0; j < kGrpSess / 2; ++j)
                            Sacc[j] = make_float2(__double2float_rn(Dacc[2 * j] * kUnscale),
                                           __double2float_rn(Dacc[2 * j + 1] * kUnscale));
                    }
                    mma_block_epilogue<EPI>(a, t, lane, h, Sacc);
                }
                named_sync(1, 128 * groups);  // S.last is reused by the next block
            }
#pragma unroll
            for (int j = 0; j < kGrpSess / 2; ++j) Sacc[j] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < kGrpSess; ++j) Dacc[j] = 0.0;
        }
        tc_fence_before();
    }

    __syncthreads();
    if (tid == 0 && S.abort) raise_error(a.status, kErrTmaTimeout);
    if (warp == kCtlWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kMmaTmemCols);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t batch_mma_smem_bytes() { return sizeof(MmaSmem); }

static long long host_unit_lo(long long U, int G, int c) { return U * c / G; }
static int host_cta_of(long long u, long long U, int G) { return static_cast<int>(((u + 1) * G + U - 1) / U) - 1; }

int batch_mma_grid(const QMatDesc &m, int sms) {
    const long long U = static_cast<long long>((m.n_tiles + kMmaTiles - 1) / kMmaTiles) * m.cpt;
    return static_cast<int>(U < sms ? U : sms);
}

int batch_mma_max_contrib(const QMatDesc &m, int sms) {
    const int n_super = (m.n_tiles + kMmaTiles - 1) / kMmaTiles;
    const long long U = static_cast<long long>(n_super) * m.cpt;
    const int G = batch_mma_grid(m, sms);
    int mx = 1;
    for (int st = 0; st < n_super; ++st) {
        const int n = host_cta_of(static_cast<long long>(st + 1) * m.cpt - 1, U, G) -
                      host_cta_of(static_cast<long long>(st) * m.cpt, U, G) + 1;
        mx = n > mx ? n : mx;
    }
    (void)host_unit_lo;
    return mx;
}

size_t batch_mma_ws_floats(const QMatDesc &m, int sms) {
    const int n_super = (m.n_tiles + kMmaTiles - 1) / kMmaTiles;
    return static_cast<size_t>(n_super) * batch_mma_max_contrib(m, sms) * 2 * kBatchMax * kMmaRows;
}

// Sets the shared-memory opt-in and checks that the compiled kernel launches
// with exactly the registers the setmaxnreg split is computed from (a launch
// with fewer would leave the epilogue warpgroups waiting for registers).
template <int EPI, bool EXACT>
static cudaError_t configure_mma_one() {
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, batch_mma_kernel<EPI, EXACT>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegs || fa.maxThreadsPerBlock < kMmaThreads) return cudaErrorInvalidDeviceFunction;
    return cudaFuncSetAttribute(batch_mma_kernel<EPI, EXACT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(MmaSmem)));
}

template <int EPI>
static cudaError_t configure_mma() {
    const cudaError_t e = configure_mma_one<EPI, true>();
    return e != cudaSuccess ? e : configure_mma_one<EPI, false>();
}

static std::atomic<unsigned long long> g_mma_configured{0};  // bit per device

cudaError_t configure_batch_mma() {
    const cudaError_t es[] = {configure_mma<kEpiStore>(), configure_mma<kEpiResid>(), configure_mma<kEpiSwiGLU>(),
                              configure_mma<kEpiQKV>(),   configure_mma<kEpiLogits>(), configure_mma<kEpiEmbAdd>()};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return e;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev < 64) g_mma_configured.fetch_or(1ull << dev);
    return cudaSuccess;
}

// The shared-memory opt-in of the kernels on the current device, set once.
static cudaError_t ensure_mma_configured() {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev < 64 && (g_mma_configured.load() & (1ull << dev))) return cudaSuccess;
    return configure_batch_mma();
}

template <int EPI>
static void launch_mma_t(const BatchGemmArgs &a, int G, bool exact, cudaStream_t s) {
    if (exact) batch_mma_kernel<EPI, true><<<G, kMmaThreads, sizeof(MmaSmem), s>>>(a);
    else batch_mma_kernel<EPI, false><<<G, kMmaThreads, sizeof(MmaSmem), s>>>(a);
}

cudaError_t launch_batch_mma(const BatchGemmArgs &a, int epi, int sms, bool exact, cudaStream_t s) {
    if (a.n_sess < 1 || a.n_sess > kBatchMax || a.W.cpt <= 0 || a.W.n_tiles <= 0 || sms <= 0)
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a.xq) & 15) || (reinterpret_cast<uintptr_t>(a.xds) & 15) ||
        (reinterpret_cast<uintptr_t>(a.W.tiles) & 15))
        return cudaErrorInvalidValue;
    const int G = batch_mma_grid(a.W, sms);
    if (batch_mma_max_contrib(a.W, sms) > 1 && (!a.ws || !a.cnt || a.max_contrib < batch_mma_max_contrib(a.W, sms)))
        return cudaErrorInvalidValue;
    if (epi == kEpiQKV && (a.head_dim % 32 || a.q_dim % 32 || a.kv_dim % 32)) return cudaErrorInvalidValue;
    const cudaError_t ce = ensure_mma_configured();
    if (ce != cudaSuccess) return ce;
    switch (epi) {
    case kEpiStore: launch_mma_t<kEpiStore>(a, G, exact, s); break;
    case kEpiResid: launch_mma_t<kEpiResid>(a, G, exact, s); break;
    case kEpiSwiGLU: launch_mma_t<kEpiSwiGLU>(a, G, exact, s); break;
    case kEpiQKV: launch_mma_t<kEpiQKV>(a, G, exact, s); break;
    case kEpiLogits: launch_mma_t<kEpiLogits>(a, G, exact, s); break;
    case kEpiEmbAdd: launch_mma_t<kEpiEmbAdd>(a, G, exact, s); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace bmo
