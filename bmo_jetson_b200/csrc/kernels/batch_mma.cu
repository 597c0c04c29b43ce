// batch_mma.cu -- the batched skinny GEMM Y[S][rows] = X[S][cols] . W^T on
// the 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Arithmetic (Q4_0 x Q8_1 per block b of 32 columns, row r, session s):
//     y[s][r] = sum_b d4[r][b] * (sumi[r][s][b] * d8[s][b] - 8 * s8[s][b])
// with sumi the integer dot of the row's 32 unsigned nibbles and the
// session's 32 int8 codes -- the reference's vec_dot_q4_0_q8_1 term
// (bmo_cuda_kernels.cu:560-683) taken over the whole block.  The tensor core
// computes every sumi exactly (kind::i8, unsigned nibbles x signed codes,
// int32 accumulators): one M=128 x N=P x K=32 MMA per block, each into its
// own TMEM slot.  The CUDA cores then apply the two per-block scales in fp32
// (sumi -> float exactly through the 2^23 + 2^22 bias, one fma with d8 and
// -8 s8, one fma with d4 into the running sum), two sessions per packed
// f32x2 instruction.  Unlike the batch-1 GEMV the block terms are rounded
// once each and summed in fp32, so results agree with the reference to fp32
// rounding (well inside the 1e-3 relative bar), not bit for bit.
//
// CTA (one per SM, 14 warps):
//   warp 12      bulk-copy producer: per 8-block chunk the four 32-row tiles'
//                Q4_0 chunks of a 128-row block (4 x 4608 B, HBM), the
//                sessions' Q8_1 codes (P x 256 B) and scales (P x 64 B, L2)
//   warps 8-11   unpack nibbles into the MMA's K-major int8 layout (A)
//   warp 13      TMEM owner and MMA issuer (one thread)
//   warps 0-7    read the int32 block sums from TMEM (warp w: TMEM lanes
//                32(w%4).., sessions 32(w/4)..), scale and accumulate, then
//                run the fused epilogue of layout.h's Epilogue per (row, session)
// Work is split stream-K: the (128-row block, chunk) units are cut evenly
// over the CTAs; a row block shared by several CTAs is combined by the last
// one to finish, summing the fp32 partials in contributor order (so the
// result does not depend on timing).  Every wait is bounded and any timeout
// makes all roles stop, drain the copies and MMAs in flight, free TMEM and
// raise the status word.
#include <atomic>

#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

constexpr int kMmaTiles = 4;                     // row tiles per 128-row block
constexpr int kMmaRows = kMmaTiles * kTileRows;  // MMA M
constexpr int kMmaStages = 4;
constexpr int kMmaABufs = 2;
constexpr int kMmaSlots = kChunkBlocks;          // one TMEM slot per block of a chunk
constexpr int kMmaSlotCols = 64;                 // >= P
constexpr int kMmaTmemCols = kMmaSlots * kMmaSlotCols;  // 512: all of TMEM
constexpr int kRawW = kMmaTiles * kChunkBytes;   // 18432
constexpr int kRawB = kBatchMax * 8 * 32;        // 16384
constexpr int kRawS = kBatchMax * 8 * 8;         // 4096
constexpr int kRawBytes = kRawW + kRawB + kRawS;
constexpr int kABlockBytes = kMmaRows * 32;      // one block of A: 128 rows x 32 int8
constexpr int kABytes = kChunkBlocks * kABlockBytes;
constexpr int kEpiWarps = 8, kUnpackWarps = 4, kProdWarp = 12, kMmaWarp = 13;
constexpr int kMmaThreads = 14 * 32;
static_assert(kRawBytes % 1024 == 0 && kABytes % 1024 == 0, "stage buffers stay 1 KB aligned");

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
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

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

// Bounded mbarrier wait that also gives up when another role has aborted.
__device__ __forceinline__ bool wait_ab(uint64_t *bar, uint32_t parity, volatile int *abort) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (i > 32) __nanosleep(64);
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

template <int EPI>
__device__ __forceinline__ void mma_block_epilogue(const BatchGemmArgs &a, int t, int lane, int h, const float2 (&v)[16]) {
    if (t >= a.W.n_tiles) return;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int s = 32 * h + 2 * j;
        if (s < a.n_sess) mma_row_epilogue<EPI>(a, t, lane, s, v[j].x);
        if (s + 1 < a.n_sess) mma_row_epilogue<EPI>(a, t, lane, s + 1, v[j].y);
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int EPI>
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
    const int halves = (ns + 31) / 32;  // epilogue warp groups with sessions
    volatile int *abort = &S.abort;

    if (tid == 0) {
        for (int i = 0; i < kMmaStages; ++i) {
            mbar_init(&S.raw_full[i], 1);
            mbar_init(&S.raw_empty[i], kUnpackWarps + 4 * halves + 1);
        }
        for (int i = 0; i < kMmaABufs; ++i) {
            mbar_init(&S.a_full[i], kUnpackWarps);
            mbar_init(&S.a_empty[i], 1);
        }
        for (int i = 0; i < kMmaSlots; ++i) {
            mbar_init(&S.tm_full[i], 1);
            mbar_init(&S.tm_empty[i], 4 * halves);
        }
        mbar_init(&S.mma_done, 1);
        S.abort = 0;
        S.last = 0;
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&S.tmem_base, kMmaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;

    if (warp == kProdWarp) {
        // ---------------- bulk-copy producer ----------------
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
                mbar_arrive_expect_tx(&S.raw_full[sg],
                                      static_cast<uint32_t>(n_t * kChunkBytes + P * 256 + P * 64));
                for (int q = 0; q < n_t; ++q)
                    bulk_load(dst + q * kChunkBytes,
                              a.W.tiles + (static_cast<size_t>(st * kMmaTiles + q) * cpt + kc) * kChunkBytes,
                              kChunkBytes, &S.raw_full[sg], pol_w);
                bulk_load(dst + kRawW, a.xq + static_cast<size_t>(kc) * 8 * P * 32, P * 256, &S.raw_full[sg], pol_x);
                bulk_load(dst + kRawW + kRawB, a.xds + static_cast<size_t>(kc) * 8 * P * 2, P * 64, &S.raw_full[sg],
                          pol_x);
                ++issued;
            }
            // copies in flight land before the CTA can exit (bounded)
            for (int g = max(0, issued - kMmaStages); g < issued; ++g)
                mbar_wait(&S.raw_full[g % kMmaStages], (g / kMmaStages) & 1);
        }
        __syncwarp();
    } else if (warp >= kEpiWarps && warp < kEpiWarps + kUnpackWarps) {
        // ---------------- unpack: Q4_0 nibbles -> K-major unsigned int8 ----------------
        const int m = tid - kEpiWarps * 32;  // row of the 128-row block
        const int q = m >> 5, rl = m & 31;
        for (int g = 0; g < n_units; ++g) {
            const long long u = u0 + g;
            const int st = static_cast<int>(u / cpt);
            const int sg = g % kMmaStages, ab = g % kMmaABufs;
            bool ok = wait_ab(&S.raw_full[sg], (g / kMmaStages) & 1, abort);
            if (ok && g >= kMmaABufs) ok = wait_ab(&S.a_empty[ab], ((g / kMmaABufs) + 1) & 1, abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            const bool present = st * kMmaTiles + q < a.W.n_tiles;
            const uint8_t *src = S.raw[sg] + q * kChunkBytes + rl * 16;
            uint8_t *dst = S.a[ab] + (m >> 3) * 256 + (m & 7) * 16;
#pragma unroll
            for (int b = 0; b < kChunkBlocks; ++b) {
                uint4 w = present ? *reinterpret_cast<const uint4 *>(src + b * 512) : make_uint4(0, 0, 0, 0);
                // byte j holds element j (low nibble) and element j + 16 (high nibble)
                const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
                const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                            (w.w >> 4) & 0x0F0F0F0Fu);
                *reinterpret_cast<uint4 *>(dst + b * kABlockBytes) = lo;
                *reinterpret_cast<uint4 *>(dst + b * kABlockBytes + 128) = hi;
            }
            fence_proxy_async();  // generic-proxy writes -> the tensor core's reads
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&S.a_full[ab]);
                mbar_arrive(&S.raw_empty[sg]);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(P);
            for (int g = 0; g < n_units; ++g) {
                const int sg = g % kMmaStages, ab = g % kMmaABufs;
                if (!wait_ab(&S.a_full[ab], (g / kMmaABufs) & 1, abort)) break;
                tc_fence_after();
                bool ok = true;
                for (int b = 0; b < kMmaSlots; ++b) {
                    if (g >= 1 && !wait_ab(&S.tm_empty[b], (g + 1) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_i8(tmem + b * kMmaSlotCols, kmajor_desc(S.a[ab] + b * kABlockBytes),
                           kmajor_desc(S.raw[sg] + kRawW + b * P * 32), idesc);
                    mma_commit(&S.tm_full[b]);
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
    } else {
        // ---------------- epilogue warps ----------------
        const int q = warp & 3, h = warp >> 2;
        const bool active = h < halves;
        float2 acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = make_float2(0.0f, 0.0f);
        const float2 bias2 = make_float2(-12582912.0f, -12582912.0f);
        for (int g = 0; active && g < n_units; ++g) {
            const long long u = u0 + g;
            const int st = static_cast<int>(u / cpt), kc = static_cast<int>(u % cpt);
            const int sg = g % kMmaStages;
            bool ok = wait_ab(&S.raw_full[sg], (g / kMmaStages) & 1, abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            const uint8_t *raw = S.raw[sg];
            const __half *d4p = reinterpret_cast<const __half *>(raw + q * kChunkBytes + kChunkQsBytes) + lane;
            for (int b = 0; b < kMmaSlots; ++b) {
                ok = wait_ab(&S.tm_full[b], g & 1, abort);
                if (!__all_sync(0xffffffffu, ok)) break;
                tc_fence_after();
                uint32_t r[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * kMmaSlotCols + 32 * h, r);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.tm_empty[b]);
                const float d4 = __half2float(d4p[b * 32]);
                const float2 d44 = make_float2(d4, d4);
                const float4 *sc = reinterpret_cast<const float4 *>(raw + kRawW + kRawB + b * P * 8) + 16 * h;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float4 p = sc[j];  // (d8, d8', -8 s8, -8 s8') of sessions 32h+2j, +1
                    // int32 -> float exactly: bits of 2^23 + 2^22 + sumi, minus the bias
                    float2 f = make_float2(__int_as_float(static_cast<int>(r[2 * j]) + 0x4B400000),
                                           __int_as_float(static_cast<int>(r[2 * j + 1]) + 0x4B400000));
                    f = __fadd2_rn(f, bias2);
                    const float2 t = __ffma2_rn(f, make_float2(p.x, p.y), make_float2(p.z, p.w));
                    acc[j] = __ffma2_rn(d44, t, acc[j]);
                }
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
                mma_block_epilogue<EPI>(a, t, lane, h, acc);
            } else {
                const int cf = cta_of(first, U, G), cl = cta_of(lastu, U, G);
                const int n_c = cl - cf + 1;
                const size_t slab = static_cast<size_t>(P) * kMmaRows;
                float *part = a.ws + (static_cast<size_t>(st) * a.max_contrib + (c - cf)) * slab;
                // the slab holds P sessions: rows of padding sessions beyond P are not stored
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (32 * h + 2 * j < P) {
                        part[(32 * h + 2 * j) * kMmaRows + 32 * q + lane] = acc[j].x;
                        part[(32 * h + 2 * j + 1) * kMmaRows + 32 * q + lane] = acc[j].y;
                    }
                }
                __threadfence();
                named_sync(1, 128 * halves);
                if (tid == 0) {
                    const int old = atomicAdd(&a.cnt[st], 1);
                    S.last = old == n_c - 1;
                    if (S.last) a.cnt[st] = 0;  // every contributor has counted: ready for the next launch
                    __threadfence();
                }
                named_sync(1, 128 * halves);
                if (S.last) {
                    float2 tot[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) tot[j] = make_float2(0.0f, 0.0f);
                    const float *base = a.ws + static_cast<size_t>(st) * a.max_contrib * slab;
                    for (int k = 0; k < n_c; ++k) {
                        const float *pk = base + k * slab;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (32 * h + 2 * j < P) {
                                tot[j].x = __fadd_rn(tot[j].x, __ldcg(pk + (32 * h + 2 * j) * kMmaRows + 32 * q + lane));
                                tot[j].y = __fadd_rn(tot[j].y, __ldcg(pk + (32 * h + 2 * j + 1) * kMmaRows + 32 * q + lane));
                            }
                        }
                    }
                    mma_block_epilogue<EPI>(a, t, lane, h, tot);
                }
                named_sync(1, 128 * halves);  // S.last is reused by the next block
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = make_float2(0.0f, 0.0f);
        }
        tc_fence_before();
    }

    __syncthreads();
    if (tid == 0 && S.abort) raise_error(a.status, kErrTmaTimeout);
    if (warp == kMmaWarp) {
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
    return static_cast<size_t>(n_super) * batch_mma_max_contrib(m, sms) * kBatchMax * kMmaRows;
}

template <int EPI>
static cudaError_t configure_mma() {
    return cudaFuncSetAttribute(batch_mma_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(MmaSmem)));
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

cudaError_t launch_batch_mma(const BatchGemmArgs &a, int epi, int sms, cudaStream_t s) {
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
    const size_t smem = sizeof(MmaSmem);
    switch (epi) {
    case kEpiStore: batch_mma_kernel<kEpiStore><<<G, kMmaThreads, smem, s>>>(a); break;
    case kEpiResid: batch_mma_kernel<kEpiResid><<<G, kMmaThreads, smem, s>>>(a); break;
    case kEpiSwiGLU: batch_mma_kernel<kEpiSwiGLU><<<G, kMmaThreads, smem, s>>>(a); break;
    case kEpiQKV: batch_mma_kernel<kEpiQKV><<<G, kMmaThreads, smem, s>>>(a); break;
    case kEpiLogits: batch_mma_kernel<kEpiLogits><<<G, kMmaThreads, smem, s>>>(a); break;
    case kEpiEmbAdd: batch_mma_kernel<kEpiEmbAdd><<<G, kMmaThreads, smem, s>>>(a); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace bmo
