// gemv_ref.cu -- batch-1 Q4_0 x Q8_1 GEMV computing every output row with
// the reference kernel's own fp32 operations in the reference's own order,
// so that its results are bit-identical to bmo_gemv_q4_0_q8_1_kernel
// (src/bmo_cuda_kernels.cu:560-683) on the same weights and activation.
//
// The reference's order.  A warp owns a row; lane l takes half block
// h = l % 2 of the blocks whose index within each group of 16 is m = l / 2.
// Its accumulator j (0..3) chains, in increasing order, the blocks
// 64 i + 16 j + m of the main loop; blocks past the last whole group of 64
// (the tail, in steps of 16) continue accumulator 0.  Each block adds
// acc = fma(d4, fma((float)sumi, d8, -4 s8), acc).  The lane's value is
// ((acc0 + acc1) + acc2) + acc3 and the row is the __shfl_down_sync tree of
// the 32 lane values.  So one row is 128 independent fp32 chains ("keys":
// block position within 64 x half block) joined by a fixed tree.
//
// B200 design.  The weights keep the engine's tiled layout (32 rows x
// 8-block chunks, one 4608-byte bulk copy each).  A chunk's 8 blocks share
// one key group G = 2 j + m / 8: main chunk c (tile-local) has G = c % 8 and
// chain position c / 8; tail chunk c = nm + t has G = t % 2 (j = 0) and
// position nm / 8 + t / 2.  So warp w of a CTA owns key group w of every
// tile of the CTA, streams exactly that group's chunks in chain order
// through a private TMA ring, and keeps the 16 chains of each row (8 blocks
// x 2 half blocks) in registers -- no chain ever crosses a warp.  After a
// tile, each warp leaves its 16 chain values per row in shared memory and a
// combiner warp (rotating with the tile) adds them in the reference's lane
// order, runs the 32-leaf tree in registers (lane = row) and applies the
// fused epilogue.  Named barriers hand the shared buffer over: the combiner
// waits until all warps have written ("full"); the writers of the next tile
// wait until the combiner has read ("empty"), which it signals before its
// tree and epilogue; each tile parity has its own pair.  Each CTA owns whole tiles (the chains must
// not be split), two CTAs per SM (registers <= 128, shared memory < half an
// SM; see gemv_ref_grid).
//
// The prologue is the RMSNorm of rmsnorm_kernel (:244-295) in its own order
// -- thread t of 256 sums x[t + 256 k]^2 with fma, a shfl_down tree per warp,
// the 8 warp sums by the tree ((w0+w4)+(w2+w6))+((w1+w5)+(w3+w7)), scale =
// rsqrtf(total / n + eps), y = (x * scale) * gamma -- then the Q8_1
// quantiser of :529-558, bit-exact, spread over all warps (element per lane,
// block statistics per lane).
#include <algorithm>

#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRing = 2;                  // chunks in flight per warp
constexpr int kMaxNbx = 384;              // activations up to 12288 elements
constexpr int kMaxNormCols = 4096;        // RMSNorm weight staged in the chain buffer's space
// Named barrier ids (0 is __syncthreads), one pair per tile parity: tile t
// hands over through FULL[t % 2] and EMPTY[t % 2].  With one pair, the
// combiner of tile t (which arrives at EMPTY without waiting and skips the
// next tile's EMPTY wait) could reach EMPTY again while a warp two tiles
// behind had not yet completed the earlier instance, and be counted into it.
// With the parity split the next use of an id cannot start before its
// previous instance completed (every path to it passes the other parity's
// barrier, which completes only after this one).
constexpr int kBarFull0 = 1, kBarEmpty0 = 3;
// Ring chunks each warp issues before griddepcontrol.wait; the rest of the
// ring is issued after the prologue.  Measured on B200 (frames/s of the
// decode frame, same box, alternating runs): 1 chunk 328-335, 2 chunks
// 317-325, none 316 -- with the whole ring in flight the activation load of
// the prologue queues behind the weight copies, with none the weight stream
// starts late.  A look-ahead of 3 or 6 more chunks into L2
// (cp.async.bulk.prefetch.L2) measured 308-310.
#ifndef BMO_GEMV_REF_PRE_WAIT
#define BMO_GEMV_REF_PRE_WAIT 1
#endif
// The prologue uses each warp's second ring slot as scratch (32 padded
// blocks of 33 floats and their 32 reciprocal scales).
static_assert(kRing == 2 && BMO_GEMV_REF_PRE_WAIT == 1, "ring slot 1 is the prologue's scratch");
static_assert((32 * 33 + 32) * 4 <= kChunkBytes, "prologue scratch fits one ring slot");

struct GemvRefSmem {
    uint64_t bar[kWarps][kRing];
    uint64_t gbar;  // RMSNorm weight bulk copy
    alignas(128) uint8_t ring[kWarps][kRing][kChunkBytes];
    alignas(16) int8_t xq[kMaxNbx * 32];
    float2 xds[kMaxNbx];  // (d8, 4 * s8) of each Q8_1 block
    union {
        float part[kWarps][2 * kChunkBlocks][32];  // [key group][block * 2 + half][row]: one tile's chains
        float gamma[kMaxNormCols];                 // prologue only
    };
    float red[kWarps];
    float tok_v[kWarps];
    int tok_i[kWarps];
    int err;
};

}  // namespace

template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_ref_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    GemvRefSmem &S = *reinterpret_cast<GemvRefSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int cpt = a.W.cpt;
    const int t0 = static_cast<int>(static_cast<long long>(a.W.n_tiles) * c / G);
    const int t1 = static_cast<int>(static_cast<long long>(a.W.n_tiles) * (c + 1) / G);
    const int nb = a.W.cols / 32, nbx = a.W.nbx;
    const KeyChains kc = KeyChains::of(nb, cpt);
    const int my_len = kc.len(warp);
    const int n_mine = my_len * (t1 - t0);
    const bool gbulk = PRO == kProNorm && (reinterpret_cast<uintptr_t>(a.gamma) & 15) == 0;

    if (tid < kWarps * kRing) mbar_init(&S.bar[tid / kRing][tid % kRing], 1);
    if (tid == kWarps * kRing) mbar_init(&S.gbar, 1);
    if (tid == 0) S.err = 0;
    fence_barrier_init();
    __syncthreads();

    // Weights never depend on earlier kernels: start streaming them now.
    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](int i) {
        const int tile = t0 + i / my_len;
        const long long k = static_cast<long long>(tile) * cpt + kc.chunk(warp, i % my_len);
        uint64_t *bar = &S.bar[warp][i % kRing];
        mbar_arrive_expect_tx(bar, kChunkBytes);
        bulk_load(S.ring[warp][i % kRing], a.W.tiles + k * kChunkBytes, kChunkBytes, bar, pol);
    };
    if (lane == 0)
        for (int i = 0; i < BMO_GEMV_REF_PRE_WAIT && i < n_mine; ++i) issue(i);
    if (gbulk && tid == 0) {
        const uint32_t gb = static_cast<uint32_t>(a.W.cols) * 4u;
        mbar_arrive_expect_tx(&S.gbar, gb);
        bulk_load(S.gamma, a.gamma, gb, &S.gbar, l2_evict_last_policy());
    }

    pdl_wait();

    // ---- prologue: activation -> Q8_1 blocks in shared memory ----
    // Warp w takes blocks w + 8 m, one element per lane, in rounds of up to
    // 32 blocks staged by cp.async into its padded scratch (its second ring
    // slot, refilled with weights only after the prologue).  Thread t thus
    // holds x[t + 256 m]: exactly its share of the reference RMSNorm's sum of
    // squares (an RMSNorm input has at most 4096 elements: one round).  Lane
    // m then takes the amax, d, 1/d and the in-order sum of block m (the
    // operations of quant_block_q8_1), and every lane quantises its element
    // of each block.  Measured on B200 against one thread per block (its
    // 32-element loops serial): 348 vs 327 frames/s, temporal 1.76 vs 1.94 ms.
    // A fully unrolled register version of the same arithmetic measured slower
    // (313 frames/s): short kernels pay for their code size, since the code
    // after griddepcontrol.wait is fetched cold on every SM.
    int tok = -1;
    if constexpr (EPI == kEpiEmbAdd) {
        tok = resolve_token<kThreads>(a.tok, S.tok_v, S.tok_i, [] { __syncthreads(); });
        if (c == 0 && tid == 0 && a.tok.tok_out) *a.tok.tok_out = tok;
    }
    const int nbw = nb > warp ? (nb - warp + kWarps - 1) / kWarps : 0;  // blocks of this warp
    float *scr = reinterpret_cast<float *>(S.ring[warp][1]);
    float *sid = scr + 32 * 33;  // 1/d of the round's blocks
    const float *gam = a.gamma;
    float scale = 1.0f;
    for (int m0 = 0; m0 < nbw || (PRO == kProNorm && m0 == 0); m0 += 32) {
        const int nr = nbw - m0 < 32 ? nbw - m0 : 32;  // blocks in this round
#pragma unroll 4
        for (int mm = 0; mm < nr; ++mm)
            cp_async4(scr + mm * 33 + lane, a.x + (warp + kWarps * (m0 + mm)) * 32 + lane);
        cp_async_wait_all();
        if constexpr (PRO == kProNorm) {  // (m0 == 0, the only round)
            float ss = 0.0f;
            for (int mm = 0; mm < nr; ++mm) {
                const float xv = scr[mm * 33 + lane];
                ss = __fmaf_rn(xv, xv, ss);
            }
            ss = shfl_down_tree(ss);
            if (lane == 0) S.red[warp] = ss;
            __syncthreads();
            const float total = __fadd_rn(__fadd_rn(__fadd_rn(S.red[0], S.red[4]), __fadd_rn(S.red[2], S.red[6])),
                                          __fadd_rn(__fadd_rn(S.red[1], S.red[5]), __fadd_rn(S.red[3], S.red[7])));
            scale = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(a.W.cols)), a.eps));
            if (gbulk) {
                if (!mbar_wait(&S.gbar, 0)) atomicOr(&S.err, 1);
                gam = S.gamma;
            }
#pragma unroll 4
            for (int mm = 0; mm < nr; ++mm) {
                float *e = scr + mm * 33 + lane;
                *e = __fmul_rn(__fmul_rn(*e, scale), gam[(warp + kWarps * mm) * 32 + lane]);
            }
        }
        if (c == 0 && a.xn_out)
#pragma unroll 4
            for (int mm = 0; mm < nr; ++mm) a.xn_out[(warp + kWarps * (m0 + mm)) * 32 + lane] = scr[mm * 33 + lane];
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
            const float id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;
            const __half2 ds = __halves2half2(__float2half_rn(d), __float2half_rn(sum));
            const int b = warp + kWarps * (m0 + lane);
            S.xds[b] = make_float2(__low2float(ds), 4.0f * __high2float(ds));
            if (c == 0 && a.q8_out) *reinterpret_cast<__half2 *>(a.q8_out + static_cast<size_t>(b) * 36) = ds;
            sid[lane] = id;
        }
        __syncwarp();
        const bool q8o = c == 0 && a.q8_out;
#pragma unroll 4
        for (int mm = 0; mm < nr; ++mm) {
            int qi = __float2int_rz(roundf(__fmul_rn(scr[mm * 33 + lane], sid[mm])));
            qi = max(-128, min(127, qi));
            const int b = warp + kWarps * (m0 + mm);
            S.xq[b * 32 + lane] = static_cast<int8_t>(qi);
            if (q8o) a.q8_out[static_cast<size_t>(b) * 36 + 4 + lane] = static_cast<uint8_t>(qi);
        }
        __syncwarp();
    }
    for (int b = nb + warp; b < nbx; b += kWarps) {  // padding blocks
        S.xq[b * 32 + lane] = 0;
        if (lane == 0) S.xds[b] = make_float2(0.0f, 0.0f);
    }
    __syncthreads();  // also ends the prologue's use of S.gamma, which S.part overlays
    if (lane == 0) {  // the rest of the ring (slot 1 held the prologue's scratch)
        fence_proxy_async();
        for (int i = BMO_GEMV_REF_PRE_WAIT; i < kRing && i < n_mine; ++i) issue(i);
    }

    // ---- main loop: each tile's key-group chains, then the combine ----
    int i = 0;           // chunks of this warp passed through
    int issued = n_mine < kRing ? n_mine : kRing;
    int first_bad = n_mine;  // first chunk whose wait gave up
    bool bad = false;
    for (int tt = 0; tt < t1 - t0; ++tt) {
        float acc[kChunkBlocks][2];
#pragma unroll
        for (int b = 0; b < kChunkBlocks; ++b) acc[b][0] = acc[b][1] = 0.0f;
        for (int p = 0; p < my_len; ++p, ++i) {
            if (!bad && !mbar_wait(&S.bar[warp][i % kRing], (i / kRing) & 1)) {
                bad = true;
                first_bad = i;
                if (lane == 0) atomicOr(&S.err, 1);
            }
            if (!bad) {
                const int ch = kc.chunk(warp, p);
                chunk_acc_ref(S.ring[warp][i % kRing], S.xq + ch * kChunkBlocks * 32, S.xds + ch * kChunkBlocks,
                              lane, acc);
            }
            __syncwarp();
            if (!bad && i + kRing < n_mine) {
                if (lane == 0) {
                    fence_proxy_async();
                    issue(i + kRing);
                }
                ++issued;
            }
        }
        // hand the tile's chains to the combiner warp
        const int comb = tt % kWarps;
        const int bar_full = kBarFull0 + (tt & 1), bar_empty = kBarEmpty0 + (tt & 1);
        if (tt > 0 && warp != (tt - 1) % kWarps) named_sync(kBarEmpty0 + ((tt - 1) & 1), kThreads);
#pragma unroll
        for (int b = 0; b < kChunkBlocks; ++b) {
            S.part[warp][2 * b][lane] = acc[b][0];
            S.part[warp][2 * b + 1][lane] = acc[b][1];
        }
        if (warp != comb) {
            named_arrive(bar_full, kThreads);
            continue;
        }
        named_sync(bar_full, kThreads);
        // lane value L[2m + h] = ((A0 + A1) + A2) + A3, A_j from key group 2j + m/8
        float L[32];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int kk = 2 * (m & 7) + h, mh = m >> 3;
                float s = __fadd_rn(S.part[mh][kk][lane], S.part[2 + mh][kk][lane]);
                s = __fadd_rn(s, S.part[4 + mh][kk][lane]);
                L[2 * m + h] = __fadd_rn(s, S.part[6 + mh][kk][lane]);
            }
        }
        if (tt + 1 < t1 - t0) named_arrive(bar_empty, kThreads);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int q = 0; q < o; ++q) L[q] = __fadd_rn(L[q], L[q + o]);
        if (!bad && !S.err) tile_epilogue<EPI, true>(a, t0 + tt, lane, L[0], tok, a.rope_cs);
    }
    // The next kernel may start: its weight prefetch overlaps this kernel's tail.
    // Triggering earlier (after the prologue, or at entry) let the next
    // kernel's CTAs compete with this one's weight stream: 317 and 297
    // frames/s against 328-335 here.
    pdl_launch_dependents();
    if (bad) {  // let this warp's copies in flight land before the CTA exits
        for (int j = first_bad; j < issued; ++j) mbar_wait(&S.bar[warp][j % kRing], (j / kRing) & 1);
    }
    __syncthreads();
    if (S.err && tid == 0) raise_error(a.status, kErrTmaTimeout);
}

// ---------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------
cudaError_t configure_gemv_ref();

// Shared memory a launch asks for: a grid no larger than the SM count asks
// for more than half an SM, so that no SM holds two of its CTAs (the
// scheduler otherwise packed pairs onto SMs its predecessor had left while
// others stayed idle: 383 vs 376 frames/s on B200); larger grids run two per
// SM (gemv_ref_grid).
constexpr size_t kSpreadSmemBytes = 118 * 1024;
static_assert(sizeof(GemvRefSmem) <= kSpreadSmemBytes, "the spread request covers the kernel's layout");

template <int PRO, int EPI>
static cudaError_t launch_ref_t(const GemvArgs &a, int grid, cudaStream_t s, bool pdl) {
    // The shared-memory opt-in is per device; the first launch on a device
    // sets it and records the device's SM count.
    static unsigned long long configured = 0;
    static int sm_count[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(configured & (1ull << dev))) {
        cudaError_t e = configure_gemv_ref();
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        configured |= 1ull << dev;
    }
    const bool spread = dev < 64 && grid <= sm_count[dev];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = spread ? kSpreadSmemBytes : sizeof(GemvRefSmem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_ref_kernel<PRO, EPI>, a);
}

#define BMO_GEMV_REF_VARIANTS(X) \
    X(kProNorm, kEpiQKV)         \
    X(kProPlain, kEpiResid)      \
    X(kProNorm, kEpiSwiGLU)      \
    X(kProNorm, kEpiLogits)      \
    X(kProPlain, kEpiLogits)     \
    X(kProPlain, kEpiEmbAdd)     \
    X(kProPlain, kEpiStore)      \
    X(kProNorm, kEpiStore)       \
    X(kProPlain, kEpiSwiGLU)     \
    X(kProNorm, kEpiResid)

cudaError_t configure_gemv_ref() {
    cudaError_t e = cudaSuccess;
#define BMO_GEMV_REF_CFG(P, E)                                                                              \
    if ((e = cudaFuncSetAttribute(gemv_ref_kernel<P, E>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                  static_cast<int>(kSpreadSmemBytes))) != cudaSuccess)                      \
        return e;
    BMO_GEMV_REF_VARIANTS(BMO_GEMV_REF_CFG)
#undef BMO_GEMV_REF_CFG
    return e;
}

size_t gemv_ref_smem_bytes() { return sizeof(GemvRefSmem); }
int gemv_ref_max_norm_cols() { return kMaxNormCols; }

// Two CTAs per SM (the shared-memory footprint allows two): with one per SM,
// programmatic dependent launch let the scheduler pack two CTAs of a kernel
// onto the SMs its predecessor had left (up to 34 of 148 SMs doubled, the
// rest idle) and the doubled SMs set the kernel's time.  Launching two per SM
// keeps the pairing even and doubles the bytes in flight per SM: 377 vs 351
// frames/s on B200 (one CTA per SM enforced by shared memory: 361).
int gemv_ref_grid(const QMatDesc &m, int sms) { return std::max(1, std::min(m.n_tiles, 2 * sms)); }

cudaError_t launch_gemv_ref(const GemvArgs &a, int prologue, int epilogue, int grid, cudaStream_t s, bool pdl) {
    if (a.W.nbx > kMaxNbx || grid <= 0 || grid > a.W.n_tiles || a.W.cpt <= 0 || a.W.n_tiles <= 0 ||
        a.W.cols % 32 || a.W.nbx != a.W.cpt * kChunkBlocks || a.W.nbx < a.W.cols / 32)
        return cudaErrorInvalidValue;
    if (prologue == kProNorm && a.W.cols > kMaxNormCols) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(a.x) & 15) return cudaErrorInvalidValue;
#define BMO_GEMV_REF_CASE(P, E) \
    if (prologue == P && epilogue == E) return launch_ref_t<P, E>(a, grid, s, pdl);
    BMO_GEMV_REF_VARIANTS(BMO_GEMV_REF_CASE)
#undef BMO_GEMV_REF_CASE
    return cudaErrorInvalidValue;
}

}  // namespace bmo
