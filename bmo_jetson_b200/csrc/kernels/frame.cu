// frame.cu -- the persistent decode-frame kernel for sm_100a.
//
// One cooperative launch runs a program of FramePhase steps (a frame's
// temporal layers and text head, and/or the depformer cascade) with one CTA
// of 8 warps per SM and no kernel boundaries between the steps.
//
// Streaming: every byte a CTA reads from HBM -- its row tiles of each weight
// matrix, and for attention steps the K/V ring rows of the heads it owns -- is
// cut into 4.6 KB units.  Warp w consumes units w, w + 8, ... of each step and
// keeps its own next kFwSlots units in flight through the TMA bulk-copy
// engine into a private shared-memory ring: after consuming a unit it issues
// the unit kFwSlots ahead in its sequence, walking into later steps of the
// program as needed.  So HBM keeps streaming while the warps wait at a grid
// barrier or run a prologue, and eight warps issue copies (one issuing thread
// per SM cannot keep HBM busy).
//
// Steps are separated by a grid-wide barrier: a monotone counter in global
// memory, zero at launch.  Every wait is bounded; a wait that gives up raises
// the status word and sets an abort flag that ends all other waits early, and
// each warp lets its copies in flight land before it exits.
//
// The arithmetic is that of the per-op kernels -- the GEMV pieces are shared
// (gemv_dev.cuh) and the attention follows attention.cu's exact-reduction
// semantics -- so both paths agree with the CPU oracle.  Data written by
// other CTAs during the launch is read with L2-only loads.
#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

constexpr int kFwWarps = 8;
constexpr int kFwThreads = kFwWarps * 32;
constexpr int kFwSlots = 5;                     // units in flight per warp (40 per SM, 184 KB)
constexpr int kFwMaxNbx = 384;                  // activations up to 12288 elements
constexpr int kFwMaxTiles = 10;                 // row tiles per CTA per matrix
constexpr int kFwMaxWindow = kFwMaxTiles * kFwWarps * 32 * 2;  // attention scores share `part`'s space
constexpr int kFwMaxHd = 128;
constexpr int kFwDepMaxWin = 8;                 // kProDepAttn keeps the window in registers
constexpr int kFwDepHd = 64;                    // kProDepAttn head size
constexpr uint32_t kGridPolls = 1u << 22;       // grid-barrier polls before giving up (~1 s)

// Warp w's position in its unit sequence: units w, w + 8, ... of every step,
// in program order, with the current step's copy parameters decoded once
// when the cursor enters it (no descriptor loads per unit).  Kept in shared
// memory and advanced by the warp's lane 0.
struct WarpStream {
    int p, u, n;            // next unit to issue: step, index in the step, units of that step
    uint32_t issued, consumed;
    uint64_t pol;
    // GEMV step: unit u is kChunkBytes at base + u * kChunkBytes
    const uint8_t *base;
    // attention step: units [2 uk h', 2 uk h' + uk) are K rows, then V rows, of owned head h0 + h'
    const uint8_t *kplane, *vplane;  // this layer's K / V ring planes
    int rb, rpu, uk, h0, group, n_ctx, start, n_old;
    bool attn;
};

struct FrameSmem {
    WarpStream ws[kFwWarps];
    uint64_t full[kFwWarps][kFwSlots];
    alignas(128) uint8_t ring[kFwWarps][kFwSlots][kChunkBytes];
    union {
        struct {
            alignas(16) int8_t xq[kFwMaxNbx * 32];
            float2 xds[kFwMaxNbx];
        } g;  // GEMV activation (Q8_1)
        struct {
            double ow[kFwWarps][kFwMaxHd];
            float q[kFwMaxHd];
            alignas(16) __half knew[kFwMaxHd];
            alignas(16) __half vnew[kFwMaxHd];
        } at;  // attention
    } u;
    union {
        alignas(16) double part[kFwMaxTiles][kFwWarps][32];  // GEMV per-warp tile sums
        float s[kFwMaxWindow];                               // attention scores / probabilities; kProDepAttn output
    } w;
    float2 rope[kFwMaxHd / 2];
    double red[kFwWarps];
    float tok_v[kFwWarps];
    int tok_i[kFwWarps];
    float wmax[kFwWarps];
    double lsum;
    int ok;
};

size_t frame_smem_bytes() { return sizeof(FrameSmem); }
int frame_max_window() { return kFwMaxWindow; }
int frame_max_tiles_per_cta() { return kFwMaxTiles; }
int frame_dep_max_window() { return kFwDepMaxWin; }
int frame_dep_head_dim() { return kFwDepHd; }

__device__ __forceinline__ void csync() { named_sync(1, kFwThreads); }

__device__ __forceinline__ void tile_range(int n_tiles, int c, int G, int &t0, int &t1) {
    t0 = static_cast<int>(static_cast<long long>(n_tiles) * c / G);
    t1 = static_cast<int>(static_cast<long long>(n_tiles) * (c + 1) / G);
}

// Heads of an attention step owned by CTA c: h with floor(h * G / n) == c, the
// range [ceil(c n / G), ceil((c + 1) n / G)).
__device__ __forceinline__ void head_range(int n_heads, int c, int G, int &h0, int &h1) {
    h0 = static_cast<int>((static_cast<long long>(c) * n_heads + G - 1) / G);
    h1 = static_cast<int>((static_cast<long long>(c + 1) * n_heads + G - 1) / G);
}

struct Window {
    int pos, window, start, n_old;
};

__device__ __forceinline__ Window attn_window(const AttnArgs &at) {
    Window w;
    w.pos = *at.pos;
    const int total = w.pos + 1;
    w.window = total > at.n_ctx ? at.n_ctx : total;
    w.start = total - w.window;
    w.n_old = w.window - 1;  // the newest row is this frame's, read after the barrier
    return w;
}

// K (or V) units per owned head of an attention step: rows of the window
// except the newest, kChunkBytes / (2 * head_dim) rows per unit.
__device__ __forceinline__ int attn_units_per_head(const FramePhase &ph, const Window &w) {
    if (w.window <= 1) return 0;
    const int rpu = kChunkBytes / (ph.head_dim * 2);
    return (w.n_old + rpu - 1) / rpu;
}

// Units a step gives this CTA.
__device__ int phase_units(const FramePhase &ph, int c, int G) {
    if (ph.kind == kPhGemv) {
        int t0, t1;
        tile_range(ph.g.W.n_tiles, c, G, t0, t1);
        return (t1 - t0) * ph.g.W.cpt;
    }
    if (ph.kind == kPhAttn) {
        int h0, h1;
        head_range(ph.at.n_heads, c, G, h0, h1);
        return (h1 - h0) * 2 * attn_units_per_head(ph, attn_window(ph.at));
    }
    return 0;
}

// Bounded mbarrier wait that also gives up once another CTA has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, const int *abort) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && ld_relaxed_gpu(abort)) return false;
        if (i > 32) __nanosleep(64);
    }
    return false;
}

__device__ __forceinline__ void fail(const FrameArgs &fa, int code) {
    atomicExch(fa.abort, 1);
    raise_error(fa.status, code);
}

// ---------------------------------------------------------------------------
// per-warp unit streams
// ---------------------------------------------------------------------------
// Decodes step st.p for this CTA (or finds there is none left).
__device__ __forceinline__ void stream_enter(WarpStream &st, const FrameArgs &fa, int c, int G) {
    st.n = 0;
    st.attn = false;
    if (st.p >= fa.n_phases) return;
    const FramePhase &ph = fa.prog[st.p];
    if (ph.kind == kPhGemv) {
        int t0, t1;
        tile_range(ph.g.W.n_tiles, c, G, t0, t1);
        st.base = ph.g.W.tiles + static_cast<size_t>(t0) * ph.g.W.cpt * kChunkBytes;
        st.n = (t1 - t0) * ph.g.W.cpt;
    } else if (ph.kind == kPhAttn) {
        const AttnArgs &at = ph.at;
        const Window w = attn_window(at);
        int h1;
        head_range(at.n_heads, c, G, st.h0, h1);
        st.rb = ph.head_dim * 2;
        st.rpu = kChunkBytes / st.rb;
        st.uk = attn_units_per_head(ph, w);
        st.group = at.n_heads / at.n_kv_heads;
        st.n_ctx = at.n_ctx;
        st.start = w.start;
        st.n_old = w.n_old;
        st.kplane = static_cast<const uint8_t *>(at.k_cache) + at.kv_layer_off * 2;
        st.vplane = static_cast<const uint8_t *>(at.v_cache) + at.kv_layer_off * 2;
        st.n = (h1 - st.h0) * 2 * st.uk;
        st.attn = true;
    }
}

// Issues the warp's next unit into its slot (lane 0 only).
__device__ __forceinline__ void stream_issue(FrameSmem &S, WarpStream &st, const FrameArgs &fa, int c, int G, int warp) {
    while (st.p < fa.n_phases && st.u >= st.n) {
        ++st.p;
        st.u = warp;
        stream_enter(st, fa, c, G);
    }
    if (st.p >= fa.n_phases) return;
    const int slot = st.issued % kFwSlots;
    uint8_t *dst = S.ring[warp][slot];
    uint64_t *bar = &S.full[warp][slot];
    if ((threadIdx.x & 31) != 0) {
        // other lanes only advance their copy of the cursor
    } else if (!st.attn) {
        fence_proxy_async();  // this warp's reads of the slot before the copy that overwrites it
        mbar_arrive_expect_tx(bar, kChunkBytes);
        bulk_load(dst, st.base + static_cast<size_t>(st.u) * kChunkBytes, kChunkBytes, bar, st.pol);
    } else {
        fence_proxy_async();
        const int hh = st.u / (2 * st.uk), r = st.u - hh * 2 * st.uk;
        const bool is_v = r >= st.uk;
        const int j0 = (is_v ? r - st.uk : r) * st.rpu;
        const int kh = (st.h0 + hh) / st.group;
        const uint8_t *ring = (is_v ? st.vplane : st.kplane) + static_cast<long long>(kh) * st.n_ctx * st.rb;
        const int nr = min(st.rpu, st.n_old - j0);
        const int s0 = (st.start + j0) % st.n_ctx;
        const int run_a = min(nr, st.n_ctx - s0);
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nr * st.rb));
        bulk_load(dst, ring + static_cast<long long>(s0) * st.rb, run_a * st.rb, bar, st.pol);
        if (nr > run_a) bulk_load(dst + run_a * st.rb, ring, (nr - run_a) * st.rb, bar, st.pol);
    }
    st.u += kFwWarps;
    ++st.issued;
}

// The next unit of this warp's sequence once it has landed (null: gave up).
__device__ __forceinline__ const uint8_t *stream_wait(FrameSmem &S, const WarpStream &st, const FrameArgs &fa) {
    const int warp = threadIdx.x >> 5;
    const int slot = st.consumed % kFwSlots;
    if (!wait_or_abort(&S.full[warp][slot], (st.consumed / kFwSlots) & 1, fa.abort)) return nullptr;
    return S.ring[warp][slot];
}

// Done with the unit: its slot takes the unit kFwSlots further on.
__device__ __forceinline__ void stream_release(FrameSmem &S, WarpStream &st, const FrameArgs &fa, int c, int G) {
    __syncwarp();
    ++st.consumed;
    stream_issue(S, st, fa, c, G, threadIdx.x >> 5);
}

// ---------------------------------------------------------------------------
// consumers: grid barrier
// ---------------------------------------------------------------------------
__device__ bool grid_sync(FrameSmem &S, const FrameArgs &fa, unsigned target, bool ok_in) {
    csync();
    if (threadIdx.x == 0) {
        int ok = ok_in ? 1 : 0;
        if (ok) {
            __threadfence();
            atomicAdd(fa.bar, 1u);
            for (uint32_t i = 0;; ++i) {
                if (ld_acquire_gpu(fa.bar) >= target) break;
                if ((i & 63) == 63 && ld_relaxed_gpu(fa.abort)) { ok = 0; break; }
                if (i >= kGridPolls) {
                    ok = 0;
                    fail(fa, kErrBarrierTimeout);
                    break;
                }
                if (i > 16) __nanosleep(32);
            }
        } else {
            atomicExch(fa.abort, 1);
        }
        S.ok = ok;
    }
    csync();
    return S.ok != 0;
}

// ---------------------------------------------------------------------------
// consumers: GEMV step
// ---------------------------------------------------------------------------
template <int PRO, int EPI>
__device__ __noinline__ bool gemv_phase(FrameSmem &S, const FramePhase &ph, const FrameArgs &fa, int c, int G) {
    WarpStream st = S.ws[threadIdx.x >> 5];  // this warp's cursor, in registers for the step
    const GemvArgs &a = ph.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cpt = a.W.cpt;
    int t0, t1;
    tile_range(a.W.n_tiles, c, G, t0, t1);
    const int n = (t1 - t0) * cpt;
    const int nb = a.W.cols / 32, nbx = a.W.nbx;
    bool ok = true;

    // ---- prologue: the activation as Q8_1 blocks in shared memory ----
    // Thread t converts block t from registers and, for activations longer
    // than 256 blocks, block t + 256 staged by an async copy into the score
    // buffer (idle until the main loop); both loads leave together.
    float v[32];
    const bool h0 = tid < nb, h1 = tid + kFwThreads < nb;
    float *stage1 = S.w.s + tid * 32;
    if constexpr (PRO == kProDepAttn) {
        dep_attention_block<kFwWarps, kFwDepHd, kFwDepMaxWin>(ph.at, S.w.s);
        csync();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = h0 ? S.w.s[tid * 32 + j] : 0.0f;
        csync();  // the attention output aliases the partial-sum table
    } else {
        if (h1)
#pragma unroll
            for (int j = 0; j < 8; ++j) cp_async16(stage1 + 4 * j, a.x + (tid + kFwThreads) * 32 + 4 * j);
        if (h0) load_block32(a.x + tid * 32, v);
    }
    int tok = -1;
    if constexpr (EPI == kEpiEmbAdd) {
        tok = resolve_token<kFwThreads>(a.tok, S.tok_v, S.tok_i, [] { csync(); });
        if (c == 0 && tid == 0 && a.tok.tok_out) *a.tok.tok_out = tok;
    }
    float scale = 1.0f;
    if constexpr (PRO == kProNorm) {
        // nb <= 160 (cols <= 5120): every block is in a register set
        double ss = h0 ? sum_sq_double(v) : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) S.red[warp] = ss;
        csync();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kFwWarps; ++w) tot += S.red[w];
        const float total = __double2float_rn(tot);
        const float mean_eps = __fadd_rn(__fdiv_rn(total, static_cast<float>(a.W.cols)), a.eps);
        scale = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(static_cast<double>(mean_eps))));
    }
    constexpr int QP = PRO == kProNorm ? kProNorm : kProPlain;
    if (tid < nbx) quantize_x_block<QP>(a, S.u.g.xq, S.u.g.xds, tid, h0, v, scale, a.gamma, c == 0);
    if (tid + kFwThreads < nbx) {
        if constexpr (PRO != kProDepAttn) {
            cp_async_wait_all();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = h1 ? stage1[j] : 0.0f;
        }
        quantize_x_block<QP>(a, S.u.g.xq, S.u.g.xds, tid + kFwThreads, h1, v, scale, a.gamma, c == 0);
    }
    csync();

    // ---- main loop: warp w takes units w, w + 8, ... of this step ----
    const int t_first = t0, t_last = t1 - 1;
    int next_unwritten = t_first, cur = -1;
    double acc = 0.0;
    auto flush = [&](int upto) {
        for (int t = next_unwritten; t <= upto; ++t) S.w.part[t - t_first][warp][lane] = t == cur ? acc : 0.0;
        next_unwritten = upto + 1;
    };
    for (int u = warp; u < n; u += kFwWarps) {
        const int k = t0 * cpt + u;
        const int tile = k / cpt, kc = k - tile * cpt;
        if (tile != cur) {
            if (cur >= 0) flush(cur);
            acc = 0.0;
            cur = tile;
        }
        const uint8_t *ch = stream_wait(S, st, fa);
        if (!ch) {
            ok = false;
            break;
        }
        acc += chunk_dot(ch, S.u.g.xq + kc * kChunkBlocks * 32, S.u.g.xds + kc * kChunkBlocks, lane);
        stream_release(S, st, fa, c, G);
    }
    if (cur >= 0) flush(cur);
    flush(t_last);
    if (lane == 0) {
        S.ws[warp] = st;
        if (!ok) S.ok = 0;
    }
    csync();
    if (!ok || S.ok == 0) return false;

    // ---- per-tile reduction (fixed order, double) and epilogue ----
    for (int tl = warp; tl < t1 - t0; tl += kFwWarps) {
        double v = 0.0;
#pragma unroll
        for (int w = 0; w < kFwWarps; ++w) v += S.w.part[tl][w][lane];
        tile_epilogue<EPI>(a, t0 + tl, lane, __double2float_rn(v), tok, a.rope_cs ? S.rope : nullptr);
    }
    return true;
}

// ---------------------------------------------------------------------------
// consumers: temporal attention step (one CTA per head, window from the ring)
// ---------------------------------------------------------------------------
template <int HD>
__device__ __noinline__ bool attn_phase(FrameSmem &S, const FramePhase &ph, const FrameArgs &fa, int c, int G) {
    WarpStream st = S.ws[threadIdx.x >> 5];  // this warp's cursor, in registers for the step
    const AttnArgs &at = ph.at;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Window w = attn_window(at);
    constexpr int kRb = HD * 2, kRpu = kChunkBytes / kRb;
    const int uk = attn_units_per_head(ph, w);
    // this warp's first unit at or after `base` (units u = warp mod 8)
    auto first_unit = [&](int base) { return base + (((warp - base) % kFwWarps) + kFwWarps) % kFwWarps; };
    int h0, h1;
    head_range(at.n_heads, c, G, h0, h1);
    bool ok = true;
    for (int h = h0; h < h1; ++h) {
        const int kbase = (h - h0) * 2 * uk, vbase = kbase + uk;
        const int kh = at.n_kv_heads == at.n_heads ? h : h / (at.n_heads / at.n_kv_heads);
        if (w.window == 1) {
            for (int d = tid; d < HD; d += kFwThreads) at.out[h * HD + d] = __ldcg(at.v_raw + kh * HD + d);
            continue;
        }
        // q and this frame's K/V rows (written by the QKV step): one round trip
        const long long newest = at.kv_layer_off / HD + static_cast<long long>(kh) * at.n_ctx + w.pos % at.n_ctx;
        if (tid < HD) S.u.at.q[tid] = __ldcg(at.q + h * HD + tid);
        if (tid < kRb / 16)
            reinterpret_cast<uint4 *>(S.u.at.knew)[tid] =
                __ldcg(reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(at.k_cache) + newest * kRb) + tid);
        else if (tid < 2 * (kRb / 16))
            reinterpret_cast<uint4 *>(S.u.at.vnew)[tid - kRb / 16] = __ldcg(
                reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(at.v_cache) + newest * kRb) + tid - kRb / 16);
        csync();
        float qr[HD / 32];
#pragma unroll
        for (int i = 0; i < HD / 32; ++i) qr[i] = S.u.at.q[lane + 32 * i];
        float *s = S.w.s;

        // ---- scores: warp w takes K units w, w + 8, ...; 4 positions at a time ----
        auto score4 = [&](const uint8_t *base, int nr, int j0) {
            for (int jb = 0; jb < nr; jb += 4) {
                double dot[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __half *row = reinterpret_cast<const __half *>(base + min(jb + e, nr - 1) * kRb);
                    dot[e] = 0.0;
#pragma unroll
                    for (int i = 0; i < HD / 32; ++i)
                        dot[e] = fma(static_cast<double>(qr[i]), static_cast<double>(__half2float(row[lane + 32 * i])), dot[e]);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int e = 0; e < 4; ++e) dot[e] += __shfl_xor_sync(0xffffffffu, dot[e], o);
                if (lane < 4 && jb + lane < nr) {
                    double mine = dot[0];
#pragma unroll
                    for (int e = 1; e < 4; ++e) mine = lane == e ? dot[e] : mine;
                    s[j0 + jb + lane] = __fmul_rn(__double2float_rn(mine), at.scale);
                }
            }
        };
        for (int u = first_unit(kbase); u < kbase + uk; u += kFwWarps) {
            const uint8_t *ch = stream_wait(S, st, fa);
            if (!ch) { ok = false; break; }
            const int j = u - kbase;
            score4(ch, min(kRpu, w.n_old - j * kRpu), j * kRpu);
            stream_release(S, st, fa, c, G);
        }
        if (warp == kFwWarps - 1) score4(reinterpret_cast<const uint8_t *>(S.u.at.knew), 1, w.n_old);
        if (lane == 0) S.ws[warp] = st;
        if (lane == 0 && !ok) S.ok = 0;
        csync();
        if (!ok || S.ok == 0) return false;

        // ---- softmax over the window (exact two-pass) ----
        float m = -INFINITY;
        for (int j = tid; j < w.window; j += kFwThreads) m = fmaxf(m, s[j]);
        m = warp_max(m);
        if (lane == 0) S.wmax[warp] = m;
        csync();
        float M = S.wmax[0];
#pragma unroll
        for (int i = 1; i < kFwWarps; ++i) M = fmaxf(M, S.wmax[i]);
        for (int j = tid; j < w.window; j += kFwThreads)
            s[j] = __double2float_rn(exp(static_cast<double>(__fsub_rn(s[j], M))));
        csync();

        // ---- weighted sum: warp w takes V units w, w + 8, ...; lanes split head_dim ----
        double o[HD / 32];
#pragma unroll
        for (int i = 0; i < HD / 32; ++i) o[i] = 0.0;
        auto pv = [&](const uint8_t *base, int nr, int j0) {
            for (int j = 0; j < nr; ++j) {
                const double p = static_cast<double>(s[j0 + j]);
                const __half *row = reinterpret_cast<const __half *>(base + j * kRb);
#pragma unroll
                for (int i = 0; i < HD / 32; ++i) o[i] = fma(p, static_cast<double>(__half2float(row[lane + 32 * i])), o[i]);
            }
        };
        for (int u = first_unit(vbase); u < vbase + uk; u += kFwWarps) {
            const uint8_t *ch = stream_wait(S, st, fa);
            if (!ch) { ok = false; break; }
            const int j = u - vbase;
            pv(ch, min(kRpu, w.n_old - j * kRpu), j * kRpu);
            stream_release(S, st, fa, c, G);
        }
        if (warp == kFwWarps - 1) pv(reinterpret_cast<const uint8_t *>(S.u.at.vnew), 1, w.n_old);
#pragma unroll
        for (int i = 0; i < HD / 32; ++i) S.u.at.ow[warp][lane + 32 * i] = o[i];
        if (warp == 0) {
            double l = 0.0;
            for (int j = lane; j < w.window; j += 32) l += static_cast<double>(s[j]);
#pragma unroll
            for (int k = 16; k > 0; k >>= 1) l += __shfl_xor_sync(0xffffffffu, l, k);
            if (lane == 0) S.lsum = l;
        }
        if (lane == 0) S.ws[warp] = st;
        if (lane == 0 && !ok) S.ok = 0;
        csync();
        if (!ok || S.ok == 0) return false;
        if (tid < HD) {
            double ot = 0.0;
#pragma unroll
            for (int i = 0; i < kFwWarps; ++i) ot += S.u.at.ow[i][tid];
            at.out[h * HD + tid] = __double2float_rn(__ddiv_rn(ot, S.lsum));
        }
        csync();  // shared buffers are reused by the next head
    }
    return ok;
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kFwThreads, 1) frame_kernel(const __grid_constant__ FrameArgs fa) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    FrameSmem &S = *reinterpret_cast<FrameSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int c = blockIdx.x, G = gridDim.x;
    if (tid < kFwWarps * kFwSlots) mbar_init(&S.full[tid / kFwSlots][tid % kFwSlots], 1);
    if (tid < fa.rope_pairs) S.rope[tid] = fa.rope[tid];
    if (tid == 0) S.ok = 1;
    fence_barrier_init();
    __syncthreads();

    if ((tid & 31) == 0) {
        WarpStream &st = S.ws[warp];
        st = WarpStream{};
        st.u = warp;
        st.pol = l2_evict_first_policy();
        stream_enter(st, fa, c, G);
        for (int k = 0; k < kFwSlots; ++k) stream_issue(S, st, fa, c, G, warp);
    }
    __syncwarp();

    for (int p = 0; p < fa.n_phases; ++p) {
        const FramePhase &ph = fa.prog[p];
        // the next step's descriptor reaches L1 while this step runs
        constexpr int kDescLines = static_cast<int>((sizeof(FramePhase) + 127) / 128);
        if (tid < kDescLines && p + 1 < fa.n_phases) prefetch_l1(reinterpret_cast<const char *>(&fa.prog[p + 1]) + tid * 128);
        bool ok = true;
        if (ph.kind == kPhGemv) {
            const int pr = ph.pro, ep = ph.epi;
            if (pr == kProNorm && ep == kEpiQKV) ok = gemv_phase<kProNorm, kEpiQKV>(S, ph, fa, c, G);
            else if (pr == kProPlain && ep == kEpiResid) ok = gemv_phase<kProPlain, kEpiResid>(S, ph, fa, c, G);
            else if (pr == kProNorm && ep == kEpiSwiGLU) ok = gemv_phase<kProNorm, kEpiSwiGLU>(S, ph, fa, c, G);
            else if (pr == kProDepAttn && ep == kEpiResid) ok = gemv_phase<kProDepAttn, kEpiResid>(S, ph, fa, c, G);
            else if (pr == kProNorm && ep == kEpiLogits) ok = gemv_phase<kProNorm, kEpiLogits>(S, ph, fa, c, G);
            else if (pr == kProPlain && ep == kEpiLogits) ok = gemv_phase<kProPlain, kEpiLogits>(S, ph, fa, c, G);
            else if (pr == kProPlain && ep == kEpiEmbAdd) ok = gemv_phase<kProPlain, kEpiEmbAdd>(S, ph, fa, c, G);
            else ok = false;  // rejected by the host; never reached
        } else if (ph.kind == kPhAttn) {
            ok = ph.head_dim == 128 ? attn_phase<128>(S, ph, fa, c, G) : attn_phase<64>(S, ph, fa, c, G);
        } else if (ph.kind == kPhTokenOut) {
            if (c == 0) {
                const int t = resolve_token<kFwThreads>(ph.tok, S.tok_v, S.tok_i, [] { csync(); });
                if (tid == 0 && ph.tok.tok_out) *ph.tok.tok_out = t;
            }
        }
        if (!ok && tid == 0) fail(fa, kErrTmaTimeout);
        if (!ok || (p + 1 < fa.n_phases && !grid_sync(S, fa, static_cast<unsigned>(G) * (p + 1), ok))) break;
    }
    // copies still in flight land before the warp exits
    __syncwarp();
    for (uint32_t k = S.ws[warp].consumed; k < S.ws[warp].issued; ++k)
        mbar_wait(&S.full[warp][k % kFwSlots], (k / kFwSlots) & 1);
}

static unsigned long long g_frame_configured = 0;

cudaError_t configure_frame() {
    return cudaFuncSetAttribute(frame_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(FrameSmem)));
}

int frame_max_grid() {
    int blocks = 0, dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (configure_frame() != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, frame_kernel, kFwThreads, sizeof(FrameSmem)) != cudaSuccess)
        return 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return blocks >= 1 ? sms : 0;
}

cudaError_t launch_frame(const FrameArgs &fa, int grid, cudaStream_t s) {
    if (grid <= 0 || !fa.prog || fa.n_phases <= 0 || !fa.bar || !fa.abort) return cudaErrorInvalidValue;
    if (fa.rope_pairs > kFwMaxHd / 2) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(g_frame_configured & (1ull << dev))) {
        const cudaError_t e = configure_frame();
        if (e != cudaSuccess) return e;
        g_frame_configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kFwThreads);
    cfg.dynamicSmemBytes = sizeof(FrameSmem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, frame_kernel, fa);
}

}  // namespace bmo
