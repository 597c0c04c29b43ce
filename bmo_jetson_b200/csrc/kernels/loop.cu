// loop.cu -- the caller's frame loop on the device: the 17-channel
// interleave and delay of bmo_daemon.cpp:727-742, its token samplers
// (sample_token_cpp, :147-175, with the loop's one std::mt19937) and its
// per-frame state update (:811-816), so that a whole conversational frame --
// interleave, temporal step, text sample, 8 depformer steps each with its
// audio sample, codec tokens -- is one CUDA graph with no host round trip.
//
//   frame 0:   [pad_text, pad_audio x 16]
//   frame 1:   [prev_text, prev_audio[0], pad_audio x 7, user[0], pad_audio x 7]
//   frame >1:  [prev_text, prev_audio[0..7], user[0], prev_user[1..7]]
//   text:      top1 = first argmax; a pause (3 or 0) or greedy mode keeps top1,
//              else top-k / temperature sampling
//   audio:     per step, first argmax (greedy) or top-k / temperature sampling
//   codec:     [prev_cb0, audio[1..7]]; then prev_cb0 = audio[0],
//              prev_audio = audio, prev_user = user, prev_text = text.
//
// The sampler reproduces sample_token_cpp's arithmetic: the top_k logits in
// descending order (ties by lower index: std::partial_sort leaves the order of
// equal logits unspecified), probs_i = exp(l_i / temp - l_0 / temp) in float
// (the exponential evaluated in double and rounded once), their float sum
// checked for zero or NaN, then std::discrete_distribution's draw -- the
// probabilities widened to double, divided by their sequential double sum,
// the running sums as the cumulative table with its last entry 1, u =
// generate_canonical<double, 53> from two 32-bit outputs, the first index
// whose cumulative value is >= u.  The generator is the standard's mt19937.
#include <algorithm>

#include "common.cuh"
#include "gemv_dev.cuh"
#include "../launch.h"

namespace bmo {

namespace {

constexpr int kSampleThreads = 1024;
constexpr unsigned kMtUpper = 0x80000000u, kMtLower = 0x7fffffffu, kMtMatrix = 0x9908b0dfu;

// The standard's mt19937: the output transform of one state word, and the
// next output (state in shared memory, one thread).
__device__ __forceinline__ unsigned mt_temper(unsigned y) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}


__device__ unsigned mt_next(unsigned *mt, int &mti) {
    if (mti >= 624) {
        for (int i = 0; i < 624; ++i) {
            const unsigned y = (mt[i] & kMtUpper) | (mt[(i + 1) % 624] & kMtLower);
            mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? kMtMatrix : 0u);
        }
        mti = 0;
    }
    return mt_temper(mt[mti++]);
}

}  // namespace

// Builds this frame's input tokens and position from the loop state.
__global__ void loop_begin_kernel(LoopState *st, LoopConfig cfg, int *tokens, int *n_tok, int *pos) {
    if (threadIdx.x != 0) return;
    // the daemon's silence tokens when the caller has no user audio
    const int silence[kLoopCb] = {1049, 243, 783, 1562, 340, 2010, 183, 1665};
    const int f = st->frame;
    const LoopParams &in = st->in[f % kLoopRing];
    for (int i = 0; i < kLoopCb; ++i) st->user[i] = in.user_valid ? in.user[i] : silence[i];
    int t[1 + 2 * kLoopCb];
    if (f == 0) {
        t[0] = cfg.text_pad;
        for (int i = 1; i <= 2 * kLoopCb; ++i) t[i] = cfg.audio_pad;
    } else if (f == 1) {
        t[0] = st->prev_text;
        t[1] = st->prev_audio[0];
        for (int i = 2; i <= kLoopCb; ++i) t[i] = cfg.audio_pad;
        t[1 + kLoopCb] = st->user[0];
        for (int i = 2 + kLoopCb; i <= 2 * kLoopCb; ++i) t[i] = cfg.audio_pad;
    } else {
        t[0] = st->prev_text;
        for (int i = 0; i < kLoopCb; ++i) t[1 + i] = st->prev_audio[i];
        t[1 + kLoopCb] = st->user[0];
        for (int i = 1; i < kLoopCb; ++i) t[1 + kLoopCb + i] = st->prev_user[i];
    }
    for (int i = 0; i < cfg.n_tok; ++i) tokens[i] = t[i];
    *n_tok = cfg.n_tok;
    *pos = f;
}

// Codec input, state update, and the frame's results in row frame % kLoopRing
// of st->out: [0] text token, [1..8] audio tokens, [9..16] codec input
// (meaningful from frame 1 on: the daemon decodes nothing at frame 0).
__global__ void loop_end_kernel(LoopState *st) {
    if (threadIdx.x != 0) return;
    int *out = st->out[st->frame % kLoopRing];
    out[0] = st->next_text;
    out[1 + kLoopCb] = st->prev_cb0;
    for (int i = 0; i < kLoopCb; ++i) out[1 + i] = st->audio[i];
    for (int i = 1; i < kLoopCb; ++i) out[1 + kLoopCb + i] = st->audio[i];
    st->prev_cb0 = st->audio[0];
    for (int i = 0; i < kLoopCb; ++i) {
        st->prev_audio[i] = st->audio[i];
        st->prev_user[i] = st->user[i];
    }
    st->prev_text = st->next_text;
    st->frame += 1;
}

namespace {

// Order-preserving key of a float (larger float, larger key; no NaNs) and back.
__device__ __forceinline__ unsigned fkey(float v) {
    const unsigned u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_value(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct alignas(16) SampleSmem {
    // selected entries as (key << 32) | ~index -- descending order = value
    // descending, index ascending -- then, after the sort, p_i / total
    union alignas(16) {
        unsigned long long sel[kLoopTopKMax + 2];
        double q[kLoopTopKMax];
    };
    unsigned long long srt[kLoopTopKMax];  // the entries in descending order
    alignas(16) float prob[kLoopTopKMax];
    unsigned mt[624];
    int hist[256];
    int wsum[32];
    float red_v[32];
    int red_i[32];
    int n_sel, n_eq_taken, n_eq, kk, tok, draw, mti;
    unsigned long long units;
    unsigned prefix;
    double total;
};

// Adds 1 to bin `b` for every lane with `take`, one atomic per distinct bin
// of the warp.
__device__ __forceinline__ void hist_add(int *hist, bool take, unsigned b) {
    const unsigned act = __ballot_sync(0xffffffffu, take);
    if (!take) return;
    const unsigned same = __match_any_sync(act, b);
    if ((threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[b], __popc(same));
}

// The kk-th largest (1-based) of the keys the block offers, by radix select
// over 8-bit digits: `each(f)` calls f(valid, key) for each of the calling
// thread's keys.  Returns the key; *n_eq is the number of offered keys equal
// to it and *kk_eq how many of those the kk largest take.  All threads call.
template <class Each>
__device__ unsigned radix_kth(SampleSmem &S, int kk, Each each, int *n_eq, int *kk_eq) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned prefix = 0, mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (tid < 256) S.hist[tid] = 0;
        __syncthreads();
        each([&](bool valid, unsigned key) { hist_add(S.hist, valid && (key & mask) == prefix, (key >> shift) & 255u); });
        __syncthreads();
        if (tid < 256) {
            // suffix sum s(b) = sum of hist[b'] over b' >= b; the bin with
            // s(b + 1) < kk <= s(b) holds the kk-th largest
            const int h = S.hist[tid];
            int s = h;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_down_sync(0xffffffffu, s, o);
                if (lane + o < 32) s += t;
            }
            if (lane == 0) S.wsum[warp] = s;
            named_sync(1, 256);
            for (int w = warp + 1; w < 8; ++w) s += S.wsum[w];
            if (s >= kk && s - h < kk) {
                S.kk = kk - (s - h);
                S.n_eq = h;
                S.prefix = prefix | (static_cast<unsigned>(tid) << shift);
            }
        }
        __syncthreads();
        kk = S.kk;
        prefix = S.prefix;
        mask |= 255u << shift;
    }
    *n_eq = S.n_eq;
    *kk_eq = kk;
    return prefix;
}

// Appends the keys for which `take` holds to S.sel as (key << 32) | ~index
// (one atomic per warp and call).
__device__ __forceinline__ void sel_push(SampleSmem &S, bool take, unsigned key, int i) {
    const int lane = threadIdx.x & 31;
    const unsigned act = __ballot_sync(0xffffffffu, take);
    int base = 0;
    if (lane == 0 && act) base = atomicAdd(&S.n_sel, __popc(act));
    base = __shfl_sync(0xffffffffu, base, 0);
    const int at = base + __popc(act & ((1u << lane) - 1u));
    if (take && at < kLoopTopKMax)
        S.sel[at] = (static_cast<unsigned long long>(key) << 32) | (~static_cast<unsigned>(i));
}

// Ranks the m entries of S.sel (each one's rank is the number of larger
// entries) and writes those of rank < k to S.srt in order.  (Measured on
// B200 for 250 entries: 2.3 µs; a warp per entry 4.6 µs, 4 threads per entry
// 3.1 µs.)
__device__ __forceinline__ void rank_sort(SampleSmem &S, int m, int k) {
    const int tid = threadIdx.x;
    if (tid < 2) S.sel[m + tid] = 0;  // padding below every entry
    __syncthreads();
    const ulonglong2 *p2 = reinterpret_cast<const ulonglong2 *>(S.sel);
    for (int i = tid; i < m; i += kSampleThreads) {
        const unsigned long long x = S.sel[i];
        int r = 0;
#pragma unroll 4
        for (int j = 0; j < (m + 1) / 2; ++j) {
            const ulonglong2 y = p2[j];
            r += (y.x > x) + (y.y > x);
        }
        if (r < k) S.srt[r] = x;
    }
    __syncthreads();
}

}  // namespace

// One token draw (the daemon's sample_token_cpp; first argmax when greedy).
// One CTA of kSampleThreads threads; thread t takes elements t + j *
// kSampleThreads, j < ITEMS.  With ITEMS = 2 (the audio logits) the keys stay
// in registers; with more (the text logits) each thread keeps only its
// largest key: the k-th largest of those 1024 maxima bounds the k largest
// logits from below (k of them reach it), so only the logits at or above it
// -- a few more than k for any spread of values -- are ranked.  The full
// radix select over every logit remains for k above 1024 or more than 2048
// such candidates (many equal logits).
template <int ITEMS>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
    __shared__ SampleSmem S;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kWarpsS = kSampleThreads / 32;
    constexpr bool kRegs = ITEMS <= 2;
    constexpr int kRollU = kRegs ? ITEMS : 1;  // register-held keys need unrolled loops; reloaded ones do not
    // Launched as a programmatic dependent of the logits' GEMV: wait for it,
    // then let the next step's kernels launch and stage their weights while
    // the draw runs (they wait for this grid before reading its token).
    pdl_wait();
    pdl_launch_dependents();

    // ---- the first argmax (std::max_element), the keys or their maximum ----
    unsigned key[kRegs ? ITEMS : 1];
    unsigned kmax = 0;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    // in groups of up to 8 loads issued together: a fully unrolled loop over
    // 32 elements measured slower (its code is fetched cold on every launch)
    constexpr int kG = ITEMS < 8 ? ITEMS : 8;
#pragma unroll 1
    for (int j0 = 0; j0 < ITEMS; j0 += kG) {
        float v[kG];
#pragma unroll
        for (int j = 0; j < kG; ++j) {
            const int i = tid + (j0 + j) * kSampleThreads;
            v[j] = i < a.n ? __ldcg(a.logits + i) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kG; ++j) {
            const int i = tid + (j0 + j) * kSampleThreads;
            const unsigned kj = i < a.n ? fkey(v[j]) : 0u;
            if (i < a.n) argmax_merge(bv, bi, v[j], i);
            if constexpr (kRegs) key[j0 + j] = kj;
            kmax = kj > kmax ? kj : kmax;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    if (lane == 0) {
        S.red_v[warp] = bv;
        S.red_i[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        float fv = S.red_v[0];
        int fi = S.red_i[0];
        for (int w = 1; w < kWarpsS; ++w) argmax_merge(fv, fi, S.red_v[w], S.red_i[w]);
        S.tok = fi;
        S.n_sel = 0;
        S.units = 0;
        S.mti = *a.mti;
    }
    __syncthreads();
    const int top1 = S.tok;
    int sampling = a.sampling, top_k = a.top_k;
    float temp = a.temp;
    if (a.st) {
        const LoopParams &in = a.st->in[a.st->frame % kLoopRing];
        sampling = in.sampling;
        top_k = a.text ? in.top_k_text : in.top_k_audio;
        temp = a.text ? in.temp_text : in.temp_audio;
    }
    const bool greedy = !sampling || top_k <= 0 || temp <= 1e-4f || (a.text && (top1 == 3 || top1 == 0));
    if (greedy) {
        if (tid == 0) *a.out = top1;
        return;
    }
    const int k = min(min(top_k, a.n), kLoopTopKMax);  // the host keeps top_k within kLoopTopKMax
    auto key_at = [&](int j) -> unsigned {
        if constexpr (kRegs) return key[j];
        else return fkey(__ldcg(a.logits + tid + j * kSampleThreads));
    };
    int n_eq, kk;

    // ---- the k largest logits, in order, into S.srt ----
    bool done = false;
    if constexpr (!kRegs) {
        if (k <= kSampleThreads) {
            const unsigned lb = radix_kth(S, k, [&](auto f) { f(true, kmax); }, &n_eq, &kk);
#pragma unroll 1
            for (int j0 = 0; j0 < ITEMS; j0 += kG) {
                unsigned kv[kG];
#pragma unroll
                for (int j = 0; j < kG; ++j) kv[j] = tid + (j0 + j) * kSampleThreads < a.n ? key_at(j0 + j) : 0u;
#pragma unroll
                for (int j = 0; j < kG; ++j) {
                    const int i = tid + (j0 + j) * kSampleThreads;
                    sel_push(S, i < a.n && kv[j] >= lb, kv[j], i);
                }
            }
            __syncthreads();
            const int m = S.n_sel;
            if (m <= kLoopTopKMax) {
                rank_sort(S, m, k);
                done = true;
            }
            __syncthreads();
            if (tid == 0) S.n_sel = 0;
            __syncthreads();
        }
    }
    if (!done) {
        // every key above the k-th largest, and of those equal to it the
        // lowest-index ones (block-scanned in index order only when the
        // threshold value occurs more often than it is needed)
        const unsigned thr = radix_kth(
            S, k,
            [&](auto f) {
#pragma unroll kRollU
                for (int j = 0; j < ITEMS; ++j) {
                    const bool valid = tid + j * kSampleThreads < a.n;
                    f(valid, valid ? key_at(j) : 0u);
                }
            },
            &n_eq, &kk);
        const bool all_eq = n_eq == kk;
#pragma unroll kRollU
        for (int j = 0; j < ITEMS; ++j) {
            const int i = tid + j * kSampleThreads;
            const unsigned kj = i < a.n ? key_at(j) : 0u;
            sel_push(S, i < a.n && (kj > thr || (all_eq && kj == thr)), kj, i);
        }
        if (!all_eq) {
            if (tid == 0) S.n_eq_taken = 0;
            __syncthreads();
#pragma unroll 1
            for (int j = 0; j < ITEMS; ++j) {
                const int i = tid + j * kSampleThreads;
                const bool eq = i < a.n && key_at(j) == thr;
                const unsigned bal = __ballot_sync(0xffffffffu, eq);
                if (lane == 0) S.wsum[warp] = __popc(bal);
                __syncthreads();
                int before = S.n_eq_taken;
                for (int w = 0; w < warp; ++w) before += S.wsum[w];
                before += __popc(bal & ((1u << lane) - 1u));
                if (eq && before < kk)
                    S.sel[atomicAdd(&S.n_sel, 1)] =
                        (static_cast<unsigned long long>(thr) << 32) | (~static_cast<unsigned>(i));
                __syncthreads();
                if (tid == 0) {
                    int t = 0;
                    for (int w = 0; w < kWarpsS; ++w) t += S.wsum[w];
                    S.n_eq_taken += t;
                }
                __syncthreads();
            }
        }
        __syncthreads();
        rank_sort(S, k, k);
    }

    // ---- probabilities: exp(l_i / temp - l_0 / temp), rounded to float ----
    // p_0 is exactly 1, so their float sum in order is positive unless a
    // term is NaN (a NaN or infinite logit): then the reference keeps the
    // first entry.  std::discrete_distribution normalises by the double sum
    // in order and draws nothing for one weight.
    const float max_l = __fdiv_rn(fkey_value(static_cast<unsigned>(S.srt[0] >> 32)), temp);
    bool nan_p = false;
    for (int i = tid; i < k; i += kSampleThreads) {
        const float li = fkey_value(static_cast<unsigned>(S.srt[i] >> 32));
        const float p = static_cast<float>(exp(static_cast<double>(__fsub_rn(__fdiv_rn(li, temp), max_l))));
        S.prob[i] = p;
        nan_p |= isnan(p);
    }
    const bool any_nan = __syncthreads_or(nan_p);
    const int tok0 = static_cast<int>(~static_cast<unsigned>(S.srt[0]));
    if (any_nan || k < 2) {
        if (tid == 0) *a.out = tok0;
        return;
    }
    // The double sum in order.  Every partial sum is below 2^e, e = bits of
    // k (p_i <= 1); when every p_i is zero or a multiple of 2^(e - 53) (its
    // exponent at least e - 30), every partial sum is a multiple of 2^(e - 53)
    // below 2^e, hence exact, and the sum in order is the exact sum: then it
    // is formed in parallel as an integer count of 2^(e - 53).  Otherwise
    // one thread adds in order.
    const int e = 32 - __clz(k);
    const double unit = ldexp(1.0, e - 53);
    bool on_grid = true;
    unsigned long long units = 0;
    for (int i = tid; i < k; i += kSampleThreads) {
        const float p = S.prob[i];
        const int ex = static_cast<int>((__float_as_uint(p) >> 23) & 255u) - 127;
        if (p != 0.0f && ex < e - 30) on_grid = false;
        units += static_cast<unsigned long long>(__dmul_rn(static_cast<double>(p), ldexp(1.0, 53 - e)));
    }
    const bool exact = __syncthreads_and(on_grid);
    if (exact) {
        for (int o = 16; o > 0; o >>= 1) units += __shfl_xor_sync(0xffffffffu, units, o);
        if (lane == 0) atomicAdd(&S.units, units);
    }
    __syncthreads();
    if (exact && tid == 0) S.total = __dmul_rn(static_cast<double>(S.units), unit);  // below 2^53 units: exact
    if (!exact && tid == 0) {
        double total = 0.0;
        int i = 0;
        for (; i + 4 <= k; i += 4) {
            const float4 p = *reinterpret_cast<const float4 *>(S.prob + i);
            total = __dadd_rn(__dadd_rn(__dadd_rn(__dadd_rn(total, static_cast<double>(p.x)), static_cast<double>(p.y)),
                                        static_cast<double>(p.z)),
                              static_cast<double>(p.w));
        }
        for (; i < k; ++i) total = __dadd_rn(total, static_cast<double>(S.prob[i]));
        S.total = total;
    }
    __syncthreads();
    const double total = S.total;
    for (int i = tid; i < k; i += kSampleThreads) S.q[i] = __ddiv_rn(static_cast<double>(S.prob[i]), total);
    // the generator: two outputs; its 624 words pass through shared memory
    // only when they are regenerated (every 312 draws)
    const bool twist = S.mti + 2 > 624;
    if (twist)
        for (int i = tid; i < 624; i += kSampleThreads) S.mt[i] = a.mt[i];
    __syncthreads();
    if (tid == 0) {
        int mti = S.mti;
        unsigned g1, g2;
        if (twist) {
            g1 = mt_next(S.mt, mti);
            g2 = mt_next(S.mt, mti);
        } else {
            g1 = mt_temper(a.mt[mti]);
            g2 = mt_temper(a.mt[mti + 1]);
            mti += 2;
        }
        double u = __dadd_rn(static_cast<double>(g1), __dmul_rn(static_cast<double>(g2), 4294967296.0));
        u = __ddiv_rn(u, 18446744073709551616.0);
        if (u >= 1.0) u = 0x1.fffffffffffffp-1;  // the largest double below 1
        // the first running sum >= u (the last one counts as 1)
        double run = 0.0;
        int pick = k - 1;
        for (int i = 0; i < k - 1; ++i) {
            run = __dadd_rn(run, S.q[i]);
            if (run >= u) {
                pick = i;
                break;
            }
        }
        *a.out = static_cast<int>(~static_cast<unsigned>(S.srt[pick]));
        *a.mti = mti;
    }
    if (twist) {
        __syncthreads();
        for (int i = tid; i < 624; i += kSampleThreads) a.mt[i] = S.mt[i];
    }
}

cudaError_t launch_loop_begin(LoopState *st, const LoopConfig &cfg, int *tokens, int *n_tok, int *pos,
                              cudaStream_t s) {
    loop_begin_kernel<<<1, 32, 0, s>>>(st, cfg, tokens, n_tok, pos);
    return cudaGetLastError();
}

cudaError_t launch_loop_end(LoopState *st, cudaStream_t s) {
    loop_end_kernel<<<1, 32, 0, s>>>(st);
    return cudaGetLastError();
}

// The sampler takes n up to kSampleMaxN and min(top_k, n) up to
// kLoopTopKMax; the host checks the caller's values before they reach the
// device.
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s, bool pdl) {
    if (a.n <= 0 || a.n > kSampleMaxN || !a.logits || !a.mt || !a.mti || !a.out ||
        (!a.st && a.sampling && std::min(a.top_k, a.n) > kLoopTopKMax))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kSampleThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a.n <= 2 * kSampleThreads) return cudaLaunchKernelEx(&cfg, sample_kernel<2>, a);
    return cudaLaunchKernelEx(&cfg, sample_kernel<kSampleMaxN / kSampleThreads>, a);
}

}  // namespace bmo
