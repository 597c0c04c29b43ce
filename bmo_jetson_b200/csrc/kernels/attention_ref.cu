// attention_ref.cu -- single-token decode attention over the fp16 KV ring
// with the reference kernel's own fp32 operations in the reference's own
// order, bit-identical to bmo_decode_attention_kernel
// (src/bmo_cuda_kernels.cu:713-848) on the same ring and inputs.
//
// The reference's arithmetic (one CTA of head_dim threads per head, thread
// = dimension): window W = min(pos + 1, n_ctx), positions i = 0..W-1 at
// slots (pos + 1 - W + i) % n_ctx, oldest first, the current token's K/V
// read back from the ring as fp16.  Score s_i = fl(T_i * scale), where T_i
// adds, in warp order starting from 0, the __shfl_down_sync tree of each
// 32-dimension group's products fl(q_d * k_d).  M = max(-1e20, max s_i);
// e_i = expf(s_i - M); thread t (< head_dim) sums e_{t + head_dim k} in
// order, each warp reduces its threads by a shfl_down tree and the warp
// sums are added in order; inv = 1 / sum; p_i = fl(e_i * inv); out_d =
// sequential fma chain over i of p_i * v_{i,d}.  A window of one returns the
// raw fp32 v.  Measured bit-exact against the reference kernel on B200.
//
// B200 design: a thread-block cluster of NSPLIT CTAs per head.  Rows written
// by earlier frames -- K rows of this CTA's share of the positions, and the
// V columns of its share of the dimensions for every position -- are
// cp.async-staged before griddepcontrol.wait, overlapping the QKV GEMV; the
// newest row (written by that GEMV's epilogue) and q after it.  CTA r scores
// positions [r W / NSPLIT ...) one (position, 32-dimension group) per thread
// with the tree in registers, and pushes each score into every CTA's shared
// memory (distributed shared memory, one cluster barrier).  Every CTA then
// runs the (cheap) softmax over the whole window in the reference's thread
// pattern, and CTA r runs the head_dim / NSPLIT sequential V chains of its
// dimensions.  The depformer (window <= 8) runs with NSPLIT = 1.
#include <cooperative_groups.h>

#include "attention_ref_dev.cuh"
#include "../launch.h"

namespace cg = cooperative_groups;

namespace bmo {

namespace {

constexpr int kThreads = 128;
constexpr int kMaxCtx = 1024;       // the reference kernel's score buffer (s_scores[1024])
constexpr int kMaxCtxSingle = 64;   // one CTA per head (the depformer's short rings)

template <int HD, int NSPLIT>
struct RefAttnLayout {
    static constexpr int kDims = HD / NSPLIT;  // V dimensions per CTA
    static constexpr int kKStride = HD + 8;    // halves per staged K row: rows 16 bytes apart in the banks
    int n_ctx, rows;                           // rows: positions scored per CTA
    size_t off_s, off_k, off_v, off_red, bytes;
    __host__ __device__ explicit RefAttnLayout(int n) : n_ctx(n), rows((n + NSPLIT - 1) / NSPLIT) {
        size_t o = HD * 4;  // q
        off_s = o;
        o += static_cast<size_t>(n) * 4;
        o = (o + 127) & ~static_cast<size_t>(127);
        off_k = o;
        o += static_cast<size_t>(rows) * kKStride * 2;
        off_v = o;
        o += static_cast<size_t>(n) * kDims * 2;
        off_red = o;
        bytes = o + 16 * 4;
    }
};

}  // namespace

template <int HD, int NSPLIT>
__global__ void __launch_bounds__(kThreads) attn_ref_kernel(const __grid_constant__ AttnArgs a) {
    using Lay = RefAttnLayout<HD, NSPLIT>;
    constexpr int kDims = Lay::kDims, kKS = Lay::kKStride;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Lay lay(a.n_ctx);
    float *sq = reinterpret_cast<float *>(smem_raw);
    float *ss = reinterpret_cast<float *>(smem_raw + lay.off_s);
    __half *kb = reinterpret_cast<__half *>(smem_raw + lay.off_k);
    __half *vb = reinterpret_cast<__half *>(smem_raw + lay.off_v);
    float *red = reinterpret_cast<float *>(smem_raw + lay.off_red);
    const int tid = threadIdx.x;
    const int r = blockIdx.x, h = blockIdx.y;

    const int pos = *a.pos;  // copied to the device before this graph's first kernel
    const int total = pos + 1;
    const int W = total > a.n_ctx ? a.n_ctx : total;
    const int start = total - W;
    const int per = (W + NSPLIT - 1) / NSPLIT;
    const int i0 = min(W, r * per), i1 = min(W, i0 + per);
    const int kh = (a.n_kv_heads == a.n_heads) ? h : h / (a.n_heads / a.n_kv_heads);
    const long long row0 = a.kv_layer_off / HD + static_cast<long long>(kh) * a.n_ctx;  // ring row of slot 0
    const __half *kc = static_cast<const __half *>(a.k_cache) + row0 * HD;
    const __half *vc = static_cast<const __half *>(a.v_cache) + row0 * HD + r * kDims;

    // K rows of positions [i0, i1) and V columns of all positions, except the
    // newest (written by this frame's QKV kernel), staged before the wait.
    if (W > 1) {
        constexpr int kKPieces = HD / 8, kVPieces = kDims / 8;  // 16-byte pieces per row
        const int nk = (min(i1, W - 1) - i0) * kKPieces;
        for (int e = tid; e < nk; e += kThreads) {
            const int i = i0 + e / kKPieces, pc = e % kKPieces;
            const int slot = (start + i) % a.n_ctx;
            cp_async16(kb + (i - i0) * kKS + pc * 8, kc + static_cast<long long>(slot) * HD + pc * 8);
        }
        const int nv = (W - 1) * kVPieces;
        for (int e = tid; e < nv; e += kThreads) {
            const int i = e / kVPieces, pc = e % kVPieces;
            const int slot = (start + i) % a.n_ctx;
            cp_async16(vb + i * kDims + pc * 8, vc + static_cast<long long>(slot) * HD + pc * 8);
        }
    }

    pdl_wait();
    pdl_launch_dependents();

    float *out = a.out + h * HD;
    if (W == 1) {  // fast path of the reference: the raw fp32 v
        for (int d = tid; d < kDims; d += kThreads) out[r * kDims + d] = __ldcg(a.v_raw + kh * HD + r * kDims + d);
        return;
    }
    for (int d = tid; d < HD; d += kThreads) sq[d] = __ldcg(a.q + h * HD + d);
    const int cur = pos % a.n_ctx;
    if (i0 < i1 && i1 == W)
        for (int d = tid; d < HD; d += kThreads) kb[(W - 1 - i0) * kKS + d] = __ldcg(kc + static_cast<long long>(cur) * HD + d);
    for (int d = tid; d < kDims; d += kThreads) vb[(W - 1) * kDims + d] = __ldcg(vc + static_cast<long long>(cur) * HD + d);
    cp_async_wait_all();
    __syncthreads();

    // ---- scores of positions [i0, i1): thread = (position, 32-dim group) ----
    attn_ref_scores<HD, kThreads, kKS>(sq, kb, i0, i1, a.scale, tid, [&](int i, float s) {
        if constexpr (NSPLIT == 1) {
            ss[i] = s;
        } else {
            cg::cluster_group cl = cg::this_cluster();
#pragma unroll
            for (int rr = 0; rr < NSPLIT; ++rr) *cl.map_shared_rank(ss + i, rr) = s;
        }
    });
    if constexpr (NSPLIT == 1) __syncthreads();
    else cg::this_cluster().sync();

    // ---- softmax over the whole window, the reference's thread pattern ----
    attn_ref_softmax<HD, kThreads>(ss, W, red, tid, [] { __syncthreads(); });

    // ---- weighted sum of V: one sequential chain per dimension ----
    if (tid < kDims) out[r * kDims + tid] = attn_ref_vchain(ss, vb + tid, W, kDims);
}

// ---------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------
cudaError_t configure_attention_ref();

template <int HD, int NSPLIT>
static cudaError_t launch_ref_attn_t(const AttnArgs &a, cudaStream_t s, bool pdl) {
    // The shared-memory opt-in is per device; the first launch on a device sets it.
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(configured & (1ull << dev))) {
        const cudaError_t e = configure_attention_ref();
        if (e != cudaSuccess) return e;
        configured |= 1ull << dev;
    }
    const RefAttnLayout<HD, NSPLIT> lay(a.n_ctx);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(NSPLIT, a.n_heads);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = lay.bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na++].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    if (NSPLIT > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = NSPLIT;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, attn_ref_kernel<HD, NSPLIT>, a);
}

template <int HD, int NSPLIT>
static cudaError_t configure_ref_attn_t() {
    const RefAttnLayout<HD, NSPLIT> lay(NSPLIT > 1 ? kMaxCtx : kMaxCtxSingle);
    return cudaFuncSetAttribute(attn_ref_kernel<HD, NSPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(lay.bytes));
}

cudaError_t configure_attention_ref() {
    cudaError_t e;
    if ((e = configure_ref_attn_t<128, 8>()) != cudaSuccess) return e;
    if ((e = configure_ref_attn_t<64, 8>()) != cudaSuccess) return e;
    if ((e = configure_ref_attn_t<128, 1>()) != cudaSuccess) return e;
    return configure_ref_attn_t<64, 1>();
}

int attn_ref_max_ctx() { return kMaxCtx; }

bool attn_ref_supported(int head_dim, int n_ctx, bool split) {
    return (head_dim == 64 || head_dim == 128) && n_ctx >= 1 && n_ctx <= (split ? kMaxCtx : kMaxCtxSingle);
}

cudaError_t launch_attention_ref(const AttnArgs &a, int head_dim, bool split, cudaStream_t s, bool pdl) {
    if (!attn_ref_supported(head_dim, a.n_ctx, split) || a.kv_type != kKvF16 || a.n_heads <= 0 ||
        a.n_kv_heads <= 0 || a.n_heads % a.n_kv_heads)
        return cudaErrorInvalidValue;
    if (head_dim == 128) return split ? launch_ref_attn_t<128, 8>(a, s, pdl) : launch_ref_attn_t<128, 1>(a, s, pdl);
    return split ? launch_ref_attn_t<64, 8>(a, s, pdl) : launch_ref_attn_t<64, 1>(a, s, pdl);
}

}  // namespace bmo
