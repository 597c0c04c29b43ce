// rvq.cu -- Mimi residual vector quantiser on caller device buffers, behind
// bmo_rvq_decode / bmo_rvq_encode (reference src/bmo_cuda_kernels.cu:886-1063).
//
// decode: out[d] = sum over the 8 codebooks of proj[cb][code_cb][d] (codes
//         outside [0, 2048) skipped), summed in codebook order.
// encode: r = W_in0 x; code_0 = argmax_k (r . e0[k] - norm0[k]); r -= e0[code_0];
//         then r = W_rest x and for stages 1..7 the same search on e_rest[s-1]
//         / norm_rest[s-1] with r -= e[code_s].  Ties resolve to the lowest
//         code (the reference keeps the first maximum).
// Fixed sizes as in the reference: 8 codebooks of 2048 entries, 256-d codes,
// 512-d input.  Scratch (>= 384 floats): r[256], per-block bests [2][64].
#include "../../../include/bmo_api.h"
#include "common.cuh"

namespace bmo {

constexpr int kRvqCodes = 2048, kRvqDim = 256, kRvqIn = 512, kRvqStages = 8, kRvqBlocks = 64;

__global__ void rvq_decode_kernel(const int32_t *codes, const float *proj, float *out) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= kRvqIn) return;
    float sum = 0.0f;
#pragma unroll
    for (int cb = 0; cb < kRvqStages; ++cb) {
        const int code = codes[cb];
        if (code >= 0 && code < kRvqCodes) sum += proj[(static_cast<size_t>(cb) * kRvqCodes + code) * kRvqIn + d];
    }
    out[d] = sum;
}

// r[row] = W[row] . x, one warp per row.
__global__ void rvq_in_proj_kernel(const float *x, const float *W, float *r) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= kRvqDim) return;
    float s = 0.0f;
    for (int i = lane; i < kRvqIn; i += 32) s = fmaf(x[i], W[static_cast<size_t>(warp) * kRvqIn + i], s);
    s = warp_sum(s);
    if (lane == 0) r[warp] = s;
}

// Scores a 32-code slice per block: one warp per code, best (value, code) per block.
__global__ void rvq_search_kernel(const float *r, const float *emb, const float *norms, float *bval, int *bidx) {
    __shared__ float sr[kRvqDim];
    __shared__ float wv[8];
    __shared__ int wi[8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < kRvqDim; i += blockDim.x) sr[i] = r[i];
    __syncthreads();
    float best = -INFINITY;
    int besti = 0x7fffffff;
    for (int c = warp; c < kRvqCodes / kRvqBlocks; c += 8) {
        const int k = blockIdx.x * (kRvqCodes / kRvqBlocks) + c;
        float s = 0.0f;
        for (int d = lane; d < kRvqDim; d += 32) s = fmaf(sr[d], emb[static_cast<size_t>(k) * kRvqDim + d], s);
        s = warp_sum(s) - norms[k];
        if (s > best || (s == best && k < besti)) { best = s; besti = k; }
    }
    if (lane == 0) { wv[warp] = best; wi[warp] = besti; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; ++w)
            if (wv[w] > best || (wv[w] == best && wi[w] < besti)) { best = wv[w]; besti = wi[w]; }
        bval[blockIdx.x] = best;
        bidx[blockIdx.x] = besti;
    }
}

// Picks the winning code over the blocks, records it and subtracts its entry from r.
__global__ void rvq_select_kernel(const float *bval, const int *bidx, const float *emb, float *r, int32_t *codes,
                                  int stage) {
    __shared__ int win;
    if (threadIdx.x == 0) {
        float best = bval[0];
        int bi = bidx[0];
        for (int b = 1; b < kRvqBlocks; ++b)
            if (bval[b] > best || (bval[b] == best && bidx[b] < bi)) { best = bval[b]; bi = bidx[b]; }
        win = bi;
        codes[stage] = bi;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kRvqDim; d += blockDim.x) r[d] -= emb[static_cast<size_t>(win) * kRvqDim + d];
}

}  // namespace bmo

using namespace bmo;

extern "C" {

int bmo_rvq_decode(const int32_t *codes_dev, const float *proj_tables_dev, float *out_dev, void *stream) {
    if (!codes_dev || !proj_tables_dev || !out_dev) return 1;
    cudaGetLastError();  // report only this call's launch errors
    rvq_decode_kernel<<<2, 256, 0, static_cast<cudaStream_t>(stream)>>>(codes_dev, proj_tables_dev, out_dev);
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int bmo_rvq_encode(const float *in_vec_dev, const float *w_in0_dev, const float *e0_dev, const float *norm0_dev,
                   const float *w_in_rest_dev, const float *e_rest_dev, const float *norm_rest_dev,
                   int32_t *out_codes_dev, float *scratch_dev, void *stream) {
    if (!in_vec_dev || !w_in0_dev || !e0_dev || !norm0_dev || !w_in_rest_dev || !e_rest_dev || !norm_rest_dev ||
        !out_codes_dev || !scratch_dev)
        return 1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaGetLastError();  // report only this call's launch errors
    float *r = scratch_dev;
    float *bval = r + kRvqDim;
    int *bidx = reinterpret_cast<int *>(bval + kRvqBlocks);
    rvq_in_proj_kernel<<<kRvqDim * 32 / 256, 256, 0, s>>>(in_vec_dev, w_in0_dev, r);
    rvq_search_kernel<<<kRvqBlocks, 256, 0, s>>>(r, e0_dev, norm0_dev, bval, bidx);
    rvq_select_kernel<<<1, 256, 0, s>>>(bval, bidx, e0_dev, r, out_codes_dev, 0);
    rvq_in_proj_kernel<<<kRvqDim * 32 / 256, 256, 0, s>>>(in_vec_dev, w_in_rest_dev, r);
    for (int stage = 1; stage < kRvqStages; ++stage) {
        const float *e = e_rest_dev + static_cast<size_t>(stage - 1) * kRvqCodes * kRvqDim;
        const float *nrm = norm_rest_dev + static_cast<size_t>(stage - 1) * kRvqCodes;
        rvq_search_kernel<<<kRvqBlocks, 256, 0, s>>>(r, e, nrm, bval, bidx);
        rvq_select_kernel<<<1, 256, 0, s>>>(bval, bidx, e, r, out_codes_dev, stage);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // extern "C"
