// common.cuh -- device helpers shared by the decode-step kernels (sm_100a).
//
// PTX wrappers for mbarriers, the bulk-copy (TMA) engine, programmatic
// dependent launch, and the Q8_1 / Q4_0 block quantisers whose bit patterns
// must match the reference (src/bmo_cuda_kernels.cu:529-558 for Q8_1; ggml's
// quantize_row_q4_0_ref for the Q4_0 KV mode).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../layout.h"

namespace bmo {

// Error codes a kernel may raise in the per-handle status word.
enum : int {
    kErrNone = 0,
    kErrTmaTimeout = 1,    // a bulk copy did not land within the wait bound
    kErrBadShape = 2,      // launch arguments inconsistent with the weight layout
    kErrReserved3 = 3,     // unused (no kernel raises it); kept so the other codes keep their bits
    kErrPeerTimeout = 4,   // a tensor-parallel peer's partial sums did not arrive within the wait bound
};

// Upper bound on mbarrier polls before a wait gives up (~1-2 s with back-off).
constexpr uint32_t kWaitPolls = 1u << 24;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false if the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 32) __nanosleep(64);
    }
    return false;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Global -> shared bulk copy on the TMA engine, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Asks the TMA engine to bring [src, src + bytes) into L2 (no shared-memory
// destination, no completion to wait for).  src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_relaxed_gpu(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 16-byte global -> shared async copy through L2 only (cp.async.cg), and the
// wait for all of this thread's outstanding copies.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// 4-byte global -> shared async copy (through L1: cp.async.ca; 4-byte aligned).
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void prefetch_l1(const void *p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

// Named barrier over `n` threads of the CTA (n a multiple of 32): wait, or
// arrive without waiting.
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void named_arrive(int id, int n) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Split thread-block-cluster barrier (all threads of every CTA take part).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The reference's warp reduction: v += __shfl_down_sync(v, o) for o = 16 .. 1
// (lane 0 holds the sum), each add rounded.
__device__ __forceinline__ float shfl_down_tree(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ void raise_error(int *status, int code) {
    if (status) atomicOr(status, 1 << code);
}

// Quantises one block of 32 floats to Q8_1 exactly as the reference
// (bmo_cuda_kernels.cu:529-558): d = amax/127 (IEEE), id = d ? 1/d : 0,
// q = clamp(roundf(v*id)), s = sequential fp32 sum v[0] + ... + v[31].
// Writes the 32 int8 values and returns (half(d), half(s)).
__device__ __forceinline__ __half2 quant_block_q8_1(const float (&v)[32], int8_t (&q)[32]) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(v[j]);
        amax = a > amax ? a : amax;
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        int qi = __float2int_rz(roundf(__fmul_rn(v[j], id)));
        qi = max(-128, min(127, qi));
        q[j] = static_cast<int8_t>(qi);
        sum = __fadd_rn(sum, v[j]);
    }
    return __halves2half2(__float2half_rn(d), __float2half_rn(sum));
}

// Q4_0 quantisation of one 32-value block held one value per lane (ggml
// quantize_row_q4_0_ref: signed max by magnitude, first occurrence; d = max/-8;
// q = min(15, trunc(x*id + 8.5)); byte j = q[j] | q[j+16] << 4).  All 32
// lanes must call it.
__device__ __forceinline__ void warp_store_q4_0(float x, int lane, uint8_t *qs_dst, __half *d_dst) {
    float am = fabsf(x), mx = x;
    int idx = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oam = __shfl_xor_sync(0xffffffffu, am, o);
        const float omx = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oidx = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oam > am || (oam == am && oidx < idx)) { am = oam; mx = omx; idx = oidx; }
    }
    const float d = __fdiv_rn(mx, -8.0f);
    const float id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;
    int q = __float2int_rz(__fadd_rn(__fmul_rn(x, id), 8.5f));
    q = min(15, q);
    const int hi = __shfl_down_sync(0xffffffffu, q, 16);
    if (lane < 16) qs_dst[lane] = static_cast<uint8_t>(q | (hi << 4));
    if (lane == 0) *d_dst = __float2half_rn(d);
}

}  // namespace bmo
