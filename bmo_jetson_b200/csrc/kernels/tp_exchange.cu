// tp_exchange.cu -- the tensor-parallel sum over NVLink peer memory, fused
// with the residual add: y = resid + fl(sum over ranks of the split
// projection's double partial sums), summed in rank order so that every rank
// computes the same bits.  Replaces an NCCL all-reduce plus a separate
// residual kernel with one small kernel that exchanges flags and reads the
// peers' partial buffers directly (plain loads; no multicast).
//
// Protocol (exchange number e, the same on every rank because all ranks run
// the same op sequence; each CTA derives it from an arrival counter that the
// kTpCtas CTAs of every launch bump once each): after the producing GEMV has
// completed (griddepcontrol.wait), CTA 0 publishes e into this rank's arrival
// word of every peer's block with a system-scope release; in every CTA,
// threads 1..size-1 each wait, bounded by %globaltimer, until one peer's word
// in this rank's block reaches e (system-scope acquire).  Then every thread
// re-reads the words with acquire semantics, loads its elements of all ranks'
// buffers at once and sums them in rank order.  A rank
// only overwrites a buffer two exchanges later, and it cannot start exchange
// e + 1 before every peer has published e + 1, which each peer does only after
// finishing its reads of exchange e -- so the two alternating buffers per rank
// never race.  A wait that runs out raises kErrPeerTimeout and the kernel
// returns without touching y; while that bit is set in the status word the
// following exchanges return at once, so a lost peer costs one bound, not one
// per exchange.
#include "common.cuh"
#include "../launch.h"

namespace bmo {

constexpr int kTpThreads = 256;
constexpr int kTpCtas = 8;                                            // 2048 threads per exchange
constexpr int kTpPerThread = kTpBufDoubles / (kTpThreads * kTpCtas);  // elements per thread, at most
constexpr uint64_t kTpWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(kTpThreads) tp_exchange_kernel(const __grid_constant__ TpExchangeArgs a) {
    __shared__ unsigned long long e_s;
    __shared__ int ok_s;
    const int tid = threadIdx.x;
    pdl_wait();  // the GEMV that wrote this rank's partial buffer has completed
    // the next GEMV's CTAs (which fit beside these 8) may launch and stream
    // their weights while this kernel waits for the peers
    pdl_launch_dependents();
    if (tid == 0) {
        // exchange number: the CTAs of the k-th launch draw arrival counts [kG, kG + G)
        const unsigned long long old = atomicAdd(a.seq, 1ull);
        e_s = old / kTpCtas + 1;
        // after a peer timed out, the rest of this call's exchanges return at once
        ok_s = (*reinterpret_cast<volatile int *>(a.status) & (1 << kErrPeerTimeout)) == 0;
        if (ok_s && blockIdx.x == 0) {
            __threadfence_system();
            for (int r = 0; r < a.size; ++r)
                if (r != a.rank) st_release_sys(a.flag_out[r], e_s);
        }
    }
    __syncthreads();
    if (!ok_s) return;
    const unsigned long long e = e_s;
    if (tid >= 1 && tid < a.size) {
        const int r = (a.rank + tid) % a.size;  // every peer, each by its own thread
        if (ld_acquire_sys(a.flag_in + r) < e) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_sys(a.flag_in + r) < e) {
                if (globaltimer_ns() - t0 > kTpWaitNs) {
                    ok_s = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
    }
    __syncthreads();
    if (!ok_s) {
        if (tid == 0) raise_error(a.status, kErrPeerTimeout);
        return;
    }
    // this thread's own acquire of every word before its peer loads
    for (int r = 0; r < a.size; ++r)
        if (r != a.rank) (void)ld_acquire_sys(a.flag_in + r);
    // every rank's values of this thread's elements loaded before any is added
    // (one NVLink round trip), then summed in rank order
    const int i0 = blockIdx.x * kTpThreads + tid, stride = kTpThreads * kTpCtas;
    double v[kTpMaxRanks][kTpPerThread];
#pragma unroll
    for (int r = 0; r < kTpMaxRanks; ++r)
#pragma unroll
        for (int k = 0; k < kTpPerThread; ++k) {
            const int i = i0 + k * stride;
            v[r][k] = (r < a.size && i < a.n) ? __ldcg(a.part[r] + i) : 0.0;
        }
#pragma unroll
    for (int k = 0; k < kTpPerThread; ++k) {
        const int i = i0 + k * stride;
        if (i >= a.n) break;
        double acc = 0.0;
#pragma unroll
        for (int r = 0; r < kTpMaxRanks; ++r)
            if (r < a.size) acc += v[r][k];
        a.y[i] = __fadd_rn(__ldcg(a.resid + i), __double2float_rn(acc));
    }
}

cudaError_t launch_tp_exchange(const TpExchangeArgs &a, cudaStream_t s, bool pdl) {
    if (a.size < 2 || a.size > kTpMaxRanks || a.rank < 0 || a.rank >= a.size || a.n <= 0 || a.n > kTpBufDoubles)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kTpCtas);
    cfg.blockDim = dim3(kTpThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tp_exchange_kernel, a);
}

}  // namespace bmo
