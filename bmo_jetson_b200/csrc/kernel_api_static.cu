// kernel_api_static.cu -- bmo_k_gemv_q4_0_static: the GEMV of the kernel
// layer without caller-provided scratch.
//
// Some callers of a decode kernel cannot allocate device memory at the point
// where they run it: code inside a real-time audio callback that must not
// block, a host framework that owns every allocation through its own pool,
// or a process running under a device-memory cap that forbids further
// cudaMalloc calls.  For them the split-K partial sums, tile counters and
// status word of the GEMV live in a fixed buffer inside this library, sized
// once at load time and kept by every GPU that loads the library until the
// process exits.
//
// Rules for the caller:
//   * The buffer is shared by all calls on a device and keeps the previous
//     call's contents; the tile counters and status word are cleared (an
//     asynchronous memset on the caller's stream) before each launch, the
//     partial sums are always written before they are read.
//   * Calls whose kernels can overlap on the GPU (different streams, or no
//     ordering between them) race on the buffer and give wrong results;
//     issue them on one stream or order them with events.
//   * The first call on each device looks up the buffer's device address
//     (cudaGetSymbolAddress with that device current); make that first call
//     before any stream capture on that device.  The address is kept for the
//     life of the process: after cudaDeviceReset on a device it is stale, so
//     do not use this entry point on that device again.
//   * A call that breaks an argument rule is rejected before it touches the
//     shared buffer.
//   * Matrices whose scratch need exceeds BMO_K_GEMV_STATIC_SCRATCH_BYTES
//     are rejected with BMO_K_ERR_SCRATCH_TOO_SMALL; no memory is allocated
//     or freed by this entry point.
#include <climits>
#include <mutex>

#include "../../include/bmo_kernels.h"
#include "kernels/common.cuh"
#include "launch.h"

namespace bmo {
namespace {

// The fixed scratch: partial sums, then tile counters, then the status word.
static __device__ __align__(256) unsigned char g_gemv_scratch[BMO_K_GEMV_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
unsigned char *g_scratch_ptr[kMaxDevices] = {};

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Device address of g_gemv_scratch on the current device (looked up once).
cudaError_t scratch_for_current_device(unsigned char **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gemv_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = static_cast<unsigned char *>(p);
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace bmo

using namespace bmo;

extern "C" {

int bmo_k_gemv_q4_0_static(const void *tiled_dev, int rows, int cols, int perm, int swiglu_f, const float *x_dev,
                           const float *gamma_dev, float eps, const float *resid_dev, float *y_dev, void *q8_out_dev,
                           float *xn_out_dev, int grid, void *stream) {
    const size_t need = bmo_k_gemv_scratch_bytes(rows, cols, perm, swiglu_f);
    if (need == 0 || !gemv_kernel_args_ok(tiled_dev, rows, cols, perm, swiglu_f, x_dev, gamma_dev, y_dev, xn_out_dev))
        return static_cast<int>(cudaErrorInvalidValue);
    if (need > BMO_K_GEMV_STATIC_SCRATCH_BYTES) return BMO_K_ERR_SCRATCH_TOO_SMALL;
    unsigned char *scratch = nullptr;
    cudaError_t e = scratch_for_current_device(&scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    // Same layout as the caller-provided scratch of bmo_k_gemv_q4_0: partials,
    // then counters and the status word, which must start at zero.
    const int n_tiles = perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows;
    const int cpt = ((cols / 32) + kChunkBlocks - 1) / kChunkBlocks;
    const size_t part = align256(static_cast<size_t>(n_tiles) * (cpt + 1) * 32 * sizeof(double));
    e = cudaMemsetAsync(scratch + part, 0, need - part, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return static_cast<int>(e);
    return bmo_k_gemv_q4_0(tiled_dev, rows, cols, perm, swiglu_f, x_dev, gamma_dev, eps, resid_dev, y_dev, q8_out_dev,
                           xn_out_dev, scratch, need, grid, stream);
}

}  // extern "C"
