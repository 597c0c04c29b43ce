// tiling.cpp -- the row-tile layout of Q4_0 weights (layout.h) computed on the
// host, for offline repacking: the same bytes as the load-time device repack
// (kernels/misc.cu, repack_q4_0_kernel), padding included, so a repacked GGUF
// can be copied into the weight arena as it is.
#include <cuda_fp16.h>
#include <vector_types.h>

#include <cstring>

#include "../../include/bmo_ext.h"
#include "layout.h"

namespace bmo {

// Bytes of the tiled form of a rows x cols Q4_0 matrix, or 0 for a shape the
// GEMV does not take.
size_t q4_0_tiled_bytes_host(int64_t rows, int64_t cols, int perm, int swiglu_f) {
    if (rows <= 0 || cols <= 0 || cols % 32) return 0;
    if (perm == kPermSwiGLU && (swiglu_f <= 0 || swiglu_f % 16 || rows != 2LL * swiglu_f)) return 0;
    if (perm != kPermSwiGLU && perm != kPermIdentity) return 0;
    const int64_t nb = cols / 32;
    const int64_t nbx = (nb + kChunkBlocks - 1) / kChunkBlocks * kChunkBlocks;
    const int64_t n_tiles = perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows;
    return static_cast<size_t>(n_tiles * (nbx / kChunkBlocks) * kChunkBytes);
}

// Tile t's chunk c holds blocks 8c..8c+7 of its 32 rows: row lane l of the
// tile is row 32 t + l (identity) or, for the SwiGLU pairing, gate row
// 16 t + l (l < 16) and up row F + 16 t + (l - 16).  Missing rows and blocks
// past the row length are zero scales with nibbles 8.
void q4_0_tile_host(const uint8_t *raw, int64_t rows, int64_t cols, int perm, int swiglu_f, uint8_t *dst) {
    const int64_t nb = cols / 32;
    const int64_t nbx = (nb + kChunkBlocks - 1) / kChunkBlocks * kChunkBlocks;
    const int64_t cpt = nbx / kChunkBlocks;
    const int64_t n_tiles = perm == kPermSwiGLU ? swiglu_f / 16 : (rows + kTileRows - 1) / kTileRows;
    for (int64_t t = 0; t < n_tiles; ++t) {
        for (int64_t b = 0; b < nbx; ++b) {
            uint8_t *chunk = dst + (t * cpt + b / kChunkBlocks) * kChunkBytes;
            const int64_t blk = b % kChunkBlocks;
            for (int lane = 0; lane < kTileRows; ++lane) {
                int64_t r;
                bool live;
                if (perm == kPermSwiGLU) {
                    r = lane < 16 ? t * 16 + lane : swiglu_f + t * 16 + (lane - 16);
                    live = t * 16 + (lane & 15) < swiglu_f;
                } else {
                    r = t * kTileRows + lane;
                    live = true;
                }
                live = live && r < rows && b < nb;
                uint8_t *qs = chunk + blk * 512 + lane * 16;
                uint8_t *dd = chunk + kChunkQsBytes + blk * 64 + lane * 2;
                if (live) {
                    const uint8_t *src = raw + (r * nb + b) * 18;
                    std::memcpy(dd, src, 2);
                    std::memcpy(qs, src + 2, 16);
                } else {
                    dd[0] = dd[1] = 0;
                    std::memset(qs, 0x88, 16);
                }
            }
        }
    }
}

}  // namespace bmo

extern "C" {

long long bmo_q4_0_tile_host(const uint8_t *raw, long long rows, long long cols, int perm, int swiglu_f,
                             uint8_t *dst) {
    const size_t bytes = bmo::q4_0_tiled_bytes_host(rows, cols, perm, swiglu_f);
    if (bytes == 0) return -1;
    if (!dst) return static_cast<long long>(bytes);
    if (!raw) return -1;
    bmo::q4_0_tile_host(raw, rows, cols, perm, swiglu_f, dst);
    return static_cast<long long>(bytes);
}

}  // extern "C"
