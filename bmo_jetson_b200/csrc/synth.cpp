// synth.cpp -- deterministic synthetic tensors for benchmark and test models,
// and ggml's Q4_0 reference quantiser.
//
// Values come from a counter-based generator (splitmix64 finaliser over
// (seed, stream, index)) and Box-Muller, so any element range can be filled
// in parallel and the same (seed, stream) gives the same tensor on any host.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/bmo_ext.h"

namespace {

inline uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

struct Gen {
    uint64_t key;
    Gen(uint64_t seed, uint64_t stream) : key(mix64(seed) ^ mix64(stream + 0x632be59bd9b4e019ull)) {}
    // uniform in (0, 1]
    double uniform(uint64_t i) const { return (static_cast<double>(mix64(key ^ mix64(i)) >> 11) + 1.0) * 0x1.0p-53; }
    // Box-Muller pair p gives elements 2p (cosine branch) and 2p + 1 (sine branch).
    void normal_pair(uint64_t p, double &z0, double &z1) const {
        const double r = std::sqrt(-2.0 * std::log(uniform(2 * p)));
        const double t = 6.283185307179586 * uniform(2 * p + 1);
        z0 = r * std::cos(t);
        z1 = r * std::sin(t);
    }
    double normal(uint64_t i) const {
        double z0, z1;
        normal_pair(i >> 1, z0, z1);
        return (i & 1) ? z1 : z0;
    }
};

// Runs f(i) for i in [0, n) on up to hardware_concurrency threads, with at
// least `grain` items per thread.
template <class F>
void parallel_for(long long n, long long grain, F f) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const long long nt = std::min<long long>(hw, std::max<long long>(1, n / grain));
    std::vector<std::thread> ts;
    for (long long t = 0; t < nt; ++t)
        ts.emplace_back([=] {
            for (long long i = n * t / nt; i < n * (t + 1) / nt; ++i) f(i);
        });
    for (auto &th : ts) th.join();
}

// ggml quantize_row_q4_0_ref: per 32-block, the value of largest magnitude
// (first occurrence) sets d = max / -8; q = min(15, trunc(x / d + 8.5)).
void q4_0_block(const float *x, uint8_t *out) {
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < 32; ++j)
        if (amax < std::fabs(x[j])) {
            amax = std::fabs(x[j]);
            mx = x[j];
        }
    const float d = mx / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const __half hd = __float2half_rn(d);
    std::memcpy(out, &hd, 2);
    for (int j = 0; j < 16; ++j) {
        const float p0 = x[j] * id;
        const float p1 = x[16 + j] * id;
        const float s0 = p0 + 8.5f;
        const float s1 = p1 + 8.5f;
        const int q0 = std::min(15, static_cast<int>(static_cast<int8_t>(s0)));
        const int q1 = std::min(15, static_cast<int>(static_cast<int8_t>(s1)));
        out[2 + j] = static_cast<uint8_t>(q0 | (q1 << 4));
    }
}

}  // namespace

extern "C" {

void bmo_quantize_q4_0_ref(const float *x, long long n, uint8_t *out) {
    for (long long b = 0; b < n / 32; ++b) q4_0_block(x + b * 32, out + b * 18);
}

void bmo_synth_normal_f32(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, float *out) {
    const Gen g(seed, stream);
    parallel_for(n, 4096, [&](long long i) {
        out[i] = static_cast<float>(static_cast<double>(mean) + static_cast<double>(sigma) * g.normal(static_cast<uint64_t>(i)));
    });
}

void bmo_synth_f16(uint64_t seed, uint64_t stream, long long n, float mean, float sigma, uint16_t *out) {
    const Gen g(seed, stream);
    parallel_for((n + 1) / 2, 2048, [&](long long p) {
        double z[2];
        g.normal_pair(static_cast<uint64_t>(p), z[0], z[1]);
        for (int k = 0; k < 2 && 2 * p + k < n; ++k) {
            const float v = static_cast<float>(static_cast<double>(mean) + static_cast<double>(sigma) * z[k]);
            const __half h = __float2half_rn(v);
            std::memcpy(&out[2 * p + k], &h, 2);
        }
    });
}

void bmo_synth_q4_0(uint64_t seed, uint64_t stream, long long rows, long long cols, float sigma, uint8_t *out) {
    const Gen g(seed, stream);
    const long long nb = cols / 32;
    parallel_for(rows, 1, [&](long long r) {
        float blk[32];
        for (long long b = 0; b < nb; ++b) {
            const uint64_t base = static_cast<uint64_t>(r * cols + b * 32);  // even: cols % 32 == 0
            for (int j = 0; j < 32; j += 2) {
                double z0, z1;
                g.normal_pair((base + j) >> 1, z0, z1);
                blk[j] = static_cast<float>(static_cast<double>(sigma) * z0);
                blk[j + 1] = static_cast<float>(static_cast<double>(sigma) * z1);
            }
            q4_0_block(blk, out + (r * nb + b) * 18);
        }
    });
}

}  // extern "C"
