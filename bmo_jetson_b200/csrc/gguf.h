// gguf.h -- read-only GGUF (v2/v3) container reader over an mmap'd file.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace bmo {

struct GgufTensor {
    std::string name;
    int type = -1;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    const uint8_t *data = nullptr;  // null for a Q4_0 matrix stored only in tiled form
    size_t nbytes = 0;
    // the matrix in the device's row-tile layout (a repacked file), or null
    const uint8_t *tiled = nullptr;
    size_t tiled_bytes = 0;
    int tiled_perm = -1, tiled_f = 0;
    int64_t rows() const { return ne[1] * ne[2] * ne[3]; }
};

// Bytes per row of ne0 elements for the ggml types this engine reads, or -1.
int64_t ggml_row_bytes(int type, int64_t ne0);

class GgufFile {
public:
    GgufFile() = default;
    ~GgufFile();
    GgufFile(const GgufFile &) = delete;
    GgufFile &operator=(const GgufFile &) = delete;

    // Throws std::runtime_error with a description on any format problem.
    void open(const std::string &path);
    // bmo.tiled.version of a repacked file (0 for a plain GGUF).
    uint32_t tiled_version() const { return tiled_version_; }
    const GgufTensor *find(const std::string &name) const;
    const std::vector<GgufTensor> &tensors() const { return tensors_; }
    int32_t scalar_i32(const std::string &name, int32_t fallback) const;
    float scalar_f32(const std::string &name, float fallback) const;

private:
    uint8_t *map_ = nullptr;
    size_t size_ = 0;
    std::vector<GgufTensor> tensors_;
    std::unordered_map<std::string, size_t> index_;
    uint32_t tiled_version_ = 0;
    void attach_tiled();
};

}  // namespace bmo
