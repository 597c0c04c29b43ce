// gguf.cpp -- GGUF container reader (header, key/values, tensor infos, aligned
// data section), written from the published GGUF layout.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace bmo {

size_t q4_0_tiled_bytes_host(int64_t rows, int64_t cols, int perm, int swiglu_f);  // tiling.cpp

namespace {

enum : uint32_t {
    kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kString, kArray, kU64, kI64, kF64
};

struct Reader {
    const uint8_t *p, *end;
    template <class T> T get() {
        if (static_cast<size_t>(end - p) < sizeof(T)) throw std::runtime_error("gguf: truncated header");
        T v;
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    void skip(uint64_t n) {
        if (static_cast<uint64_t>(end - p) < n) throw std::runtime_error("gguf: truncated header");
        p += n;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > (1u << 20)) throw std::runtime_error("gguf: implausible string length");
        const char *s = reinterpret_cast<const char *>(p);
        skip(n);
        return std::string(s, n);
    }
    void skip_value(uint32_t type, int depth = 0) {
        static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (depth > 4) throw std::runtime_error("gguf: nested arrays too deep");
        if (type == kString) { str(); return; }
        if (type == kArray) {
            const uint32_t et = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            if (et != kString && et != kArray && et <= kF64) { skip(n * static_cast<uint64_t>(sz[et])); return; }
            for (uint64_t i = 0; i < n; ++i) skip_value(et, depth + 1);
            return;
        }
        if (type > kF64) throw std::runtime_error("gguf: unknown value type");
        skip(static_cast<uint64_t>(sz[type]));
    }
};

}  // namespace

int64_t ggml_row_bytes(int type, int64_t ne0) {
    switch (type) {
    case 0: case 26: return ne0 * 4;      // F32, I32
    case 1: case 30: return ne0 * 2;      // F16, BF16
    case 2: return ne0 / 32 * 18;          // Q4_0
    case 8: return ne0 / 32 * 34;          // Q8_0
    case 24: return ne0;                   // I8
    case 25: return ne0 * 2;               // I16
    case 27: case 28: return ne0 * 8;      // I64, F64
    default: return -1;
    }
}

GgufFile::~GgufFile() {
    if (map_) munmap(map_, size_);
}

void GgufFile::open(const std::string &path) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw std::runtime_error("gguf: cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        throw std::runtime_error("gguf: cannot stat or file too small: " + path);
    }
    size_ = static_cast<size_t>(st.st_size);
    void *m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) throw std::runtime_error("gguf: mmap failed: " + path);
    map_ = static_cast<uint8_t *>(m);

    Reader r{map_, map_ + size_};
    if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("gguf: bad magic in " + path);
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) throw std::runtime_error("gguf: unsupported version");
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (n_tensors > 1000000 || n_kv > 1000000) throw std::runtime_error("gguf: implausible counts");
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; ++i) {
        const std::string key = r.str();
        const uint32_t type = r.get<uint32_t>();
        if (key == "general.alignment" && type == kU32) {
            alignment = r.get<uint32_t>();
            if (alignment == 0 || (alignment & (alignment - 1))) throw std::runtime_error("gguf: bad alignment");
        } else if (key == "bmo.tiled.version" && type == kU32) {
            tiled_version_ = r.get<uint32_t>();
            if (tiled_version_ != 1)
                throw std::runtime_error("gguf: repacked with tiled layout version " + std::to_string(tiled_version_) +
                                         "; this build reads version 1");
        } else {
            r.skip_value(type);
        }
    }
    tensors_.resize(n_tensors);
    std::vector<uint64_t> offsets(n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
        GgufTensor &t = tensors_[i];
        t.name = r.str();
        t.n_dims = static_cast<int>(r.get<uint32_t>());
        if (t.n_dims < 1 || t.n_dims > 4) throw std::runtime_error("gguf: bad rank for " + t.name);
        for (int d = 0; d < t.n_dims; ++d) t.ne[d] = static_cast<int64_t>(r.get<uint64_t>());
        t.type = static_cast<int>(r.get<uint32_t>());
        offsets[i] = r.get<uint64_t>();
    }
    const size_t header = static_cast<size_t>(r.p - map_);
    const size_t data0 = (header + alignment - 1) / alignment * alignment;
    for (uint64_t i = 0; i < n_tensors; ++i) {
        GgufTensor &t = tensors_[i];
        const int64_t rb = ggml_row_bytes(t.type, t.ne[0]);
        if (rb >= 0) {
            for (int d = 0; d < 4; ++d)
                if (t.ne[d] < 0) throw std::runtime_error("gguf: negative dim in " + t.name);
            t.nbytes = static_cast<size_t>(rb) * static_cast<size_t>(t.rows());
            if (data0 + offsets[i] + t.nbytes > size_) throw std::runtime_error("gguf: tensor data past EOF: " + t.name);
            t.data = map_ + data0 + offsets[i];
        }
        index_[t.name] = i;
    }
    if (tiled_version_) attach_tiled();
}

// Pairs each "bmo.tiled:N" with its descriptor and hangs it on N, adding N
// (without raw rows) when the file dropped them.
void GgufFile::attach_tiled() {
    static const std::string kTiled = "bmo.tiled:", kDesc = "bmo.tiled_desc:";
    const size_t n0 = tensors_.size();
    std::vector<GgufTensor> added;
    for (size_t i = 0; i < n0; ++i) {
        const GgufTensor &tt = tensors_[i];
        if (tt.name.compare(0, kTiled.size(), kTiled) != 0) continue;
        const std::string name = tt.name.substr(kTiled.size());
        auto di = index_.find(kDesc + name);
        if (tt.type != 24 || !tt.data || di == index_.end())
            throw std::runtime_error("gguf: tiled tensor without its descriptor: " + name);
        const GgufTensor &d = tensors_[di->second];
        if (d.type != 26 || !d.data || d.ne[0] != 4) throw std::runtime_error("gguf: bad tiled descriptor: " + name);
        int32_t v[4];
        std::memcpy(v, d.data, sizeof(v));
        const int64_t cols = v[0], rows = v[1];
        const int perm = v[2], f = v[3];
        const size_t want = q4_0_tiled_bytes_host(rows, cols, perm, f);
        if (want == 0 || want != tt.nbytes) throw std::runtime_error("gguf: tiled tensor size does not match its shape: " + name);
        auto ri = index_.find(name);
        GgufTensor *raw = ri == index_.end() ? nullptr : &tensors_[ri->second];
        if (raw && (raw->type != 2 || raw->ne[0] != cols || raw->rows() != rows))
            throw std::runtime_error("gguf: tiled tensor does not match its raw rows: " + name);
        GgufTensor v2;
        GgufTensor &t = raw ? *raw : v2;
        if (!raw) {
            t.name = name;
            t.type = 2;  // Q4_0
            t.n_dims = 2;
            t.ne[0] = cols;
            t.ne[1] = rows;
            t.nbytes = static_cast<size_t>(rows * (cols / 32) * 18);
        }
        t.tiled = tt.data;
        t.tiled_bytes = tt.nbytes;
        t.tiled_perm = perm;
        t.tiled_f = f;
        if (!raw) added.push_back(t);
    }
    for (auto &t : added) {
        index_[t.name] = tensors_.size();
        tensors_.push_back(t);
    }
}

const GgufTensor *GgufFile::find(const std::string &name) const {
    auto it = index_.find(name);
    if (it == index_.end()) return nullptr;
    const GgufTensor *t = &tensors_[it->second];
    return (t->data || t->tiled) ? t : nullptr;
}

int32_t GgufFile::scalar_i32(const std::string &name, int32_t fallback) const {
    // Like the reference loader (bmo.cpp:62-70) the first four bytes are read
    // whatever the element type.
    const GgufTensor *t = find(name);
    if (!t || !t->data || t->nbytes < 4) return fallback;
    int32_t v;
    std::memcpy(&v, t->data, 4);
    return v;
}

float GgufFile::scalar_f32(const std::string &name, float fallback) const {
    const GgufTensor *t = find(name);
    if (!t || !t->data || t->nbytes < 4) return fallback;
    float v;
    std::memcpy(&v, t->data, 4);
    return v;
}

}  // namespace bmo
