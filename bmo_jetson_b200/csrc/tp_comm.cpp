// tp_comm.cpp -- NCCL through dlopen for the tensor-parallel mode.
#include "tp_comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <stdexcept>

namespace bmo {

namespace {

struct NcclApi {
    void *lib = nullptr;
    std::string error;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        a.lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!a.lib) {
            const char *e = dlerror();
            a.error = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown");
            return;
        }
        auto sym = [&](const char *n) {
            void *p = dlsym(a.lib, n);
            if (!p && a.error.empty()) a.error = std::string("libnccl.so.2 lacks ") + n;
            return p;
        };
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(sym("ncclGetUniqueId"));
        a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(sym("ncclCommInitRank"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(sym("ncclAllReduce"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(sym("ncclAllGather"));
        a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(sym("ncclCommDestroy"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(sym("ncclGetErrorString"));
    });
    return a;
}

void check(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return;
    const NcclApi &a = api();
    throw std::runtime_error(std::string(what) + ": " + (a.error_string ? a.error_string(r) : "NCCL error"));
}

const NcclApi &need() {
    const NcclApi &a = api();
    if (!a.error.empty()) throw std::runtime_error(a.error);
    return a;
}

}  // namespace

std::string tp_unavailable() { return api().error; }

void tp_unique_id(void *out) {
    static_assert(sizeof(ncclUniqueId) == kTpIdBytes, "NCCL unique id size");
    ncclUniqueId id;
    check(need().get_unique_id(&id), "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof id);
}

TpComm::TpComm(const void *id, int rank, int size) : rank_(rank), size_(size) {
    if (size < 1 || rank < 0 || rank >= size) throw std::runtime_error("tensor parallel: rank outside [0, size)");
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclComm_t c = nullptr;
    check(need().comm_init_rank(&c, size, uid, rank), "ncclCommInitRank");
    comm_ = c;
}

TpComm::~TpComm() {
    if (comm_) api().comm_destroy(static_cast<ncclComm_t>(comm_));
}

void TpComm::all_reduce_sum(double *buf, size_t n, cudaStream_t s) {
    check(need().all_reduce(buf, buf, n, ncclFloat64, ncclSum, static_cast<ncclComm_t>(comm_), s), "ncclAllReduce");
}

namespace {
void cuda_ok(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
// A device scratch and stream for the synchronous setup collectives.
struct SetupScratch {
    void *d = nullptr;
    cudaStream_t s = nullptr;
    explicit SetupScratch(size_t bytes) {
        cuda_ok(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "setup stream");
        cuda_ok(cudaMalloc(&d, bytes), "setup scratch");
    }
    ~SetupScratch() {
        if (d) cudaFree(d);
        if (s) cudaStreamDestroy(s);
    }
};
}  // namespace

void TpComm::all_gather_bytes(const void *send, void *recv, size_t bytes) {
    SetupScratch t(bytes * (static_cast<size_t>(size_) + 1));
    uint8_t *in = static_cast<uint8_t *>(t.d), *out = in + bytes;
    cuda_ok(cudaMemcpyAsync(in, send, bytes, cudaMemcpyHostToDevice, t.s), "all-gather input");
    check(need().all_gather(in, out, bytes, ncclUint8, static_cast<ncclComm_t>(comm_), t.s), "ncclAllGather");
    cuda_ok(cudaMemcpyAsync(recv, out, bytes * static_cast<size_t>(size_), cudaMemcpyDeviceToHost, t.s),
            "all-gather output");
    cuda_ok(cudaStreamSynchronize(t.s), "all-gather");
}

int TpComm::all_min(int v) {
    SetupScratch t(sizeof(int));
    cuda_ok(cudaMemcpyAsync(t.d, &v, sizeof v, cudaMemcpyHostToDevice, t.s), "all-min input");
    check(need().all_reduce(t.d, t.d, 1, ncclInt32, ncclMin, static_cast<ncclComm_t>(comm_), t.s), "ncclAllReduce");
    int r = 0;
    cuda_ok(cudaMemcpyAsync(&r, t.d, sizeof r, cudaMemcpyDeviceToHost, t.s), "all-min output");
    cuda_ok(cudaStreamSynchronize(t.s), "all-min");
    return r;
}

}  // namespace bmo
