// NCCL through dlopen: the few entry points the tensor-parallel decoder uses.
#include "wl_nccl.h"
#include <dlfcn.h>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <nccl.h>
#include "wl_common.h"

namespace wl {

namespace {
struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    std::string load_error;
};

const Nccl& nccl()
{
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = nullptr;
        const char* env = getenv("WL_NCCL_LIBRARY");
        for (const char* name : {env, "libnccl.so.2", "libnccl.so"}) {
            if (!name || !*name) continue;
            h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
            if (h) break;
        }
        if (!h) {
            const char* e = dlerror();
            n.load_error = std::string("NCCL (libnccl.so.2) cannot be loaded: ") + (e ? e : "not found");
            return;
        }
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn && n.load_error.empty()) n.load_error = std::string("NCCL has no symbol ") + name;
        };
        sym(n.get_unique_id, "ncclGetUniqueId");
        sym(n.comm_init_rank, "ncclCommInitRank");
        sym(n.comm_destroy, "ncclCommDestroy");
        sym(n.all_reduce, "ncclAllReduce");
        sym(n.all_gather, "ncclAllGather");
        sym(n.error_string, "ncclGetErrorString");
    });
    if (!n.load_error.empty()) WL_THROW(WL_ENCCL, n.load_error);
    return n;
}

void check(ncclResult_t r, const char* what)
{
    if (r == ncclSuccess) return;
    const Nccl& n = nccl();
    WL_THROW(WL_ENCCL, std::string(what) + " failed: " + (n.error_string ? n.error_string(r) : "error") + " (" +
                           std::to_string((int)r) + ")");
}
}  // namespace

void Comm::unique_id(uint8_t out[TP_ID_BYTES])
{
    static_assert(sizeof(ncclUniqueId) == TP_ID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    check(nccl().get_unique_id(&id), "ncclGetUniqueId");
    memcpy(out, &id, TP_ID_BYTES);
}

Comm::Comm(const uint8_t id[TP_ID_BYTES], int size_, int rank_) : size(size_), rank(rank_)
{
    ncclUniqueId u;
    memcpy(&u, id, TP_ID_BYTES);
    ncclComm_t c = nullptr;
    check(nccl().comm_init_rank(&c, size, u, rank), "ncclCommInitRank");
    comm_ = c;
}

Comm::~Comm()
{
    if (comm_) nccl().comm_destroy((ncclComm_t)comm_);
}

void Comm::allreduce_sum(float* buf, int64_t n, cudaStream_t s)
{
    check(nccl().all_reduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, (ncclComm_t)comm_, s), "ncclAllReduce");
}

void Comm::allreduce_max(int32_t* buf, int64_t n, cudaStream_t s)
{
    check(nccl().all_reduce(buf, buf, (size_t)n, ncclInt32, ncclMax, (ncclComm_t)comm_, s), "ncclAllReduce");
}

void Comm::allgather(const void* send, void* recv, int64_t bytes_per_rank, cudaStream_t s)
{
    check(nccl().all_gather(send, recv, (size_t)bytes_per_rank, ncclUint8, (ncclComm_t)comm_, s), "ncclAllGather");
}

}  // namespace wl
