// nf_nccl.h -- NCCL, loaded with dlopen on first use, for the library's
// multi-GPU handles (expert parallelism in nf_ep.cu, tensor-parallel linears
// in nf_tp.cu).  A process that already loaded NCCL (e.g. through PyTorch)
// shares that copy, and processes that never use a multi-GPU handle never
// load it.
#pragma once

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

namespace nf {

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

inline NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) {
            api.why = "libnccl.so.2 not found";
            return;
        }
        auto sym = [&](const char* name) { return dlsym(lib, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.group_start && api.group_end &&
                 api.send && api.recv && api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks the point-to-point API";
    });
    return api;
}

inline const char* nccl_str(ncclResult_t r) { return nccl().error_string ? nccl().error_string(r) : "unknown"; }

// Every rank sends `bytes` bytes from host `mine` to every rank (its own
// slot included) and receives every rank's into host all[world][bytes]: a
// gather of small set-up records through `stage` (a device buffer of at
// least bytes * (world + 1) bytes, allocated before the communicator, so
// that every exchange has a buffer on every rank).  The sends and receives
// are posted whatever happened locally, so a rank whose copy failed never
// leaves the others waiting: its slot is cleared first, so the others then
// receive a zeroed record (records carry an `ok` word that reads as a
// failure when zero).  Returns false when this rank's copy or the exchange
// failed.
inline bool nccl_allgather_records(void* comm_v, uint8_t* stage, cudaStream_t st, int world, const void* mine,
                                   size_t bytes, void* all) {
    NcclApi& api = nccl();
    ncclComm_t comm = static_cast<ncclComm_t>(comm_v);
    if (!stage || !comm) return false;  // the same on every rank: no exchange is posted anywhere
    const bool local = cudaMemset(stage, 0, bytes) == cudaSuccess &&
                       cudaMemcpy(stage, mine, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
    if (!local) cudaGetLastError();
    ncclResult_t r = api.group_start();
    for (int p = 0; p < world && r == ncclSuccess; ++p) {
        r = api.send(stage, bytes, ncclUint8, p, comm, st);
        if (r == ncclSuccess) r = api.recv(stage + bytes * (p + 1), bytes, ncclUint8, p, comm, st);
    }
    const ncclResult_t r2 = api.group_end();
    const bool ok = r == ncclSuccess && r2 == ncclSuccess && cudaStreamSynchronize(st) == cudaSuccess &&
                    cudaMemcpy(all, stage + bytes, bytes * world, cudaMemcpyDeviceToHost) == cudaSuccess;
    return ok && local;
}

}  // namespace nf
