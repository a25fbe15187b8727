// sd_nccl.cu -- NCCL for tensor-parallel contexts, loaded at run time (dlopen) so that single-GPU use of
// the library has no NCCL dependency.  One process per GPU: the caller creates one communicator per
// rank from a unique id that it distributes itself (e.g. over torch.distributed).
#include <dlfcn.h>
#include <cstring>
#include <mutex>
#include <nccl.h>

#include "sd_host.h"
#include "specdec_b200.h"

namespace sd {

namespace {

struct NcclApi {
    bool tried = false, ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi& api() {
    static NcclApi a;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (a.tried) return a;
    a.tried = true;
    // a libnccl already loaded into the process (e.g. by torch) is reused through its soname
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_reduce && a.error_string;
    return a;
}

int nccl_fail(ncclResult_t r, const char* what) {
    NcclApi& a = api();
    return fail(SD_ERR_CUDA, "%s: %s", what, a.error_string ? a.error_string(r) : "nccl error");
}

}  // namespace

// Sum-all-reduce of n fp32 values in place on stream st.
int nccl_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st) {
    NcclApi& a = api();
    if (!a.ok) return fail(SD_ERR_UNSUPPORTED, "NCCL is not available");
    ncclResult_t r = a.all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st);
    return r == ncclSuccess ? SD_OK : nccl_fail(r, "ncclAllReduce");
}

}  // namespace sd

using namespace sd;

extern "C" {

int sd_nccl_unique_id(void* id_out) {
    clear_error();
    if (!id_out) return fail(SD_ERR_INVALID, "null argument");
    NcclApi& a = api();
    if (!a.ok) return fail(SD_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
    ncclUniqueId id;
    ncclResult_t r = a.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id_out, &id, sizeof(id));
    return SD_OK;
}

int sd_nccl_comm_create(const void* id, int nranks, int rank, int device, void** comm_out) {
    clear_error();
    if (!id || !comm_out || nranks < 1 || rank < 0 || rank >= nranks) return fail(SD_ERR_INVALID, "bad arguments");
    NcclApi& a = api();
    if (!a.ok) return fail(SD_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    ncclResult_t r = a.comm_init_rank(&comm, nranks, uid, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm_out = comm;
    return SD_OK;
}

void sd_nccl_comm_destroy(void* comm) {
    NcclApi& a = api();
    if (comm && a.ok) a.comm_destroy(static_cast<ncclComm_t>(comm));
}

}  // extern "C"
