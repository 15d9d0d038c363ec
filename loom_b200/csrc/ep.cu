// ep.cu -- expert parallelism over NCCL (NVLink/NVSwitch inside one node).
//
// Experts are sharded contiguously: rank r holds experts
// [r*E/R, (r+1)*E/R). Routing is replicated (every rank computes identical
// logits and ids), each rank runs only its local experts, and the combine is a
// sum-all-reduce of the [T, dim] partial outputs (the residual is added on one
// rank only). NCCL is loaded at run time (dlopen) so the process shares the
// copy the framework already loaded, if any.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>

#include "../../include/loom_cuda.h"
#include "ep.cuh"

namespace loom {
namespace {

struct Nccl {
    void *h = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*groupStart)() = nullptr;
    ncclResult_t (*groupEnd)() = nullptr;
    const char *(*getErrorString)(ncclResult_t) = nullptr;
} N;

ncclComm_t g_comm = nullptr;
int g_rank = 0, g_size = 1;
std::string g_ep_err;

bool load_nccl(std::string &err) {
    if (N.h) return true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        err = std::string("cannot load NCCL: ") + dlerror();
        return false;
    }
    N.getUniqueId = reinterpret_cast<decltype(N.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    N.commInitRank = reinterpret_cast<decltype(N.commInitRank)>(dlsym(h, "ncclCommInitRank"));
    N.allReduce = reinterpret_cast<decltype(N.allReduce)>(dlsym(h, "ncclAllReduce"));
    N.commDestroy = reinterpret_cast<decltype(N.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    N.getErrorString = reinterpret_cast<decltype(N.getErrorString)>(dlsym(h, "ncclGetErrorString"));
    N.send = reinterpret_cast<decltype(N.send)>(dlsym(h, "ncclSend"));
    N.recv = reinterpret_cast<decltype(N.recv)>(dlsym(h, "ncclRecv"));
    N.groupStart = reinterpret_cast<decltype(N.groupStart)>(dlsym(h, "ncclGroupStart"));
    N.groupEnd = reinterpret_cast<decltype(N.groupEnd)>(dlsym(h, "ncclGroupEnd"));
    if (!N.getUniqueId || !N.commInitRank || !N.allReduce || !N.commDestroy || !N.getErrorString || !N.send ||
        !N.recv || !N.groupStart || !N.groupEnd) {
        err = "NCCL library lacks an expected symbol";
        return false;
    }
    N.h = h;
    return true;
}

}  // namespace

bool ep_active() { return g_comm != nullptr && g_size > 1; }
int ep_rank() { return g_rank; }
int ep_size() { return g_size; }

int ep_allreduce_sum(float *buf, size_t n, cudaStream_t st, std::string &err) {
    if (!ep_active()) return LOOM_CUDA_OK;
    ncclResult_t r = N.allReduce(buf, buf, n, ncclFloat32, ncclSum, g_comm, st);
    if (r != ncclSuccess) {
        err = std::string("ncclAllReduce: ") + N.getErrorString(r);
        return LOOM_CUDA_ERROR;
    }
    return LOOM_CUDA_OK;
}

int ep_alltoallv(const void *send, const size_t *soff, const size_t *scnt, void *recv, const size_t *roff,
                 const size_t *rcnt, size_t unit_bytes, cudaStream_t st, std::string &err) {
    const int world = ep_active() ? g_size : 1, me = ep_active() ? g_rank : 0;
    const uint8_t *s = static_cast<const uint8_t *>(send);
    uint8_t *d = static_cast<uint8_t *>(recv);
    if (scnt[me] != rcnt[me]) {
        err = "all-to-all: the run to this rank and the run from it differ in size";
        return LOOM_CUDA_ERROR;
    }
    if (scnt[me]) {
        cudaError_t e = cudaMemcpyAsync(d + roff[me] * unit_bytes, s + soff[me] * unit_bytes, scnt[me] * unit_bytes,
                                        cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) {
            err = std::string("all-to-all self copy: ") + cudaGetErrorString(e);
            return LOOM_CUDA_ERROR;
        }
    }
    if (world == 1) return LOOM_CUDA_OK;
    ncclResult_t r = N.groupStart();
    for (int p = 0; p < world && r == ncclSuccess; p++) {
        if (p == me) continue;
        if (scnt[p]) r = N.send(s + soff[p] * unit_bytes, scnt[p] * unit_bytes, ncclUint8, p, g_comm, st);
        if (r == ncclSuccess && rcnt[p]) r = N.recv(d + roff[p] * unit_bytes, rcnt[p] * unit_bytes, ncclUint8, p, g_comm, st);
    }
    const ncclResult_t r2 = N.groupEnd();
    if (r == ncclSuccess) r = r2;
    if (r != ncclSuccess) {
        err = std::string("ncclSend/ncclRecv: ") + N.getErrorString(r);
        return LOOM_CUDA_ERROR;
    }
    return LOOM_CUDA_OK;
}

}  // namespace loom

using namespace loom;

extern "C" {

int loom_cuda_ep_unique_id(void *out, size_t bytes) {
    if (bytes < sizeof(ncclUniqueId)) return LOOM_CUDA_DECLINED;
    if (!load_nccl(g_ep_err)) return LOOM_CUDA_DECLINED;
    ncclUniqueId id;
    if (N.getUniqueId(&id) != ncclSuccess) return LOOM_CUDA_ERROR;
    memcpy(out, &id, sizeof id);
    return LOOM_CUDA_OK;
}

int loom_cuda_ep_init(int nranks, int rank, const void *id_bytes, size_t bytes) {
    if (nranks < 1 || rank < 0 || rank >= nranks || bytes < sizeof(ncclUniqueId)) return LOOM_CUDA_DECLINED;
    if (nranks == 1) {
        g_rank = 0;
        g_size = 1;
        return LOOM_CUDA_OK;
    }
    if (!load_nccl(g_ep_err)) return LOOM_CUDA_DECLINED;
    ncclUniqueId id;
    memcpy(&id, id_bytes, sizeof id);
    ncclComm_t c = nullptr;
    ncclResult_t r = N.commInitRank(&c, nranks, id, rank);
    if (r != ncclSuccess) {
        g_ep_err = std::string("ncclCommInitRank: ") + N.getErrorString(r);
        return LOOM_CUDA_ERROR;
    }
    g_comm = c;
    g_rank = rank;
    g_size = nranks;
    return LOOM_CUDA_OK;
}

void loom_cuda_ep_shutdown(void) {
    if (g_comm) N.commDestroy(g_comm);
    g_comm = nullptr;
    g_rank = 0;
    g_size = 1;
}

int loom_cuda_ep_rank(void) { return g_rank; }
int loom_cuda_ep_size(void) { return g_size; }

}  // extern "C"
