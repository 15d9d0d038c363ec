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

#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/loom_cuda.h"
#include "ep.cuh"
#include "kernels.cuh"

namespace loom {
namespace {

struct Nccl {
    void *h = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
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
    N.allGather = reinterpret_cast<decltype(N.allGather)>(dlsym(h, "ncclAllGather"));
    N.commDestroy = reinterpret_cast<decltype(N.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    N.getErrorString = reinterpret_cast<decltype(N.getErrorString)>(dlsym(h, "ncclGetErrorString"));
    N.send = reinterpret_cast<decltype(N.send)>(dlsym(h, "ncclSend"));
    N.recv = reinterpret_cast<decltype(N.recv)>(dlsym(h, "ncclRecv"));
    N.groupStart = reinterpret_cast<decltype(N.groupStart)>(dlsym(h, "ncclGroupStart"));
    N.groupEnd = reinterpret_cast<decltype(N.groupEnd)>(dlsym(h, "ncclGroupEnd"));
    if (!N.getUniqueId || !N.commInitRank || !N.allReduce || !N.allGather || !N.commDestroy || !N.getErrorString || !N.send ||
        !N.recv || !N.groupStart || !N.groupEnd) {
        err = "NCCL library lacks an expected symbol";
        return false;
    }
    N.h = h;
    return true;
}

// ---- one-shot combine over peer memory (NVLink / NVSwitch) ------------------------------
// For the small partials of decode (T x dim floats), an NCCL all-reduce costs
// far more than the bytes: each rank stores its partial straight into every
// rank's receive slot over NVLink, publishes an epoch flag on every rank
// (release, system scope), waits for every rank's flag on its own side
// (acquire, bounded), and sums the slots in rank order, so every rank gets
// the same bits. The epoch is a device counter each rank's kernel advances,
// so a CUDA graph replays it correctly; a ring of slots keeps a fast rank
// from overwriting a slot a slow rank is still reading.
constexpr int P2P_SLOTS = 4;
constexpr size_t P2P_MAXN = 16384;  // floats per combine
constexpr int P2P_MAX_RANKS = 8;
constexpr uint32_t P2P_POLLS = 1u << 22;

struct P2PArgs {
    float *peer_recv[P2P_MAX_RANKS];                // every rank's receive slots [SLOTS][R][MAXN]
    unsigned long long *peer_flags[P2P_MAX_RANKS];  // every rank's flags [SLOTS][R]
    unsigned long long *epoch;                      // this rank's counter
    int *err;
    int me, R;
};
struct P2PState {
    bool ready = false;
    void *base = nullptr;  // own allocation: receive slots, then flags
    unsigned long long *epoch = nullptr;
    int *err = nullptr;
    void *peer_base[P2P_MAX_RANKS] = {};
    P2PArgs args{};
} P2;

__global__ void __launch_bounds__(1024) k_p2p_combine(P2PArgs a, float *buf, int n) {
    __shared__ unsigned long long e_s;
    __shared__ int ok_s;
    const int tid = threadIdx.x;
    if (tid == 0) {
        e_s = *reinterpret_cast<volatile unsigned long long *>(a.epoch) + 1;
        ok_s = 1;
    }
    __syncthreads();
    const unsigned long long e = e_s;
    const int slot = (int)(e % P2P_SLOTS);
    for (int p = 0; p < a.R; p++) {  // push: this rank's partial into slot [slot][me] of every rank
        float4 *dst = reinterpret_cast<float4 *>(a.peer_recv[p] + ((size_t)slot * a.R + a.me) * P2P_MAXN);
        const float4 *src = reinterpret_cast<const float4 *>(buf);
        for (int i = tid; i < n / 4; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    if (tid < a.R) {  // publish on rank tid
        __threadfence_system();
        unsigned long long *f = a.peer_flags[tid] + (size_t)slot * a.R + a.me;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(e) : "memory");
    }
    if (tid < a.R) {  // wait for rank tid's partial on this side
        const unsigned long long *f = a.peer_flags[a.me] + (size_t)slot * a.R + tid;
        uint32_t i = 0;
        for (; i < P2P_POLLS; i++) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
            if (v >= e) break;
        }
        if (i >= P2P_POLLS) {
            atomicOr(a.err, 1);
            ok_s = 0;
        }
    }
    __syncthreads();
    if (ok_s) {  // sum in rank order from +0
        const float *own = a.peer_recv[a.me] + (size_t)slot * a.R * P2P_MAXN;
        for (int i = tid; i < n; i += blockDim.x) {
            float acc = 0.0f;
            for (int r = 0; r < a.R; r++) acc = __fadd_rn(acc, __ldcv(own + (size_t)r * P2P_MAXN + i));
            buf[i] = acc;
        }
    }
    if (tid == 0) *a.epoch = e;
}

// Collective over the communicator: every rank allocates its slots, the IPC
// handles go round with an NCCL all-gather, every rank opens the others'; the
// path is enabled only if every rank succeeded (an NCCL min over the flags).
void p2p_setup() {
    if (g_size > P2P_MAX_RANKS) return;
    const int R = g_size;
    int ok = 1;
    const size_t recv_bytes = (size_t)P2P_SLOTS * R * P2P_MAXN * 4, flag_bytes = (size_t)P2P_SLOTS * R * 8;
    cudaIpcMemHandle_t mine{};
    if (cudaMalloc(&P2.base, recv_bytes + flag_bytes) != cudaSuccess ||
        cudaMemset(P2.base, 0, recv_bytes + flag_bytes) != cudaSuccess ||
        cudaMalloc(&P2.epoch, 256) != cudaSuccess || cudaMemset(P2.epoch, 0, 256) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine, P2.base) != cudaSuccess)
        ok = 0;
    P2.err = reinterpret_cast<int *>(P2.epoch + 8);
    uint8_t *d_h = nullptr;
    int *d_ok = nullptr;
    cudaStream_t st = nullptr;
    std::vector<cudaIpcMemHandle_t> all(R);
    if (cudaMalloc(&d_h, (size_t)R * sizeof(cudaIpcMemHandle_t)) != cudaSuccess || cudaMalloc(&d_ok, 4) != cudaSuccess ||
        cudaStreamCreate(&st) != cudaSuccess) {
        if (d_h) cudaFree(d_h);
        if (d_ok) cudaFree(d_ok);
        return;  // (a few bytes: NCCL's own initialisation allocated far more; not expected to fail)
    }
    cudaMemcpy(d_h + (size_t)g_rank * sizeof mine, &mine, sizeof mine, cudaMemcpyHostToDevice);
    if (N.allGather(d_h + (size_t)g_rank * sizeof mine, d_h, sizeof mine, ncclUint8, g_comm, st) != ncclSuccess) ok = 0;
    cudaStreamSynchronize(st);
    cudaMemcpy(all.data(), d_h, (size_t)R * sizeof mine, cudaMemcpyDeviceToHost);
    for (int p = 0; p < R && ok; p++) {
        if (p == g_rank) {
            P2.peer_base[p] = P2.base;
            continue;
        }
        if (cudaIpcOpenMemHandle(&P2.peer_base[p], all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) ok = 0;
    }
    cudaMemcpy(d_ok, &ok, 4, cudaMemcpyHostToDevice);
    if (N.allReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, g_comm, st) != ncclSuccess) ok = 0;
    cudaStreamSynchronize(st);
    int all_ok = 0;
    cudaMemcpy(&all_ok, d_ok, 4, cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    cudaFree(d_ok);
    cudaStreamDestroy(st);
    cudaGetLastError();
    if (!ok || !all_ok) return;
    P2.args.me = g_rank;
    P2.args.R = R;
    P2.args.epoch = P2.epoch;
    P2.args.err = P2.err;
    for (int p = 0; p < R; p++) {
        P2.args.peer_recv[p] = static_cast<float *>(P2.peer_base[p]);
        P2.args.peer_flags[p] = reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(P2.peer_base[p]) + recv_bytes);
    }
    P2.ready = !getenv("LOOM_CUDA_EP_NCCL");  // the NCCL path can be forced (comparisons)
}

void p2p_teardown() {
    for (int p = 0; p < P2P_MAX_RANKS; p++)
        if (P2.peer_base[p] && P2.peer_base[p] != P2.base) cudaIpcCloseMemHandle(P2.peer_base[p]);
    if (P2.base) cudaFree(P2.base);
    if (P2.epoch) cudaFree(P2.epoch);
    P2 = P2PState{};
}

}  // namespace

bool ep_active() { return g_comm != nullptr && g_size > 1; }
int ep_rank() { return g_rank; }
int ep_size() { return g_size; }

bool ep_agree(const int *vals, int n, std::string &err) {
    if (!ep_active()) return true;
    if (n > 16) return false;
    // min and max of every value over the ranks: equal everywhere iff min == max
    int h[32];
    for (int i = 0; i < n; i++) {
        h[i] = vals[i];
        h[16 + i] = -vals[i];
    }
    int *d = nullptr;
    cudaStream_t st = nullptr;
    bool ok = cudaMalloc(&d, sizeof h) == cudaSuccess && cudaStreamCreate(&st) == cudaSuccess &&
              cudaMemcpyAsync(d, h, sizeof h, cudaMemcpyHostToDevice, st) == cudaSuccess &&
              N.allReduce(d, d, 32, ncclInt32, ncclMin, g_comm, st) == ncclSuccess &&
              cudaMemcpyAsync(h, d, sizeof h, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
              cudaStreamSynchronize(st) == cudaSuccess;
    if (d) cudaFree(d);
    if (st) cudaStreamDestroy(st);
    if (!ok) {
        err = "expert-parallel agreement failed";
        return false;
    }
    for (int i = 0; i < n; i++)
        if (h[i] != -h[16 + i]) return false;  // some rank's value differs
    return true;
}

int ep_allreduce_sum(float *buf, size_t n, cudaStream_t st, std::string &err) {
    if (!ep_active()) return LOOM_CUDA_OK;
    if (P2.ready && n <= P2P_MAXN && n % 4 == 0 && (reinterpret_cast<uintptr_t>(buf) & 15) == 0) {
        k_p2p_combine<<<1, 1024, 0, st>>>(P2.args, buf, (int)n);
        count_launch();
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            err = std::string("peer combine: ") + cudaGetErrorString(e);
            return LOOM_CUDA_ERROR;
        }
        return LOOM_CUDA_OK;
    }
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
    p2p_setup();
    return LOOM_CUDA_OK;
}

int loom_cuda_ep_peer_combine(void) { return P2.ready ? 1 : 0; }

int loom_cuda_ep_error(void) {
    if (!P2.err) return 0;
    int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&v, P2.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return -1;
    if (v) P2.ready = false;  // epochs may disagree after a time-out: stay on NCCL from here on
    return v;
}

void loom_cuda_ep_shutdown(void) {
    cudaDeviceSynchronize();
    p2p_teardown();
    if (g_comm) N.commDestroy(g_comm);
    g_comm = nullptr;
    g_rank = 0;
    g_size = 1;
}

int loom_cuda_ep_rank(void) { return g_rank; }
int loom_cuda_ep_size(void) { return g_size; }

}  // extern "C"
