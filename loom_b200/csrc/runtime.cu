// runtime.cu -- the C ABI of the CUDA backend (include/loom_cuda.h): device
// and stream ownership, the device weight cache, arenas, scratch, and the
// host-buffer seam entry points.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "../../include/loom_cuda.h"
#include "attn.cuh"
#include "gemv.cuh"
#include "decode.cuh"
#include "ep.cuh"
#include "kernels.cuh"

using namespace loom;

namespace {

thread_local std::string g_err;
std::string g_arena_err;
bool g_inited = false;
int g_device = -1;
cudaStream_t g_stream = nullptr;
size_t g_cmdbufs = 0;

int fail(const char *what, cudaError_t e) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
    g_err = buf;
    return LOOM_CUDA_ERROR;
}
int decline(const char *why) {
    g_err = why;
    return LOOM_CUDA_DECLINED;
}
#define CK(call)                                     \
    do {                                             \
        cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return fail(#call, e_); \
    } while (0)

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }
bool type_ok(int t) {
    return t == T_F32 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0 || is_kquant(t);
}
// types stored as their GGUF blocks unchanged (16-byte multiples)
bool raw_layout(int t) { return t == T_F32 || t == T_Q4_K || t == T_Q5_K; }

// ---- device tensors ---------------------------------------------------------------

struct Tensor {
    int type = 0;
    uint64_t nblk = 0;
    uint8_t *base = nullptr;
    size_t dev_bytes = 0;
    WDev w{};
};
std::unordered_map<uint64_t, Tensor> g_tensors;
uint64_t g_next_handle = 1;

// weight cache: (host pointer, bytes, type) -> tensor handle
std::map<std::tuple<const void *, size_t, int>, uint64_t> g_cache;

struct Arena {
    const uint8_t *host;
    size_t bytes;
    uint8_t *dev;
};
std::vector<Arena> g_arenas;

// Bumped whenever a scratch or staging buffer moves or a cached weight is
// freed: seam graphs captured before then point at stale memory.
uint64_t g_buf_gen = 1;

// growable device buffer
struct DBuf {
    void *p = nullptr;
    size_t cap = 0;
    int ensure(size_t n, bool zero = false) {
        if (n <= cap) return 0;
        if (p) {
            cudaStreamSynchronize(g_stream);
            cudaFree(p);
            p = nullptr;
            cap = 0;
        }
        size_t want = std::max<size_t>(align256(n + n / 4), 256);
        g_buf_gen++;
        cudaError_t e = cudaMalloc(&p, want);
        if (e != cudaSuccess) return fail("cudaMalloc(scratch)", e);
        if (zero) {
            e = cudaMemset(p, 0, want);
            if (e != cudaSuccess) return fail("cudaMemset(scratch)", e);
        }
        cap = want;
        return 0;
    }
    template <class T> T *as() const { return reinterpret_cast<T *>(p); }
};
struct HBuf {  // pinned host staging
    void *p = nullptr;
    size_t cap = 0;
    int ensure(size_t n) {
        if (n <= cap) return 0;
        if (p) {
            cudaStreamSynchronize(g_stream);
            cudaFreeHost(p);
            p = nullptr;
            cap = 0;
        }
        size_t want = std::max<size_t>(align256(n + n / 4), 4096);
        g_buf_gen++;
        cudaError_t e = cudaHostAlloc(&p, want, cudaHostAllocDefault);
        if (e != cudaSuccess) return fail("cudaHostAlloc(staging)", e);
        cap = want;
        return 0;
    }
    template <class T> T *as() const { return reinterpret_cast<T *>(p); }
};

struct Scratch {
    DBuf xq256_q, xq256_d, xq256_s, xq32_q, xq32_d, xq32_s;
    DBuf logits, ids, gates, slots, act, aq, ad, as, counters, grp, ybuf;
    DBuf io_in, io_out, io_aux, raw;
    // all-to-all expert parallelism: home-side lists and rows, receive-side rows
    DBuf tmp;  // small synchronous scratch (tensor scans)
    DBuf prenormed;  // the FFN input when a layer's RMSNorm is not folded into its router kernel
    DBuf amax;  // argmax slot + counter (zeroed once, left zeroed by the kernel); lm_head logits
    DBuf head_logits;
    DBuf a2a_i, a2a_sx, a2a_yb, a2a_ysh, a2a_rx, a2a_re, a2a_yr, a2a_g1;
    HBuf h_in, h_out, h_cnt;
} S;

int alloc_tensor(int type, uint64_t nblk, Tensor &t) {
    t.type = type;
    t.nblk = nblk;
    const size_t qb = align256(nblk * (size_t)layout_qbytes(type));
    const size_t scb = (type == T_Q6_K || type == T_Q3_K) ? align256(nblk * 16)
                     : (type == T_Q5_1 || type == T_Q5_0) ? align256(nblk * 4) : 0;  // Q5_x: the 32 high bits
    const size_t db = (type == T_Q6_K || type == T_Q8_0 || type == T_Q4_0 || type == T_Q3_K || type == T_Q5_0)
                        ? align256(nblk * 2)
                    : (type == T_Q2_K || type == T_Q4_1 || type == T_Q5_1) ? align256(nblk * 4) : 0;  // d and dmin / m
    t.dev_bytes = qb + scb + db;
    cudaError_t e = cudaMalloc(&t.base, std::max<size_t>(t.dev_bytes, 256));
    if (e != cudaSuccess) return fail("cudaMalloc(tensor)", e);
    t.w.type = type;
    t.w.q = t.base;
    t.w.sc = scb ? t.base + qb : nullptr;
    t.w.d = db ? reinterpret_cast<uint16_t *>(t.base + qb + scb) : nullptr;
    return 0;
}

// Fill a tensor from GGUF bytes already on the device (`raw_dev`).
int fill_from_raw_dev(Tensor &t, const uint8_t *raw_dev) {
    if (raw_layout(t.type)) {
        CK(cudaMemcpyAsync(t.base, raw_dev, t.nblk * (size_t)block_bytes(t.type), cudaMemcpyDeviceToDevice, g_stream));
    } else {
        launch_repack(t.type, raw_dev, t.base, const_cast<uint8_t *>(t.w.sc), const_cast<uint16_t *>(t.w.d), t.nblk,
                      g_stream);
    }
    CK(cudaGetLastError());
    return 0;
}

// Q6_K: record whether every sub-block scale is within +-32 (the tensor-core
// path folds sc * (q - 32) into fp16 and sums 128 such products times int8
// activations in f32: exact only then). Synchronises g_stream.
int mark_q6k(Tensor &t) {
    if (t.type != T_Q6_K) return 0;
    if (int rc = S.tmp.ensure(64)) return rc;
    const int m = q6k_max_scale(t.w.sc, t.nblk, S.tmp.as<int>(), g_stream);
    if (m < 0) return fail("q6k scale scan", cudaGetLastError());
    if (m <= 32) t.w.pad_ |= WDEV_Q6K_SMALL_SCALES;
    return 0;
}

const uint8_t *arena_lookup(const void *p, size_t bytes) {
    const uint8_t *hp = static_cast<const uint8_t *>(p);
    for (auto &a : g_arenas)
        if (a.dev && hp >= a.host && hp + bytes <= a.host + a.bytes) return a.dev + (hp - a.host);
    return nullptr;
}

int upload_tensor(int type, const void *data, size_t bytes, uint64_t &handle) {
    const size_t bb = block_bytes(type);
    if (!type_ok(type) || bb == 0) return decline("unsupported ggml type");
    if (bytes % bb != 0) return decline("tensor bytes are not a whole number of blocks");
    Tensor t;
    if (int rc = alloc_tensor(type, bytes / bb, t)) return rc;
    const uint8_t *raw_dev = arena_lookup(data, bytes);
    if (!raw_dev && raw_layout(type)) {
        CK(cudaMemcpyAsync(t.base, data, bytes, cudaMemcpyHostToDevice, g_stream));
    } else {
        if (!raw_dev) {
            if (int rc = S.raw.ensure(bytes)) return rc;
            CK(cudaMemcpyAsync(S.raw.p, data, bytes, cudaMemcpyHostToDevice, g_stream));
            raw_dev = S.raw.as<uint8_t>();
        }
        if (int rc = fill_from_raw_dev(t, raw_dev)) return rc;
    }
    CK(cudaStreamSynchronize(g_stream));  // the host bytes are only borrowed
    if (int rc = mark_q6k(t)) return rc;
    handle = g_next_handle++;
    g_tensors[handle] = t;
    return 0;
}

// Resolve a seam weight (host bytes) to its cached device tensor.
int resolve(int type, const void *data, size_t bytes, Tensor *&out) {
    auto key = std::make_tuple(data, bytes, type);
    auto it = g_cache.find(key);
    if (it != g_cache.end()) {
        out = &g_tensors[it->second];
        return 0;
    }
    uint64_t h = 0;
    if (int rc = upload_tensor(type, data, bytes, h)) return rc;
    g_cache[key] = h;
    out = &g_tensors[h];
    return 0;
}

Tensor *lookup(loom_tensor h) {
    auto it = g_tensors.find(h);
    return it == g_tensors.end() ? nullptr : &it->second;
}

int need_init() { return g_inited ? 0 : decline("loom_cuda_init has not been called"); }

// The seam calls return with their outputs on the host. Waiting on the stream
// with cudaStreamSynchronize wakes the host tens of microseconds after the
// copy lands under the default (yielding) scheduling; a seam call is a few
// kernels of ~10 us, so the wake-up dominated. Instead the host polls an event
// it recorded after the last copy (bounded to ~2 s of polling, then a blocking
// wait), which returns within a microsecond or two of completion.
cudaEvent_t g_seam_ev = nullptr;

cudaError_t seam_wait() {
    if (!g_seam_ev) {
        cudaError_t e = cudaEventCreateWithFlags(&g_seam_ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaEventRecord(g_seam_ev, g_stream);
    if (e != cudaSuccess) return e;
    const auto t0 = std::chrono::steady_clock::now();
    while ((e = cudaEventQuery(g_seam_ev)) == cudaErrorNotReady) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2)) return cudaEventSynchronize(g_seam_ev);
    }
    return e;
}

// Scratch for quantizing T activation vectors of width `cols`.
int ensure_xq(size_t T, size_t cols) {
    if (int rc = S.xq256_q.ensure(T * cols)) return rc;
    if (int rc = S.xq256_d.ensure(T * (cols / 256 + 1) * 4)) return rc;
    if (int rc = S.xq256_s.ensure(T * (cols / 16 + 1) * 4)) return rc;
    if (int rc = S.xq32_q.ensure(T * cols)) return rc;
    if (int rc = S.xq32_d.ensure(T * (cols / 32 + 1) * 4)) return rc;
    if (int rc = S.xq32_s.ensure(T * (cols / 32 + 1) * 4)) return rc;
    return 0;
}

XQ make_xq(bool k256, size_t cols) {
    XQ x;
    x.cols = (int)cols;
    x.kind256 = k256;
    if (k256) {
        x.q = S.xq256_q.as<int8_t>();
        x.d = S.xq256_d.as<float>();
        x.s = S.xq256_s.as<int32_t>();
        x.dstride = (int)(cols / 256);
        x.sstride = (int)(cols / 16);
    } else {
        x.q = S.xq32_q.as<int8_t>();
        x.d = S.xq32_d.as<float>();
        x.s = S.xq32_s.as<int32_t>();
        x.dstride = (int)(cols / 32);
        x.sstride = (int)(cols / 32);
    }
    return x;
}

void quantize_into(const float *x, size_t T, size_t cols, bool k256, cudaStream_t st) {
    XQ q = make_xq(k256, cols);
    launch_quant_act(x, (int)T, (int)cols, (int)cols, k256, const_cast<int8_t *>(q.q), const_cast<float *>(q.d),
                     const_cast<int32_t *>(q.s), q.dstride, q.sstride, st);
}

int ensure_moe_scratch(size_t T, size_t dim, size_t max_ffn, size_t n_expert, size_t n_slots) {
    const size_t act_stride = align256(max_ffn);
    if (int rc = ensure_xq(T, dim)) return rc;
    if (int rc = S.logits.ensure(T * n_expert * 4)) return rc;
    if (int rc = S.ids.ensure(n_slots * 4)) return rc;
    if (int rc = S.gates.ensure(n_slots * 4)) return rc;
    if (int rc = S.slots.ensure(n_slots * sizeof(Slot))) return rc;
    if (int rc = S.act.ensure(n_slots * act_stride * 4)) return rc;
    if (int rc = S.aq.ensure(n_slots * act_stride)) return rc;
    if (int rc = S.ad.ensure(n_slots * act_stride / 32 * 4 + 64)) return rc;
    if (int rc = S.as.ensure(n_slots * act_stride / 16 * 4 + 64)) return rc;
    if (int rc = S.counters.ensure((T + n_slots + 1) * 4, true)) return rc;
    return 0;
}

void quantize_inputs(const float *d_x, size_t T, size_t dim, bool need256, bool need32, cudaStream_t st) {
    if (need256) quantize_into(d_x, T, dim, true, st);
    if (need32) quantize_into(d_x, T, dim, false, st);
}

int check_moe_types(const Tensor *g, const Tensor *u, const Tensor *d) {
    for (const Tensor *t : {g, u, d})
        if (!t || t->type == T_F32 || t->type == T_Q5_0)  // Q5_0 runs on f32 activations (matvecQ50)
            return decline("MoE expert tensors must be a quantized type on int8 activations (not F32 or Q5_0)");
    return 0;
}

int routed_layer(RoutedLayerDev &L, const Tensor *g, const Tensor *u, const Tensor *dn, size_t dim, size_t ffn,
                 size_t n_local, const Tensor *sh[3], size_t shexp_ffn) {
    if (int rc = check_moe_types(g, u, dn)) return rc;
    const int bg = block_elems(g->type), bu = block_elems(u->type), bd = block_elems(dn->type);
    if (dim % bg || dim % bu || ffn % bd || ffn % 32) return decline("MoE shape is not a whole number of blocks");
    const uint64_t pg = ffn * (dim / bg), pu = ffn * (dim / bu), pd = dim * (ffn / bd);
    if (g->nblk < pg * n_local || u->nblk < pu * n_local || dn->nblk < pd * n_local)
        return decline("expert tensor smaller than n_expert planes");
    L.g = g->w;
    L.u = u->w;
    L.dn = dn->w;
    L.plane_blk_g = pg;
    L.plane_blk_u = pu;
    L.plane_blk_dn = pd;
    L.ffn = (int)ffn;
    L.dim = (int)dim;
    L.has_shared = 0;
    L.shexp_ffn = 0;
    if (sh[0]) {
        if (int rc = check_moe_types(sh[0], sh[1], sh[2])) return rc;
        if (dim % block_elems(sh[0]->type) || dim % block_elems(sh[1]->type) ||
            shexp_ffn % block_elems(sh[2]->type) || shexp_ffn % 32 || shexp_ffn == 0)
            return decline("shared expert shape is not a whole number of blocks");
        L.has_shared = 1;
        L.sg = sh[0]->w;
        L.su = sh[1]->w;
        L.sdn = sh[2]->w;
        L.shexp_ffn = (int)shexp_ffn;
    }
    return 0;
}

bool any_type(const RoutedLayerDev &L, bool k256) {
    bool r = act256(L.g.type) == k256 || act256(L.u.type) == k256;
    if (L.has_shared) r = r || act256(L.sg.type) == k256 || act256(L.su.type) == k256;
    return r;
}

// The fused decode kernels take up to this many tokens per layer (the
// allocation-free entry point runs them up to this size).
constexpr size_t DECODE_MAX_T = 16;
// Above this many tokens the expert-major batch kernels win (one read of each
// selected expert for all its tokens; measured on B200 at the Qwen3 layer:
// T = 2 decode 1.86 ms vs batch 2.15 ms per 48 layers, T = 4 3.13 vs 2.51).
constexpr size_t DECODE_AUTO_T = 2;

int g_force_generic = 0;  // test hook: 0 auto, 1 slot kernels, 2 int8 batch kernels, 3 tensor cores, 4 dp4a tiles
int g_last_path = -1;      // kernel family of the last routed layer (loom_cuda_last_path)
const uint8_t *g_next_router = nullptr;  // L2-prefetch hint for the layer being launched
size_t g_next_router_bytes = 0;
// phase trace: [2*n] (first start, last end) per traced kernel, see loom_cuda_trace_*
unsigned long long *g_trace = nullptr;
size_t g_trace_cap = 0, g_trace_next = 0;  // test hook: route every layer through the slot kernels

// Kernel family of an expert-major batch layer with `slots` routed slots:
// the tensor cores once the experts average 16 or more slots each (prefill),
// else the tiled dp4a kernels, else the per-expert int8 kernels; the test
// hook g_force_generic (2, 3, 4) selects one where the layer's types allow.
int batch_path(const DecodeArgs &A, size_t slots, int n_local) {
    if (g_force_generic == 2) return BATCH_GRP;
    if (g_force_generic == 3) return moe_mma_supported(A) ? BATCH_MMA : BATCH_GRP;
    if (g_force_generic == 4) return moe_dp4a_supported(A) ? BATCH_DP4A : BATCH_GRP;
    if (moe_mma_supported(A) && slots >= 16 * (size_t)n_local) return BATCH_MMA;
    if (moe_dp4a_supported(A)) return BATCH_DP4A;
    return BATCH_GRP;
}

// Group-limited selection of a layer (DeepSeek-V3 routing): n_group 0 or 1 is
// plain top-k; otherwise n_group <= 32 groups dividing n_expert, 1 <=
// topk_group <= n_group, and n_used no more than the kept experts.
int group_cfg(const loom_moe_desc &D, RoutedLayerDev &L) {
    const size_t ng = D.n_group ? D.n_group : 1, tg = D.n_group > 1 ? D.topk_group : 1;
    if (ng > 32 || D.n_expert % ng || tg == 0 || tg > ng || D.n_used > tg * (D.n_expert / ng))
        return decline("expert groups out of range (n_group <= 32 dividing n_expert, 1 <= topk_group <= n_group)");
    L.n_group = (int)ng;
    L.topk_group = (int)tg;
    return 0;
}

DecodeArgs decode_args(const RoutedLayerDev &L, size_t T, const float *router, const float *d_x,
                       const float *d_logits_in, const float *d_bias, float *d_out, const float *d_residual,
                       uint32_t *d_ids_out, size_t act_stride) {
    DecodeArgs A{};
    A.T = (int)T;
    A.dim = L.dim;
    A.ffn = L.ffn;
    A.n_expert = L.n_expert;
    A.n_used = L.n_used;
    A.gating = L.gating;
    A.weights_norm = L.weights_norm;
    A.weights_scale = L.weights_scale;
    A.n_group = L.n_group;
    A.topk_group = L.topk_group;
    A.expert0 = L.expert0;
    A.n_local = L.n_local;
    A.router = router;
    A.bias = d_bias;
    A.logits_in = d_logits_in;
    A.x = d_x;
    A.out = d_out;
    A.residual = d_residual;
    A.logits = S.logits.as<float>();
    A.ids = S.ids.as<int>();
    A.gates = S.gates.as<float>();
    A.ids_out = d_ids_out;
    A.cnt_tok = S.counters.as<int>();
    A.cnt_slot = S.counters.as<int>() + T;
    A.err = S.counters.as<int>() + T + (T * L.n_used + (L.has_shared ? T : 0));
    A.x256 = XQW{S.xq256_q.as<int8_t>(), S.xq256_d.as<float>(), S.xq256_s.as<int32_t>()};
    A.x32 = XQW{S.xq32_q.as<int8_t>(), S.xq32_d.as<float>(), S.xq32_s.as<int32_t>()};
    A.need256 = any_type(L, true);
    A.need32 = any_type(L, false);
    A.g = L.g;
    A.u = L.u;
    A.dn = L.dn;
    A.has_shared = L.has_shared;
    A.sg = L.sg;
    A.su = L.su;
    A.sdn = L.sdn;
    A.shexp_ffn = L.shexp_ffn;
    A.act = S.act.as<float>();
    A.aq = S.aq.as<int8_t>();
    A.ad = S.ad.as<float>();
    A.as = S.as.as<int32_t>();
    A.act_stride = (int)act_stride;
    A.next_router = g_next_router;
    A.next_router_bytes = g_next_router_bytes;
    if (g_trace && g_trace_next + 12 <= g_trace_cap) {
        A.trace = g_trace;
        A.trace_slot = (int)g_trace_next;
        g_trace_next += 12;
    }
    return A;
}

// Device-side forward of a routed MoE layer (routing on the device). `router`
// (f32 [n_expert][dim]) computes the logits; otherwise d_logits holds them.
// Seam calls repeat the same few shapes on the same weights every token, so
// each (operation, weights, shape, configuration) gets a CUDA graph of its
// copies and kernels: the first call runs eagerly (sizing every buffer), the
// second captures and instantiates, later calls are one graph launch. A graph
// is dropped when a buffer it points at moves or a weight is freed
// (g_buf_gen). The host side of a call (staging the inputs in pinned memory,
// reading the result back after seam_wait) stays outside the graph.
struct SeamGraph {
    uint64_t gen = 0;
    cudaGraphExec_t exec = nullptr;
    bool seen = false, bad = false;  // bad: capture failed once, always run eagerly
    uint64_t launches = 0;
    int last_path = 0;
};
std::map<std::vector<uint64_t>, SeamGraph> g_seam_graphs;

template <class F>
int seam_run(const std::vector<uint64_t> &key, F &&body) {
    if (g_trace) return body();  // traced kernels record into a buffer that is re-armed per call
    SeamGraph &G = g_seam_graphs[key];
    if (G.exec && G.gen == g_buf_gen) {
        cudaError_t e = cudaGraphLaunch(G.exec, g_stream);
        if (e != cudaSuccess) return fail("cudaGraphLaunch(seam)", e);
        count_launches(G.launches);
        g_last_path = G.last_path;
        return 0;
    }
    if (G.exec) {
        cudaGraphExecDestroy(G.exec);
        G.exec = nullptr;
    }
    if (G.bad) return body();
    if (!G.seen || G.gen != g_buf_gen) {  // first sighting at this buffer generation: eager
        const int rc = body();
        G.seen = rc == 0;
        G.gen = g_buf_gen;  // after the eager run's allocations
        return rc;
    }
    cudaError_t e = cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) {
        cudaGetLastError();
        G.bad = true;
        return body();
    }
    const uint64_t l0 = launches();
    const int rc = body();
    cudaGraph_t graph = nullptr;
    e = cudaStreamEndCapture(g_stream, &graph);
    G.launches = launches() - l0;
    G.last_path = g_last_path;
    if (rc || e != cudaSuccess || !graph || G.gen != g_buf_gen) {  // nothing ran: run eagerly
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        G.bad = G.gen == g_buf_gen;  // a buffer move is retried, anything else is not
        G.seen = false;
        return body();
    }
    e = cudaGraphInstantiate(&G.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
        G.exec = nullptr;
        G.bad = true;
        cudaGetLastError();
        return body();
    }
    e = cudaGraphLaunch(G.exec, g_stream);
    if (e != cudaSuccess) return fail("cudaGraphLaunch(seam)", e);
    return 0;
}

void seam_graphs_clear() {
    for (auto &kv : g_seam_graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    g_seam_graphs.clear();
}

inline uint64_t fbits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

// The layer's FFN RMSNorm weight for the next moe_routed_dev call (model.cu):
// x is then the raw residual stream. One-token decode folds the norm into the
// router kernel; every other path normalizes into a scratch row first.
const float *g_prenorm_w = nullptr;
float g_prenorm_eps = 0.0f;

int moe_routed_dev(const RoutedLayerDev &L, size_t T, const float *router, const float *d_x, const float *d_logits,
                   const float *d_bias, float *d_out, const float *d_residual, uint32_t *d_ids_out, cudaStream_t st) {
    const size_t max_ffn = std::max<size_t>(L.ffn, L.has_shared ? L.shexp_ffn : 0);
    const size_t n_slots = T * L.n_used + (L.has_shared ? T : 0);
    if (int rc = ensure_moe_scratch(T, L.dim, max_ffn, L.n_expert, n_slots)) return rc;
    const size_t act_stride = align256(max_ffn);
    const float *pre_w = g_prenorm_w;
    g_prenorm_w = nullptr;
    auto prenorm_scratch = [&]() -> int {  // the unfolded form: RMSNorm rows into scratch
        if (int rc = S.prenormed.ensure(T * (size_t)L.dim * 4)) return rc;
        const XQW none{nullptr, nullptr, nullptr};
        for (size_t t = 0; t < T; t++)
            launch_rmsnorm_q(const_cast<float *>(d_x) + t * L.dim, nullptr, pre_w, L.dim, g_prenorm_eps,
                             S.prenormed.as<float>() + t * L.dim, none, none, false, st);
        CK(cudaGetLastError());
        d_x = S.prenormed.as<float>();
        pre_w = nullptr;
        return 0;
    };
    if (g_force_generic != 1) {
        DecodeArgs A = decode_args(L, T, router, d_x, d_logits, d_bias, d_out, d_residual, d_ids_out, act_stride);
        const bool batch_ok = router && batch_supported(A);
        if (g_force_generic == 0 && (T <= DECODE_AUTO_T || (!batch_ok && T <= DECODE_MAX_T)) && decode_supported(A)) {
            g_last_path = 0;
            if (pre_w && T == 1) {
                A.prenorm_w = pre_w;
                A.prenorm_eps = g_prenorm_eps;
            } else if (pre_w) {
                if (int rc = prenorm_scratch()) return rc;
                A.x = d_x;
            }
            CK(launch_decode(A, st));
            return 0;
        }
        if (pre_w) {
            if (int rc = prenorm_scratch()) return rc;
            A.x = d_x;
        }
        if (batch_ok) {
            const int path = batch_path(A, T * L.n_used, L.n_local);
            if (int rc = S.grp.ensure((3 * (size_t)L.n_local + T * L.n_used + 4) * 4)) return rc;
            if (int rc = S.ybuf.ensure(n_slots * (size_t)L.dim * 4)) return rc;
            A.grp_cnt = S.grp.as<int>();
            A.grp_off = A.grp_cnt + L.n_local;
            A.grp_list = A.grp_off + L.n_local;
            A.tc_pre = A.grp_list + T * L.n_used;
            A.y = S.ybuf.as<float>();
            g_last_path = path;
            CK(launch_batch(A, path, st));
            return 0;
        }
    }
    if (pre_w)
        if (int rc = prenorm_scratch()) return rc;
    if (router) {
        launch_mm_f32(router, L.n_expert, L.dim, d_x, (int)T, S.logits.as<float>(), st);
        d_logits = S.logits.as<float>();
    }
    g_last_path = 1;
    launch_route(d_logits, d_bias, (int)T, L.n_expert, L.n_used, L.gating, L.weights_norm, L.weights_scale,
                 S.ids.as<int>(), S.gates.as<float>(), st, L.n_group, L.topk_group);
    quantize_inputs(d_x, T, L.dim, any_type(L, true), any_type(L, false), st);
    launch_experts_routed(L, S.ids.as<int>(), S.gates.as<float>(), (int)T, (int)act_stride, make_xq(true, L.dim),
                          make_xq(false, L.dim), S.act.as<float>(), S.aq.as<int8_t>(), S.ad.as<float>(),
                          S.as.as<int32_t>(), d_out, d_residual, st);
    if (d_ids_out) CK(cudaMemcpyAsync(d_ids_out, S.ids.p, T * L.n_used * 4, cudaMemcpyDeviceToDevice, st));
    CK(cudaGetLastError());
    return 0;
}

}  // namespace

// Internal hooks for the other host files of the library (model.cu).
namespace loom {
bool rt_tensor(uint64_t h, WDev *w, int *type, uint64_t *nblk) {
    Tensor *t = lookup(h);
    if (!t) return false;
    *w = t->w;
    *type = t->type;
    *nblk = t->nblk;
    return true;
}
cudaStream_t rt_stream(void *s) { return s ? static_cast<cudaStream_t>(s) : g_stream; }
int rt_need_init() { return need_init(); }
int rt_decline(const char *why) { return decline(why); }
int rt_fail(const char *what, cudaError_t e) { return fail(what, e); }
uint64_t rt_buf_gen() { return g_buf_gen; }
cudaError_t rt_wait() { return seam_wait(); }  // completion of the backend's stream, polled
// The next loom_cuda_moe_forward takes the raw residual row and applies the
// layer's FFN RMSNorm (weight w, f32 [dim]) itself.
void rt_moe_prenorm(const float *w, float eps) {
    g_prenorm_w = w;
    g_prenorm_eps = eps;
}

// A host weight range -> the cached device tensor that holds it (uploading it
// as its own tensor when no cached tensor of that type contains it) and its
// first block and block count there.
int rt_place(int type, const void *data, size_t bytes, uint64_t *handle, uint64_t *blk0, uint64_t *nblk) {
    const size_t bb = block_bytes(type);
    if (!type_ok(type) || bb == 0) return decline("unsupported ggml type");
    if (bytes == 0 || bytes % bb != 0) return decline("extent is not a whole number of blocks");
    const uint8_t *p = static_cast<const uint8_t *>(data);
    for (auto &kv : g_cache) {
        const uint8_t *hp = static_cast<const uint8_t *>(std::get<0>(kv.first));
        const size_t hb = std::get<1>(kv.first);
        if (std::get<2>(kv.first) != type || p < hp || p + bytes > hp + hb) continue;
        if ((size_t)(p - hp) % bb != 0) continue;
        *handle = kv.second;
        *blk0 = (size_t)(p - hp) / bb;
        *nblk = bytes / bb;
        return 0;
    }
    Tensor *t = nullptr;
    if (int rc = resolve(type, data, bytes, t)) return rc;
    *handle = g_cache[std::make_tuple(data, bytes, type)];
    *blk0 = 0;
    *nblk = bytes / bb;
    return 0;
}
// Drop a cached weight tensor: the next seam call that names its bytes
// uploads them again.
void rt_evict(uint64_t handle) {
    cudaStreamSynchronize(g_stream);
    for (auto it = g_cache.begin(); it != g_cache.end();) {
        if (it->second == handle) it = g_cache.erase(it);
        else ++it;
    }
    auto it = g_tensors.find(handle);
    if (it != g_tensors.end()) {
        cudaFree(it->second.base);
        g_tensors.erase(it);
    }
    g_buf_gen++;
}
}  // namespace loom

extern "C" {

int loom_cuda_init(int device) {
    if (const char *e = getenv("LOOM_CUDA_GENERIC")) g_force_generic = e[0] - '0';
    if (g_inited) return device == g_device ? LOOM_CUDA_OK : decline("already initialised on another device");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return decline("no CUDA device");
    if (device < 0 || device >= n) return decline("device index out of range");
    CK(cudaSetDevice(device));
    cudaDeviceProp p;
    CK(cudaGetDeviceProperties(&p, device));
    if (p.major != 10) return decline("this backend is built for sm_100a (B200)");
    // A blocking stream: work on the legacy default stream (where torch and most
    // C callers queue their copies) is ordered before and after it.
    CK(cudaStreamCreateWithFlags(&g_stream, cudaStreamDefault));
    g_device = device;
    g_inited = true;
    return LOOM_CUDA_OK;
}

void loom_cuda_clear_weight_cache(void) {
    if (!g_inited) return;
    cudaStreamSynchronize(g_stream);
    g_buf_gen++;
    for (auto &kv : g_cache) {
        auto it = g_tensors.find(kv.second);
        if (it != g_tensors.end()) {
            cudaFree(it->second.base);
            g_tensors.erase(it);
        }
    }
    g_cache.clear();
}

void loom_cuda_shutdown(void) {
    if (!g_inited) return;
    cudaStreamSynchronize(g_stream);
    seam_graphs_clear();
    for (auto &kv : g_tensors) cudaFree(kv.second.base);
    g_tensors.clear();
    g_cache.clear();
    for (auto &a : g_arenas)
        if (a.dev) cudaFree(a.dev);
    g_arenas.clear();
    for (DBuf *b : {&S.xq256_q, &S.xq256_d, &S.xq256_s, &S.xq32_q, &S.xq32_d, &S.xq32_s, &S.logits, &S.ids, &S.gates,
                    &S.slots, &S.act, &S.aq, &S.ad, &S.as, &S.counters, &S.grp, &S.ybuf, &S.io_in, &S.io_out, &S.io_aux, &S.raw, &S.a2a_i, &S.a2a_sx,
                    &S.a2a_yb, &S.a2a_ysh, &S.a2a_rx, &S.a2a_re, &S.a2a_yr, &S.a2a_g1, &S.tmp, &S.amax, &S.head_logits, &S.prenormed}) {
        if (b->p) cudaFree(b->p);
        b->p = nullptr;
        b->cap = 0;
    }
    for (HBuf *b : {&S.h_in, &S.h_out}) {
        if (b->p) cudaFreeHost(b->p);
        b->p = nullptr;
        b->cap = 0;
    }
    if (g_seam_ev) cudaEventDestroy(g_seam_ev);
    g_seam_ev = nullptr;
    cudaStreamDestroy(g_stream);
    g_stream = nullptr;
    g_inited = false;
    g_device = -1;
}

void loom_cuda_parallel_begin(size_t n) {
    (void)n;
    if (!g_inited) loom_cuda_init(0);
}
void loom_cuda_parallel_end(void) {}
size_t loom_cuda_max_batch(void) { return 64; }

int loom_cuda_register_arena(const void *mem, size_t bytes) {
    if (int rc = need_init()) return rc;
    if (!mem || bytes == 0) return decline("empty arena");
    g_arenas.push_back(Arena{static_cast<const uint8_t *>(mem), bytes, nullptr});
    return LOOM_CUDA_OK;
}

size_t loom_cuda_materialize_arenas(void) {
    if (!g_inited) {
        g_arena_err = "backend not initialised";
        return 0;
    }
    size_t total = 0;
    for (auto &a : g_arenas) {
        if (!a.dev) {
            cudaError_t e = cudaMalloc(&a.dev, a.bytes);
            if (e != cudaSuccess) {
                a.dev = nullptr;
                g_arena_err = std::string("cudaMalloc(arena): ") + cudaGetErrorString(e);
                return 0;
            }
            e = cudaMemcpy(a.dev, a.host, a.bytes, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) {
                cudaFree(a.dev);
                a.dev = nullptr;
                g_arena_err = std::string("arena upload: ") + cudaGetErrorString(e);
                return 0;
            }
        }
        total += a.bytes;
    }
    g_arena_err.clear();
    return total;
}

const char *loom_cuda_arena_error(void) { return g_arena_err.empty() ? nullptr : g_arena_err.c_str(); }

size_t loom_cuda_take_cmdbuf_count(void) {
    size_t n = g_cmdbufs;
    g_cmdbufs = 0;
    return n;
}

uint64_t loom_cuda_kernel_launches(void) { return loom::launches(); }

size_t loom_cuda_last_error(char *buf, size_t len) {
    if (buf && len) {
        size_t n = std::min(len - 1, g_err.size());
        memcpy(buf, g_err.data(), n);
        buf[n] = 0;
    }
    return g_err.size();
}

void *loom_cuda_stream(void) { return g_stream; }

int loom_cuda_trace_enable(size_t n_kernels) {
    if (int rc = need_init()) return rc;
    CK(cudaStreamSynchronize(g_stream));
    if (g_trace) cudaFree(g_trace);
    g_trace = nullptr;
    g_trace_cap = g_trace_next = 0;
    if (n_kernels == 0) return LOOM_CUDA_OK;
    CK(cudaMalloc(&g_trace, n_kernels * 16));
    g_trace_cap = n_kernels;
    return loom_cuda_trace_reset();
}

int loom_cuda_trace_reset(void) {
    if (int rc = need_init()) return rc;
    if (!g_trace) return decline("tracing is off");
    std::vector<unsigned long long> init(2 * g_trace_cap);
    for (size_t i = 0; i < g_trace_cap; i++) {  // per layer: 7 (start, end) spans, then 5 cycle-count pairs
        init[2 * i] = i % 12 < 7 ? ~0ull : 0;
        init[2 * i + 1] = 0;
    }
    CK(cudaMemcpy(g_trace, init.data(), init.size() * 8, cudaMemcpyHostToDevice));
    return LOOM_CUDA_OK;
}

size_t loom_cuda_trace_read(uint64_t *out, size_t n_kernels) {
    if (!g_inited || !g_trace) return 0;
    const size_t n = std::min(n_kernels, g_trace_next);
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) return 0;
    if (cudaMemcpy(out, g_trace, n * 16, cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    return n;
}

int loom_cuda_device_error(void) {
    if (!g_inited || !S.counters.p) return 0;
    int v = 0;
    // the error word sits after the counters of the last layer shape reserved
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) return -1;
    std::vector<int> all(S.counters.cap / 4);
    if (cudaMemcpy(all.data(), S.counters.p, all.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    for (int x : all) v |= x;
    return v;
}

int loom_cuda_last_path(void) { return g_last_path; }

int loom_cuda_force_generic(int on) {
    const int prev = g_force_generic;
    g_force_generic = on;
    return prev;
}

int loom_cuda_sync(void) {
    if (int rc = need_init()) return rc;
    CK(cudaStreamSynchronize(g_stream));
    return LOOM_CUDA_OK;
}

// ---- seam ops -------------------------------------------------------------------

int loom_cuda_matvec(int type, float *out, const void *w, size_t w_bytes, const float *x, size_t rows, size_t cols) {
    return loom_cuda_matmul(type, out, w, w_bytes, x, 1, rows, cols);
}

int loom_cuda_matmul(int type, float *out, const void *w, size_t w_bytes, const float *xs, size_t n, size_t rows,
                     size_t cols) {
    if (int rc = need_init()) return rc;
    if (!type_ok(type)) return decline("unsupported ggml type");
    const size_t be = block_elems(type);
    if (cols == 0 || cols % be) return decline("cols is not a whole number of blocks");
    if (rows > (1u << 30) || cols > (1u << 24) || n > (1u << 20)) return decline("shape out of range");
    if (w_bytes < rows * (cols / be) * (size_t)block_bytes(type)) return decline("weight slice shorter than rows x cols");
    if (n == 0 || rows == 0) return LOOM_CUDA_OK;
    Tensor *t;
    if (int rc = resolve(type, w, w_bytes, t)) return rc;
    const size_t in_b = n * cols * 4, out_b = n * rows * 4;
    if (int rc = S.h_in.ensure(in_b)) return rc;
    if (int rc = S.h_out.ensure(out_b)) return rc;
    if (int rc = S.io_in.ensure(in_b)) return rc;
    if (int rc = S.io_out.ensure(out_b)) return rc;
    memcpy(S.h_in.p, xs, in_b);
    const std::vector<uint64_t> key = {1, (uint64_t)type, (uint64_t)(uintptr_t)t->base, n, rows, cols};
    if (int rc = seam_run(key, [&]() -> int {
            CK(cudaMemcpyAsync(S.io_in.p, S.h_in.p, in_b, cudaMemcpyHostToDevice, g_stream));
            if (type == T_F32) {
                launch_mm_f32(reinterpret_cast<const float *>(t->base), (int)rows, (int)cols, S.io_in.as<float>(),
                              (int)n, S.io_out.as<float>(), g_stream);
            } else if (type == T_Q5_0) {
                launch_mm_q50(t->w, 0, (int)rows, (int)cols, S.io_in.as<float>(), (int)n, S.io_out.as<float>(),
                              g_stream);
            } else {
                if (int rc = ensure_xq(n, cols)) return rc;
                quantize_into(S.io_in.as<float>(), n, cols, act256(type), g_stream);
                launch_mm(t->w, 0, (int)rows, (int)cols, make_xq(act256(type), cols), (int)n, S.io_out.as<float>(),
                          g_stream);
            }
            CK(cudaGetLastError());
            CK(cudaMemcpyAsync(S.h_out.p, S.io_out.p, out_b, cudaMemcpyDeviceToHost, g_stream));
            return 0;
        }))
        return rc;
    CK(seam_wait());  // the seam returns with `out` written
    memcpy(out, S.h_out.p, out_b);
    g_cmdbufs++;
    return LOOM_CUDA_OK;
}

int loom_cuda_dequant_row(int type, float *out, const void *w, size_t w_bytes, size_t r, size_t cols) {
    if (int rc = need_init()) return rc;
    if (!type_ok(type)) return decline("unsupported ggml type");
    const size_t be = block_elems(type);
    if (cols == 0 || cols % be) return decline("cols is not a whole number of blocks");
    const size_t rb = (cols / be) * block_bytes(type);
    if (w_bytes < (r + 1) * rb) return decline("row out of range");
    Tensor *t;
    if (int rc = resolve(type, w, w_bytes, t)) return rc;
    if (int rc = S.io_out.ensure(cols * 4)) return rc;
    if (int rc = S.h_out.ensure(cols * 4)) return rc;
    launch_dequant(t->w, (uint64_t)r * (cols / be), cols / be, S.io_out.as<float>(), g_stream);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(S.h_out.p, S.io_out.p, cols * 4, cudaMemcpyDeviceToHost, g_stream));
    CK(seam_wait());  // the seam returns with `out` written
    memcpy(out, S.h_out.p, cols * 4);
    g_cmdbufs++;
    return LOOM_CUDA_OK;
}

int loom_cuda_moe_route(const float *logits, const float *bias, size_t n_expert, uint32_t *ids_out, float *gates_out,
                        size_t n_used, int gating_sigmoid, int weights_norm, float weights_scale) {
    if (int rc = need_init()) return rc;
    if (n_expert == 0 || n_expert > 1024 || n_used == 0 || n_used > 64 || n_used > n_expert)
        return decline("router shape out of range (moe.zig:48-49)");
    const size_t in_b = n_expert * 4 * 2, out_b = n_used * 8;
    if (int rc = S.h_in.ensure(in_b)) return rc;
    if (int rc = S.h_out.ensure(out_b)) return rc;
    if (int rc = S.io_in.ensure(in_b)) return rc;
    if (int rc = S.io_out.ensure(out_b)) return rc;
    memcpy(S.h_in.p, logits, n_expert * 4);
    if (bias) memcpy(S.h_in.as<float>() + n_expert, bias, n_expert * 4);
    CK(cudaMemcpyAsync(S.io_in.p, S.h_in.p, bias ? in_b : n_expert * 4, cudaMemcpyHostToDevice, g_stream));
    int *d_ids = S.io_out.as<int>();
    float *d_g = S.io_out.as<float>() + n_used;
    launch_route(S.io_in.as<float>(), bias ? S.io_in.as<float>() + n_expert : nullptr, 1, (int)n_expert, (int)n_used,
                 gating_sigmoid ? 2 : 1, weights_norm, weights_scale, d_ids, d_g, g_stream);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(S.h_out.p, S.io_out.p, out_b, cudaMemcpyDeviceToHost, g_stream));
    CK(seam_wait());  // the seam returns with `out` written
    memcpy(ids_out, S.h_out.p, n_used * 4);
    memcpy(gates_out, S.h_out.as<float>() + n_used, n_used * 4);
    g_cmdbufs++;
    return LOOM_CUDA_OK;
}

int loom_cuda_moe_ffn_block(const float *normed, size_t dim, const loom_expert *experts, size_t n, float *out) {
    if (int rc = need_init()) return rc;
    if (n == 0 || n > 65) return decline("expert count out of range");
    if (dim == 0 || dim % 32) return decline("dim is not a whole number of blocks");
    // Resolve everything before launching anything: a decline leaves no work behind.
    std::vector<Slot> host(n);
    size_t max_ffn = 0;
    bool need256 = false, need32 = false;
    for (size_t k = 0; k < n; k++) {
        const loom_expert &e = experts[k];
        Tensor *g, *u, *d;
        if (int rc = resolve(e.gate.ggml_type, e.gate.data, e.gate.bytes, g)) return rc;
        if (int rc = resolve(e.up.ggml_type, e.up.data, e.up.bytes, u)) return rc;
        if (int rc = resolve(e.down.ggml_type, e.down.data, e.down.bytes, d)) return rc;
        if (int rc = check_moe_types(g, u, d)) return rc;
        if (dim % block_elems(g->type) || dim % block_elems(u->type) || e.ffn % block_elems(d->type) || e.ffn % 32 ||
            e.ffn == 0)
            return decline("expert shape is not a whole number of blocks");
        if (g->nblk < e.ffn * (dim / block_elems(g->type)) || u->nblk < e.ffn * (dim / block_elems(u->type)) ||
            d->nblk < dim * (e.ffn / block_elems(d->type)))
            return decline("expert slice shorter than its shape");
        max_ffn = std::max(max_ffn, e.ffn);
        need256 |= act256(g->type) || act256(u->type);
        need32 |= !act256(g->type) || !act256(u->type);
        host[k].g = g->w;
        host[k].u = u->w;
        host[k].dn = d->w;
        host[k].gb_g = host[k].gb_u = host[k].gb_dn = 0;
        host[k].ffn = (int)e.ffn;
        host[k].token = 0;
        host[k].weight = e.weight;
    }
    const size_t act_stride = align256(max_ffn);
    for (size_t k = 0; k < n; k++) host[k].act_off = (int)(k * act_stride);
    if (int rc = ensure_moe_scratch(1, dim, max_ffn, 1, n)) return rc;
    const size_t slot_b = n * sizeof(Slot);
    if (int rc = S.h_in.ensure(align256(slot_b) + dim * 4)) return rc;
    if (int rc = S.h_out.ensure(dim * 4)) return rc;
    if (int rc = S.io_in.ensure(dim * 4)) return rc;
    if (int rc = S.io_out.ensure(dim * 4)) return rc;
    memcpy(S.h_in.p, host.data(), slot_b);
    memcpy(S.h_in.as<uint8_t>() + align256(slot_b), normed, dim * 4);
    CK(cudaMemcpyAsync(S.slots.p, S.h_in.p, slot_b, cudaMemcpyHostToDevice, g_stream));
    CK(cudaMemcpyAsync(S.io_in.p, S.h_in.as<uint8_t>() + align256(slot_b), dim * 4, cudaMemcpyHostToDevice, g_stream));
    quantize_inputs(S.io_in.as<float>(), 1, dim, need256, need32, g_stream);
    launch_experts_host(S.slots.as<Slot>(), (int)n, (int)max_ffn, (int)dim, make_xq(true, dim), make_xq(false, dim),
                        S.act.as<float>(), S.aq.as<int8_t>(), S.ad.as<float>(), S.as.as<int32_t>(), S.io_out.as<float>(),
                        g_stream);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(S.h_out.p, S.io_out.p, dim * 4, cudaMemcpyDeviceToHost, g_stream));
    CK(seam_wait());  // the seam returns with `out` written
    memcpy(out, S.h_out.p, dim * 4);
    g_cmdbufs++;
    return LOOM_CUDA_OK;
}

int loom_cuda_moe_ffn_routed(const float *normed, size_t dim, const float *logits, const float *bias, loom_weight gate,
                             loom_weight up, loom_weight down, const loom_weight *shexp3, size_t ffn, size_t shexp_ffn,
                             loom_routed_cfg cfg, float *out) {
    if (int rc = need_init()) return rc;
    if (cfg.n_expert == 0 || cfg.n_expert > 1024 || cfg.n_used == 0 || cfg.n_used > 64 || cfg.n_used > cfg.n_expert)
        return decline("router shape out of range (moe.zig:48-49)");
    if (dim == 0 || ffn == 0) return decline("empty layer");
    Tensor *g, *u, *d;
    if (int rc = resolve(gate.ggml_type, gate.data, gate.bytes, g)) return rc;
    if (int rc = resolve(up.ggml_type, up.data, up.bytes, u)) return rc;
    if (int rc = resolve(down.ggml_type, down.data, down.bytes, d)) return rc;
    const Tensor *sh[3] = {nullptr, nullptr, nullptr};
    if (shexp3) {
        for (int i = 0; i < 3; i++) {
            Tensor *t;
            if (int rc = resolve(shexp3[i].ggml_type, shexp3[i].data, shexp3[i].bytes, t)) return rc;
            sh[i] = t;
        }
    }
    RoutedLayerDev L{};
    if (int rc = routed_layer(L, g, u, d, dim, ffn, cfg.n_expert, sh, shexp_ffn)) return rc;
    L.n_expert = (int)cfg.n_expert;
    L.n_used = (int)cfg.n_used;
    L.gating = cfg.gating_sigmoid ? 2 : 1;
    L.weights_norm = cfg.weights_norm;
    L.weights_scale = cfg.weights_scale;
    L.n_group = L.topk_group = 1;
    L.expert0 = 0;
    L.n_local = (int)cfg.n_expert;
    const size_t in_b = (dim + 2 * cfg.n_expert) * 4;
    if (int rc = S.h_in.ensure(in_b)) return rc;
    if (int rc = S.h_out.ensure(dim * 4)) return rc;
    if (int rc = S.io_in.ensure(in_b)) return rc;
    if (int rc = S.io_out.ensure(dim * 4)) return rc;
    float *hin = S.h_in.as<float>();
    memcpy(hin, normed, dim * 4);
    memcpy(hin + dim, logits, cfg.n_expert * 4);
    if (bias) memcpy(hin + dim + cfg.n_expert, bias, cfg.n_expert * 4);
    auto base = [](const Tensor *t) -> uint64_t { return t ? (uint64_t)(uintptr_t)t->base : 0; };
    const std::vector<uint64_t> key = {2, (uint64_t)g->type, base(g), (uint64_t)u->type, base(u), (uint64_t)d->type,
                                       base(d), base(sh[0]), base(sh[1]), base(sh[2]), dim, ffn, shexp_ffn,
                                       cfg.n_expert, cfg.n_used, (uint64_t)cfg.gating_sigmoid,
                                       (uint64_t)cfg.weights_norm, fbits(cfg.weights_scale), bias ? 1u : 0u,
                                       (uint64_t)g_force_generic | (uint64_t)g_tc_exact << 8};
    if (int rc = seam_run(key, [&]() -> int {
            CK(cudaMemcpyAsync(S.io_in.p, S.h_in.p, in_b, cudaMemcpyHostToDevice, g_stream));
            const float *dx = S.io_in.as<float>();
            if (int rc = moe_routed_dev(L, 1, nullptr, dx, dx + dim, bias ? dx + dim + cfg.n_expert : nullptr,
                                        S.io_out.as<float>(), nullptr, nullptr, g_stream))
                return rc;
            CK(cudaMemcpyAsync(S.h_out.p, S.io_out.p, dim * 4, cudaMemcpyDeviceToHost, g_stream));
            return 0;
        }))
        return rc;
    CK(seam_wait());  // the seam returns with `out` written
    memcpy(out, S.h_out.p, dim * 4);
    g_cmdbufs++;
    return LOOM_CUDA_OK;
}

// ---- device-resident API ------------------------------------------------------------

int loom_cuda_tensor_upload(int type, const void *data, size_t bytes, loom_tensor *out) {
    if (int rc = need_init()) return rc;
    uint64_t h = 0;
    if (int rc = upload_tensor(type, data, bytes, h)) return rc;
    *out = h;
    return LOOM_CUDA_OK;
}

int loom_cuda_tensor_synth(int type, uint64_t nblk, uint64_t seed, float sigma, loom_tensor *out) {
    return loom_cuda_tensor_synth_range(type, 0, nblk, seed, sigma, out);
}

int loom_cuda_tensor_synth_range(int type, uint64_t blk0, uint64_t nblk, uint64_t seed, float sigma, loom_tensor *out) {
    if (int rc = need_init()) return rc;
    if (!type_ok(type)) return decline("unsupported ggml type");
    Tensor t;
    if (int rc = alloc_tensor(type, nblk, t)) return rc;
    const size_t bb = block_bytes(type);
    if (raw_layout(type)) {
        launch_synth(type, t.base, blk0, nblk, seed, sigma, g_stream);
    } else {
        // generate GGUF bytes in bounded chunks, then repack each into the layout
        const uint64_t chunk = std::max<uint64_t>(1, (256ull << 20) / bb);
        if (int rc = S.raw.ensure(std::min<uint64_t>(chunk, nblk) * bb)) {
            cudaFree(t.base);
            return rc;
        }
        for (uint64_t b0 = 0; b0 < nblk; b0 += chunk) {
            const uint64_t nb = std::min(chunk, nblk - b0);
            launch_synth(type, S.raw.as<uint8_t>(), blk0 + b0, nb, seed, sigma, g_stream);
            uint8_t *q = t.base + b0 * layout_qbytes(type);
            uint8_t *sc = t.w.sc ? const_cast<uint8_t *>(t.w.sc) + b0 * 16 : nullptr;
            uint16_t *d = t.w.d ? const_cast<uint16_t *>(t.w.d) + b0 : nullptr;
            launch_repack(type, S.raw.as<uint8_t>(), q, sc, d, nb, g_stream);
        }
    }
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) {
        cudaFree(t.base);
        return fail("tensor_synth", e);
    }
    if (int rc = mark_q6k(t)) {
        cudaFree(t.base);
        return rc;
    }
    uint64_t h = g_next_handle++;
    g_tensors[h] = t;
    *out = h;
    return LOOM_CUDA_OK;
}

int loom_cuda_tensor_download(loom_tensor h, void *dst, size_t bytes) {
    if (int rc = need_init()) return rc;
    Tensor *t = lookup(h);
    if (!t) return decline("unknown tensor");
    const size_t raw_b = t->nblk * (size_t)block_bytes(t->type);
    if (bytes != raw_b) return decline("size mismatch");
    if (raw_layout(t->type)) {
        CK(cudaMemcpyAsync(dst, t->base, raw_b, cudaMemcpyDeviceToHost, g_stream));
    } else {
        if (int rc = S.raw.ensure(raw_b)) return rc;
        launch_unpack(t->type, t->w, S.raw.as<uint8_t>(), t->nblk, g_stream);
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(dst, S.raw.p, raw_b, cudaMemcpyDeviceToHost, g_stream));
    }
    CK(cudaStreamSynchronize(g_stream));
    return LOOM_CUDA_OK;
}

int loom_cuda_tensor_free(loom_tensor h) {
    if (int rc = need_init()) return rc;
    Tensor *t = lookup(h);
    if (!t) return decline("unknown tensor");
    CK(cudaStreamSynchronize(g_stream));
    cudaFree(t->base);
    g_buf_gen++;
    for (auto it = g_cache.begin(); it != g_cache.end();)
        it = it->second == h ? g_cache.erase(it) : std::next(it);
    g_tensors.erase(h);
    return LOOM_CUDA_OK;
}

size_t loom_cuda_tensor_device_bytes(loom_tensor h) {
    Tensor *t = lookup(h);
    return t ? t->dev_bytes : 0;
}

int loom_cuda_reserve(size_t T, size_t dim, size_t ffn, size_t n_expert, size_t n_used) {
    if (int rc = need_init()) return rc;
    const size_t n_slots = T * (n_used + 1);
    if (int rc = ensure_moe_scratch(T, dim, ffn, n_expert, n_slots)) return rc;
    if (int rc = S.grp.ensure((3 * n_expert + T * n_used + 4) * 4)) return rc;
    if (int rc = S.ybuf.ensure(n_slots * dim * 4)) return rc;
    CK(cudaStreamSynchronize(g_stream));
    return LOOM_CUDA_OK;
}

int loom_cuda_moe_forward(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out, const float *d_residual,
                          const float *d_logits, uint32_t *d_ids, void *stream) {
    struct PrenormOnce {  // a pending FFN-norm fold applies to this call only, whatever it returns
        ~PrenormOnce() { g_prenorm_w = nullptr; }
    } prenorm_once;
    if (int rc = need_init()) return rc;
    if (!desc || T == 0) return decline("empty forward");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    const loom_moe_desc &D = *desc;
    if (D.n_expert == 0 || D.n_expert > 1024 || D.n_used == 0 || D.n_used > 64 || D.n_used > D.n_expert)
        return decline("router shape out of range (moe.zig:48-49)");
    const size_t n_local = D.n_local ? D.n_local : D.n_expert;
    if (D.expert0 + n_local > D.n_expert) return decline("expert range out of bounds");
    Tensor *g = lookup(D.gate), *u = lookup(D.up), *dn = lookup(D.down);
    const Tensor *sh[3] = {nullptr, nullptr, nullptr};
    if (D.shexp_gate) {
        sh[0] = lookup(D.shexp_gate);
        sh[1] = lookup(D.shexp_up);
        sh[2] = lookup(D.shexp_down);
        if (!sh[0] || !sh[1] || !sh[2]) return decline("unknown shared-expert tensor");
    }
    RoutedLayerDev L{};
    if (int rc = routed_layer(L, g, u, dn, D.dim, D.ffn, n_local, sh, D.shexp_ffn)) return rc;
    L.n_expert = (int)D.n_expert;
    L.n_used = (int)D.n_used;
    L.gating = D.gating ? D.gating : 1;
    L.weights_norm = D.weights_norm;
    L.weights_scale = D.weights_scale;
    if (int rc = group_cfg(D, L)) return rc;
    L.expert0 = (int)D.expert0;
    L.n_local = (int)n_local;
    const float *bias = nullptr;
    if (D.router_bias) {
        Tensor *b = lookup(D.router_bias);
        if (!b || b->type != T_F32 || b->nblk < D.n_expert) return decline("router bias must be f32 [n_expert]");
        bias = reinterpret_cast<const float *>(b->base);
    }
    const size_t max_ffn = std::max<size_t>(D.ffn, sh[0] ? D.shexp_ffn : 0);
    const size_t n_slots = T * D.n_used + (sh[0] ? T : 0);
    if (int rc = ensure_moe_scratch(T, D.dim, max_ffn, D.n_expert, n_slots)) return rc;
    const float *router = nullptr;
    if (!d_logits) {
        Tensor *r = lookup(D.router);
        if (!r || r->type != T_F32 || r->nblk < D.n_expert * D.dim) return decline("router must be f32 [n_expert][dim]");
        router = reinterpret_cast<const float *>(r->base);
    }
    g_next_router = nullptr;
    g_next_router_bytes = 0;
    if (D.next_router) {
        Tensor *nr = lookup(D.next_router);
        if (nr && nr->type == T_F32) {
            g_next_router = nr->base;
            g_next_router_bytes = nr->nblk * 4;
        }
    }
    // expert parallel: this rank's partial, then the sum over ranks (residual once)
    const bool sharded = ep_active() && n_local < D.n_expert;
    const float *res = sharded && ep_rank() != 0 ? nullptr : d_residual;
    const int rc = moe_routed_dev(L, T, router, d_x, d_logits, bias, d_out, res, d_ids, st);
    g_next_router = nullptr;
    if (rc) return rc;
    if (sharded) {
        if (int e = ep_allreduce_sum(d_out, T * D.dim, st, g_err)) return e;
    }
    CK(cudaGetLastError());
    return LOOM_CUDA_OK;
}

// All-to-all expert parallelism (a2a.cu): route this rank's own tokens, send
// each routed row to the expert's owner, run the rows that arrive through
// this rank's experts, send the outputs back, combine in selection order.
}  // extern "C"

namespace {

// Both all-to-all forms: t_cap == 0 sends exactly the routed rows (their
// counts go to the host once per layer); t_cap > 0 sends fixed runs of
// t_cap * n_used rows to every rank (no host synchronisation).
// The all-to-all layer is a collective: a rank that declined alone would leave
// its peers blocked in the exchange. So every layer shape is agreed once
// (every rank valid, the same t_cap and shapes) before its first exchange,
// and declined on every rank otherwise; and a rank with more tokens than the
// fixed capacity still takes part (it sends none of its rows, runs the rows
// its peers send it) and then declines for its own tokens.
std::set<std::vector<int>> g_a2a_agreed;

int ep_a2a_checked(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out, const float *d_residual,
                   const float *d_logits, uint32_t *d_ids, void *stream, size_t t_cap);

int ep_a2a(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out, const float *d_residual,
           const float *d_logits, uint32_t *d_ids, void *stream, size_t t_cap) {
    if (int rc = need_init()) return rc;
    if (!ep_active()) return ep_a2a_checked(desc, d_x, T, d_out, d_residual, d_logits, d_ids, stream, t_cap);
    // this rank's verdict on the layer shape (the local checks, no work), then the agreement
    const int local = ep_a2a_checked(desc, nullptr, 0, nullptr, nullptr, d_logits, nullptr, stream, t_cap | (1ull << 62));
    std::vector<int> key{local == LOOM_CUDA_OK ? 1 : 0, (int)t_cap, desc ? (int)desc->n_expert : 0,
                         desc ? (int)desc->n_used : 0, desc ? (int)desc->dim : 0, desc ? (int)desc->ffn : 0,
                         desc && desc->shexp_gate ? (int)desc->shexp_ffn : -1, d_logits ? 1 : 0};
    if (!g_a2a_agreed.count(key)) {
        if (!ep_agree(key.data(), (int)key.size(), g_err)) return decline("the ranks disagree on the all-to-all layer (shape, t_cap or a local check)");
        if (key[0] == 0) return local;  // every rank declined alike
        g_a2a_agreed.insert(key);
    }
    if (local != LOOM_CUDA_OK) return local;
    return ep_a2a_checked(desc, d_x, T, d_out, d_residual, d_logits, d_ids, stream, t_cap);
}

// t_cap's bit 62: validate only (no launches, no exchange).
int ep_a2a_checked(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out, const float *d_residual,
                   const float *d_logits, uint32_t *d_ids, void *stream, size_t t_cap) {
    const bool check_only = (t_cap >> 62) & 1;
    t_cap &= ~(1ull << 62);
    if (!desc) return decline("no layer description");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    const loom_moe_desc &D = *desc;
    if (D.n_expert == 0 || D.n_expert > 1024 || D.n_used == 0 || D.n_used > 64 || D.n_used > D.n_expert)
        return decline("router shape out of range (moe.zig:48-49)");
    const int world = ep_active() ? ep_size() : 1, me = ep_active() ? ep_rank() : 0;
    if (world > A2A_MAX_RANKS) return decline("too many ranks for the all-to-all layer");
    const size_t e0 = (size_t)me * D.n_expert / world, e1 = (size_t)(me + 1) * D.n_expert / world;
    const size_t n_local = D.n_local ? D.n_local : D.n_expert;
    if (D.expert0 != e0 || n_local != e1 - e0)
        return decline("the all-to-all layer needs this rank's contiguous shard [r*E/R, (r+1)*E/R)");
    if (D.dim % 4) return decline("dim must be a multiple of 4");
    Tensor *g = lookup(D.gate), *u = lookup(D.up), *dn = lookup(D.down);
    const Tensor *sh[3] = {nullptr, nullptr, nullptr};
    if (D.shexp_gate) {
        sh[0] = lookup(D.shexp_gate);
        sh[1] = lookup(D.shexp_up);
        sh[2] = lookup(D.shexp_down);
        if (!sh[0] || !sh[1] || !sh[2]) return decline("unknown shared-expert tensor");
    }
    RoutedLayerDev L{};
    if (int rc = routed_layer(L, g, u, dn, D.dim, D.ffn, n_local, sh, D.shexp_ffn)) return rc;
    L.n_expert = (int)D.n_expert;
    L.n_used = (int)D.n_used;
    L.gating = D.gating ? D.gating : 1;
    L.weights_norm = D.weights_norm;
    L.weights_scale = D.weights_scale;
    if (int rc = group_cfg(D, L)) return rc;
    L.expert0 = (int)e0;
    L.n_local = (int)n_local;
    const float *bias = nullptr;
    if (D.router_bias) {
        Tensor *b = lookup(D.router_bias);
        if (!b || b->type != T_F32 || b->nblk < D.n_expert) return decline("router bias must be f32 [n_expert]");
        bias = reinterpret_cast<const float *>(b->base);
    }
    const float *router = nullptr;
    if (!d_logits) {
        Tensor *r = lookup(D.router);
        if (!r || r->type != T_F32 || r->nblk < D.n_expert * D.dim) return decline("router must be f32 [n_expert][dim]");
        router = reinterpret_cast<const float *>(r->base);
    }
    const size_t dim = D.dim, k = D.n_used;
    if (t_cap && (size_t)world * t_cap * k > (1u << 24)) return decline("all-to-all capacity out of range");
    if (check_only) return LOOM_CUDA_OK;
    // more tokens than the capacity: take part without sending any of this rank's rows, then decline
    const bool over = t_cap && T > t_cap;
    if (over) T = 0;
    const size_t ns = T * k;
    const size_t cap = t_cap * k, nsend = std::max(ns, (size_t)world * cap);  // send-list entries
    const size_t max_ffn = std::max<size_t>(D.ffn, sh[0] ? D.shexp_ffn : 0), act_stride = align256(max_ffn);
    // home side: route, then the destination-ordered send lists
    if (int rc = ensure_moe_scratch(std::max<size_t>(T, 1), dim, max_ffn, D.n_expert, std::max<size_t>(T, 1) * (k + 1)))
        return rc;
    const size_t ni = align256(nsend + 1);
    if (int rc = S.a2a_i.ensure((4 * ni + 2 * A2A_MAX_RANKS) * 4)) return rc;
    if (int rc = S.a2a_sx.ensure(std::max<size_t>(nsend, 1) * dim * 4)) return rc;
    if (int rc = S.a2a_yb.ensure(std::max<size_t>(nsend, 1) * dim * 4)) return rc;
    if (int rc = S.a2a_ysh.ensure(std::max<size_t>(T, 1) * dim * 4)) return rc;
    if (int rc = S.h_cnt.ensure(2 * A2A_MAX_RANKS * 4)) return rc;
    int *send_eid = S.a2a_i.as<int>(), *send_tok = send_eid + ni, *slot_pos = send_tok + ni;
    float *home_gates = reinterpret_cast<float *>(slot_pos + ni);
    int *cnt = slot_pos + 2 * ni;  // [A2A_MAX_RANKS] sent, then [A2A_MAX_RANKS] received
    if (T) {
        if (router) {
            launch_mm_f32(router, L.n_expert, L.dim, d_x, (int)T, S.logits.as<float>(), st);
            d_logits = S.logits.as<float>();
        }
        launch_route(d_logits, bias, (int)T, L.n_expert, L.n_used, L.gating, L.weights_norm, L.weights_scale,
                     S.ids.as<int>(), S.gates.as<float>(), st, L.n_group, L.topk_group);
        CK(cudaMemcpyAsync(home_gates, S.gates.p, ns * 4, cudaMemcpyDeviceToDevice, st));
        if (d_ids) CK(cudaMemcpyAsync(d_ids, S.ids.p, ns * 4, cudaMemcpyDeviceToDevice, st));
    }
    launch_a2a_pack(S.ids.as<int>(), (int)T, (int)k, (int)D.n_expert, world, (int)cap, d_x, (int)dim, send_eid,
                    send_tok, slot_pos, cnt, S.a2a_sx.as<float>(), st);
    std::vector<size_t> scnt(world), soff(world), rcnt(world), roff(world);
    size_t nr = 0;
    if (cap) {  // fixed runs: every size is known without looking at the routing
        for (int r = 0; r < world; r++) {
            scnt[r] = rcnt[r] = cap;
            soff[r] = roff[r] = (size_t)r * cap;
        }
        nr = (size_t)world * cap;
    } else {  // counts: one int to and from every rank, then to the host
        std::vector<size_t> one(world, 1), idx(world);
        for (int r = 0; r < world; r++) idx[r] = r;
        if (int e = ep_alltoallv(cnt, idx.data(), one.data(), cnt + A2A_MAX_RANKS, idx.data(), one.data(), 4, st,
                                 g_err))
            return e;
        CK(cudaMemcpyAsync(S.h_cnt.p, cnt, 2 * A2A_MAX_RANKS * 4, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        const int *hc = S.h_cnt.as<int>();
        size_t so = 0;
        for (int r = 0; r < world; r++) {
            scnt[r] = (size_t)hc[r];
            rcnt[r] = (size_t)hc[A2A_MAX_RANKS + r];
            soff[r] = so;
            roff[r] = nr;
            so += scnt[r];
            nr += rcnt[r];
        }
        if (so != ns) return fail("all-to-all pack", cudaErrorUnknown);
    }
    // receive side buffers (sized now that the counts are known)
    if (int rc = S.a2a_rx.ensure(std::max<size_t>(nr, 1) * dim * 4)) return rc;
    if (int rc = S.a2a_re.ensure(std::max<size_t>(nr, 1) * 4)) return rc;
    if (int rc = S.a2a_yr.ensure(std::max<size_t>(nr, 1) * dim * 4)) return rc;
    if (int rc = S.a2a_g1.ensure(std::max<size_t>(nr, 1) * 4)) return rc;
    const size_t nmax = std::max<size_t>(std::max(T, nr), 1);
    if (int rc = ensure_moe_scratch(nmax, dim, max_ffn, D.n_expert, nmax * (k + 1))) return rc;
    if (int e = ep_alltoallv(S.a2a_sx.p, soff.data(), scnt.data(), S.a2a_rx.p, roff.data(), rcnt.data(), dim * 4, st,
                             g_err))
        return e;
    if (int e = ep_alltoallv(send_eid, soff.data(), scnt.data(), S.a2a_re.p, roff.data(), rcnt.data(), 4, st, g_err))
        return e;
    // the shared expert of this rank's own tokens (replicated weights)
    const float *y_sh = nullptr;
    if (sh[0] && T) {
        RoutedLayerDev Ls = L;
        Ls.n_used = 0;
        quantize_inputs(d_x, T, dim, any_type(Ls, true), any_type(Ls, false), st);
        launch_experts_routed(Ls, nullptr, nullptr, (int)T, (int)act_stride, make_xq(true, dim), make_xq(false, dim),
                              S.act.as<float>(), S.aq.as<int8_t>(), S.ad.as<float>(), S.as.as<int32_t>(),
                              S.a2a_ysh.as<float>(), nullptr, st);
        y_sh = S.a2a_ysh.as<float>();
    }
    // the rows that arrived, each through its one local expert with weight 1
    if (nr) {
        RoutedLayerDev Lr = L;
        Lr.n_used = 1;
        Lr.has_shared = 0;
        DecodeArgs A = decode_args(Lr, nr, nullptr, S.a2a_rx.as<float>(), nullptr, nullptr, S.a2a_yr.as<float>(),
                                   nullptr, nullptr, act_stride);
        A.ids_in = S.a2a_re.as<int>();
        A.trace = nullptr;
        if (g_force_generic != 1 && batch_supported(A)) {
            // expert-major: each local expert's rows against one read of its weights
            const int path = batch_path(A, nr, Lr.n_local);
            if (int rc = S.grp.ensure((3 * (size_t)Lr.n_local + nr + 4) * 4)) return rc;
            if (int rc = S.ybuf.ensure(nr * dim * 4)) return rc;
            A.grp_cnt = S.grp.as<int>();
            A.grp_off = A.grp_cnt + Lr.n_local;
            A.grp_list = A.grp_off + Lr.n_local;
            A.tc_pre = A.grp_list + nr;
            g_last_path = path;
            A.y = S.ybuf.as<float>();
            CK(launch_batch(A, path, st));
        } else {  // per-row slot kernels
            launch_a2a_fill(S.a2a_g1.as<float>(), (int)nr, 1.0f, st);
            quantize_inputs(S.a2a_rx.as<float>(), nr, dim, any_type(Lr, true), any_type(Lr, false), st);
            launch_experts_routed(Lr, S.a2a_re.as<int>(), S.a2a_g1.as<float>(), (int)nr, (int)act_stride,
                                  make_xq(true, dim), make_xq(false, dim), S.act.as<float>(), S.aq.as<int8_t>(),
                                  S.ad.as<float>(), S.as.as<int32_t>(), S.a2a_yr.as<float>(), nullptr, st);
        }
    }
    // outputs back to the rows' home ranks (the reverse of the dispatch)
    if (int e = ep_alltoallv(S.a2a_yr.p, roff.data(), rcnt.data(), S.a2a_yb.p, soff.data(), scnt.data(), dim * 4, st,
                             g_err))
        return e;
    launch_a2a_combine(S.a2a_yb.as<float>(), slot_pos, home_gates, y_sh, d_residual, d_out, (int)T, (int)k, (int)dim,
                       st);
    CK(cudaGetLastError());
    if (over) return decline("more tokens than the all-to-all capacity (this rank's rows were not sent; its peers' were run)");
    return LOOM_CUDA_OK;
}

}  // namespace

extern "C" {

int loom_cuda_ep_a2a_forward(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out,
                             const float *d_residual, const float *d_logits, uint32_t *d_ids, void *stream) {
    return ep_a2a(desc, d_x, T, d_out, d_residual, d_logits, d_ids, stream, 0);
}

int loom_cuda_ep_a2a_forward_cap(const loom_moe_desc *desc, const float *d_x, size_t T, size_t t_cap, float *d_out,
                                 const float *d_residual, const float *d_logits, uint32_t *d_ids, void *stream) {
    if (t_cap == 0) return decline("the fixed-capacity all-to-all needs t_cap >= 1");
    return ep_a2a(desc, d_x, T, d_out, d_residual, d_logits, d_ids, stream, t_cap);
}

int loom_cuda_tensor_matmul(loom_tensor h, size_t rows, size_t cols, const float *d_xs, size_t n, float *d_out,
                            void *stream) {
    if (int rc = need_init()) return rc;
    Tensor *t = lookup(h);
    if (!t) return decline("unknown tensor");
    const size_t be = block_elems(t->type);
    if (cols == 0 || cols % be || t->nblk < rows * (cols / be)) return decline("shape does not fit the tensor");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    if (t->type == T_F32) {
        launch_mm_f32(reinterpret_cast<const float *>(t->base), (int)rows, (int)cols, d_xs, (int)n, d_out, st);
    } else if (t->type == T_Q5_0) {
        launch_mm_q50(t->w, 0, (int)rows, (int)cols, d_xs, (int)n, d_out, st);
    } else {
        if (int rc = ensure_xq(n, cols)) return rc;
        quantize_into(d_xs, n, cols, act256(t->type), st);
        if (n == 1 && gemv_stream_supported(t->type, (int)rows, (int)cols))  // one vector, a large matrix
            CK(launch_gemv_stream(t->w, (int)rows, (int)cols, make_xq(act256(t->type), cols), d_out, st));
        else
            launch_mm(t->w, 0, (int)rows, (int)cols, make_xq(act256(t->type), cols), (int)n, d_out, st);
    }
    CK(cudaGetLastError());
    return LOOM_CUDA_OK;
}

// sampler.zig:7-15 argmax on device logits.
int loom_cuda_argmax(const float *d_logits, size_t n, uint32_t *d_index, void *stream) {
    if (int rc = need_init()) return rc;
    if (!d_logits || !d_index || n == 0 || n > 0x7FFFFFFFu) return decline("argmax needs 1 <= n < 2^31 logits");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    if (int rc = S.amax.ensure(16, true)) return rc;
    launch_argmax(d_logits, (int)n, S.amax.as<unsigned long long>(), reinterpret_cast<unsigned *>(S.amax.as<uint8_t>() + 8),
                  d_index, st);
    CK(cudaGetLastError());
    return LOOM_CUDA_OK;
}

// The output head and greedy sampling of one token (llama.zig:1225-1226 +
// sampler.zig:7-15): logits = W x through the bit-exact matvec of the
// tensor's type, then their argmax.
int loom_cuda_lm_head_argmax(loom_tensor w, size_t vocab, size_t dim, const float *d_x, float *d_logits,
                             uint32_t *d_index, void *stream) {
    if (int rc = need_init()) return rc;
    if (!d_index || vocab == 0 || vocab > 0x7FFFFFFFu) return decline("lm_head needs 1 <= vocab < 2^31");
    if (!d_logits) {
        if (int rc = S.head_logits.ensure(vocab * 4)) return rc;
        d_logits = S.head_logits.as<float>();
    }
    if (int rc = loom_cuda_tensor_matmul(w, vocab, dim, d_x, 1, d_logits, stream)) return rc;
    return loom_cuda_argmax(d_logits, vocab, d_index, stream);
}

}  // extern "C"

// ---- allocation-free MoE layer ----------------------------------------------------
// For callers that must not allocate device memory while they run: code that
// executes inside a CUDA stream capture owned by someone else, a host engine
// whose memory is budgeted up front, or a process sharing the GPU under a
// fixed allocation. The layer's scratch lives in one fixed array that the
// library image carries on every device it is loaded on, so this entry point
// never calls cudaMalloc/cudaFree and never grows the backend's own scratch.

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(1) << 20;  // LOOM_CUDA_NOALLOC_SCRATCH_BYTES
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];
constexpr int NOALLOC_MAX_DEVICES = 64;
uint8_t *g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};  // device address of g_noalloc_scratch, per device

// Carve the decode-path scratch out of [base, base + NOALLOC_SCRATCH_BYTES);
// returns the bytes used (0 when it does not fit).
size_t noalloc_layout(uint8_t *base, size_t T, size_t dim, size_t n_expert, size_t n_used, size_t n_slots,
                      size_t act_stride, DecodeArgs &A) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *p = base + off;
        off += align256(bytes);
        return p;
    };
    A.x256 = XQW{reinterpret_cast<int8_t *>(take(T * dim)), reinterpret_cast<float *>(take(T * (dim / 256 + 1) * 4)),
                 reinterpret_cast<int32_t *>(take(T * (dim / 16 + 1) * 4))};
    A.x32 = XQW{reinterpret_cast<int8_t *>(take(T * dim)), reinterpret_cast<float *>(take(T * (dim / 32 + 1) * 4)),
                reinterpret_cast<int32_t *>(take(T * (dim / 32 + 1) * 4))};
    A.logits = reinterpret_cast<float *>(take(T * n_expert * 4));
    A.ids = reinterpret_cast<int *>(take(T * n_used * 4));
    A.gates = reinterpret_cast<float *>(take(T * n_used * 4));
    A.act = reinterpret_cast<float *>(take(n_slots * act_stride * 4));
    A.aq = reinterpret_cast<int8_t *>(take(n_slots * act_stride));
    A.ad = reinterpret_cast<float *>(take(n_slots * (act_stride / 32) * 4));
    A.as = reinterpret_cast<int32_t *>(take(n_slots * (act_stride / 16) * 4));
    return off <= NOALLOC_SCRATCH_BYTES ? off : 0;
}

}  // namespace

extern "C" int loom_cuda_moe_forward_noalloc(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out,
                                             const float *d_residual, void *stream) {
    if (int rc = need_init()) return rc;
    if (!desc || T == 0) return decline("empty forward");
    if (g_device < 0 || g_device >= NOALLOC_MAX_DEVICES) return decline("device index out of range for the fixed scratch");
    // once per device, with that device current: the device address of the
    // fixed array (host code only has a stand-in symbol for it)
    if (!g_noalloc_ptr[g_device]) {
        void *p = nullptr;
        CK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[g_device] = static_cast<uint8_t *>(p);
    }
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    const loom_moe_desc &D = *desc;
    if (D.n_expert == 0 || D.n_expert > 1024 || D.n_used == 0 || D.n_used > 64 || D.n_used > D.n_expert)
        return decline("router shape out of range (moe.zig:48-49)");
    const size_t n_local = D.n_local ? D.n_local : D.n_expert;
    if (D.expert0 + n_local > D.n_expert) return decline("expert range out of bounds");
    Tensor *g = lookup(D.gate), *u = lookup(D.up), *dn = lookup(D.down), *r = lookup(D.router);
    const Tensor *sh[3] = {nullptr, nullptr, nullptr};
    if (D.shexp_gate) {
        sh[0] = lookup(D.shexp_gate);
        sh[1] = lookup(D.shexp_up);
        sh[2] = lookup(D.shexp_down);
        if (!sh[0] || !sh[1] || !sh[2]) return decline("unknown shared-expert tensor");
    }
    if (!r || r->type != T_F32 || r->nblk < D.n_expert * D.dim) return decline("router must be f32 [n_expert][dim]");
    RoutedLayerDev L{};
    if (int rc = routed_layer(L, g, u, dn, D.dim, D.ffn, n_local, sh, D.shexp_ffn)) return rc;
    L.n_expert = (int)D.n_expert;
    L.n_used = (int)D.n_used;
    L.gating = D.gating ? D.gating : 1;
    L.weights_norm = D.weights_norm;
    L.weights_scale = D.weights_scale;
    if (int rc = group_cfg(D, L)) return rc;
    L.expert0 = (int)D.expert0;
    L.n_local = (int)n_local;
    const float *bias = nullptr;
    if (D.router_bias) {
        Tensor *b = lookup(D.router_bias);
        if (!b || b->type != T_F32 || b->nblk < D.n_expert) return decline("router bias must be f32 [n_expert]");
        bias = reinterpret_cast<const float *>(b->base);
    }
    const size_t max_ffn = std::max<size_t>(D.ffn, sh[0] ? D.shexp_ffn : 0);
    const size_t n_slots = T * D.n_used + (sh[0] ? T : 0);
    const size_t act_stride = align256(max_ffn);
    if (T > DECODE_MAX_T) return decline("the allocation-free layer takes at most 16 tokens");
    DecodeArgs A{};
    if (!noalloc_layout(g_noalloc_ptr[g_device], T, D.dim, D.n_expert, D.n_used, n_slots, act_stride, A))
        return decline("layer scratch exceeds the 1 MiB fixed array of the allocation-free entry point");
    A.T = (int)T;
    A.dim = L.dim;
    A.ffn = L.ffn;
    A.n_expert = L.n_expert;
    A.n_used = L.n_used;
    A.gating = L.gating;
    A.weights_norm = L.weights_norm;
    A.weights_scale = L.weights_scale;
    A.n_group = L.n_group;
    A.topk_group = L.topk_group;
    A.expert0 = L.expert0;
    A.n_local = L.n_local;
    A.router = reinterpret_cast<const float *>(r->base);
    A.bias = bias;
    A.x = d_x;
    A.out = d_out;
    A.residual = d_residual;
    A.need256 = any_type(L, true);
    A.need32 = any_type(L, false);
    A.g = L.g;
    A.u = L.u;
    A.dn = L.dn;
    A.has_shared = L.has_shared;
    A.sg = L.sg;
    A.su = L.su;
    A.sdn = L.sdn;
    A.shexp_ffn = L.shexp_ffn;
    A.act_stride = (int)act_stride;
    if (!decode_supported(A)) return decline("layer shape not covered by the fused decode kernels");
    CK(launch_decode(A, st));
    return LOOM_CUDA_OK;
}

// ---- persistent decode stack --------------------------------------------------------

namespace {
struct StackRec {
    StackArgs args{};
    size_t tagged_bytes = 0;  // logits + act, contiguous from args.logits
    size_t part_bytes = 0;    // tagged partial outputs at args.part
    int gty = 0, dty = 0;
    void *mem = nullptr;  // layers + buffers, one allocation
};
std::unordered_map<uint64_t, StackRec> g_stacks;
uint64_t g_next_stack = 1;
}  // namespace

extern "C" int loom_cuda_stack_prepare(const loom_moe_desc *descs, size_t n_layers, uint64_t *handle) {
    if (int rc = need_init()) return rc;
    if (!descs || n_layers == 0) return decline("empty stack");
    const loom_moe_desc &D0 = descs[0];
    std::vector<StackLayer> host(n_layers);
    int gty = -1, dty = -1;
    for (size_t l = 0; l < n_layers; l++) {
        const loom_moe_desc &D = descs[l];
        if (D.dim != D0.dim || D.ffn != D0.ffn || D.n_expert != D0.n_expert || D.n_used != D0.n_used ||
            D.gating != D0.gating || D.weights_norm != D0.weights_norm || D.weights_scale != D0.weights_scale)
            return decline("stack layers must share one shape and routing configuration");
        if (D.router_bias || D.shexp_gate || (D.n_local && D.n_local != D.n_expert) || D.expert0 ||
            (D.n_group > 1 && D.topk_group < D.n_group))
            return decline("the stack kernel takes plain routed layers (no bias, shared expert, sharding or groups)");
        Tensor *r = lookup(D.router), *g = lookup(D.gate), *u = lookup(D.up), *dn = lookup(D.down);
        const Tensor *sh[3] = {nullptr, nullptr, nullptr};
        RoutedLayerDev L{};
        if (!r || r->type != T_F32 || r->nblk < D.n_expert * D.dim) return decline("router must be f32 [n_expert][dim]");
        if (int rc = routed_layer(L, g, u, dn, D.dim, D.ffn, D.n_expert, sh, 0)) return rc;
        if (g->type != u->type) return decline("gate and up types differ");
        if (l == 0) {
            gty = g->type;
            dty = dn->type;
        } else if (g->type != gty || dn->type != dty) {
            return decline("stack layers must share block types");
        }
        host[l] = StackLayer{reinterpret_cast<const float *>(r->base), g->w, u->w, dn->w};
    }
    StackRec S;
    StackArgs &A = S.args;
    A.n_layers = (int)n_layers;
    A.dim = (int)D0.dim;
    A.ffn = (int)D0.ffn;
    A.n_expert = (int)D0.n_expert;
    A.n_used = (int)D0.n_used;
    A.gating = D0.gating ? D0.gating : 1;
    A.weights_norm = D0.weights_norm;
    A.weights_scale = D0.weights_scale;
    A.act_stride = (int)align256(D0.ffn);
    if (!stack_supported(A, gty, dty)) return decline("layer shape not covered by the stack kernel");
    const size_t lay_b = align256(n_layers * sizeof(StackLayer)), part_b = align256(2 * D0.n_used * D0.dim * 4);
    const size_t lg_b = align256((D0.n_expert + 32) * 8 * LOGIT_REPLICAS), act_b = align256(D0.n_used * (size_t)A.act_stride * 8);
    const size_t total = lay_b + part_b + lg_b + act_b + 256;
    CK(cudaMalloc(&S.mem, total));
    uint8_t *p = static_cast<uint8_t *>(S.mem);
    A.layers = reinterpret_cast<const StackLayer *>(p);
    A.part = reinterpret_cast<float *>(p + lay_b);
    A.logits = reinterpret_cast<unsigned long long *>(p + lay_b + part_b);
    A.act = reinterpret_cast<unsigned long long *>(p + lay_b + part_b + lg_b);
    A.bar = reinterpret_cast<unsigned *>(p + lay_b + part_b + lg_b + act_b);
    A.err = reinterpret_cast<int *>(A.bar + 2);
    CK(cudaMemcpy(p, host.data(), n_layers * sizeof(StackLayer), cudaMemcpyHostToDevice));
    CK(cudaMemset(p + lay_b, 0, total - lay_b));  // tagged words, barrier words, epoch
    S.tagged_bytes = lg_b + act_b;
    S.part_bytes = part_b;
    S.gty = gty;
    S.dty = dty;
    const uint64_t h = g_next_stack++;
    g_stacks[h] = S;
    *handle = h;
    return LOOM_CUDA_OK;
}

extern "C" int loom_cuda_stack_forward(uint64_t handle, const float *d_x, float *d_out, uint32_t *d_ids, void *stream) {
    if (int rc = need_init()) return rc;
    auto it = g_stacks.find(handle);
    if (it == g_stacks.end()) return decline("unknown stack");
    StackArgs A = it->second.args;
    A.x_in = d_x;
    A.residual = nullptr;
    A.out = d_out;
    A.ids_out = d_ids;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    CK(launch_stack(A, it->second.gty, it->second.dty, st));
    return LOOM_CUDA_OK;
}

extern "C" int loom_cuda_stack_forward_residual(uint64_t handle, const float *d_x, const float *d_residual,
                                                float *d_out, uint32_t *d_ids, void *stream) {
    if (int rc = need_init()) return rc;
    auto it = g_stacks.find(handle);
    if (it == g_stacks.end()) return decline("unknown stack");
    if (!d_residual) return decline("no residual");
    StackArgs A = it->second.args;
    A.x_in = d_x;
    A.residual = d_residual;
    A.out = d_out;
    A.ids_out = d_ids;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_stream;
    CK(launch_stack(A, it->second.gty, it->second.dty, st));
    return LOOM_CUDA_OK;
}

extern "C" int loom_cuda_stack_error(uint64_t handle) {
    auto it = g_stacks.find(handle);
    if (it == g_stacks.end()) return -1;
    int v = 0;
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) return -1;
    if (cudaMemcpy(&v, it->second.args.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v) {  // re-arm: barrier words, epoch, and every tagged word (so no stale tag can match)
        if (cudaMemset(it->second.args.bar, 0, 256) != cudaSuccess) return -1;
        if (cudaMemset(it->second.args.logits, 0, it->second.tagged_bytes) != cudaSuccess) return -1;
        if (cudaMemset(it->second.args.part, 0, it->second.part_bytes) != cudaSuccess) return -1;
    }
    return v;
}

extern "C" int loom_cuda_stack_trace(uint64_t handle, int enable, uint64_t *out, size_t n) {
    auto it = g_stacks.find(handle);
    if (it == g_stacks.end()) return decline("unknown stack");
    StackArgs &A = it->second.args;
    const size_t slots = (size_t)A.n_layers * STACK_TRACE_WORDS;
    if (enable && !A.trace) CK(cudaMalloc(&A.trace, slots * 8));
    if (enable) {
        CK(cudaMemset(A.trace, 0, slots * 8));
        return LOOM_CUDA_OK;
    }
    if (!A.trace) return decline("stack trace not enabled");
    CK(cudaDeviceSynchronize());
    if (out) CK(cudaMemcpy(out, A.trace, (n < slots ? n : slots) * 8, cudaMemcpyDeviceToHost));
    cudaFree(A.trace);
    A.trace = nullptr;
    return LOOM_CUDA_OK;
}

extern "C" int loom_cuda_stack_free(uint64_t handle) {
    auto it = g_stacks.find(handle);
    if (it == g_stacks.end()) return decline("unknown stack");
    cudaDeviceSynchronize();
    cudaFree(it->second.mem);
    if (it->second.args.trace) cudaFree(it->second.args.trace);
    g_stacks.erase(it);
    return LOOM_CUDA_OK;
}
