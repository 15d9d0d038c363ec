// decode.cu -- the fused MoE decode path: three kernels per layer chained
// with programmatic dependent launch (PDL), each issuing its weight loads
// before it waits for its producer.
//
//   k_router_route  one 8-CTA cluster per token: router GEMV (dotF32 order),
//                   logits gathered in CTA 0 through distributed shared
//                   memory, then route (moe.zig:106) and the token's
//                   activation quantization. Router weights are loaded BEFORE
//                   waiting for the previous layer.
//   k_gateup_dec    gate and up rows of every (token, expert) slot + SwiGLU.
//   k_down_dec      per output row: the token's expert activations quantized
//                   into shared memory, the local experts' down rows (weights
//                   loaded BEFORE waiting for k_gateup_dec), the weighted
//                   combine in selection order, the shared expert, the
//                   residual.
//
// Scratch that an earlier kernel wrote before this one's producer ran is read
// through L2 (ld.global.cg).
#include <cuda_runtime.h>

#include "decode.cuh"
#include "devutil.cuh"
#include "tma.cuh"
#include "warpdot.cuh"

namespace loom {

static inline unsigned cdivu(uint64_t a, uint64_t b) { return (unsigned)((a + b - 1) / b); }

// Phase tracing (off unless the caller passes a trace buffer): the first CTA
// start and the last CTA end of each kernel, in globaltimer nanoseconds.
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void trace_begin(const DecodeArgs &A, int k) {
    if (A.trace && threadIdx.x == 0) atomicMin(A.trace + 2 * (A.trace_slot + k), gtimer());
}
__device__ __forceinline__ void trace_end(const DecodeArgs &A, int k) {
    if (A.trace && threadIdx.x == 0) atomicMax(A.trace + 2 * (A.trace_slot + k) + 1, gtimer());
}

// Bulk prefetch of [p, p+bytes) into L2 (no data returned to the SM). p is
// rounded down and the end up to 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes + 15) & ~uintptr_t(15);
    while (a < e) {
        const uint32_t n = (uint32_t)((e - a) < 32768 ? (e - a) : 32768);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
        a += n;
    }
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---- router + route + activation quantization ---------------------------------------
// One thread-block cluster of RR_CLUSTER CTAs per token: warp w of the cluster
// computes router rows w, w + RR_WARPS_ALL, ... and writes each logit straight
// into CTA 0's shared memory (distributed shared memory); after one cluster
// barrier CTA 0 routes (warp 0) and quantizes the token's activation (the
// other warps). No global atomics or fences sit on this path.

constexpr int RR_CLUSTER = 8;
constexpr int RR_WARPS = 16;
constexpr int RR_WARPS_ALL = RR_CLUSTER * RR_WARPS;
constexpr int RR_CHUNK = 64;  // router weights per lane held in registers (2048 columns)

__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// store a float into CTA `rank`'s shared memory at the address of `local` in this CTA
__device__ __forceinline__ void st_cluster_f32(float *local, unsigned rank, float v) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// dotF32 (ggml.zig:198) of router row `wr` with x in shared memory; lane j is
// accumulator lane j. `w` holds the row's first RR_CHUNK*32 weights.
__device__ __forceinline__ float router_dot(const float (&w)[RR_CHUNK], const float *wr, const float *smx, int dim,
                                            int lane) {
    const int nfull = dim / 32;
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < RR_CHUNK; i++)
        if (i < nfull) a = fadd(a, fmul(w[i], smx[i * 32 + lane]));
    for (int i = RR_CHUNK; i < nfull; i++) a = fadd(a, fmul(__ldg(wr + i * 32 + lane), smx[i * 32 + lane]));
    int i = nfull * 32;
    for (; i + 8 <= dim; i += 8)
        if (lane < 8) a = fadd(a, fmul(__ldg(wr + i + lane), smx[i + lane]));
    const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
    const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
    const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
    const float v = fadd(fadd(fadd(a, a8), a16), a24);
    float r = __shfl_sync(0xffffffffu, v, 0);
#pragma unroll
    for (int jj = 1; jj < 8; jj++) r = fadd(r, __shfl_sync(0xffffffffu, v, jj));
    for (; i < dim; i++) r = fadd(r, fmul(__ldg(wr + i), smx[i]));
    return r;
}

__device__ __forceinline__ void load_row_chunk(float (&w)[RR_CHUNK], const float *wr, int dim, int lane) {
    const int nfull = dim / 32;
#pragma unroll
    for (int i = 0; i < RR_CHUNK; i++)
        if (i < nfull) w[i] = __ldg(wr + i * 32 + lane);
}

// CTA 0 of a token's router cluster, once every logit is in `choice`:
// route (moe.zig:106) and quantize the token's activation (smx) for the expert
// kernels. nw = warps in the CTA.
// The FFN RMSNorm of the layer folded into the router kernel's prologue
// (llama.zig:1198 before the MoE block): sx holds the raw residual row; every
// CTA of the cluster normalizes its own copy, sums of squares as a tree (per
// thread, then warps in order), out = x * (1 / sqrt(ss / dim + eps)) * w.
__device__ __noinline__ void prenorm_smem(float *sx, const float *w, int dim, float eps) {
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float ss = 0.0f;
    for (int i = tid; i < dim; i += blockDim.x) ss = fadd(ss, fmul(sx[i], sx[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = fadd(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int i = 0; i < nw; i++) t = fadd(t, red[i]);
        red[0] = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(t, (float)dim), eps)));
    }
    __syncthreads();
    const float scale = red[0];
    for (int i = tid; i < dim; i += blockDim.x) sx[i] = fmul(fmul(sx[i], scale), w[i]);
    __syncthreads();
}

// every expert of a pre-routed row is -1 (an unused fixed-capacity entry)
__device__ __forceinline__ bool row_unused(const int *ids, int n) {
    for (int k = 0; k < n; k++)
        if (__ldcg(ids + k) >= 0) return false;
    return true;
}

// x quantization of token t's row smx into the format(s) the expert types read, 256-value blocks
// b0, b0 + step, ... (and the 32-value groups likewise) by one warp each (warp index wi of nwq)
__device__ __forceinline__ void quant_x_rows(const DecodeArgs &A, int t, const float *smx, int b0, int step, int wi,
                                             int nwq, int lane) {
    const int dim = A.dim;
    if (A.need256)
        for (int b = b0 + step * wi; b < dim / 256; b += step * nwq)
            quant_lane8(smx + b * 256 + lane * 8, true, 32, A.x256.q + (size_t)t * dim + b * 256 + lane * 8,
                        A.x256.d + (size_t)t * (dim / 256) + b, A.x256.s + (size_t)t * (dim / 16) + b * 16 + lane / 2,
                        nullptr, lane);
    if (A.need32) {
        const int nb = dim / 32, ng = (nb + 7) / 8;
        for (int g = b0 + step * wi; g < ng; g += step * nwq) {
            const int b = g * 8 + lane / 4;
            const int off = b * 32 + (lane & 3) * 8;
            quant_lane8(smx + off, b < nb, 4, A.x32.q + (size_t)t * dim + off, A.x32.d + (size_t)t * (dim / 32) + b,
                        nullptr, A.x32.s + (size_t)t * (dim / 32) + b, lane);
        }
    }
}

// quant: also quantize x here (false when the cluster's CTAs quantized it already)
__device__ __forceinline__ void router_tail(const DecodeArgs &A, int t, const float *smx, float *scores, float *choice,
                                            int nw, bool quant = true) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int dim = A.dim, ne = A.n_expert;
    int *sid = reinterpret_cast<int *>(choice + ne);
    float *sg = choice + ne + 64;
    float *red = choice + ne + 128;
    // the route by one warp (logits in registers) where the layer allows, else by ROUTE_THREADS threads
    const bool wroute = !A.ids_in && (A.n_group <= 1 || A.topk_group >= A.n_group) && ne <= 32 * RW_MAX;
    if (threadIdx.x < ROUTE_THREADS && A.ids_in) {  // rows routed elsewhere: take their experts and gates
        for (int k = threadIdx.x; k < A.n_used; k += ROUTE_THREADS) {
            const size_t i = (size_t)t * A.n_used + k;
            A.ids[i] = A.ids_in[i];
            A.gates[i] = A.gates_in ? A.gates_in[i] : 1.0f;
            if (A.ids_out) A.ids_out[i] = A.ids_in[i];
        }
    } else if (wroute ? warp == 0 : threadIdx.x < ROUTE_THREADS) {
        if (wroute) {
            // one warp on logits in registers (the stack kernel's route; same order, same results);
            // the CTA's other warps quantize meanwhile
            if (ne <= 128)
                route_warp_regs<false, 4>(choice, A.bias, ne, A.n_used, A.gating, A.weights_norm, A.weights_scale,
                                          scores, choice, sid, sg, A.ids + (size_t)t * A.n_used,
                                          A.gates + (size_t)t * A.n_used, lane);
            else
                route_warp_regs<false, RW_MAX>(choice, A.bias, ne, A.n_used, A.gating, A.weights_norm,
                                               A.weights_scale, scores, choice, sid, sg,
                                               A.ids + (size_t)t * A.n_used, A.gates + (size_t)t * A.n_used, lane);
            __syncwarp();
            if (A.ids_out)
                for (int k = lane; k < A.n_used; k += 32) A.ids_out[(size_t)t * A.n_used + k] = sid[k];
        } else {
            route_block(choice, A.bias, ne, A.n_used, A.gating, A.weights_norm, A.weights_scale, scores, choice, sid,
                        sg, red, A.ids + (size_t)t * A.n_used, A.gates + (size_t)t * A.n_used, A.n_group, A.topk_group);
            if (A.ids_out)
                for (int k = threadIdx.x; k < A.n_used; k += ROUTE_THREADS)
                    A.ids_out[(size_t)t * A.n_used + k] = sid[k];
        }
        if (A.trace && threadIdx.x == 0) atomicMin(A.trace + 2 * (A.trace_slot + 6), gtimer());
    } else if (quant && !(A.ids_in && row_unused(A.ids_in + (size_t)t * A.n_used, A.n_used))) {
        // quantize x in the format(s) the expert types read (not for the unused
        // entries of a fixed-capacity exchange: expert -1, no expert reads them)
        const int nrw = wroute ? 1 : ROUTE_THREADS / 32;  // warps routing
        quant_x_rows(A, t, smx, 0, 1, warp - nrw, nw - nrw, lane);
        if (A.trace && lane == 0) atomicMax(A.trace + 2 * (A.trace_slot + 6) + 1, gtimer());
    }
    (void)dim;
}

__global__ void __launch_bounds__(RR_WARPS * 32) k_router_route(DecodeArgs A) {
    extern __shared__ float smx[];  // x[dim] | scores[ne] | choice[ne] | ids[64] | gates[64]
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int dim = A.dim, ne = A.n_expert;
    const unsigned rank = A.router ? cluster_rank() : 0;
    const int gw = (int)rank * RR_WARPS + warp;  // warp index within the cluster
    float *scores = smx + dim, *choice = scores + ne;
    trace_begin(A, 0);
    // 1. the first row's leading weights, before the wait
    float w[RR_CHUNK];
    if (A.router && gw < ne) load_row_chunk(w, A.router + (size_t)gw * dim, dim, lane);
    pdl_wait();
    pdl_trigger();
    // 2. this token's activation into shared memory
    const float *xt = A.x + (size_t)t * dim;
    trace_begin(A, 3);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) smx[i] = xt[i];
    __syncthreads();
    if (A.prenorm_w) prenorm_smem(smx, A.prenorm_w, dim, A.prenorm_eps);
    if (A.router) {
        for (int row = gw; row < ne; row += RR_WARPS_ALL) {
            const float *wr = A.router + (size_t)row * dim;
            if (row != gw) load_row_chunk(w, wr, dim, lane);
            const float r = router_dot(w, wr, smx, dim, lane);
            if (lane == 0) {
                st_cluster_f32(choice + row, 0, r);
                A.logits[(size_t)t * ne + row] = r;
            }
        }
        cluster_sync_all();  // every logit is in CTA 0's `choice`
        trace_end(A, 3);
        if (rank != 0) return;
    } else {
        for (int e = threadIdx.x; e < ne; e += blockDim.x) choice[e] = A.logits_in[(size_t)t * ne + e];
        __syncthreads();
    }
    router_tail(A, t, smx, scores, choice, RR_WARPS);
    __syncthreads();
    trace_end(A, 0);
}

// TMA variant: one cluster of RR2_CLUSTER CTAs per token; each CTA copies its
// slice of router rows into shared memory with bulk asynchronous copies issued
// BEFORE the wait, so the 1 MiB of router weights streams while the previous
// layer finishes; after the wait the dots read shared memory only.
constexpr int RR2_WARPS = 8;
constexpr uint32_t WAIT_POLLS = 1u << 22;  // bounded mbarrier wait (far beyond any legitimate latency)

__global__ void __launch_bounds__(RR2_WARPS * 32) k_router_tma(DecodeArgs A) {
    extern __shared__ __align__(16) float smw[];  // W rows [rpc][dim] | x[dim] | scores | choice | ids | gates | norm w
    __shared__ __align__(8) uint64_t bar, bar_x;
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int dim = A.dim, ne = A.n_expert;
    const unsigned rank = cluster_rank();
    const int ncl = (int)gridDim.x;
    const int rpc = (ne + ncl - 1) / ncl;  // rows per CTA
    const int row0 = (int)rank * rpc;
    const int nrows = row0 >= ne ? 0 : (ne - row0 < rpc ? ne - row0 : rpc);
    float *smx = smw + (size_t)rpc * dim;
    float *scores = smx + dim, *choice = scores + ne;
    float *snw = choice + ne + 136;  // the FFN norm weights, bulk-copied when 16-byte aligned
    const bool wbulk = A.prenorm_w && (size_t)(snw - smw) % 4 == 0;
    trace_begin(A, 0);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init(&bar_x, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0 && (nrows > 0 || wbulk)) {
        // the router rows and the norm weights (neither depends on the previous kernel)
        mbar_expect_tx(&bar, (uint32_t)(nrows * dim * 4) + (wbulk ? (uint32_t)dim * 4 : 0u));
        for (int r = 0; r < nrows; r++)
            bulk_g2s(smw + (size_t)r * dim, A.router + (size_t)(row0 + r) * dim, (uint32_t)(dim * 4), &bar);
        if (wbulk) bulk_g2s(snw, A.prenorm_w, (uint32_t)dim * 4, &bar);
    }
    pdl_wait();

    const float *xt = A.x + (size_t)t * dim;
    trace_begin(A, 3);
    if (threadIdx.x == 0) {  // the row the previous kernel wrote, as one bulk copy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_expect_tx(&bar_x, (uint32_t)dim * 4);
        bulk_g2s(smx, xt, (uint32_t)dim * 4, &bar_x);
    }
    if (!mbar_wait(&bar_x, 0, WAIT_POLLS) && threadIdx.x == 0 && A.err) atomicOr(A.err, 1);
    if (A.prenorm_w) {
        if (wbulk && !mbar_wait(&bar, 0, WAIT_POLLS) && threadIdx.x == 0 && A.err) atomicOr(A.err, 1);
        prenorm_smem(smx, wbulk ? snw : A.prenorm_w, dim, A.prenorm_eps);
    }
    const long long c0 = clock64();
    if (nrows > 0 && !mbar_wait(&bar, 0, WAIT_POLLS)) {
        if (threadIdx.x == 0 && A.err) atomicOr(A.err, 1);
    }
    const long long c1 = clock64();
    for (int r = warp; r < nrows; r += RR2_WARPS) {  // dotF32 (ggml.zig:198), lane j = accumulator lane j
        const float *wr = smw + (size_t)r * dim;
        const int nfull = dim / 32;
        float a = 0.0f;
        for (int i = 0; i < nfull; i++) a = fadd(a, fmul(wr[i * 32 + lane], smx[i * 32 + lane]));
        int i = nfull * 32;
        for (; i + 8 <= dim; i += 8)
            if (lane < 8) a = fadd(a, fmul(wr[i + lane], smx[i + lane]));
        const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
        const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
        const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
        const float v = fadd(fadd(fadd(a, a8), a16), a24);
        float res = __shfl_sync(0xffffffffu, v, 0);
#pragma unroll
        for (int jj = 1; jj < 8; jj++) res = fadd(res, __shfl_sync(0xffffffffu, v, jj));
        for (; i < dim; i++) res = fadd(res, fmul(wr[i], smx[i]));
        if (lane == 0) {
            st_cluster_f32(choice + row0 + r, 0, res);
            A.logits[(size_t)t * ne + row0 + r] = res;
        }
    }
    const long long c2 = clock64();
    cluster_sync_all();  // every logit is in CTA 0's `choice`
    trace_end(A, 3);
    if (A.trace && threadIdx.x == 0) {  // cycles: TMA wait, dots (max over the cluster)
        atomicMax(A.trace + 2 * (A.trace_slot + 7), (unsigned long long)(c1 - c0));
        atomicMax(A.trace + 2 * (A.trace_slot + 7) + 1, (unsigned long long)(c2 - c1));
    }
    if (rank != 0) {
        // the x quantization, split over the cluster's other CTAs (each holds the normalized row):
        // block b by CTA 1 + b % (ncl - 1), one warp a block, while CTA 0 routes
        if (ncl > 1 && !(A.ids_in && row_unused(A.ids_in + (size_t)t * A.n_used, A.n_used))) {
            quant_x_rows(A, t, smx, (int)rank - 1, ncl - 1, warp, RR2_WARPS, lane);
            if (A.trace && lane == 0) atomicMax(A.trace + 2 * (A.trace_slot + 6) + 1, gtimer());
        }
        __syncthreads();
        pdl_trigger();
        return;
    }
    const long long c3 = clock64();
    router_tail(A, t, smx, scores, choice, RR2_WARPS, ncl == 1);
    if (A.trace && threadIdx.x == 0) atomicMax(A.trace + 2 * (A.trace_slot + 8) + 1, (unsigned long long)(clock64() - c3));
    __syncthreads();
    pdl_trigger();  // late: the expert kernel's CTAs would only wait on this SM's issue slots
    trace_end(A, 0);
}

// ---- slot description -------------------------------------------------------------

struct SlotInfo {
    int expert_local;  // -1 when not held here
    int token;
    int ffn;
    bool shared;
};

__device__ __forceinline__ SlotInfo slot_info(const DecodeArgs &A, int slot) {
    SlotInfo si;
    const int nr = A.T * A.n_used;
    if (slot < nr) {
        si.token = slot / A.n_used;
        const int le = __ldcg(A.ids + slot) - A.expert0;
        si.expert_local = (le >= 0 && le < A.n_local) ? le : -1;
        si.ffn = si.expert_local >= 0 ? A.ffn : 0;
        si.shared = false;
    } else {
        si.token = slot - nr;
        si.expert_local = 0;
        si.ffn = A.shexp_ffn;
        si.shared = true;
    }
    return si;
}

// stage `n` bytes (multiple of 16) from global (through L2) into shared memory
__device__ __forceinline__ void stage16(void *dst, const void *src, int n) {
    const int4 *s = reinterpret_cast<const int4 *>(src);
    int4 *d = reinterpret_cast<int4 *>(dst);
    for (int i = threadIdx.x; i < n / 16; i += blockDim.x) d[i] = __ldcg(s + i);
}

// ---- gate/up + SwiGLU ---------------------------------------------------------------

constexpr int GU_WARPS = 4;
// rows per warp (streams = NR gate rows + NR up rows): 3 for rows of up to 8
// super-blocks (one wave of CTAs at the Qwen shape), 1 for wider rows
template <int NB> constexpr int gu_nr() { return NB <= 8 ? 3 : 1; }

template <int GU_NR> struct GateUpStreams {
    WDev wg, wu;
    uint64_t gb_g, gb_u;  // first block of the warp's first row
    int nb;
    XV xv;
    __device__ __forceinline__ WDev w(int s) const { return s < GU_NR ? wg : wu; }
    __device__ __forceinline__ uint64_t gb(int s) const {
        return s < GU_NR ? gb_g + (uint64_t)s * nb : gb_u + (uint64_t)(s - GU_NR) * nb;
    }
    __device__ __forceinline__ XV x(int) const { return xv; }
};

template <int TY, int NB>
__global__ void __launch_bounds__(GU_WARPS * 32) k_gateup_dec(DecodeArgs A) {
    constexpr int GU_NR = gu_nr<NB>();
    using E = CEng<TY, 2 * GU_NR, NB>;
    static_assert(E::OK, "unit mapping");
    extern __shared__ __align__(16) uint8_t sm[];
    trace_begin(A, 1);
    pdl_wait();
    pdl_trigger();
    trace_begin(A, 4);
    const long long gc0 = clock64();
    const int slot = blockIdx.y;
    const SlotInfo si = slot_info(A, slot);
    const int rows_cta = GU_WARPS * GU_NR;
    const int nctas = (si.ffn + rows_cta - 1) / rows_cta;
    if ((int)blockIdx.x >= nctas) return;
    constexpr int dim = NB * 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // stage the token's quantized activation (gate and up share the K format)
    int8_t *xq = reinterpret_cast<int8_t *>(sm);
    float *xd = reinterpret_cast<float *>(sm + dim);
    int32_t *xs = reinterpret_cast<int32_t *>(sm + dim + NB * 4);
    // (written by the router kernel: three bulk copies, landing while the weights load)
    constexpr bool XBULK = NB % 4 == 0;  // 16-byte sizes and offsets
    __shared__ __align__(8) uint64_t bx;
    if (XBULK) {
        if (threadIdx.x == 0) {
            mbar_init(&bx, 1);
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_expect_tx(&bx, (uint32_t)(dim + NB * 4 + NB * 64));
            bulk_g2s(xq, A.x256.q + (size_t)si.token * dim, (uint32_t)dim, &bx);
            bulk_g2s(xd, A.x256.d + (size_t)si.token * NB, (uint32_t)NB * 4, &bx);
            bulk_g2s(xs, A.x256.s + (size_t)si.token * NB * 16, (uint32_t)NB * 64, &bx);
        }
    } else {
        stage16(xq, A.x256.q + (size_t)si.token * dim, dim);
        for (int i = threadIdx.x; i < NB; i += blockDim.x) xd[i] = __ldcg(A.x256.d + (size_t)si.token * NB + i);
        for (int i = threadIdx.x; i < NB * 16; i += blockDim.x) xs[i] = __ldcg(A.x256.s + (size_t)si.token * NB * 16 + i);
    }
    const WDev wg = si.shared ? A.sg : A.g, wu = si.shared ? A.su : A.u;
    const uint64_t plane = si.shared ? 0 : (uint64_t)si.expert_local * si.ffn * NB;
    const int r0 = blockIdx.x * rows_cta + warp * GU_NR;
    const int rmax = si.ffn - GU_NR;
    const int rl = r0 <= rmax ? r0 : rmax;  // clamp the last (partial) group; its extra rows are not stored
    GateUpStreams<GU_NR> st{wg, wu, plane + (uint64_t)rl * NB, plane + (uint64_t)rl * NB, NB, XV{xq, xd, xs}};
    typename E::Frags fr;
    const long long gc1 = clock64();
    E::load(st, fr, lane);  // weight loads are in flight while the activation lands in shared memory
    if (threadIdx.x == 0) {
        // warm L2 with this CTA's share of the slot's down plane for k_down_dec
        // (and, from the first CTA, the next layer's router weights)
        const WDev wd = si.shared ? A.sdn : A.dn;
        const int f = si.shared ? A.shexp_ffn : A.ffn;
        const uint64_t pb = (uint64_t)A.dim * (f / block_elems(wd.type));  // blocks per down plane
        const uint64_t e0 = si.shared ? 0 : (uint64_t)si.expert_local * pb;
        const uint64_t qb = pb * layout_qbytes(wd.type), chunk = (qb / nctas + 15) & ~uint64_t(15);
        const uint64_t off = chunk * blockIdx.x;
        if (off < qb) prefetch_l2(wd.q + e0 * layout_qbytes(wd.type) + off, off + chunk <= qb ? chunk : qb - off);
        if (blockIdx.x == 0) {
            if (wd.sc) prefetch_l2(wd.sc + e0 * 16, pb * 16);
            if (wd.d) prefetch_l2(wd.d + e0, pb * 2);
            if (A.next_router && blockIdx.y == 0) prefetch_l2(A.next_router, A.next_router_bytes);
        }
    }
    __syncthreads();
    if (XBULK && !mbar_wait(&bx, 0, WAIT_POLLS) && threadIdx.x == 0 && A.err) atomicOr(A.err, 1);
    float acc[2 * GU_NR];
    E::finish(st, fr, acc, lane);
    float *act = A.act + (size_t)slot * A.act_stride;
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < GU_NR; i++) {
            const int r = rl + i;
            if (r >= r0 && r < si.ffn) {
                const float g = acc[i], u = acc[GU_NR + i];
                act[r] = fmul(fdiv(g, fadd(1.0f, exp_f(-g))), u);  // silu(g) * u (tensor.zig:30,53)
            }
        }
    }
    if (A.trace && lane == 0) {  // cycles: ids + activation staging, weights in + dots
        atomicMax(A.trace + 2 * (A.trace_slot + 9), (unsigned long long)(gc1 - gc0));
        atomicMax(A.trace + 2 * (A.trace_slot + 9) + 1, (unsigned long long)(clock64() - gc1));
    }
    __syncthreads();
    trace_end(A, 1);
}

// ---- down + combine ------------------------------------------------------------------

constexpr int DN_WARPS = 4;    // grouped down kernel
constexpr int DND_WARPS = 16;  // decode down kernel: one 512-thread CTA per SM, so each CTA
                               // quantizes the token's activations once for 16 rows

struct DownStreams {
    WDev wd;
    const uint64_t *g;   // per stream: first block of this output row (shared memory)
    const int *sl;       // per stream: staged activation index (shared memory)
    const int8_t *aq;    // staged activations: index j at aq + j*stride
    const float *ad;
    const int32_t *as;
    int stride;
    int nvalid;          // streams beyond this repeat stream 0 (their result is unused)
    __device__ __forceinline__ WDev w(int) const { return wd; }
    __device__ __forceinline__ uint64_t gb(int s) const { return g[s < nvalid ? s : 0]; }
    __device__ __forceinline__ XV x(int s) const {
        const int j = sl[s < nvalid ? s : 0];
        return XV{aq + (size_t)j * stride, ad + (size_t)j * (stride / 32), as + (size_t)j * (stride / 16)};
    }
    // run-time engine interface
    __device__ __forceinline__ void at(int s, WDev &wo, uint64_t &gg, XV &xv) const {
        wo = wd;
        gg = gb(s);
        xv = x(s);
    }
};

// SC streams (experts) per chunk of NB blocks; NBSH = shared expert blocks (0: none)
template <int TY, int SC, int NB, int NBSH>
__global__ void __launch_bounds__(DND_WARPS * 32) k_down_dec(DecodeArgs A) {
    using E = CEng<TY, SC, NB>;
    using ES = CEng<TY, 1, (NBSH > 0 ? NBSH : QT<TY>::LPB == 8 ? 4 : 32 / QT<TY>::LPB)>;
    static_assert(E::OK, "unit mapping");
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_slot[64];  // local routed slots of this token, selection order
    __shared__ float s_gate[64];
    __shared__ int s_nloc;
    __shared__ int s_shidx;
    __shared__ uint64_t s_gb[DND_WARPS][SC];
    const int t = blockIdx.y;
    trace_begin(A, 2);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.x * DND_WARPS + warp;
    const int rr = r < A.dim ? r : A.dim - 1;
    const int nk = A.n_used;
    // Routing is final before this kernel may start: k_gateup_dec triggers its
    // dependents only after its own wait on the router, so ids/gates are read now.
    if (threadIdx.x == 0) {
        int n = 0;
        for (int k = 0; k < nk; k++) {
            const int le = __ldcg(A.ids + (size_t)t * nk + k) - A.expert0;
            if (le >= 0 && le < A.n_local) {
                s_slot[n] = k;
                s_gate[n] = __ldcg(A.gates + (size_t)t * nk + k);
                n++;
            }
        }
        s_nloc = n;
        s_shidx = nk;
    }
    __syncthreads();
    const int nloc = s_nloc;
    auto set_gb = [&](int c0, int n) {
        __syncwarp();
        if (lane < n) {
            const int le = __ldcg(A.ids + (size_t)t * nk + s_slot[c0 + lane]) - A.expert0;
            s_gb[warp][lane] = ((uint64_t)le * A.dim + rr) * NB;
        }
        __syncwarp();
    };
    int8_t *aq = reinterpret_cast<int8_t *>(sm);
    const int stride = A.act_stride;
    const int nk1 = nk + (NBSH > 0 ? 1 : 0);  // staged: the token's routed slots, then its shared one
    float *ad = reinterpret_cast<float *>(sm + (size_t)nk1 * stride);
    int32_t *as = reinterpret_cast<int32_t *>(sm + (size_t)nk1 * stride + (size_t)nk1 * (stride / 32) * 4);
    typename E::Frags fr;
    const int n0 = nloc < SC ? nloc : SC;
    DownStreams st{A.dn, s_gb[warp], s_slot, aq, ad, as, stride, n0};
    if (n0 > 0) {  // the first chunk's weights, before the wait
        set_gb(0, n0);
        if (n0 == SC) E::load(st, fr, lane);
        else wd_load<TY, SC, E::MAXU>(st, NB, n0, fr, lane);
    }
    pdl_wait();
    pdl_trigger();
    trace_begin(A, 5);
    const long long dc0 = clock64();
    // quantize the token's expert activations into shared memory, in the down
    // type's format (quantizeX256 / quantizeX): routed slot k at k*stride, the
    // shared expert's at nk*stride
    {
        // every (slot, block) pair of this token; each warp loads QB blocks' values
        // before quantizing any, so the L2 reads overlap
        constexpr int QB = 4;
        constexpr int BEQ = act256(TY) ? 256 : 32;  // quantization block
        constexpr int LPQ = BEQ / 8;                // lanes per quantization block
        constexpr int BPW = 32 / LPQ;               // blocks per warp step
        const int nbr = A.ffn / BEQ, nbs = NBSH > 0 ? A.shexp_ffn / BEQ : 0;
        const int nunits = nk * nbr + nbs;  // warp units of BPW blocks
        const int nsteps = (nunits + BPW - 1) / BPW;
        for (int s0 = warp; s0 < nsteps; s0 += DND_WARPS * QB) {
            float v[QB][8];
            int kk[QB], bb[QB];
            bool live[QB];
#pragma unroll
            for (int i = 0; i < QB; i++) {
                const int st_ = s0 + i * DND_WARPS;
                const int u = st_ * BPW + lane / LPQ;
                live[i] = st_ < nsteps && u < nunits;
                kk[i] = u < nk * nbr ? u / nbr : nk;
                bb[i] = u < nk * nbr ? u % nbr : u - nk * nbr;
                const size_t slot = kk[i] < nk ? (size_t)t * nk + kk[i] : (size_t)A.T * nk + t;
                const float *src = A.act + slot * stride + bb[i] * BEQ + (lane % LPQ) * 8;
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b4 = a;
                if (live[i]) {
                    a = reinterpret_cast<const float4 *>(src)[0];
                    b4 = reinterpret_cast<const float4 *>(src)[1];
                }
                v[i][0] = a.x, v[i][1] = a.y, v[i][2] = a.z, v[i][3] = a.w;
                v[i][4] = b4.x, v[i][5] = b4.y, v[i][6] = b4.z, v[i][7] = b4.w;
            }
#pragma unroll
            for (int i = 0; i < QB; i++) {
                if (s0 + i * DND_WARPS >= nsteps) break;  // warp-uniform
                const int k = kk[i], b = bb[i];
                int8_t *q = aq + (size_t)k * stride + b * BEQ + (lane % LPQ) * 8;
                float *dd = ad + (size_t)k * (stride / 32) + b;
                int32_t *ss = as + (size_t)k * (stride / 16);
                if (BEQ == 256) quant_vals8(v[i], live[i], 32, q, dd, ss + b * 16 + lane / 2, nullptr, lane);
                else quant_vals8(v[i], live[i], 4, q, dd, nullptr, ss + b, lane);
            }
        }
    }
    __syncthreads();
    const long long dc1 = clock64();
    float acc = 0.0f;
    for (int c0 = 0; c0 < nloc; c0 += SC) {
        const int n = nloc - c0 < SC ? nloc - c0 : SC;
        st.sl = s_slot + c0;
        st.nvalid = n;
        if (c0 > 0) {
            set_gb(c0, n);
            if (n == SC) E::load(st, fr, lane);
            else wd_load<TY, SC, E::MAXU>(st, NB, n, fr, lane);
        }
        float y[SC];
        if (n == SC) E::finish(st, fr, y, lane);
        else wd_finish<TY, SC, E::MAXU>(st, NB, n, fr, y, lane);
#pragma unroll
        for (int k = 0; k < SC; k++)
            if (k < n) acc = fadd(acc, fmul(s_gate[c0 + k], y[k]));  // moeRun: acc += gate * out (llama.zig:1397)
    }
    if constexpr (NBSH > 0) {  // shared expert added plainly after the routed sum (deepseek.zig:1498-1508)
        __syncwarp();
        if (lane == 0) s_gb[warp][0] = (uint64_t)rr * NBSH;
        __syncwarp();
        DownStreams sh{A.sdn, s_gb[warp], &s_shidx, aq, ad, as, stride, 1};
        typename ES::Frags fs;
        ES::load(sh, fs, lane);
        float y[1];
        ES::finish(sh, fs, y, lane);
        acc = fadd(acc, y[0]);
    }
    if (lane == 0 && r < A.dim) {
        const size_t o = (size_t)t * A.dim + r;
        A.out[o] = A.residual ? fadd(__ldcg(A.residual + o), acc) : acc;
    }
    if (A.trace && lane == 0) {  // cycles: activation quantization, dots + combine
        atomicMax(A.trace + 2 * (A.trace_slot + 10), (unsigned long long)(dc1 - dc0));
        atomicMax(A.trace + 2 * (A.trace_slot + 10) + 1, (unsigned long long)(clock64() - dc1));
    }
    __syncthreads();
    trace_end(A, 2);
}

// ---- dispatch ---------------------------------------------------------------------
// The instantiated shapes: gate/up blocks per row (dim/256) and, for the down
// projection, (type, experts per chunk, blocks per row, shared-expert blocks).
// Other shapes run on the general slot kernels (same arithmetic).

using GUFn = void (*)(DecodeArgs);
static GUFn gateup_fn(int ty, int nb) {
    if (ty == T_Q4_K) switch (nb) {
            case 4: return k_gateup_dec<T_Q4_K, 4>;
            case 8: return k_gateup_dec<T_Q4_KW, 8>;
            case 16: return k_gateup_dec<T_Q4_KW, 16>;
            case 28: return k_gateup_dec<T_Q4_K, 28>;
        }
    if (ty == T_Q6_K && nb == 8) return k_gateup_dec<T_Q6_K, 8>;
    return nullptr;
}

static GUFn down_fn(int ty, int nb, int nbsh) {
    if (ty == T_Q6_K && nbsh == 0) switch (nb) {  // 8 experts per chunk, block-major units
            case 1: return k_down_dec<T_Q6_K, 8, 1, 0>;
            case 2: return k_down_dec<T_Q6_K, 8, 2, 0>;
            case 3: return k_down_dec<T_Q6_K, 8, 3, 0>;
            case 4: return k_down_dec<T_Q6_K, 8, 4, 0>;
        }
    if (ty == T_Q4_K) {  // 4 experts per chunk, stream-major units
        if (nb == 4 && nbsh == 0) return k_down_dec<T_Q4_K, 4, 4, 0>;
        if (nb == 4 && nbsh == 4) return k_down_dec<T_Q4_K, 4, 4, 4>;
        if (nb == 8 && nbsh == 0) return k_down_dec<T_Q4_KW, 4, 8, 0>;
        if (nb == 8 && nbsh == 8) return k_down_dec<T_Q4_KW, 4, 8, 8>;
    }
    return nullptr;
}

static size_t down_smem(const DecodeArgs &A) {
    const size_t nk1 = A.n_used + (A.has_shared ? 1 : 0);
    return nk1 * A.act_stride + nk1 * (A.act_stride / 32) * 4 + nk1 * (A.act_stride / 16) * 4;
}

static int shared_nb(const DecodeArgs &A) { return A.has_shared ? A.shexp_ffn / block_elems(A.sdn.type) : 0; }

bool decode_supported(const DecodeArgs &A) {
    if (A.g.type != A.u.type || A.dim % 256 || A.n_used > 64) return false;
    if (!gateup_fn(A.g.type, A.dim / 256)) return false;
    const int dty = A.dn.type;
    if (block_elems(dty) == 0 || A.ffn % block_elems(dty)) return false;
    if (A.has_shared) {
        if (A.sg.type != A.g.type || A.su.type != A.g.type || A.sdn.type != dty) return false;
        if (A.shexp_ffn % block_elems(dty) || A.shexp_ffn > A.act_stride) return false;
    }
    if (!down_fn(dty, A.ffn / block_elems(dty), shared_nb(A))) return false;
    const size_t max_ffn = A.has_shared && A.shexp_ffn > A.ffn ? A.shexp_ffn : A.ffn;
    return down_smem(A) <= 48 * 1024 && (size_t)(A.dim + 2 * A.n_expert + 136) * 4 <= 48 * 1024 &&
           max_ffn * 4 <= 48 * 1024;
}

// Router cluster shape for the TMA variant: 16 CTAs when the device can place
// a 16-CTA cluster (non-portable size), else 8; 0 when the rows do not fit.
// dotF32 (ggml.zig:198) of a router row and x, both in shared memory, dim a
// multiple of 32 (the stack kernel's router_dot_smem, same order)
// ---- batch router (T > 16 tokens): router GEMV tiled over experts x tokens,
// then one block per token for route + activation quantization. The logits
// are dotF32 (ggml.zig:198) in the same order as the decode router, and the
// route is router_tail's, so every path routes identically.
constexpr int RB_WARPS = 16, RB_TOK = 4;

static int rb_experts(int dim) {  // router rows a CTA keeps in shared memory (<= RB_WARPS, ~190 KB)
    int et = (int)((190 * 1024 - RB_TOK * (size_t)dim * 4) / ((size_t)dim * 4));
    return et < 1 ? 1 : et > RB_WARPS ? RB_WARPS : et;
}

// dotF32 order (as router_dot_smem_) for RB_TOK tokens at once: the warp's
// lanes read each weight once and carry one accumulator per token
__device__ __forceinline__ void router_dot_smem_tok(const float *wr, const float *x, int dim, int lane, int nt,
                                                    float (&out)[RB_TOK]) {
    float a[RB_TOK];
#pragma unroll
    for (int t = 0; t < RB_TOK; t++) a[t] = 0.0f;
#pragma unroll 4
    for (int i = lane; i < dim; i += 32) {
        const float w = wr[i];
#pragma unroll
        for (int t = 0; t < RB_TOK; t++) a[t] = fadd(a[t], fmul(w, x[(size_t)t * dim + i]));
    }
#pragma unroll
    for (int t = 0; t < RB_TOK; t++) {
        const float a8 = __shfl_down_sync(0xffffffffu, a[t], 8);
        const float a16 = __shfl_down_sync(0xffffffffu, a[t], 16);
        const float a24 = __shfl_down_sync(0xffffffffu, a[t], 24);
        const float v = fadd(fadd(fadd(a[t], a8), a16), a24);
        float r = __shfl_sync(0xffffffffu, v, 0);
#pragma unroll
        for (int jj = 1; jj < 8; jj++) r = fadd(r, __shfl_sync(0xffffffffu, v, jj));
        out[t] = r;
    }
    (void)nt;
}

__global__ void __launch_bounds__(RB_WARPS * 32) k_router_batch(DecodeArgs A, int et) {
    extern __shared__ __align__(16) float rbs[];  // rows [et][dim] | x [2][dim]
    pdl_wait();
    pdl_trigger();
    const int dim = A.dim, ne = A.n_expert;
    const int e0 = blockIdx.x * et, t0 = blockIdx.y * RB_TOK;
    const int ne_here = ne - e0 < et ? ne - e0 : et;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *rows = rbs, *xb = rbs + (size_t)et * dim;  // x: [RB_TOK][dim], zero past the last token
    const int nt = A.T - t0 < RB_TOK ? A.T - t0 : RB_TOK;
    for (int i = threadIdx.x; i < ne_here * dim / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(rows)[i] = __ldg(reinterpret_cast<const float4 *>(A.router + (size_t)e0 * dim) + i);
    for (int i = threadIdx.x; i < RB_TOK * dim / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xb)[i] = i < nt * dim / 4
            ? __ldg(reinterpret_cast<const float4 *>(A.x + (size_t)t0 * dim) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    if (warp < ne_here) {
        float r[RB_TOK];
        router_dot_smem_tok(rows + (size_t)warp * dim, xb, dim, lane, nt, r);
        if (lane == 0)
#pragma unroll
            for (int t = 0; t < RB_TOK; t++)
                if (t < nt) A.logits[(size_t)(t0 + t) * ne + e0 + warp] = r[t];
    }
}

__global__ void __launch_bounds__(256) k_route_batch(DecodeArgs A) {
    extern __shared__ float smx[];  // x[dim] | scores[ne] | choice[ne] | ids[64] | gates[64] | red
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, dim = A.dim, ne = A.n_expert;
    float *scores = smx + dim, *choice = scores + ne;
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(smx)[i] = __ldg(reinterpret_cast<const float4 *>(A.x + (size_t)t * dim) + i);
    if (!A.ids_in)
        for (int e = threadIdx.x; e < ne; e += blockDim.x) choice[e] = __ldcg(A.logits + (size_t)t * ne + e);
    __syncthreads();
    router_tail(A, t, smx, scores, choice, 8);
}

static int tma_cluster(const DecodeArgs &A, size_t &smem) {
    static int c16 = -1, ok = 0;
    if (c16 < 0) {
        c16 = 0;
        ok = cudaFuncSetAttribute(k_router_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) == cudaSuccess;
        if (ok && cudaFuncSetAttribute(k_router_tma, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(16);
            cfg.blockDim = dim3(RR2_WARPS * 32);
            cfg.dynamicSmemBytes = 96 * 1024;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 16;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, k_router_tma, &cfg) == cudaSuccess && n > 0) c16 = 1;
        }
        cudaGetLastError();
    }
    if (!ok) return 0;
    for (int c : {c16 ? 16 : 8, 8}) {
        const int rpc = (A.n_expert + c - 1) / c;
        smem = ((size_t)rpc * A.dim + A.dim + 2 * A.n_expert + 136 + A.dim) * 4;
        if (A.dim % 4 == 0 && smem <= 200 * 1024) return c;
    }
    return 0;
}

static cudaError_t launch_router(const DecodeArgs &A, cudaStream_t st) {
    if (A.ids_in) {  // pre-routed rows: copy the routing, quantize the rows
        const size_t rs = (size_t)(A.dim + 2 * A.n_expert + 136) * 4;
        cudaError_t e = cudaSuccess;
        if (rs > 48 * 1024 &&
            (e = cudaFuncSetAttribute(k_route_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rs)) != cudaSuccess)
            return e;
        return launch_pdl(k_route_batch, dim3(A.T), dim3(256), rs, st, A);
    }
    // batch router: many tokens, or a router too large for one cluster's shared memory (DeepSeek-V3:
    // 256 x 7168 f32 = 7.3 MB), tiled over experts across the GPU
    const bool big_router = (size_t)A.n_expert * A.dim * 4 > (4u << 20) && !A.prenorm_w;
    if (A.router && (A.T > 16 || big_router) && A.dim % 32 == 0 && A.dim <= 8192 && !A.trace_reg) {
        const int et = rb_experts(A.dim);
        const size_t smem = ((size_t)et + RB_TOK) * A.dim * 4;
        cudaError_t e = cudaFuncSetAttribute(k_router_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if ((e = launch_pdl(k_router_batch, dim3(cdivu(A.n_expert, et), cdivu(A.T, RB_TOK)), dim3(RB_WARPS * 32), smem,
                            st, A, et)) != cudaSuccess)
            return e;
        const size_t rs = (size_t)(A.dim + 2 * A.n_expert + 136) * 4;
        if (rs > 48 * 1024 &&
            (e = cudaFuncSetAttribute(k_route_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rs)) != cudaSuccess)
            return e;
        return launch_pdl(k_route_batch, dim3(A.T), dim3(256), rs, st, A);
    }
    size_t smem = 0;
    const int tc = (A.router && !A.trace_reg) ? tma_cluster(A, smem) : 0;
    if (!tc) smem = (size_t)(A.dim + 2 * A.n_expert + 136) * 4;
    const int cl = tc ? tc : (A.router ? RR_CLUSTER : 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, A.T);
    cfg.blockDim = dim3((tc ? RR2_WARPS : RR_WARPS) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cl;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    count_launch();
    return cudaLaunchKernelEx(&cfg, tc ? k_router_tma : k_router_route, A);
}

cudaError_t launch_decode(const DecodeArgs &A, cudaStream_t st) {
    cudaError_t e;
    // 1. router + route + activation quantization
    e = launch_router(A, st);
    if (e != cudaSuccess) return e;
    // 2. gate/up
    {
        const int n_slots = A.T * A.n_used + (A.has_shared ? A.T : 0);
        const int max_ffn = A.has_shared && A.shexp_ffn > A.ffn ? A.shexp_ffn : A.ffn;
        const dim3 grid(cdivu(max_ffn, GU_WARPS * (A.dim / 256 <= 8 ? 3 : 1)), n_slots);
        const size_t smem_x = (size_t)A.dim + A.dim / 256 * 4 + A.dim / 16 * 4;
        const size_t smem_q = (size_t)max_ffn * 4;
        e = launch_pdl(gateup_fn(A.g.type, A.dim / 256), grid, dim3(GU_WARPS * 32), smem_x > smem_q ? smem_x : smem_q,
                       st, A);
        if (e != cudaSuccess) return e;
    }
    // 3. down + combine
    {
        const dim3 grid(cdivu(A.dim, DND_WARPS), A.T);
        e = launch_pdl(down_fn(A.dn.type, A.ffn / block_elems(A.dn.type), shared_nb(A)), grid, dim3(DND_WARPS * 32),
                       down_smem(A), st, A);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}


// ==== expert-major batch path ===========================================================
// For T tokens the routed (token, expert) slots are grouped by expert, and
// every kernel reads an expert's rows once for all the tokens that chose it
// (the reference's moeBatchUnion, llama.zig:1828-1925, and matmulK256's
// "decode once, dot n lanes", ggml.zig:1044). Per slot the arithmetic is the
// decode path's, so results are bit-identical to it and to the CPU.

// Group the local routed slots by expert (stable: slot order within a group).
__global__ void __launch_bounds__(512) k_group(DecodeArgs A) {
    pdl_wait();
    pdl_trigger();
    __shared__ int cnt[1024];
    const int ns = A.T * A.n_used;
    for (int e = threadIdx.x; e < A.n_local; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int s = threadIdx.x; s < ns; s += blockDim.x) {
        const int le = A.ids[s] - A.expert0;
        if (le >= 0 && le < A.n_local) atomicAdd(&cnt[le], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive prefix over n_local (<= 1024) counts
        int o = 0, c = 0;
        for (int e = 0; e < A.n_local; e++) {
            A.grp_off[e] = o;
            A.grp_cnt[e] = cnt[e];
            o += cnt[e];
            if (A.tc_pre && A.tc_chunk) {
                A.tc_pre[e] = c;
                c += (cnt[e] + A.tc_chunk - 1) / A.tc_chunk;
            }
        }
        if (A.tc_pre && A.tc_chunk) {
            if (A.has_shared) {
                A.tc_pre[A.n_local] = c;
                c += (A.T + A.tc_chunk - 1) / A.tc_chunk;
            }
            A.tc_pre[A.n_local + (A.has_shared ? 1 : 0)] = c;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < A.n_local; e += blockDim.x) cnt[e] = 0;  // now: fill positions
    __syncthreads();
    // the order of slots inside a group does not matter: every slot's output is
    // computed on its own and the combine adds slots in selection order
    for (int s = threadIdx.x; s < ns; s += blockDim.x) {
        const int le = A.ids[s] - A.expert0;
        if (le < 0 || le >= A.n_local) continue;
        A.grp_list[A.grp_off[le] + atomicAdd(&cnt[le], 1)] = s;
    }
}

// gate/up for expert blockIdx.y (n_local = the shared expert): the CTA's rows
// are loaded once, then dotted with each token of the expert.
template <int TY, int NB>
__global__ void __launch_bounds__(GU_WARPS * 32) k_gateup_grp(DecodeArgs A) {
    constexpr int GU_NR = gu_nr<NB>();
    using E = CEng<TY, 2 * GU_NR, NB>;
    pdl_wait();
    pdl_trigger();
    const int e = blockIdx.y;
    const bool shared = e == A.n_local;
    const int n = shared ? A.T : A.grp_cnt[e];
    const int ffn = shared ? A.shexp_ffn : A.ffn;
    const int rows_cta = GU_WARPS * GU_NR;
    if (n == 0 || (int)blockIdx.x * rows_cta >= ffn) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int dim = NB * 256;
    const WDev wg = shared ? A.sg : A.g, wu = shared ? A.su : A.u;
    const uint64_t plane = shared ? 0 : (uint64_t)e * ffn * NB;
    const int r0 = blockIdx.x * rows_cta + warp * GU_NR;
    const int rl = r0 <= ffn - GU_NR ? r0 : ffn - GU_NR;
    GateUpStreams<GU_NR> st{wg, wu, plane + (uint64_t)rl * NB, plane + (uint64_t)rl * NB, NB, XV{nullptr, nullptr, nullptr}};
    typename E::Frags fr;
    E::load(st, fr, lane);
    const int *list = shared ? nullptr : A.grp_list + A.grp_off[e];
    for (int i = 0; i < n; i++) {
        const int slot = shared ? A.T * A.n_used + i : list[i];
        const int t = shared ? i : slot / A.n_used;
        st.xv = XV{A.x256.q + (size_t)t * dim, A.x256.d + (size_t)t * NB, A.x256.s + (size_t)t * NB * 16};
        float acc[2 * GU_NR];
        E::finish(st, fr, acc, lane);
        if (lane == 0) {
            float *act = A.act + (size_t)slot * A.act_stride;
#pragma unroll
            for (int k = 0; k < GU_NR; k++) {
                const int r = rl + k;
                if (r >= r0 && r < ffn) act[r] = fmul(fdiv(acc[k], fadd(1.0f, exp_f(-acc[k]))), acc[GU_NR + k]);
            }
        }
    }
}

// quantize every live slot's activation in the down type's format
__global__ void __launch_bounds__(128) k_quant_grp(DecodeArgs A) {
    pdl_wait();
    pdl_trigger();
    const int slot = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nr = A.T * A.n_used;
    int f;
    int dty;
    if (slot < nr) {
        const int le = A.ids[slot] - A.expert0;
        if (le < 0 || le >= A.n_local) return;
        f = A.ffn;
        dty = A.dn.type;
    } else {
        f = A.shexp_ffn;
        dty = A.sdn.type;
    }
    const float *x = A.act + (size_t)slot * A.act_stride;
    int8_t *q = A.aq + (size_t)slot * A.act_stride;
    float *d = A.ad + (size_t)slot * (A.act_stride / 32);
    int32_t *s = A.as + (size_t)slot * (A.act_stride / 16);
    if (act256(dty)) {
        for (int b = warp; b < f / 256; b += 4)
            quant_lane8(x + b * 256 + lane * 8, true, 32, q + b * 256 + lane * 8, d + b, s + b * 16 + lane / 2, nullptr,
                        lane);
    } else {
        const int nb = f / 32, ng = (nb + 7) / 8;
        for (int g = warp; g < ng; g += 4) {
            const int b = g * 8 + lane / 4;
            const int off = b * 32 + (lane & 3) * 8;
            quant_lane8(x + off, b < nb, 4, q + off, d + b, nullptr, s + b, lane);
        }
    }
}

// down rows of expert blockIdx.y for each of its tokens: y[slot][row]
template <int RS> struct RowStreams {  // RS consecutive rows of one expert plane
    WDev wd;
    uint64_t gb0;
    int nb;
    XV xv;
    __device__ __forceinline__ WDev w(int) const { return wd; }
    __device__ __forceinline__ uint64_t gb(int s) const { return gb0 + (uint64_t)s * nb; }
    __device__ __forceinline__ XV x(int) const { return xv; }
};

template <int TY, int RS, int NB>
__global__ void __launch_bounds__(DN_WARPS * 32) k_down_grp(DecodeArgs A) {
    using E = CEng<TY, RS, NB>;
    pdl_wait();
    pdl_trigger();
    const int e = blockIdx.y;
    const bool shared = e == A.n_local;
    const int n = shared ? A.T : A.grp_cnt[e];
    if (n == 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = (blockIdx.x * DN_WARPS + warp) * RS;
    if (r0 >= A.dim) return;
    const int rl = r0 <= A.dim - RS ? r0 : A.dim - RS;
    const WDev wd = shared ? A.sdn : A.dn;
    const uint64_t plane = shared ? 0 : (uint64_t)e * A.dim * NB;
    RowStreams<RS> st{wd, plane + (uint64_t)rl * NB, NB, XV{nullptr, nullptr, nullptr}};
    typename E::Frags fr;
    E::load(st, fr, lane);
    const int *list = shared ? nullptr : A.grp_list + A.grp_off[e];
    const int stride = A.act_stride;
    for (int i = 0; i < n; i++) {
        const int slot = shared ? A.T * A.n_used + i : list[i];
        st.xv = XV{A.aq + (size_t)slot * stride, A.ad + (size_t)slot * (stride / 32), A.as + (size_t)slot * (stride / 16)};
        float y[RS];
        E::finish(st, fr, y, lane);
        if (lane < RS) {
            float v = y[0];
#pragma unroll
            for (int k = 1; k < RS; k++)
                if (lane == k) v = y[k];
            const int r = rl + lane;
            if (r >= r0) A.y[(size_t)slot * A.dim + r] = v;
        }
    }
}

// out[t][r] = residual + sum over the token's local slots, in selection order,
// of gate * y, then + the shared expert's y (llama.zig:1397, deepseek.zig:1498)
__global__ void __launch_bounds__(256) k_combine(DecodeArgs A) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= A.dim) return;
    float acc = 0.0f;
    for (int k = 0; k < A.n_used; k++) {
        const int slot = t * A.n_used + k;
        const int le = A.ids[slot] - A.expert0;
        if (le < 0 || le >= A.n_local) continue;
        acc = fadd(acc, fmul(A.gates[slot], A.y[(size_t)slot * A.dim + r]));
    }
    if (A.has_shared) acc = fadd(acc, A.y[((size_t)A.T * A.n_used + t) * A.dim + r]);
    const size_t o = (size_t)t * A.dim + r;
    A.out[o] = A.residual ? fadd(A.residual[o], acc) : acc;
}

static GUFn gateup_grp_fn(int ty, int nb) {
    if (ty == T_Q4_K) switch (nb) {
            case 4: return k_gateup_grp<T_Q4_K, 4>;
            case 8: return k_gateup_grp<T_Q4_KW, 8>;
            case 16: return k_gateup_grp<T_Q4_KW, 16>;
            case 28: return k_gateup_grp<T_Q4_K, 28>;
        }
    if (ty == T_Q6_K && nb == 8) return k_gateup_grp<T_Q6_K, 8>;
    return nullptr;
}

// rows per warp of the grouped down kernel: 8 (Q6_K, block-major units) or 4
// (Q4_K, stream-major units)
static GUFn down_grp_fn(int ty, int nb, int &rs) {
    if (ty == T_Q6_K) {
        rs = 8;
        switch (nb) {
            case 1: return k_down_grp<T_Q6_K, 8, 1>;
            case 2: return k_down_grp<T_Q6_K, 8, 2>;
            case 3: return k_down_grp<T_Q6_K, 8, 3>;
            case 4: return k_down_grp<T_Q6_K, 8, 4>;
            case 8: return k_down_grp<T_Q6_K, 8, 8>;
        }
    }
    if (ty == T_Q4_K) {
        rs = 4;
        switch (nb) {
            case 4: return k_down_grp<T_Q4_K, 4, 4>;
            case 8: return k_down_grp<T_Q4_KW, 4, 8>;
        }
    }
    return nullptr;
}

bool batch_supported(const DecodeArgs &A) {
    if (A.g.type != A.u.type || A.dim % 256 || A.n_local > 1024) return false;
    if (!gateup_grp_fn(A.g.type, A.dim / 256)) return false;
    const int dty = A.dn.type;
    if (block_elems(dty) == 0 || A.ffn % block_elems(dty)) return false;
    int rs;
    if (!down_grp_fn(dty, A.ffn / block_elems(dty), rs) || A.dim % rs) return false;
    if (A.has_shared) {
        if (A.sg.type != A.g.type || A.su.type != A.g.type || A.sdn.type != dty) return false;
        if (A.shexp_ffn != A.ffn) return false;  // the shared expert reuses the routed instantiation
    }
    return (size_t)(A.dim + 2 * A.n_expert + 136) * 4 <= 48 * 1024;
}

static cudaError_t launch_quant_grp(const DecodeArgs &A, cudaStream_t st) {
    const int n_slots = A.T * A.n_used + (A.has_shared ? A.T : 0);
    return launch_pdl(k_quant_grp, dim3(n_slots), dim3(128), 0, st, A);
}

cudaError_t launch_batch(const DecodeArgs &A0, int path, cudaStream_t st) {
    DecodeArgs A = A0;
    A.tc_chunk = path == BATCH_MMA ? MOE_TC_N : path == BATCH_DP4A ? MOE_DP_CH : 0;
    cudaError_t e = launch_router(A, st);
    if (e != cudaSuccess) return e;
    if ((e = launch_pdl(k_group, dim3(1), dim3(512), 0, st, A)) != cudaSuccess) return e;
    if (path == BATCH_MMA || path == BATCH_DP4A) {
        if ((e = (path == BATCH_MMA ? launch_moe_mma : launch_moe_dp4a)(A, st, launch_quant_grp)) != cudaSuccess)
            return e;
        return launch_pdl(k_combine, dim3(cdivu(A.dim, 256), A.T), dim3(256), 0, st, A);
    }
    const int nexp = A.n_local + (A.has_shared ? 1 : 0);
    const int nb = A.dim / 256;
    const int rows_cta = GU_WARPS * (nb <= 8 ? 3 : 1);
    if ((e = launch_pdl(gateup_grp_fn(A.g.type, nb), dim3(cdivu(A.ffn, rows_cta), nexp), dim3(GU_WARPS * 32), 0, st,
                        A)) != cudaSuccess)
        return e;
    const int n_slots = A.T * A.n_used + (A.has_shared ? A.T : 0);
    if ((e = launch_pdl(k_quant_grp, dim3(n_slots), dim3(128), 0, st, A)) != cudaSuccess) return e;
    int rs = 0;
    GUFn dfn = down_grp_fn(A.dn.type, A.ffn / block_elems(A.dn.type), rs);
    if ((e = launch_pdl(dfn, dim3(cdivu(A.dim, DN_WARPS * rs), nexp), dim3(DN_WARPS * 32), 0, st, A)) != cudaSuccess)
        return e;
    return launch_pdl(k_combine, dim3(cdivu(A.dim, 256), A.T), dim3(256), 0, st, A);
}


// ==== persistent decode stack ===========================================================
// One cooperative kernel runs every layer of a T = 1 decode step. Per layer:
//   P1  router rows spread one per warp over the grid (dotF32 order)     | barrier
//   P2  every CTA routes (replicated, bit-identical) and quantizes x;
//       gate/up rows of the selected experts spread over the grid;
//       each CTA warms L2 with the down rows it will read               | barrier
//   P3  every CTA quantizes the experts' activations into shared memory;
//       down rows + ordered combine + residual spread over the grid;
//       each CTA warms L2 with its router rows of the next layer         | barrier
// Data written by other CTAs inside the kernel is read through L2 (ld.cg).
// The arithmetic per element is the decode kernels', so the stack output is
// bit-identical to running the layers one by one.

constexpr int PS_WARPS = 16;
constexpr uint32_t BAR_POLLS = 1u << 21;  // bounded grid-barrier wait (~1 s of polling)
constexpr uint32_t STAGE_POLLS = 1u << 22; // bounded wait on a bulk copy into shared memory

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Trace slots of the stack kernel: the latest CTA to reach a point (max over
// CTAs), or CTA 0's time at a barrier exit.
__device__ __forceinline__ void trace_max(unsigned long long *slot) {
    if (slot && threadIdx.x == 0) atomicMax(slot, gtimer());
}

// Grid-wide barrier over gridDim.x co-resident CTAs on a monotonic 64-bit
// arrival counter: each CTA adds 1 with release semantics (no round trip) and
// polls with acquire loads until the counter reaches its target, which thread 0
// of each CTA advances by gridDim.x per barrier. Gives up after BAR_POLLS
// polls, or as soon as *err is set by another CTA, raising bit 2 of *err, and
// returns false (the caller leaves the kernel: it never traps or spins forever).
// Thread 0's section cycle counter of the stack kernel (no-op without a trace).
struct CycTrace {
    unsigned long long *base;  // this layer's cycle pairs, or null
    long long t;
    __device__ __forceinline__ void mark(int i) {
        if (threadIdx.x == 0) {
            const long long n = clock64();
            if (base) {
                atomicMax(base + 2 * i, (unsigned long long)(n - t));
                atomicAdd(base + 2 * i + 1, (unsigned long long)(n - t));
            }
            t = n;
        }
    }
};

__device__ __forceinline__ bool grid_barrier(unsigned long long *ctr, unsigned long long &target, int *err,
                                             unsigned long long *t_in = nullptr, unsigned long long *t_out = nullptr,
                                             CycTrace *cy = nullptr, int ci = 0) {
    __shared__ int s_ok;
    __syncthreads();
    trace_max(t_in);
    if (cy) cy->mark(ci);
    if (threadIdx.x == 0) {
        int ok = 1;
        target += gridDim.x;
        red_release_add_u64(ctr, 1ull);
        uint32_t i = 0;
        for (; i < BAR_POLLS; i++) {
            if (ld_acquire_u64(ctr) >= target) break;
            if ((i & 1023) == 1023 && *reinterpret_cast<volatile int *>(err)) i = BAR_POLLS;  // another CTA failed
        }
        if (i >= BAR_POLLS) {
            atomicOr(err, 2);
            ok = 0;
        }
        s_ok = ok;
        if (t_out && blockIdx.x == 0) *t_out = gtimer();
    }
    if (cy) cy->mark(ci + 1);
    __syncthreads();
    return s_ok != 0;
}

// Tagged words: a float and the tag of the layer (and launch) that wrote it,
// in one 8-byte store, so a reader that sees the tag sees the value (one
// single-copy-atomic access) and needs no barrier of its own.
constexpr uint32_t TAG_POLLS = 1u << 20;  // bounded poll on tagged data (~1 s)

__device__ __forceinline__ unsigned long long tagged(float v, uint32_t tag) {
    return ((unsigned long long)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ ulonglong2 ld_relaxed_v2u64(const unsigned long long *p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Down streams of the stack kernel: SC consecutive output rows of ONE expert
// (this CTA's expert), weights staged in shared memory as a row-major tile
// [rows][NBD blocks], the expert's int8 activations (xpad_q6k layout) shared
// by every stream.
template <int NBD> struct StackDownRows {
    WDev w_;         // the tile (quants, scales, f16 scales from doff)
    uint64_t row0;   // tile row of stream 0
    int nvalid;      // streams that are real rows
    XV xv;
    __device__ __forceinline__ WDev w(int) const { return w_; }
    __device__ __forceinline__ uint64_t gb(int s) const { return (row0 + (s < nvalid ? s : 0)) * NBD; }
    __device__ __forceinline__ XV x(int) const { return xv; }
};

__host__ __device__ constexpr size_t round_to_mod128(size_t n, size_t r) {  // smallest m >= n, m % 128 == r
    return (n + (128 - r) + 127) / 128 * 128 - (128 - r);
}

// Work split of the stack kernel over G CTAs (c = blockIdx.x):
//   gate/up  groups of NR rows of gate and up, n_used * ffn / NR of them, in
//            order (expert slot, row); CTA c takes groups [c*total/G, (c+1)*total/G)
//   down     CTA c serves expert slot kd = c*n_used/G; the CTAs of one slot
//            split the dim output rows evenly
struct StackSplit {
    int g0, g1;  // gate/up groups
    int kd;      // down: expert slot
    int ra, rb;  // down: output rows
    __device__ __forceinline__ StackSplit(int c, int G, int total, int nk, int dim) {
        g0 = (int)((long long)c * total / G);
        g1 = (int)((long long)(c + 1) * total / G);
        kd = c * nk / G;
        const int first = (kd * G + nk - 1) / nk, last = ((kd + 1) * G + nk - 1) / nk, n = last - first;
        ra = (c - first) * dim / n;
        rb = (c - first + 1) * dim / n;
    }
};

// Shared-memory map of the stack kernel (recomputed per phase so that no
// pointer stays live in registers across phases). Sizes depend on the grid:
// ngmax gate/up groups and nrmax down rows per CTA.
constexpr int MB_ROUTER = 0, MB_DOWN = 1, MB_GATEUP = 2, MB_COUNT = 4;  // MB_GATEUP, MB_GATEUP + 1: the halves
constexpr int STACK_MAX_LAYERS = 64;

template <int NBG, int NR, int NBD> struct StackSmem {
    static constexpr int dim = NBG * 256;
    static constexpr int GU_HALF = NR * NBG * 144;  // one group's NR rows of gate (or of up), Q4_K
    float *xs;        // x [dim] of the current layer
    int8_t *xq;       // [NBG * XPAD_BLOCK] (xpad_q4kw layout)
    float *xqd;       // [NBG]
    int32_t *xqs;     // [NBG*16]
    float *scores;    // [ne]
    float *choice;    // [ne]
    int *sid;         // [64]
    float *sg;        // [64]
    int *doff;        // [8]
    float *red;       // [8]
    uint64_t *mbar;   // [MB_COUNT]: router rows, down tile, gate/up tiles
    float *rbuf;      // [rpc][dim] this CTA's router rows of the current layer
    uint8_t *gub;     // gate tiles [ngmax][GU_HALF], then up tiles [ngmax][GU_HALF]
    uint8_t *dq;      // [nrmax*NBD][192] down tile quants
    uint8_t *dsc;     // [nrmax*NBD][16]
    uint16_t *dd;     // [dslot/2]
    float *af;        // [ffn] this CTA's expert's activations
    int8_t *aq;       // [ffn/256 * XPAD_BLOCK]
    float *ad;        // [ffn/256]
    int32_t *as;      // [ffn/16]
    StackLayer *lys;  // [n_layers] the layer descriptors
    float *tt;        // [PS_WARPS][2*NR*NBG] per-warp transpose of the gate/up block terms
    static __host__ __device__ size_t dslot(int nrmax) { return ((size_t)nrmax * NBD * 2 + 15) / 16 * 16 + 16; }
    __device__ __forceinline__ StackSmem(uint8_t *base, int ne, int ffn, int rpc, int ngmax, int nrmax) {
        xs = reinterpret_cast<float *>(base);
        xq = reinterpret_cast<int8_t *>(xs + dim);
        xqd = reinterpret_cast<float *>(xq + NBG * XPAD_BLOCK);
        xqs = reinterpret_cast<int32_t *>(xqd + NBG);
        scores = reinterpret_cast<float *>(xqs + NBG * 16);
        choice = scores + ne;
        sid = reinterpret_cast<int *>(choice + ne);
        sg = reinterpret_cast<float *>(sid + 64);
        doff = reinterpret_cast<int *>(sg + 64);
        red = reinterpret_cast<float *>(doff + 8);
        mbar = reinterpret_cast<uint64_t *>(red + 8);  // 16-byte aligned: ne % 4 == 0
        rbuf = reinterpret_cast<float *>(mbar + MB_COUNT);
        gub = reinterpret_cast<uint8_t *>(rbuf + (size_t)rpc * dim);
        dq = gub + (size_t)2 * ngmax * GU_HALF;
        dsc = dq + (size_t)nrmax * NBD * 192;
        dd = reinterpret_cast<uint16_t *>(dsc + (size_t)nrmax * NBD * 16);
        af = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(dd) + dslot(nrmax));
        aq = reinterpret_cast<int8_t *>(af + ffn);
        ad = reinterpret_cast<float *>(aq + (size_t)(ffn / 256) * XPAD_BLOCK);
        as = reinterpret_cast<int32_t *>(ad + ffn / 256);
        lys = reinterpret_cast<StackLayer *>(base + ((reinterpret_cast<uintptr_t>(as + ffn / 16) - reinterpret_cast<uintptr_t>(base) + 15) & ~uintptr_t(15)));
        tt = reinterpret_cast<float *>(lys + STACK_MAX_LAYERS);
    }
    static size_t bytes(int ne, int ffn, int rpc, int ngmax, int nrmax, int n_layers) {
        return (size_t)dim * 4 + NBG * XPAD_BLOCK + NBG * 4 + NBG * 64 + (size_t)2 * ne * 4 + 64 * 8 + 32 + 32 + 8 * MB_COUNT +
               16 + (size_t)STACK_MAX_LAYERS * sizeof(StackLayer) + (size_t)PS_WARPS * 2 * NR * NBG * 4 +
               (size_t)rpc * dim * 4 + (size_t)2 * ngmax * GU_HALF + (size_t)nrmax * NBD * (192 + 16) + dslot(nrmax) +
               (size_t)ffn * 4 + (size_t)(ffn / 256) * XPAD_BLOCK + (size_t)(ffn / 256) * 4 + (size_t)(ffn / 16) * 4;
    }
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Thread 0: stage this CTA's router rows of layer `l` (rows c, c+G, ...) into
// shared memory with bulk copies completing on *mbar.
__device__ __noinline__ void stage_router_rows(const StackArgs &A, int l, float *rbuf, uint64_t *mbar) {
    const int G = gridDim.x, c = blockIdx.x, dim = A.dim;
    int n = 0;
    for (int row = c; row < A.n_expert; row += G) n++;
    if (n == 0) return;
    fence_proxy_async_smem();
    mbar_expect_tx(mbar, (uint32_t)(n * dim * 4));
    int j = 0;
#pragma unroll 1
    for (int row = c; row < A.n_expert; row += G, j++)
        bulk_g2s(rbuf + (size_t)j * dim, A.layers[l].router + (size_t)row * dim, (uint32_t)(dim * 4), mbar);
}

// Stage this CTA's tiles with bulk copies, three warps issuing in parallel
// (a bulk copy takes a few hundred cycles to issue):
//   warp 0  gate/up tiles of the first half of its groups  -> mb_gu
//   warp 1  gate/up tiles of the second half               -> mb_gu + 1
//   last warp  the down tile, once the gate/up tiles have landed: rows
//           ra..rb of expert slot kd (quants, scales, and the f16 scales
//           through a 16-byte-aligned window whose offset goes to *doff)
//                                                          -> mb_dn
// Within a half, a run of groups inside one expert is contiguous in global
// memory and in the tile: lane q copies (run q/2, gate or up).
template <int NBG, int NR, int NBD>
__device__ __forceinline__ void stage_expert_tiles(const StackArgs &A, const StackLayer &Ly, const int *sid, int *doff,
                                                   uint8_t *gub, uint8_t *dq, uint8_t *dsc, uint16_t *dd,
                                                   uint64_t *mb_gu, uint64_t *mb_dn, const StackSplit &P, int ngmax,
                                                   uint32_t parity) {
    using SM = StackSmem<NBG, NR, NBD>;
    constexpr int dim = NBG * 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, ffn = A.ffn, per_e = ffn / NR;
    const int ng = P.g1 - P.g0, nr = P.rb - P.ra, gm = P.g0 + (ng + 1) / 2;
    if (warp < 2) {
        const int h = warp, ha = h ? gm : P.g0, hz = h ? P.g1 : gm;
        if (ha >= hz) return;
        if (lane == 0) mbar_expect_tx(mb_gu + h, (uint32_t)(2 * (hz - ha) * SM::GU_HALF));
        __syncwarp();
        fence_proxy_async_smem();
        const int ka = ha / per_e, kb = (hz - 1) / per_e;
        for (int q = lane; q < 2 * (kb - ka + 1); q += 32) {
            const int k = ka + q / 2, up = q & 1;
            const int ga = max(ha, k * per_e), gz = min(hz, (k + 1) * per_e);
            const uint64_t blk = ((uint64_t)sid[k] * ffn + (uint64_t)(ga - k * per_e) * NR) * NBG;
            bulk_g2s(gub + (size_t)(up ? ngmax : 0) * SM::GU_HALF + (size_t)(ga - P.g0) * SM::GU_HALF,
                     (up ? Ly.u : Ly.g).q + blk * 144, (uint32_t)(gz - ga) * SM::GU_HALF, mb_gu + h);
        }
    } else if (warp == PS_WARPS - 1 && nr) {
        // the down tile is needed only after the gate/up phase: request it once
        // the first gate/up tiles have landed, so the two do not share DRAM
        // bandwidth
        // the first half's leader (warp 0) arrives on named barrier 4 once its
        // tiles have landed; this warp waits there in hardware (no mbarrier poll)
        if (ng > 0 && ng < PS_WARPS) asm volatile("bar.sync 4, 64;" ::: "memory");
        const uint64_t b0 = ((uint64_t)sid[P.kd] * dim + P.ra) * NBD, nb = (uint64_t)nr * NBD;
        const uintptr_t d0 = reinterpret_cast<uintptr_t>(Ly.dn.d + b0);
        const uintptr_t da = d0 & ~uintptr_t(15), de = (d0 + nb * 2 + 15) & ~uintptr_t(15);
        if (lane == 0) {
            *doff = (int)((d0 - da) / 2);
            mbar_expect_tx(mb_dn, (uint32_t)(nb * (192 + 16) + (de - da)));
        }
        __syncwarp();
        fence_proxy_async_smem();
        if (lane == 0) bulk_g2s(dq, Ly.dn.q + b0 * 192, (uint32_t)(nb * 192), mb_dn);
        if (lane == 1) bulk_g2s(dsc, Ly.dn.sc + b0 * 16, (uint32_t)(nb * 16), mb_dn);
        if (lane == 2) bulk_g2s(dd, reinterpret_cast<const void *>(da), (uint32_t)(de - da), mb_dn);
    }
}

// dotF32 (ggml.zig:198) of a router row in shared memory with x in shared
// memory, dim a multiple of 32: lane j accumulates elements j, j+32, ... in
// order, then the eight-lane / four-way reduction of the CPU's 4x8 accumulators.
__device__ __forceinline__ float router_dot_smem(const float *wr, const float *x, int dim, int lane) {
    float a = 0.0f;
#pragma unroll 8
    for (int i = lane; i < dim; i += 32) a = fadd(a, fmul(wr[i], x[i]));
    const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
    const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
    const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
    const float v = fadd(fadd(fadd(a, a8), a16), a24);
    float r = __shfl_sync(0xffffffffu, v, 0);
#pragma unroll
    for (int jj = 1; jj < 8; jj++) r = fadd(r, __shfl_sync(0xffffffffu, v, jj));
    return r;
}

// Bounded wait on a staging barrier. Only thread 0 polls; the verdict is
// shared, so every thread of the CTA takes the same path. On a
// time-out bit 4 of *err is raised: the caller skips its work and the next
// grid barrier, seeing *err, lets the whole grid leave (after draining).
__device__ __noinline__ bool cta_stage_wait(uint64_t *mbar, int parity, int *err) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_ok = mbar_wait(mbar, parity, STAGE_POLLS);
        if (!s_ok) atomicOr(err, 4);
    }
    __syncthreads();
    return s_ok != 0;
}

// One activation block of 256 values (8 per lane) quantized as quantizeX256
// (one scale per block, sums per 16) into a padded int8 layout: xpad_q6k for
// the down operand (Q6K = true), xpad_q4kw for the gate/up operand.
template <bool Q6K>
__device__ __noinline__ void quant_block256_padded(const float *src, int8_t *qbase, float *d256, int32_t *s16,
                                                   int lane) {
    float v[8];
    const float4 p = *reinterpret_cast<const float4 *>(src + lane * 8);
    const float4 q = *reinterpret_cast<const float4 *>(src + lane * 8 + 4);
    v[0] = p.x, v[1] = p.y, v[2] = p.z, v[3] = p.w, v[4] = q.x, v[5] = q.y, v[6] = q.z, v[7] = q.w;
    quant_vals8(v, true, 32, qbase + (Q6K ? xpad_q6k(lane * 8) : xpad_q4kw(lane * 8)), d256, s16 + lane / 2, nullptr,
                lane);
}

// Every CTA, on every way out: count the exit; the last one to leave advances
// the launch epoch (the next launch's tags), so stale tagged words of this
// launch never match a later one.
__device__ __noinline__ void stack_exit(const StackArgs &A) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned *ex = A.bar + 6;
        if (atomicAdd(ex, 1u) == gridDim.x - 1) {
            *ex = 0;
            atomicAdd(A.bar + 4, 1u);
        }
    }
}

// Leaving early (an error): let every copy of layer l this CTA requested land
// first (bounded waits), so that no bulk copy into shared memory outlives it.
__device__ __noinline__ void stack_drain(uint64_t *mbar, const StackSplit &P, int l) {
    if (threadIdx.x != 0) return;
    if (P.g1 > P.g0) mbar_wait(mbar + MB_GATEUP, l & 1, STAGE_POLLS);
    if (P.g1 - P.g0 > 1) mbar_wait(mbar + MB_GATEUP + 1, l & 1, STAGE_POLLS);
    if (P.rb > P.ra) mbar_wait(mbar + MB_DOWN, l & 1, STAGE_POLLS);
}


constexpr int STACK_MAX_USED = 8;

// Wait (thread 0, bounded) until the parts counter of a layer has seen every
// CTA's arrival; the CTA-wide barrier after it orders every thread's reads of
// the parts after the acquire.
__device__ __forceinline__ void wait_parts(const unsigned long long *cnt, unsigned long long target, int *err) {
    if (threadIdx.x == 0) {
        uint32_t it = 0;
        for (; it < TAG_POLLS; it++)
            if (ld_acquire_u64(cnt) >= target) break;
        if (it == TAG_POLLS) atomicOr(err, 16);
    }
    __syncthreads();
}

// x of the next layer: x += sum over expert slots k (in order, from +0) of the
// gate-weighted partial outputs part[k][r] (moe.zig combine order), each
// thread on its own elements of the shared-memory x.
__device__ __forceinline__ void combine_parts(const float *part, int nk, int dim, float *xs) {
#pragma unroll 1
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) {
        float4 p[STACK_MAX_USED];
#pragma unroll
        for (int k = 0; k < STACK_MAX_USED; k++)
            if (k < nk) p[k] = __ldcg(reinterpret_cast<const float4 *>(part + (size_t)k * dim) + i);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < STACK_MAX_USED; k++)
            if (k < nk) {
                acc.x = fadd(acc.x, p[k].x);
                acc.y = fadd(acc.y, p[k].y);
                acc.z = fadd(acc.z, p[k].z);
                acc.w = fadd(acc.w, p[k].w);
            }
        float4 &x = reinterpret_cast<float4 *>(xs)[i];
        x.x = fadd(x.x, acc.x);
        x.y = fadd(x.y, acc.y);
        x.z = fadd(x.z, acc.z);
        x.w = fadd(x.w, acc.w);
    }
}

template <int TYG, int NBG, int TYD, int SC, int NBD, int RW, bool TRACE>
__global__ void __launch_bounds__(PS_WARPS * 32, 1) k_stack(StackArgs A) {
    constexpr int NR = gu_nr<NBG>();
    static_assert(TYG == T_Q4_KW && TYD == T_Q6_K, "staged tiles are laid out for Q4_K gate/up and Q6_K down");
    using SM = StackSmem<NBG, NR, NBD>;
    constexpr int dim = NBG * 256;
    extern __shared__ __align__(16) uint8_t smraw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int nk = A.n_used, ffn = A.ffn;
    const int rpc = (A.n_expert + G - 1) / G;
    const int per_e = ffn / NR, total = nk * per_e, ngmax = (total + G - 1) / G;
    const int nrmax = (dim + G / nk - 1) / (G / nk);
    const int lg_stride = A.n_expert + 32;  // one logit replica
    const StackSplit P(c, G, total, nk, dim);
#define STACK_SMEM SM S(smraw, A.n_expert, ffn, rpc, ngmax, nrmax)
    // tags of this launch: the epoch advances once per completed launch
    const uint32_t epoch = *reinterpret_cast<volatile unsigned *>(A.bar + 4);
    const uint32_t tag0 = epoch * 64u;
    // parts counters, one per layer parity: G arrivals per layer of that parity
    unsigned long long *pcnt = reinterpret_cast<unsigned long long *>(A.bar + 8);
    const unsigned long long n_par[2] = {(unsigned long long)(A.n_layers + 1) / 2, (unsigned long long)A.n_layers / 2};
    auto parts_target = [&](int l) {
        return (unsigned long long)G * ((unsigned long long)epoch * n_par[l & 1] + (unsigned long long)(l >> 1) + 1ull);
    };
    if (threadIdx.x == 0) {
        STACK_SMEM;
        for (int i = 0; i < MB_COUNT; i++) mbar_init(S.mbar + i, 1);
        stage_router_rows(A, 0, S.rbuf, S.mbar + MB_ROUTER);
    }
    {
        STACK_SMEM;
        for (int i = threadIdx.x; i < A.n_layers; i += blockDim.x) S.lys[i] = A.layers[i];
    }
    __syncthreads();
    CycTrace cy{nullptr, TRACE ? clock64() : 0};
#pragma unroll 1
    for (int l = 0; l < A.n_layers; l++) {
        unsigned long long *tr = TRACE ? A.trace + (size_t)l * STACK_TRACE_WORDS : nullptr;
        if (TRACE) cy.base = tr + STACK_TRACE_SLOTS;
        if (TRACE && c == 0 && threadIdx.x == 0) tr[0] = gtimer();  // the previous barrier's exit
        const uint32_t tag = tag0 + (uint32_t)l + 1u;
        {   // ---- P1: x of this layer (x_in, or the previous layer's x plus its combined experts), router rows . x
            STACK_SMEM;
            if (l == 0) {
#pragma unroll 1
                for (int i = threadIdx.x; i < dim / 4; i += blockDim.x)
                    reinterpret_cast<float4 *>(S.xs)[i] = __ldcg(reinterpret_cast<const float4 *>(A.x_in) + i);
            } else {
                wait_parts(pcnt + ((l - 1) & 1), parts_target(l - 1), A.err);
                combine_parts(A.part + (size_t)((l - 1) & 1) * nk * dim, nk, dim, S.xs);
            }
            __syncthreads();
            const bool ok = c >= A.n_expert || cta_stage_wait(S.mbar + MB_ROUTER, l & 1, A.err);
            if (TRACE) cy.mark(0);  // x ready, router rows landed
            // warps with a router row take it; the rest quantize x for gate/up meanwhile
            const int nrw = (A.n_expert - c + G - 1) / G;  // this CTA's router rows
            if (!ok) {
            } else if (warp < nrw) {
#pragma unroll 1
                for (int row = c + warp * G, j = warp; row < A.n_expert; row += PS_WARPS * G, j += PS_WARPS) {
                    const float r = router_dot_smem(S.rbuf + (size_t)j * dim, S.xs, dim, lane);
                    if (lane < LOGIT_REPLICAS) A.logits[(size_t)lane * lg_stride + row] = tagged(r, tag);
                }
            } else {
                const int nq = PS_WARPS - (nrw < PS_WARPS ? nrw : PS_WARPS - 1);
#pragma unroll 1
                for (int b = warp - (PS_WARPS - nq); b < NBG; b += nq)
                    quant_block256_padded<false>(S.xs + b * 256, S.xq + b * XPAD_BLOCK, S.xqd + b, S.xqs + b * 16, lane);
            }
            if (warp < nrw) {  // rbuf is free once the router warps' dots are done: stage the next layer's rows
                // (only the router warps meet: the route of P2 need not wait for x's quantization)
                if (nrw == 1) __syncwarp();
                else asm volatile("bar.sync 5, %0;" ::"r"((nrw < PS_WARPS ? nrw : PS_WARPS) * 32) : "memory");
                if (l + 1 < A.n_layers && threadIdx.x == 0) stage_router_rows(A, l + 1, S.rbuf, S.mbar + MB_ROUTER);
            }
        }
        if (TRACE) {
            __syncthreads();
            trace_max(tr + 1);
            cy.mark(1);  // router rows and x quantization done
        }
        {   // ---- P2: route (replicated in every CTA); stage gate/up and down tiles; gate/up
            STACK_SMEM;
            const int ne = A.n_expert;
            if (warp == 0) {
                // the logits of this layer, as they arrive (tagged words of replica c % R)
                const unsigned long long *lg = A.logits + (size_t)(c % LOGIT_REPLICAS) * lg_stride;
                float v[RW];
                uint32_t it = 0;
                for (; it < TAG_POLLS; it++) {
                    bool have = true;
#pragma unroll
                    for (int t = 0; t < RW; t++) {
                        const int e = lane + 32 * t;
                        v[t] = -INFINITY;
                        if (e < ne) {
                            const unsigned long long w = ld_relaxed_u64(lg + e);
                            v[t] = __uint_as_float((uint32_t)w);
                            have &= (uint32_t)(w >> 32) == tag;
                        }
                    }
                    if (__all_sync(0xffffffffu, have)) break;
                }
                if (it == TAG_POLLS && lane == 0) atomicOr(A.err, 8);
                if (TRACE) cy.mark(2);  // logits arrived
                route_warp_vals<RW>(v, nullptr, ne, nk, A.gating, A.weights_norm, A.weights_scale, S.scores, S.choice,
                                    S.sid, S.sg, S.sid, S.sg, lane);
            }
            if (TRACE) cy.mark(3);  // route (thread 0's warp)
            __syncthreads();
            if (TRACE) trace_max(tr + 3);
            if (warp < 2 || warp == PS_WARPS - 1)
                stage_expert_tiles<NBG, NR, NBD>(A, S.lys[l], S.sid, S.doff, S.gub, S.dq, S.dsc, S.dd,
                                                 S.mbar + MB_GATEUP, S.mbar + MB_DOWN, P, ngmax, l & 1);
            if (TRACE) cy.mark(4);  // tiles requested
            if (c == 0 && A.ids_out && threadIdx.x < nk) A.ids_out[(size_t)l * nk + threadIdx.x] = S.sid[threadIdx.x];
            const int ng = P.g1 - P.g0, nga = (ng + 1) / 2;  // groups, and groups in the first half
            __shared__ int s_half_ok[2];
#pragma unroll 1
            for (int g = warp; g < ng; g += PS_WARPS) {
                {   // this group's half of the tiles: ONE thread per half waits on its
                    // barrier (bounded), the half's other warps park on a named barrier
                    const int h = g >= nga, first = h ? nga : 0, nw = h ? ng - nga : nga;
                    if (lane == 0 && g == first) {
                        const int ok = mbar_wait(S.mbar + MB_GATEUP + h, l & 1, STAGE_POLLS);
                        if (!ok) atomicOr(A.err, 4);
                        s_half_ok[h] = ok;
                    }
                    if (g == 0 && ng < PS_WARPS && P.rb > P.ra)  // release the down-tile warp
                        asm volatile("bar.arrive 4, 64;" ::: "memory");
                    asm volatile("bar.sync %0, %1;" ::"r"(2 + h), "r"(nw * 32) : "memory");
                    if (!s_half_ok[h]) break;
                }
                if (TRACE && g == 0) {
                    trace_max(tr + 9);
                    cy.mark(5);  // warp 0's gate/up tiles landed
                }
                if (TRACE && g == nga && lane == 0) atomicMax(tr + 8, gtimer());  // second half landed
                const int grp = P.g0 + g, k = grp / per_e, rl = (grp % per_e) * NR;
                const float dotv = q4k_group_dot_smem<NR, NBG>(S.gub + (size_t)g * SM::GU_HALF,
                                                              S.gub + (size_t)(ngmax + g) * SM::GU_HALF, S.xq, S.xqd,
                                                              S.xqs, S.tt + warp * 2 * NR * NBG, lane);
                if (TRACE && g == 0) cy.mark(13);  // warp 0's gate/up dots
                const float u = __shfl_down_sync(0xffffffffu, dotv, NR);  // lane i < NR: up row i
                if (lane < NR)  // lane i: silu(gate row i) * up row i
                    A.act[(size_t)k * A.act_stride + rl + lane] =
                        tagged(fmul(fdiv(dotv, fadd(1.0f, exp_f(-dotv))), u), tag);
                if (TRACE && g == 0) cy.mark(14);  // warp 0's activations stored
            }
        }
        if (TRACE) {
            __syncthreads();
            trace_max(tr + 4);
            cy.mark(6);  // gate/up done
        }
        {   // ---- P3: this CTA's expert: its activations quantized, rows ra..rb of its down matrix
            STACK_SMEM;
            const int nbf = ffn / 256;
            {   // this expert's activations as they arrive (tagged words), every thread polling its share
                const unsigned long long *src = A.act + (size_t)P.kd * A.act_stride;
                constexpr int PER = 2;  // entries per thread polled together (ffn <= PER * blockDim.x)
                unsigned long long w[PER];
                bool have = false;
                uint32_t it = 0;
                for (; it < TAG_POLLS && !have; it++) {
                    have = true;
#pragma unroll
                    for (int j = 0; j < PER; j++) {
                        const int i = threadIdx.x + j * blockDim.x;
                        if (i < ffn) {
                            w[j] = ld_relaxed_u64(src + i);
                            have &= (uint32_t)(w[j] >> 32) == tag;
                        }
                    }
                }
                if (!have) atomicOr(A.err, 8);
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    const int i = threadIdx.x + j * blockDim.x;
                    if (i < ffn) S.af[i] = __uint_as_float((uint32_t)w[j]);
                }
            }
            __syncthreads();
            if (TRACE) cy.mark(8);  // activations arrived
            if (warp < nbf)
                quant_block256_padded<true>(S.af + warp * 256, S.aq + warp * XPAD_BLOCK, S.ad + warp, S.as + warp * 16,
                                            lane);
            __syncthreads();
            if (TRACE) {
                cy.mark(9);  // activations quantized
                trace_max(tr + 6);
            }
            const bool ok = P.rb <= P.ra || cta_stage_wait(S.mbar + MB_DOWN, l & 1, A.err);
            if (TRACE) {
                trace_max(tr + 10);
                cy.mark(10);  // down tile landed
            }
            const float gk = S.sg[P.kd];
            float *pout = A.part + ((size_t)(l & 1) * nk + P.kd) * dim;
            const WDev wt{S.dq, S.dsc, S.dd + *S.doff, T_Q6_K, 0};
#pragma unroll 1
            for (int r = P.ra + warp * SC; ok && r < P.rb; r += PS_WARPS * SC) {
                const int n = P.rb - r < SC ? P.rb - r : SC;
                const float yv = q6k_rows_dot_smem<SC, NBD>(wt, r - P.ra, n, S.aq, S.ad, S.as, lane);
                if ((lane & 3) == 0 && (lane >> 2) < n) pout[r + (lane >> 2)] = fmul(gk, yv);
            }
            __syncthreads();  // every row of this CTA stored: arrive on the layer's parts counter
            if (threadIdx.x == 0) red_release_add_u64(pcnt + (l & 1), 1ull);
            if (TRACE) {
                trace_max(tr + 7);
                cy.mark(11);  // down rows done
            }
        }
    }
    {   // the last layer's output: x plus its combined experts, this CTA's slice of rows
        STACK_SMEM;
        const int r0 = c * dim / G, r1 = (c + 1) * dim / G, L = A.n_layers;
        const float *pl = A.part + (size_t)((L - 1) & 1) * nk * dim;
        wait_parts(pcnt + ((L - 1) & 1), parts_target(L - 1), A.err);
        for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
            float acc = 0.0f;
            for (int k = 0; k < nk; k++) acc = fadd(acc, __ldcg(pl + (size_t)k * dim + r));
            A.out[r] = fadd(A.residual ? __ldcg(A.residual + r) : S.xs[r], acc);
        }
    }
    stack_exit(A);
#undef STACK_SMEM
}

using StackFn = void (*)(StackArgs);
static StackFn stack_fn(int gty, int nbg, int dty, int nbd, int ne, bool trace) {
    if (gty == T_Q4_K && nbg == 8 && dty == T_Q6_K && nbd == 3) {
        if (ne <= 128)
            return trace ? k_stack<T_Q4_KW, 8, T_Q6_K, 8, 3, 4, true> : k_stack<T_Q4_KW, 8, T_Q6_K, 8, 3, 4, false>;
        if (ne <= 256)
            return trace ? k_stack<T_Q4_KW, 8, T_Q6_K, 8, 3, 8, true> : k_stack<T_Q4_KW, 8, T_Q6_K, 8, 3, 8, false>;
    }
    return nullptr;
}

static size_t stack_smem(const StackArgs &S, int n_sm) {
    const int rpc = (S.n_expert + n_sm - 1) / n_sm;
    const int total = S.n_used * (S.ffn / gu_nr<8>());
    const int per_slot = n_sm / S.n_used;  // fewest CTAs serving one expert slot's down rows
    return StackSmem<8, gu_nr<8>(), 3>::bytes(S.n_expert, S.ffn, rpc, (total + n_sm - 1) / n_sm,
                                              (S.dim + per_slot - 1) / per_slot, S.n_layers);
}

static int sm_count() {
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    return nsm;
}

bool stack_supported(const StackArgs &S, int g_type, int dn_type) {
    if (S.dim % 256 || S.ffn % 256 || S.n_used > 64 || S.n_expert > 1024 || S.n_expert % 4) return false;
    if (!stack_fn(g_type, S.dim / 256, dn_type, S.ffn / block_elems(dn_type), S.n_expert, false)) return false;
    if (S.dim / 256 != 8) return false;  // the shared-memory map is instantiated for dim 2048
    const int nsm = sm_count(), total = S.n_used * (S.ffn / gu_nr<8>());
    if (S.n_used > STACK_MAX_USED || S.ffn > 2 * PS_WARPS * 32 || S.ffn / 256 > PS_WARPS || nsm < S.n_used || S.n_layers > STACK_MAX_LAYERS) return false;
    (void)total;
    return stack_smem(S, sm_count()) <= 227 * 1024;
}

cudaError_t launch_stack(const StackArgs &S, int g_type, int dn_type, cudaStream_t st) {
    StackFn fn = stack_fn(g_type, S.dim / 256, dn_type, S.ffn / block_elems(dn_type), S.n_expert, S.trace != nullptr);
    const int nsm = sm_count();
    int per_sm = 0;
    const size_t smem = stack_smem(S, nsm);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, PS_WARPS * 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nsm);
    cfg.blockDim = dim3(PS_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, fn, S);
}

}  // namespace loom
