// gemv.cu -- one-token matvec on the warp engine (warpdot.cuh): each warp
// takes S consecutive rows, issues every 16-byte weight load of those rows
// before touching the activations (so the loads are in flight while the
// producer of x is still finishing: programmatic dependent launch), then
// forms the reference's integer block dots and adds each row's block terms in
// block order (ggml.zig:1002-1042 kBlockDot / matvecK256; :1196 / :1277 for
// Q4_0 / Q8_0). Bit-identical to k_mm and to the CPU reference.
#include "gemv.cuh"
#include "pdl.cuh"
#include "step_dev.cuh"
#include "warpdot.cuh"

namespace loom {

namespace {

constexpr int GV_WARPS = 8;

struct GvRows {
    WDev w;
    int r0, nb;
    XQ x;
    __device__ __forceinline__ void at(int s, WDev &ww, uint64_t &gb, XV &xv) const {
        ww = w;
        gb = (uint64_t)(r0 + s) * nb;
        xv = XV{x.q, x.d, x.s};
    }
};

template <int TY, int S, int MAXU>
__global__ void __launch_bounds__(GV_WARPS * 32) k_gemv(WDev w, int rows, int nb, XQ x, float *out) {
    const int lane = threadIdx.x & 31;
    const int r0 = (blockIdx.x * GV_WARPS + (threadIdx.x >> 5)) * S;
    if (r0 >= rows) {
        pdl_wait_();
        return;
    }
    const int nS = min(S, rows - r0);
    const GvRows st{w, r0, nb, x};
    WFrags<TY, MAXU> fr;
    wd_load<TY, S, MAXU>(st, nb, nS, fr, lane);
    pdl_wait_();
    pdl_trigger_();
    float acc[S];
    wd_finish<TY, S, MAXU>(st, nb, nS, fr, acc, lane);
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < S; s++)
            if (s < nS) out[r0 + s] = acc[s];
    }
}

// units a warp holds: MAXU fragments x (32 / lanes per block)
template <int TY> constexpr int gv_maxu() { return TY == T_Q4_K ? 8 : TY == T_Q6_K ? 4 : TY == T_Q8_0 ? 4 : 2; }
template <int TY> constexpr int gv_units() { return gv_maxu<TY>() * (32 / QT<TY>::LPB); }

template <int TY> cudaError_t gv_launch(const WDev &w, int rows, int nb, const XQ &x, float *out, cudaStream_t st) {
    constexpr int MAXU = gv_maxu<TY>();
    const int cap = gv_units<TY>() / nb;  // rows a warp can hold
    if (cap >= 4)
        return launch_pdl_(k_gemv<TY, 4, MAXU>, dim3((rows + GV_WARPS * 4 - 1) / (GV_WARPS * 4)), dim3(GV_WARPS * 32),
                           0, st, w, rows, nb, x, out);
    if (cap >= 2)
        return launch_pdl_(k_gemv<TY, 2, MAXU>, dim3((rows + GV_WARPS * 2 - 1) / (GV_WARPS * 2)), dim3(GV_WARPS * 32),
                           0, st, w, rows, nb, x, out);
    return launch_pdl_(k_gemv<TY, 1, MAXU>, dim3((rows + GV_WARPS - 1) / GV_WARPS), dim3(GV_WARPS * 32), 0, st, w,
                       rows, nb, x, out);
}

// ---- streamed matvec for large matrices (output heads, wide projections) -----------
// Persistent CTAs (one per SM) walk tiles of TR rows: thread 0 bulk-copies each
// tile's regions (quants, Q6_K scales and f16 scales) into a two-stage ring
// (mbarrier transaction counts), so ~2 tiles per SM are in flight; the warps
// form each row's block terms one lane per (row, block) on the staged tile
// against the activation held in shared memory in the padded layout, and add
// them in block order (ab_rows: the warp engine's arithmetic). Bit-identical
// to k_gemv / k_mm. Q4_K (raw blocks) and Q6_K (nb % 8 == 0) only.
constexpr int GS_WARPS = 8, GS_STAGES = 2;
constexpr uint32_t GS_POLLS = 1u << 22;
constexpr size_t GS_STAGE_MAX = 96 * 1024;

__host__ __device__ constexpr size_t gs_row_bytes(int type, int nb) {
    return (size_t)nb * (type == T_Q6_K ? 192 + 16 + 2 : 144);
}
__host__ __device__ inline size_t gs_act_bytes(int nb) {
    return ab_al128((size_t)nb * 272) + ab_al128((size_t)nb * 4) + ab_al128((size_t)nb * 20 * 4);
}

template <int TY>
__global__ void __launch_bounds__(GS_WARPS * 32, 1) k_gemv_stream(WDev w, int rows, int nb, XQ x, float *out, int tr,
                                                                  const float *res) {
    extern __shared__ __align__(128) uint8_t gs[];
    __shared__ __align__(8) uint64_t full[GS_STAGES];
    __shared__ float tsm_all[GS_WARPS][128];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ntiles = (rows + tr - 1) / tr;
    int8_t *xq = reinterpret_cast<int8_t *>(gs);
    float *xd = reinterpret_cast<float *>(gs + ab_al128((size_t)nb * 272));
    int32_t *xs = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(xd) + ab_al128((size_t)nb * 4));
    uint8_t *stage0 = gs + gs_act_bytes(nb);
    const size_t qb = (size_t)tr * nb * layout_qbytes(TY);
    const size_t sb = TY == T_Q6_K ? (size_t)tr * nb * 16 : 0, db = TY == T_Q6_K ? (size_t)tr * nb * 2 : 0;
    const size_t stage_bytes = ab_al128(qb) + ab_al128(sb) + ab_al128(db);
    auto issue = [&](int k, int t) {  // tile t into stage k % 2 (thread 0)
        uint8_t *st = stage0 + (size_t)(k % GS_STAGES) * stage_bytes;
        const int r0 = t * tr, n = min(tr, rows - r0);
        const uint64_t gb0 = (uint64_t)r0 * nb, nbk = (uint64_t)n * nb;
        uint64_t *bar = &full[k % GS_STAGES];
        mbar_expect_tx(bar, (uint32_t)(nbk * layout_qbytes(TY) + (TY == T_Q6_K ? nbk * 18 : 0)));
        bulk_g2s(st, w.q + gb0 * layout_qbytes(TY), (uint32_t)(nbk * layout_qbytes(TY)), bar);
        if (TY == T_Q6_K) {
            bulk_g2s(st + ab_al128(qb), w.sc + gb0 * 16, (uint32_t)(nbk * 16), bar);
            bulk_g2s(st + ab_al128(qb) + ab_al128(sb), w.d + gb0, (uint32_t)(nbk * 2), bar);
        }
    };
    int issued = 0;  // tiles issued (thread 0)
    if (tid == 0) {
        for (int i = 0; i < GS_STAGES; i++) mbar_init_nf(&full[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < GS_STAGES; k++) {  // the weights do not depend on the previous kernel
            const int t = blockIdx.x + k * gridDim.x;
            if (t < ntiles) {
                issue(k, t);
                issued++;
            }
        }
    }
    pdl_wait_();
    pdl_trigger_();
    // the activation into the padded layout (quants 272 B per block, sums 20 words)
    for (int i = tid; i < nb * 16; i += blockDim.x) {
        const int b = i >> 4, c = i & 15;
        *reinterpret_cast<int4 *>(xq + (size_t)b * 272 + 16 * c) = __ldcg(reinterpret_cast<const int4 *>(x.q + (size_t)b * 256) + c);
        xs[b * 20 + c] = __ldcg(x.s + (size_t)b * 16 + c);
    }
    for (int b = tid; b < nb; b += blockDim.x) xd[b] = __ldcg(x.d + b);
    __syncthreads();
    const XV xv{xq, xd, xs};
    const int nS = max(1, min(4, 32 / nb));  // rows per warp call (<= 128 units)
    float *tsm = tsm_all[warp];
    int k = 0;
    for (;; k++) {
        const int t = blockIdx.x + k * gridDim.x;
        if (t >= ntiles) break;
        const bool ok = mbar_wait(&full[k % GS_STAGES], (k / GS_STAGES) & 1, GS_POLLS);
        if (__syncthreads_or(!ok)) break;  // a copy that never landed: every thread leaves together
        uint8_t *st = stage0 + (size_t)(k % GS_STAGES) * stage_bytes;
        const int r0 = t * tr, n = min(tr, rows - r0);
        AbStage sg;
        sg.q = st;
        sg.sc = TY == T_Q6_K ? st + ab_al128(qb) : nullptr;
        sg.d = reinterpret_cast<const uint16_t *>(st + ab_al128(qb) + ab_al128(sb));
        sg.ra = r0;
        sg.rb = r0 + n;
        sg.nb = nb;
        for (int rr = warp * nS; rr < n; rr += GS_WARPS * nS) {
            const int ns = min(nS, n - rr);
            const float a = ab_rows<TY>(sg, rr, ns, xv, tsm, lane, 272, 20);
            if (lane < ns) out[r0 + rr + lane] = res ? fadd(res[r0 + rr + lane], a) : a;
        }
        __syncthreads();  // every warp is done with this stage
        if (tid == 0) {
            const int t2 = blockIdx.x + (k + GS_STAGES) * gridDim.x;
            if (t2 < ntiles) {
                issue(k + GS_STAGES, t2);
                issued++;
            }
        }
    }
    // copies still in flight (only after a timed-out wait) land before the CTA exits (bounded)
    if (tid == 0)
        for (int kk = k; kk < issued; kk++) mbar_wait(&full[kk % GS_STAGES], (kk / GS_STAGES) & 1, GS_POLLS);
}

int gs_tile_rows(int type, int nb) {
    const size_t rb = gs_row_bytes(type, nb);
    int tr = (int)(GS_STAGE_MAX / rb) & ~7;
    return tr > 64 ? 64 : tr;
}

}  // namespace

bool gemv_stream_shape_ok(int type, int cols) {
    if (type != T_Q4_K && type != T_Q6_K) return false;
    if (cols % 256) return false;
    const int nb = cols / 256;
    if (nb > 128 || (type == T_Q6_K && nb % 8)) return false;
    return gs_tile_rows(type, nb) >= 8;
}

bool gemv_stream_supported(int type, int rows, int cols) { return rows >= 4096 && gemv_stream_shape_ok(type, cols); }

cudaError_t launch_gemv_stream(const WDev &w, int rows, int cols, const XQ &x, float *out, cudaStream_t st,
                               const float *res) {
    static int n_sm = 0;
    if (!n_sm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    }
    const int nb = cols / 256, tr = gs_tile_rows(w.type, nb);
    const size_t qb = (size_t)tr * nb * layout_qbytes(w.type);
    const size_t sb = w.type == T_Q6_K ? (size_t)tr * nb * 16 : 0, db = w.type == T_Q6_K ? (size_t)tr * nb * 2 : 0;
    const size_t smem = gs_act_bytes(nb) + GS_STAGES * (ab_al128(qb) + ab_al128(sb) + ab_al128(db));
    const int tiles = (rows + tr - 1) / tr;
    const dim3 grid(tiles < n_sm ? tiles : n_sm);
    if (w.type == T_Q6_K) {
        cudaFuncSetAttribute(k_gemv_stream<T_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        return launch_pdl_(k_gemv_stream<T_Q6_K>, grid, dim3(GS_WARPS * 32), smem, st, w, rows, nb, x, out, tr, res);
    }
    cudaFuncSetAttribute(k_gemv_stream<T_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch_pdl_(k_gemv_stream<T_Q4_K>, grid, dim3(GS_WARPS * 32), smem, st, w, rows, nb, x, out, tr, res);
}

bool gemv_supported(int type, int cols) {
    const int be = block_elems(type);
    if (be == 0 || cols % be) return false;
    const int nb = cols / be;
    switch (type) {
        case T_Q4_K: return nb <= gv_units<T_Q4_K>();
        case T_Q6_K: return nb <= gv_units<T_Q6_K>();
        case T_Q8_0: return nb <= gv_units<T_Q8_0>();
        case T_Q4_0: return nb <= gv_units<T_Q4_0>();
        default: return false;
    }
}

cudaError_t launch_gemv(const WDev &w, int rows, int cols, const XQ &x, float *out, cudaStream_t st) {
    const int nb = cols / block_elems(w.type);
    switch (w.type) {
        case T_Q4_K: return gv_launch<T_Q4_K>(w, rows, nb, x, out, st);
        case T_Q6_K: return gv_launch<T_Q6_K>(w, rows, nb, x, out, st);
        case T_Q8_0: return gv_launch<T_Q8_0>(w, rows, nb, x, out, st);
        case T_Q4_0: return gv_launch<T_Q4_0>(w, rows, nb, x, out, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace loom
