// prefill.cu -- the dense matmuls of a batched prefill (llama.zig:1698 stepBatch,
// mmul over n token rows) as a tiled kernel: each CTA stages a tile of weight
// rows (one bulk copy per region: they are contiguous in the device layout)
// and a tile of the tokens' quantized activations (the padded shared-memory
// layout of ab_quant_pad, so the dots' reads are conflict-free), then dots
// every (row, token) pair of the tile with one lane per (row, block)
// (ab_rows: the reference's integer sums and float tail, kBlockDot /
// matvecK256, ggml.zig:1002-1042 -- bit-identical to the per-token matvec).
// The weights cross L2 once per token tile and the activations once per row
// tile, instead of every row re-reading every token's activation.
#include <cuda_runtime.h>

#include "pdl.cuh"
#include "step_dev.cuh"
#include "warpdot.cuh"

namespace loom {

namespace {

constexpr int MT_WARPS = 8, MT_THREADS = MT_WARPS * 32;
constexpr size_t MT_SMEM_MAX = 200 * 1024;

struct MtPlan {
    int R = 0, NT = 0;  // rows, tokens per tile
    size_t w_bytes = 0, sc_bytes = 0, d_bytes = 0, x_bytes = 0, smem = 0;
};

__host__ __device__ inline bool mt_k256(int ty) { return ty == T_Q4_K || ty == T_Q6_K; }

inline size_t al128(size_t n) { return (n + 127) & ~size_t(127); }

// per token: quants (padded), per-16 or per-32 sums (padded), block scales
__host__ __device__ inline size_t mt_tok_bytes(int ty, int nb) {
    const bool k = mt_k256(ty);
    return (((size_t)nb * ab_pad_qs(k) + 15) & ~size_t(15)) + (((size_t)nb * ab_pad_ss(k) * 4 + 15) & ~size_t(15)) +
           (((size_t)nb * 4 + 15) & ~size_t(15));
}

MtPlan mt_plan(int ty, int nb) {
    const size_t qb = layout_qbytes(ty);
    for (int R : {64, 32, 16}) {
        for (int NT : {16, 8}) {
            MtPlan c;
            c.R = R;
            c.NT = NT;
            c.w_bytes = al128((size_t)R * nb * qb);
            c.sc_bytes = ty == T_Q6_K ? al128((size_t)R * nb * 16) : 0;
            c.d_bytes = ty == T_Q4_K ? 0 : al128((size_t)R * nb * 2);
            c.x_bytes = al128((size_t)NT * mt_tok_bytes(ty, nb));
            c.smem = c.w_bytes + c.sc_bytes + c.d_bytes + c.x_bytes;
            if (c.smem <= MT_SMEM_MAX) return c;
        }
    }
    return MtPlan{};
}

template <int TY>
__global__ void __launch_bounds__(MT_THREADS, 1) k_mm_tiled(WDev w, int rows, int nb, XQ x, int ntok, float *out,
                                                            int R, int NT, size_t w_off_sc, size_t w_off_d,
                                                            size_t x_off) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float tsm_all[MT_WARPS][64];
    constexpr bool K256 = TY == T_Q4_K || TY == T_Q6_K;
    constexpr int BE = K256 ? 256 : 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r0 = blockIdx.x * R, t0 = blockIdx.y * NT;
    const int nr = min(R, rows - r0), nt = min(NT, ntok - t0);
    uint8_t *sq = sm, *ssc = sm + w_off_sc;
    uint16_t *sd = reinterpret_cast<uint16_t *>(sm + w_off_d);
    if (tid == 0) {  // the weight rows do not depend on the previous kernel: requested before its wait
        mbar_init_nf(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint64_t gb0 = (uint64_t)r0 * nb, n = (uint64_t)nr * nb;
        const uint32_t bytes = (uint32_t)(n * layout_qbytes(TY)) + (TY == T_Q6_K ? (uint32_t)(n * 16) : 0u);
        mbar_expect_tx(&bar, bytes);
        bulk_g2s(sq, w.q + gb0 * layout_qbytes(TY), (uint32_t)(n * layout_qbytes(TY)), &bar);
        if (TY == T_Q6_K) bulk_g2s(ssc, w.sc + gb0 * 16, (uint32_t)(n * 16), &bar);
    }
    pdl_wait_();
    pdl_trigger_();
    if (TY != T_Q4_K)  // the f16 block scales: read-only loads
        for (int i = tid; i < nr * nb; i += MT_THREADS) sd[i] = __ldg(w.d + (uint64_t)r0 * nb + i);
    // the tile's tokens into the padded layout (quants 16 bytes at a time)
    const size_t tb = mt_tok_bytes(TY, nb);
    const int qs = ab_pad_qs(K256), ss = ab_pad_ss(K256), c16 = BE / 16, spb = K256 ? 16 : 1;
    const size_t q_bytes = ((size_t)nb * qs + 15) & ~size_t(15), s_bytes = ((size_t)nb * ss * 4 + 15) & ~size_t(15);
    uint8_t *xt = sm + x_off;
    for (int i = tid; i < nt * nb * c16; i += MT_THREADS) {
        const int t = i / (nb * c16), rem = i - t * nb * c16, b = rem / c16, c = rem - b * c16;
        *reinterpret_cast<int4 *>(xt + (size_t)t * tb + (size_t)b * qs + 16 * c) =
            __ldcg(reinterpret_cast<const int4 *>(x.q + (size_t)(t0 + t) * x.cols + (size_t)b * BE) + c);
    }
    if (K256 || TY == T_Q4_0)
        for (int i = tid; i < nt * nb * spb; i += MT_THREADS) {
            const int t = i / (nb * spb), rem = i - t * nb * spb, b = rem / spb, c = rem - b * spb;
            reinterpret_cast<int32_t *>(xt + (size_t)t * tb + q_bytes)[b * ss + c] =
                __ldcg(x.s + (size_t)(t0 + t) * x.sstride + (size_t)b * spb + c);
        }
    for (int i = tid; i < nt * nb; i += MT_THREADS) {
        const int t = i / nb, b = i - t * nb;
        reinterpret_cast<float *>(xt + (size_t)t * tb + q_bytes + s_bytes)[b] =
            __ldcg(x.d + (size_t)(t0 + t) * x.dstride + b);
    }
    __syncthreads();
    if (!mbar_wait(&bar, 0, 1u << 22)) return;  // a copy that never landed: the outputs stay unwritten
    const AbStage st{sq, TY == T_Q6_K ? ssc : nullptr, TY == T_Q4_K ? nullptr : sd, 0, nr, nb};
    // units: (token, chunk of rows) with at most 32 (row, block) lanes
    const int nS = max(1, min(4, 32 / nb)), nch = (nr + nS - 1) / nS;
    for (int u = warp; u < nt * nch; u += MT_WARPS) {
        const int t = u / nch, rc = (u - t * nch) * nS, n = min(nS, nr - rc);
        const uint8_t *xb = xt + (size_t)t * tb;
        const XV xv{reinterpret_cast<const int8_t *>(xb), reinterpret_cast<const float *>(xb + q_bytes + s_bytes),
                    reinterpret_cast<const int32_t *>(xb + q_bytes)};
        const float a = ab_rows<TY>(st, rc, n, xv, tsm_all[warp], lane, qs, ss);
        if (lane < n) out[(size_t)(t0 + t) * rows + r0 + rc + lane] = a;
    }
}

template <int TY>
cudaError_t mt_launch(const WDev &w, int rows, int nb, const XQ &x, int ntok, float *out, cudaStream_t st,
                      const MtPlan &p) {
    static int set = 0;
    if (!set) {
        cudaFuncSetAttribute(k_mm_tiled<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MT_SMEM_MAX);
        set = 1;
    }
    const size_t off_sc = p.w_bytes, off_d = p.w_bytes + p.sc_bytes, off_x = p.w_bytes + p.sc_bytes + p.d_bytes;
    const dim3 grid((rows + p.R - 1) / p.R, (ntok + p.NT - 1) / p.NT);
    return launch_pdl_(k_mm_tiled<TY>, grid, dim3(MT_THREADS), p.smem, st, w, rows, nb, x, ntok, out, p.R, p.NT, off_sc,
                       off_d, off_x);
}

}  // namespace

// The tiled matmul for the weight types ab_rows reads (Q4_K, Q6_K, Q8_0,
// Q4_0); false when the type or the row width does not fit (the caller runs
// launch_mm). out[k * rows + r], bit-identical to launch_mm.
bool launch_mm_tiled(const WDev &w, int rows, int cols, const XQ &x, int ntok, float *out, cudaStream_t st) {
    const int ty = w.type;
    if (ty != T_Q4_K && ty != T_Q6_K && ty != T_Q8_0 && ty != T_Q4_0) return false;
    const int be = mt_k256(ty) ? 256 : 32;
    if (cols % be || x.kind256 != (mt_k256(ty) ? 1 : 0)) return false;
    const int nb = cols / be;
    if (nb > 64) return false;  // the per-warp term buffer
    const MtPlan p = mt_plan(ty, nb);
    if (!p.R) return false;
    cudaError_t e = cudaSuccess;
    switch (ty) {
        case T_Q4_K: e = mt_launch<T_Q4_K>(w, rows, nb, x, ntok, out, st, p); break;
        case T_Q6_K: e = mt_launch<T_Q6_K>(w, rows, nb, x, ntok, out, st, p); break;
        case T_Q8_0: e = mt_launch<T_Q8_0>(w, rows, nb, x, ntok, out, st, p); break;
        default: e = mt_launch<T_Q4_0>(w, rows, nb, x, ntok, out, st, p); break;
    }
    return e == cudaSuccess;
}

}  // namespace loom
