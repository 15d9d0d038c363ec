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
constexpr size_t MT_SMEM_MAX = 200 * 1024, MT_SMEM_TWO = 92 * 1024;
constexpr int MT_NT = 16;  // tokens a lane dots against one unpacked weight fragment

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

// The largest tile that lets two CTAs share an SM (16 warps to hide the dots' latencies), else
// the largest that fits one. A matrix far beyond L2 (an output head) takes 16 tokens a tile with
// the largest row tile that fits one CTA, so its weights cross HBM as few times as that allows.
MtPlan mt_plan(int ty, int nb, int rows, int ntok) {
    const size_t qb = layout_qbytes(ty);
    const size_t wbytes = (size_t)rows * nb * (qb + (ty == T_Q6_K ? 16 : 0) + (ty == T_Q4_K ? 0 : 2));
    if (wbytes > ((size_t)32 << 20) && ntok > 16) {
        for (int R : {64, 32, 16}) {
            MtPlan c;
            c.R = R;
            c.NT = MT_NT;
            c.w_bytes = al128((size_t)R * nb * qb);
            c.sc_bytes = ty == T_Q6_K ? al128((size_t)R * nb * 16) : 0;
            c.d_bytes = ty == T_Q4_K ? 0 : al128((size_t)R * nb * 2);
            c.x_bytes = al128((size_t)MT_NT * mt_tok_bytes(ty, nb));
            c.smem = c.w_bytes + c.sc_bytes + c.d_bytes + c.x_bytes;
            if (c.smem <= MT_SMEM_MAX) return c;
        }
    }
    for (size_t cap : {MT_SMEM_TWO, MT_SMEM_MAX})
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
            if (c.smem <= cap) return c;
        }
    }
    return MtPlan{};
}

// Q4_K rows [r0, r0 + nS) of the staged tile against up to MT_NT tokens at once:
// lane u = (row, block) unpacks each 32-byte nibble fragment and its two
// sub-block scales/mins once (QT<T_Q4_K>::part's arithmetic) and runs the
// dp4a dots of every token against them; per token the integer sums I and M
// are exact, so the block terms and their block-order sums equal ab_rows'.
__device__ __noinline__ void q4k_rows_multi(const uint8_t *wq, int r0, int nS, int NB, const uint8_t *xt, size_t tb,
                                            size_t q_bytes, size_t s_bytes, int nt, float (*tsm)[32], int lane,
                                            float *out, int rows, int t0) {
    const int u = lane;
    if (u < nS * NB) {
        const int s2 = u / NB, b = u - s2 * NB;
        const uint8_t *blk = wq + ((size_t)(r0 + s2) * NB + b) * 144;
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        int I[MT_NT], M[MT_NT];
#pragma unroll
        for (int t = 0; t < MT_NT; t++) I[t] = M[t] = 0;
#pragma unroll 1
        for (int sub = 0; sub < 8; sub++) {
            const uint4 q = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * sub);
            const int j = sub >> 1, hh = sub & 1;
            const int l0 = (int)(q.x & 0x0F0F0F0Fu), l1 = (int)(q.y & 0x0F0F0F0Fu), l2 = (int)(q.z & 0x0F0F0F0Fu),
                      l3 = (int)(q.w & 0x0F0F0F0Fu);
            const int h0 = (int)((q.x >> 4) & 0x0F0F0F0Fu), h1 = (int)((q.y >> 4) & 0x0F0F0F0Fu),
                      h2 = (int)((q.z >> 4) & 0x0F0F0F0Fu), h3 = (int)((q.w >> 4) & 0x0F0F0F0Fu);
            int sc0, mn0, sc1, mn1;  // scaleMinK4 (ggml.zig:1332) for sub-blocks 2j and 2j+1
            if (j < 2) {
                const uint32_t a = h.y >> (16 * j), c = h.z >> (16 * j);
                sc0 = a & 63;
                sc1 = (a >> 8) & 63;
                mn0 = c & 63;
                mn1 = (c >> 8) & 63;
            } else {
                const int jj = j - 2;
                const uint32_t lo = h.w >> (16 * jj), hs = h.y >> (16 * jj), hm = h.z >> (16 * jj);
                sc0 = (lo & 0xF) | (((hs >> 6) & 3) << 4);
                mn0 = ((lo >> 4) & 0xF) | (((hm >> 6) & 3) << 4);
                sc1 = ((lo >> 8) & 0xF) | (((hs >> 14) & 3) << 4);
                mn1 = ((lo >> 12) & 0xF) | (((hm >> 14) & 3) << 4);
            }
#pragma unroll
            for (int t = 0; t < MT_NT; t++) {
                if (t < nt) {
                    const uint8_t *xb = xt + (size_t)t * tb;
                    const int8_t *xq = reinterpret_cast<const int8_t *>(xb) + (size_t)b * 272;
                    const int4 xl = *reinterpret_cast<const int4 *>(xq + 64 * j + 16 * hh);
                    const int4 xh = *reinterpret_cast<const int4 *>(xq + 64 * j + 32 + 16 * hh);
                    int dl = dp4a(l0, xl.x, 0);
                    dl = dp4a(l1, xl.y, dl);
                    dl = dp4a(l2, xl.z, dl);
                    dl = dp4a(l3, xl.w, dl);
                    int dh = dp4a(h0, xh.x, 0);
                    dh = dp4a(h1, xh.y, dh);
                    dh = dp4a(h2, xh.z, dh);
                    dh = dp4a(h3, xh.w, dh);
                    const int32_t *xs = reinterpret_cast<const int32_t *>(xb + q_bytes) + b * 20;
                    I[t] += sc0 * dl + sc1 * dh;
                    M[t] += mn0 * xs[4 * j + hh] + mn1 * xs[4 * j + 2 + hh];
                }
            }
        }
        const float d = f16_to_f32((uint16_t)(h.x & 0xFFFF)), dmin = f16_to_f32((uint16_t)(h.x >> 16));
#pragma unroll
        for (int t = 0; t < MT_NT; t++)
            if (t < nt) {
                const float xd = reinterpret_cast<const float *>(xt + (size_t)t * tb + q_bytes + s_bytes)[b];
                tsm[t][u] = fmul(xd, fsub(fmul(d, (float)I[t]), fmul(dmin, (float)M[t])));
            }
    }
    __syncwarp();
    if (lane < nS)
        for (int t = 0; t < nt; t++) {
            float a = 0.0f;
#pragma unroll 1
            for (int b = 0; b < NB; b++) a = fadd(b == 0 ? 0.0f : a, tsm[t][lane * NB + b]);  // from +0, block order
            out[(size_t)(t0 + t) * rows + r0 + lane] = a;
        }
    __syncwarp();
}

// Q6_K likewise (QT<T_Q6_K>::part's arithmetic): each lane's (row, block) fragment -- 6-bit
// quants rebuilt from the low and high planes, four int8 sub-block scales -- unpacked once for
// every token of the tile; per token I = sum sc (q . x - 32 sum x), exact.
__device__ __noinline__ void q6k_rows_multi(const AbStage &st, int r0, int nS, int NB, const uint8_t *xt, size_t tb,
                                            size_t q_bytes, size_t s_bytes, int nt, float (*tsm)[32], int lane,
                                            float *out, int rows, int t0) {
    const int u = lane;
    if (u < nS * NB) {
        const int s2 = u / NB, b = u - s2 * NB, gb = (r0 + s2) * NB + b;
        int I[MT_NT];
#pragma unroll
        for (int t = 0; t < MT_NT; t++) I[t] = 0;
        const uint4 sv = *reinterpret_cast<const uint4 *>(st.sc + (size_t)gb * 16);
#pragma unroll 1
        for (int sub = 0; sub < 4; sub++) {
            const int n = sub >> 1, hh = sub & 1;
            const uint8_t *qb = st.q + (size_t)gb * 192;
            const uint4 a4 = *reinterpret_cast<const uint4 *>(qb + 64 * n + 16 * hh);
            const uint4 b4 = *reinterpret_cast<const uint4 *>(qb + 64 * n + 32 + 16 * hh);
            const uint4 h4 = *reinterpret_cast<const uint4 *>(qb + 128 + 32 * n + 16 * hh);
            const uint32_t A[4] = {a4.x, a4.y, a4.z, a4.w}, Bq[4] = {b4.x, b4.y, b4.z, b4.w}, H[4] = {h4.x, h4.y, h4.z, h4.w};
            int w0[4], w1[4], w2[4], w3[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                w0[k] = (int)((A[k] & 0x0F0F0F0Fu) | ((H[k] & 0x03030303u) << 4));
                w1[k] = (int)((Bq[k] & 0x0F0F0F0Fu) | (((H[k] >> 2) & 0x03030303u) << 4));
                w2[k] = (int)(((A[k] >> 4) & 0x0F0F0F0Fu) | (((H[k] >> 4) & 0x03030303u) << 4));
                w3[k] = (int)(((Bq[k] >> 4) & 0x0F0F0F0Fu) | (((H[k] >> 6) & 0x03030303u) << 4));
            }
            const uint32_t sw0 = n ? sv.z : sv.x, sw1 = n ? sv.w : sv.y;
            const int c0 = (int)(int8_t)(sw0 >> (8 * hh)), c1 = (int)(int8_t)(sw0 >> (8 * (hh + 2)));
            const int c2 = (int)(int8_t)(sw1 >> (8 * hh)), c3 = (int)(int8_t)(sw1 >> (8 * (hh + 2)));
#pragma unroll
            for (int t = 0; t < MT_NT; t++) {
                if (t < nt) {
                    const uint8_t *xbt = xt + (size_t)t * tb;
                    const int8_t *xb = reinterpret_cast<const int8_t *>(xbt) + (size_t)b * 272 + 128 * n + 16 * hh;
                    const int4 x0 = *reinterpret_cast<const int4 *>(xb), x1 = *reinterpret_cast<const int4 *>(xb + 32);
                    const int4 x2 = *reinterpret_cast<const int4 *>(xb + 64), x3 = *reinterpret_cast<const int4 *>(xb + 96);
                    int d0 = dp4a(w0[0], x0.x, 0), d1 = dp4a(w1[0], x1.x, 0), d2 = dp4a(w2[0], x2.x, 0),
                        d3 = dp4a(w3[0], x3.x, 0);
                    d0 = dp4a(w0[1], x0.y, d0); d1 = dp4a(w1[1], x1.y, d1); d2 = dp4a(w2[1], x2.y, d2); d3 = dp4a(w3[1], x3.y, d3);
                    d0 = dp4a(w0[2], x0.z, d0); d1 = dp4a(w1[2], x1.z, d1); d2 = dp4a(w2[2], x2.z, d2); d3 = dp4a(w3[2], x3.z, d3);
                    d0 = dp4a(w0[3], x0.w, d0); d1 = dp4a(w1[3], x1.w, d1); d2 = dp4a(w2[3], x2.w, d2); d3 = dp4a(w3[3], x3.w, d3);
                    const int32_t *bs = reinterpret_cast<const int32_t *>(xbt + q_bytes) + b * 20 + 8 * n + hh;
                    I[t] += c0 * (d0 - 32 * bs[0]) + c1 * (d1 - 32 * bs[2]) + c2 * (d2 - 32 * bs[4]) + c3 * (d3 - 32 * bs[6]);
                }
            }
        }
        const float d = f16_to_f32(st.d[gb]);
#pragma unroll
        for (int t = 0; t < MT_NT; t++)
            if (t < nt) {
                const float xd = reinterpret_cast<const float *>(xt + (size_t)t * tb + q_bytes + s_bytes)[b];
                tsm[t][u] = fmul(fmul(xd, d), (float)I[t]);
            }
    }
    __syncwarp();
    if (lane < nS)
        for (int t = 0; t < nt; t++) {
            float a = 0.0f;
#pragma unroll 1
            for (int b = 0; b < NB; b++) a = fadd(b == 0 ? 0.0f : a, tsm[t][lane * NB + b]);  // from +0, block order
            out[(size_t)(t0 + t) * rows + r0 + lane] = a;
        }
    __syncwarp();
}

template <int TY>
__global__ void __launch_bounds__(MT_THREADS, 2) k_mm_tiled(WDev w, int rows, int nb, XQ x, int ntok, float *out,
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
    const int nS = max(1, min(4, 32 / nb)), nch = (nr + nS - 1) / nS;
    const AbStage st{sq, TY == T_Q6_K ? ssc : nullptr, TY == T_Q4_K ? nullptr : sd, 0, nr, nb};
    if ((TY == T_Q4_K || TY == T_Q6_K) && NT <= MT_NT) {  // fragments unpacked once for every token of the tile
        __shared__ float tsm_nt[MT_WARPS][MT_NT][32];
        for (int c = warp; c < nch; c += MT_WARPS) {
            const int rc = c * nS;
            if (TY == T_Q4_K)
                q4k_rows_multi(sq, rc, min(nS, nr - rc), nb, xt, tb, q_bytes, s_bytes, nt, tsm_nt[warp], lane, out + r0,
                               rows, t0);
            else
                q6k_rows_multi(st, rc, min(nS, nr - rc), nb, xt, tb, q_bytes, s_bytes, nt, tsm_nt[warp], lane, out + r0,
                               rows, t0);
        }
        return;
    }
    // units: (token, chunk of rows) with at most 32 (row, block) lanes
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
    const MtPlan p = mt_plan(ty, nb, rows, ntok);
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
