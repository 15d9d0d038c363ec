// step_dev.cuh -- device helpers shared by the cooperative model-step kernels
// (attn_block.cu, model_kernel.cu): the bounded grid barrier, bulk staging of
// row slices into shared memory, compact row dots on staged rows (the warp
// engine's arithmetic), RMSNorm and activation quantization by a whole CTA.
// Internal linkage: each including file gets its own copy.
#pragma once
#include "attn.cuh"
#include "devutil.cuh"
#include "tma.cuh"
#include "warpdot.cuh"

namespace loom {
namespace {

constexpr int AB_WARPS = 12, AB_THREADS = AB_WARPS * 32;  // 12 warps: up to 168 registers a thread
constexpr int AB_GRP_WARPS = 4;                       // warps of an attention group
constexpr int AB_NBAR = 4;                            // grid barriers per launch (with the FFN norm)
constexpr uint32_t AB_POLLS = 1u << 21;               // bounded grid-barrier wait (~1 s)

__device__ __forceinline__ unsigned long long ab_ld_acquire(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ab_red_release(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ float ab_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// bar[0]: u64 arrival counter; bar[1]: (u32 epoch, u32 exit count); bar[2]: u32 error word.
// Each CTA adds one arrival (release) and polls until the counter reaches the
// barrier's target (acquire); ~1.2 us for 148 CTAs on B200 (measured; a
// variant with a separate release flag written by the last arriver was slower).
__device__ __forceinline__ bool ab_barrier(unsigned long long *ctr, unsigned long long target, unsigned *err) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        ab_red_release(ctr, 1ull);
        uint32_t i = 0;
        for (; i < AB_POLLS; i++) {
            if (ab_ld_acquire(ctr) >= target) break;
            if ((i & 1023) == 1023 && *reinterpret_cast<volatile unsigned *>(err)) i = AB_POLLS;
        }
        if (i >= AB_POLLS) atomicOr(err, 1u);
        s_ok = i < AB_POLLS;
    }
    __syncthreads();
    return s_ok != 0;
}

__device__ __forceinline__ void ab_cp16(void *smem, const void *gmem) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

// L2 prefetch of bytes [0, n) at p, 128-byte lines, spread over the grid's threads
__device__ __forceinline__ void ab_prefetch(const void *p, size_t n, size_t gt, size_t nt) {
    const uint8_t *b = static_cast<const uint8_t *>(p);
    for (size_t off = gt * 128; off < n; off += nt * 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(b + off));
}
// every region of the first nblk blocks of a device tensor
__device__ __forceinline__ void ab_prefetch_w(const WDev &w, uint64_t nblk, size_t gt, size_t nt) {
    ab_prefetch(w.q, nblk * (size_t)layout_qbytes(w.type), gt, nt);
    if (w.sc) ab_prefetch(w.sc, nblk * 16, gt, nt);
    if (w.d) ab_prefetch(w.d, nblk * 2, gt, nt);
}

// rows [r0, r0 + S) of one matrix against one activation view
struct AbRows {
    WDev w;
    int r0, nb;
    XV x;
    __device__ __forceinline__ void at(int s, WDev &ww, uint64_t &gb, XV &xv) const {
        ww = w;
        gb = (uint64_t)(r0 + s) * nb;
        xv = x;
    }
};

__host__ __device__ constexpr size_t ab_al16(size_t n) { return (n + 15) & ~size_t(15); }
__host__ __device__ constexpr size_t ab_al128(size_t n) { return (n + 127) & ~size_t(127); }
constexpr uint32_t STAGE_POLLS_AB = 1u << 22;  // bounded wait on the staged rows

template <int TY> constexpr int ab_maxu() { return TY == T_Q4_K ? 8 : TY == T_Q6_K ? 4 : TY == T_Q8_0 ? 4 : 2; }

// RMSNorm of x (dim floats) by the whole CTA into sx (shared): the sum of
// squares serial (thread 0, the reference's order) or a tree; then
// out = x * scale * w. Returns after a __syncthreads with sx holding the result.
__device__ void ab_rmsnorm(const float *x, const float *w, int dim, float eps, bool serial, float *sx, float *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float ss = 0.0f;
    // the weights are requested with the row (one round trip for both), kept in registers
    constexpr int WE = 24;
    float wr[WE];
    const bool wreg = dim <= WE * AB_THREADS;
    if (wreg) {
#pragma unroll
        for (int k = 0; k < WE; k++) {
            const int i = tid + k * AB_THREADS;
            wr[k] = i < dim ? __ldg(w + i) : 0.0f;
        }
    }
    for (int i = tid; i < dim; i += AB_THREADS) {
        const float v = x[i];
        sx[i] = v;
        if (!serial) ss = fadd(ss, fmul(v, v));
    }
    __syncthreads();
    if (serial) {
        if (tid == 0) {
            float s = 0.0f;
            for (int i = 0; i < dim; i++) s = fadd(s, fmul(sx[i], sx[i]));
            red[0] = s;
        }
    } else {
        ss = ab_warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float t = 0.0f;
            for (int i = 0; i < AB_WARPS; i++) t = fadd(t, red[i]);
            red[0] = t;
        }
    }
    __syncthreads();
    const float scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(red[0], (float)dim), eps)));
    if (wreg) {
#pragma unroll
        for (int k = 0; k < WE; k++) {
            const int i = tid + k * AB_THREADS;
            if (i < dim) sx[i] = fmul(fmul(sx[i], scale), wr[k]);
        }
    } else {
        for (int i = tid; i < dim; i += AB_THREADS) sx[i] = fmul(fmul(sx[i], scale), w[i]);
    }
    __syncthreads();
}

// One head row in shared memory by one warp: optional headNorm with weight
// gamma (shared; llama.zig:938-950: inv = 1 / sqrt(ss / hd + eps), ss serial
// in the reference's order when `serial`, else a lane-strided tree), optional
// RoPE on the (cos, sin) pairs cs (shared; llama.zig:830-858; NEOX pairs j,
// j + half, else 2j, 2j + 1), and a copy to `cache` (global) when given.
__device__ __noinline__ void ab_head_smem(float *v, const float *gamma, bool rope, const float *cs, int half, int neox,
                                          int hd, float eps, int serial, float *cache, int lane) {
    if (gamma) {
        float ss = 0.0f;
        if (serial) {
            if (lane == 0)
                for (int i = 0; i < hd; i++) ss = fadd(ss, fmul(v[i], v[i]));
            ss = __shfl_sync(0xffffffffu, ss, 0);
        } else {
            for (int i = lane; i < hd; i += 32) ss = fadd(ss, fmul(v[i], v[i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss = fadd(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        }
        const float inv = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)hd), eps)));
        __syncwarp();
        for (int i = lane; i < hd; i += 32) v[i] = fmul(fmul(v[i], inv), gamma[i]);
        __syncwarp();
    }
    if (rope) {
        for (int j = lane; j < half; j += 32) {
            const int ia = neox ? j : 2 * j, ib = neox ? j + half : 2 * j + 1;
            const float a = v[ia], b = v[ib], co = cs[2 * j], si = cs[2 * j + 1];
            v[ia] = fsub(fmul(a, co), fmul(b, si));
            v[ib] = fadd(fmul(a, si), fmul(b, co));
        }
        __syncwarp();
    }
    if (cache)
        for (int i = lane; i < hd; i += 32) cache[i] = v[i];
}

// RMSNorm of the row already in sx (dim floats, shared), in place: the sum of
// squares serial (thread 0, the reference's order) or a tree (per thread, then
// warps in order); out = x * scale * w. Ends with a __syncthreads.
__device__ void ab_rmsnorm_sx(const float *w, int dim, float eps, bool serial, float *sx, float *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int WE = 24;
    float wr[WE];
    const bool wreg = dim <= WE * AB_THREADS;
    if (wreg) {
#pragma unroll
        for (int k = 0; k < WE; k++) {
            const int i = tid + k * AB_THREADS;
            wr[k] = i < dim ? __ldg(w + i) : 0.0f;
        }
    }
    float ss = 0.0f;
    if (serial) {
        if (tid == 0) {
            for (int i = 0; i < dim; i++) ss = fadd(ss, fmul(sx[i], sx[i]));
            red[0] = ss;
        }
    } else {
        for (int i = tid; i < dim; i += AB_THREADS) ss = fadd(ss, fmul(sx[i], sx[i]));
        ss = ab_warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float t = 0.0f;
            for (int i = 0; i < AB_WARPS; i++) t = fadd(t, red[i]);
            red[0] = t;
        }
    }
    __syncthreads();
    const float scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(red[0], (float)dim), eps)));
    if (wreg) {
#pragma unroll
        for (int k = 0; k < WE; k++) {
            const int i = tid + k * AB_THREADS;
            if (i < dim) sx[i] = fmul(fmul(sx[i], scale), wr[k]);
        }
    } else {
        for (int i = tid; i < dim; i += AB_THREADS) sx[i] = fmul(fmul(sx[i], scale), w[i]);
    }
    __syncthreads();
}

// quantize sx (n floats) per 256 (k256) or per 32 into q/d/s
__device__ void ab_quant(const float *sx, int n, bool k256, int8_t *q, float *d, int32_t *s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (k256) {
        for (int b = warp; b < n / 256; b += AB_WARPS) {
            const int off = b * 256 + lane * 8;
            quant_lane8(sx + off, true, 32, q + off, d + b, s + b * 16 + lane / 2, nullptr, lane);
        }
    } else {
        const int nb = n / 32, ng = (nb + 7) / 8;
        for (int g = warp; g < ng; g += AB_WARPS) {
            const int b = g * 8 + lane / 4;
            const bool live = b < nb;
            const int off = b * 32 + (lane & 3) * 8;
            quant_lane8(sx + (live ? off : 0), live, 4, q + off, d + b, nullptr, s + b, lane);
        }
    }
}

// Floats of one attention group's shared memory: K rows (padded stride hd + 4)
// and V rows of a chunk, the group's query heads, their scores, and the
// head-norm weights and (cos, sin) pairs of the head preparation.
__host__ __device__ constexpr size_t ab_att_per(int hd, int gq) {
    return (size_t)ATT_CH * (hd + 4) + (size_t)ATT_CH * hd + (size_t)gq * hd + (size_t)gq * ATT_CH + 3 * (size_t)hd;
}

// Padded activation layout (shared memory): a 256-value block's quants 272
// bytes apart and its 16 sums 20 words apart (80 bytes: bulk-copy rows); a 32-value block's quants 48
// bytes apart, one sum word each. ab_quant_pad writes it; ab_rows reads it
// with these strides.
__host__ __device__ constexpr int ab_pad_qs(bool k256) { return k256 ? 272 : 48; }
__host__ __device__ constexpr int ab_pad_ss(bool k256) { return k256 ? 20 : 1; }
__host__ __device__ constexpr size_t ab_pad_qbytes(size_t n) { return n / 32 * 48; }           // >= n / 256 * 272
__host__ __device__ constexpr size_t ab_pad_sbytes(size_t n) { return (n / 256 + 1) * 20 * 4 + n / 32 * 4; }
__device__ void ab_quant_pad(const float *sx, int n, bool k256, int8_t *q, float *d, int32_t *s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (k256) {
        for (int b = warp; b < n / 256; b += AB_WARPS)
            quant_lane8(sx + b * 256 + lane * 8, true, 32, q + b * 272 + lane * 8, d + b, s + b * 20 + lane / 2,
                        nullptr, lane);
    } else {
        const int nb = n / 32, ng = (nb + 7) / 8;
        for (int g = warp; g < ng; g += AB_WARPS) {
            const int b = g * 8 + lane / 4;
            const bool live = b < nb;
            const int off = (lane & 3) * 8;
            quant_lane8(sx + (live ? b * 32 + off : 0), live, 4, q + (live ? b : 0) * 48 + off, d + b, nullptr, s + b,
                        lane);
        }
    }
}

// A matrix's rows [ra, rb) staged in shared memory in the device layout's
// regions (quants / Q4_K blocks, Q6_K scales, f16 scales); block gb of the
// slice is global block ra * nb + gb.
struct AbStage {
    const uint8_t *q, *sc;
    const uint16_t *d;
    int ra, rb, nb;
};

__device__ __forceinline__ uint4 ab_ld16(const uint8_t *p) {
    return *reinterpret_cast<const uint4 *>(p);
}

// the fragment QT<TY>::load reads from global memory, read from a staged slice
template <int TY> __device__ __forceinline__ typename QT<TY>::Frag ab_frag(const AbStage &s, int gb, int sub);
template <> __device__ __forceinline__ QT<T_Q4_K>::Frag ab_frag<T_Q4_K>(const AbStage &s, int gb, int sub) {
    const uint8_t *blk = s.q + (size_t)gb * 144;
    return QT<T_Q4_K>::Frag{ab_ld16(blk), ab_ld16(blk + 16 + 16 * sub)};
}
template <> __device__ __forceinline__ QT<T_Q6_K>::Frag ab_frag<T_Q6_K>(const AbStage &s, int gb, int sub) {
    const int n = sub >> 1, hh = sub & 1;
    const uint8_t *qb = s.q + (size_t)gb * 192;
    QT<T_Q6_K>::Frag f;
    f.a = ab_ld16(qb + 64 * n + 16 * hh);
    f.b = ab_ld16(qb + 64 * n + 32 + 16 * hh);
    f.h = ab_ld16(qb + 128 + 32 * n + 16 * hh);
    f.s = ab_ld16(s.sc + (size_t)gb * 16);
    f.d = s.d[gb];
    return f;
}
template <> __device__ __forceinline__ QT<T_Q8_0>::Frag ab_frag<T_Q8_0>(const AbStage &s, int gb, int sub) {
    return QT<T_Q8_0>::Frag{ab_ld16(s.q + (size_t)gb * 32 + 16 * sub), (uint32_t)s.d[gb]};
}
template <> __device__ __forceinline__ QT<T_Q4_0>::Frag ab_frag<T_Q4_0>(const AbStage &s, int gb, int) {
    return QT<T_Q4_0>::Frag{ab_ld16(s.q + (size_t)gb * 16), (uint32_t)s.d[gb]};
}

// rows [r0, r0 + nS) of a staged slice (r0 local) against activations xv,
// one lane per unit (row, block): the lane walks the block's LPB fragments
// (QT<TY>::part, the warp engine's arithmetic; the integer sums I and M are
// the same integers the lane groups' shuffle trees form) and writes the
// block's float term into the warp's term buffer tsm (>= nS * nb floats);
// then lane s adds stream s's block terms in block order from +0 (kBlockDot /
// matvecK256, ggml.zig:1002-1042). Bit-identical to wd_load + wd_finish.
// One lane per unit needs no cross-lane reduction per block, so a warp
// issues about a quarter of the instructions of lane groups, with the
// fragments' shared-memory loads independent of each other.
// acc[s] for s < nS is valid in lane s.
// Activation blocks sit qs bytes (quants) and ss words (per-16 sums) apart:
// the packed layout (qs = BE, ss = SPB) or the padded shared-memory layout of
// ab_quant_pad, in which the lanes of one 8-lane phase, reading the same
// offset of eight consecutive blocks, hit eight different bank groups.
template <int TY>
__device__ __noinline__ float ab_rows(const AbStage &st, int r0, int nS, const XV &xv, float *tsm, int lane,
                                      int qs = QT<TY>::BE, int ss = QT<TY>::SPB) {
    using Q = QT<TY>;
    const int NB = st.nb, U = nS * NB;
    for (int u = lane; u < U; u += 32) {
        const int s2 = u / NB, b = u - s2 * NB, gb = (r0 + s2) * NB + b;
        int I = 0, M = 0;
        typename Q::Frag f{};
#pragma unroll 2
        for (int sub = 0; sub < Q::LPB; sub++) {
            f = ab_frag<TY>(st, gb, sub);
            int i = 0, m = 0;
            Q::part(f, sub, xv.q + b * qs, xv.s + b * ss, i, m);
            I += i;
            M += m;
        }
        tsm[u] = Q::term(f, I, M, xv.d[b]);
    }
    __syncwarp();
    float a = 0.0f;
    if (lane < nS) {
#pragma unroll 1
        for (int b = 0; b < NB; b++) a = fadd(b == 0 ? 0.0f : a, tsm[lane * NB + b]);  // from +0, block order
    }
    __syncwarp();
    return a;
}

// Issue the staging of rows [ra, rb) of w (nb blocks a row): the quant and
// Q6_K-scale regions by bulk copies on mbarrier bar (returns their bytes; the
// caller's expect_tx covers them), the f16 scales by this CTA's threads.
__device__ __forceinline__ uint32_t ab_stage_bulk(const WDev &w, int ra, int rb, int nb, uint8_t *dq, uint8_t *dsc,
                                                  uint64_t *bar) {
    const uint64_t gb0 = (uint64_t)ra * nb, n = (uint64_t)(rb - ra) * nb;
    const uint32_t qb = (uint32_t)layout_qbytes(w.type);
    uint32_t bytes = 0;
    if (n) {
        bulk_g2s(dq, w.q + gb0 * qb, (uint32_t)(n * qb), bar);
        bytes += (uint32_t)(n * qb);
        if (w.sc) {
            bulk_g2s(dsc, w.sc + gb0 * 16, (uint32_t)(n * 16), bar);
            bytes += (uint32_t)(n * 16);
        }
    }
    return bytes;
}
__device__ __forceinline__ void ab_stage_d(const WDev &w, int ra, int rb, int nb, uint16_t *dd) {
    if (!w.d) return;
    const uint64_t gb0 = (uint64_t)ra * nb, n = (uint64_t)(rb - ra) * nb;
    // read-only loads: free to run ahead of the shared-memory stores (no assumed aliasing)
    for (uint64_t i = threadIdx.x; i < n; i += AB_THREADS) dd[i] = __ldg(w.d + gb0 + i);
}

}  // namespace
}  // namespace loom
