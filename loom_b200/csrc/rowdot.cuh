// rowdot.cuh -- one warp computes the dot of one weight row against NT
// int8-quantized activation vectors, for each block type.
//
// Numerics restate the reference's int8-activation kernels exactly
// (ch4r10t33r/loom src/gguf/ggml.zig):
//   Q4_K  kDecode :882 + kBlockDot :1002   term = xd*(d*I - dmin*M)
//   Q6_K  kDecode :882 + kBlockDot :1002   term = (xd*d)*I
//   Q4_0  matvecQ40Int :1196               term = (d*xd)*(dot - 8*sum)
//   Q8_0  matvecQ80Int :1277               term = (d*xd)*dot
//   F32   dotF32 :198 (4x8 accumulators, ordered reduce, scalar tail)
// The integer partial sums are exact whatever the lane split; each block's
// float term is formed with one IEEE rounding per operation, and the row
// accumulator adds the terms in block order, so the result is bit-identical
// to the CPU reference.
//
// Lane split per block: Q4_K 8 lanes x 16 B, Q6_K 4 lanes x 48 B, Q8_0 2 lanes
// x 16 B, Q4_0 1 lane x 16 B: every weight load is a 16-byte aligned
// ld.global.nc that the warp issues fully coalesced.
#pragma once
#include "common.cuh"

namespace loom {

__device__ __forceinline__ int nib_lo(uint32_t w) { return (int)(w & 0x0F0F0F0Fu); }
__device__ __forceinline__ int nib_hi(uint32_t w) { return (int)((w >> 4) & 0x0F0F0F0Fu); }

// ---- Q4_K -------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void rowdot_q4k(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                           float (&acc)[NT], int lane) {
    const int sub = lane & 7, grp = lane >> 3;
    const int j = sub >> 1, h = sub & 1;  // 32-byte chunk j holds sub-blocks 2j (low) and 2j+1 (high)
    for (int b0 = 0; b0 < nb; b0 += 4) {
        const int b = b0 + grp;
        const bool live = b < nb;
        uint4 hdr = make_uint4(0, 0, 0, 0), qv = make_uint4(0, 0, 0, 0);
        if (live) {
            const uint8_t *blk = w.q + (gb0 + b) * 144;
            hdr = ld_stream_v4(blk);
            qv = ld_stream_v4(blk + 16 + 16 * sub);
        }
        uint8_t s[12];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            s[i] = (hdr.y >> (8 * i)) & 0xFF;
            s[4 + i] = (hdr.z >> (8 * i)) & 0xFF;
            s[8 + i] = (hdr.w >> (8 * i)) & 0xFF;
        }
        int sc0, mn0, sc1, mn1;
        scale_min_k4(2 * j, s, sc0, mn0);
        scale_min_k4(2 * j + 1, s, sc1, mn1);
        const float d = f16_to_f32((uint16_t)(hdr.x & 0xFFFF));
        const float dmin = f16_to_f32((uint16_t)(hdr.x >> 16));
#pragma unroll
        for (int k = 0; k < NT; k++) {
            int I = 0, M = 0;
            if (live && k < nt) {
                const int t = t0 + k;
                const int8_t *xb = x.q + (size_t)t * x.cols + b * 256;
                const int4 xl = ld_i4(xb + 64 * j + 16 * h);
                const int4 xh = ld_i4(xb + 64 * j + 32 + 16 * h);
                int dl = 0, dh = 0;
                dl = dp4a(nib_lo(qv.x), xl.x, dl);
                dl = dp4a(nib_lo(qv.y), xl.y, dl);
                dl = dp4a(nib_lo(qv.z), xl.z, dl);
                dl = dp4a(nib_lo(qv.w), xl.w, dl);
                dh = dp4a(nib_hi(qv.x), xh.x, dh);
                dh = dp4a(nib_hi(qv.y), xh.y, dh);
                dh = dp4a(nib_hi(qv.z), xh.z, dh);
                dh = dp4a(nib_hi(qv.w), xh.w, dh);
                const int32_t *bs = x.s + (size_t)t * x.sstride + b * 16;
                I = sc0 * dl + sc1 * dh;
                M = mn0 * __ldg(bs + 4 * j + h) + mn1 * __ldg(bs + 4 * j + 2 + h);
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                I += __shfl_xor_sync(0xffffffffu, I, o);
                M += __shfl_xor_sync(0xffffffffu, M, o);
            }
            float term = 0.0f;
            if (live && k < nt) {
                const float xd = __ldg(x.d + (size_t)(t0 + k) * x.dstride + b);
                term = fmul(xd, fsub(fmul(d, (float)I), fmul(dmin, (float)M)));
            }
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const float tg = __shfl_sync(0xffffffffu, term, 8 * g);
                if (b0 + g < nb) acc[k] = fadd(acc[k], tg);
            }
        }
    }
}

// ---- Q6_K -------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void rowdot_q6k(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                           float (&acc)[NT], int lane) {
    const int sub = lane & 3, grp = lane >> 2;
    const int n = sub >> 1, h = sub & 1;  // 128-value half n, 16-byte column h
    for (int b0 = 0; b0 < nb; b0 += 8) {
        const int b = b0 + grp;
        const bool live = b < nb;
        uint4 A = make_uint4(0, 0, 0, 0), B = A, H = A, S = A;
        float d = 0.0f;
        if (live) {
            const uint64_t gb = gb0 + b;
            const uint8_t *qb = w.q + gb * 192;
            A = ld_stream_v4(qb + 64 * n + 16 * h);
            B = ld_stream_v4(qb + 64 * n + 32 + 16 * h);
            H = ld_stream_v4(qb + 128 + 32 * n + 16 * h);
            S = ld_stream_v4(w.sc + gb * 16);
            d = f16_to_f32(__ldg(w.d + gb));
        }
        const uint32_t a4[4] = {A.x, A.y, A.z, A.w}, b4[4] = {B.x, B.y, B.z, B.w}, h4[4] = {H.x, H.y, H.z, H.w};
        const uint32_t s4[4] = {S.x, S.y, S.z, S.w};
        int sc[4];
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const int idx = 8 * n + 2 * g + h;
            sc[g] = (int)(int8_t)((s4[idx >> 2] >> (8 * (idx & 3))) & 0xFF);
        }
#pragma unroll
        for (int k = 0; k < NT; k++) {
            int I = 0;
            if (live && k < nt) {
                const int t = t0 + k;
                const int8_t *xb = x.q + (size_t)t * x.cols + b * 256 + 128 * n + 16 * h;
                const int4 x0 = ld_i4(xb), x1 = ld_i4(xb + 32), x2 = ld_i4(xb + 64), x3 = ld_i4(xb + 96);
                const int x0a[4] = {x0.x, x0.y, x0.z, x0.w}, x1a[4] = {x1.x, x1.y, x1.z, x1.w};
                const int x2a[4] = {x2.x, x2.y, x2.z, x2.w}, x3a[4] = {x3.x, x3.y, x3.z, x3.w};
                int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
                for (int wd = 0; wd < 4; wd++) {
                    const uint32_t a = a4[wd], bb = b4[wd], hh = h4[wd];
                    const int q0 = (int)((a & 0x0F0F0F0Fu) | ((hh & 0x03030303u) << 4));
                    const int q1 = (int)((bb & 0x0F0F0F0Fu) | (((hh >> 2) & 0x03030303u) << 4));
                    const int q2 = (int)(((a >> 4) & 0x0F0F0F0Fu) | (((hh >> 4) & 0x03030303u) << 4));
                    const int q3 = (int)(((bb >> 4) & 0x0F0F0F0Fu) | (((hh >> 6) & 0x03030303u) << 4));
                    d0 = dp4a(q0, x0a[wd], d0);
                    d1 = dp4a(q1, x1a[wd], d1);
                    d2 = dp4a(q2, x2a[wd], d2);
                    d3 = dp4a(q3, x3a[wd], d3);
                }
                // (q - 32) . x = q . x - 32 * sum(x); the per-16 sums come from the quantizer
                const int32_t *bs = x.s + (size_t)t * x.sstride + b * 16 + 8 * n + h;
                I = sc[0] * (d0 - 32 * __ldg(bs + 0)) + sc[1] * (d1 - 32 * __ldg(bs + 2)) +
                    sc[2] * (d2 - 32 * __ldg(bs + 4)) + sc[3] * (d3 - 32 * __ldg(bs + 6));
            }
            I += __shfl_xor_sync(0xffffffffu, I, 1);
            I += __shfl_xor_sync(0xffffffffu, I, 2);
            float term = 0.0f;
            if (live && k < nt) {
                const float xd = __ldg(x.d + (size_t)(t0 + k) * x.dstride + b);
                term = fmul(fmul(xd, d), (float)I);
            }
#pragma unroll
            for (int g = 0; g < 8; g++) {
                const float tg = __shfl_sync(0xffffffffu, term, 4 * g);
                if (b0 + g < nb) acc[k] = fadd(acc[k], tg);
            }
        }
    }
}

// ---- Q8_0 -------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void rowdot_q80(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                           float (&acc)[NT], int lane) {
    const int sub = lane & 1, grp = lane >> 1;
    for (int b0 = 0; b0 < nb; b0 += 16) {
        const int b = b0 + grp;
        const bool live = b < nb;
        uint4 qv = make_uint4(0, 0, 0, 0);
        float d = 0.0f;
        if (live) {
            const uint64_t gb = gb0 + b;
            qv = ld_stream_v4(w.q + gb * 32 + 16 * sub);
            d = f16_to_f32(__ldg(w.d + gb));
        }
#pragma unroll
        for (int k = 0; k < NT; k++) {
            int dot = 0;
            if (live && k < nt) {
                const int4 xv = ld_i4(x.q + (size_t)(t0 + k) * x.cols + b * 32 + 16 * sub);
                dot = dp4a((int)qv.x, xv.x, dot);
                dot = dp4a((int)qv.y, xv.y, dot);
                dot = dp4a((int)qv.z, xv.z, dot);
                dot = dp4a((int)qv.w, xv.w, dot);
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            float term = 0.0f;
            if (live && k < nt) term = fmul(fmul(d, __ldg(x.d + (size_t)(t0 + k) * x.dstride + b)), (float)dot);
#pragma unroll
            for (int g = 0; g < 16; g++) {
                const float tg = __shfl_sync(0xffffffffu, term, 2 * g);
                if (b0 + g < nb) acc[k] = fadd(acc[k], tg);
            }
        }
    }
}

// ---- Q4_0 -------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void rowdot_q40(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                           float (&acc)[NT], int lane) {
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        const bool live = b < nb;
        uint4 qv = make_uint4(0, 0, 0, 0);
        float d = 0.0f;
        if (live) {
            const uint64_t gb = gb0 + b;
            qv = ld_stream_v4(w.q + gb * 16);
            d = f16_to_f32(__ldg(w.d + gb));
        }
#pragma unroll
        for (int k = 0; k < NT; k++) {
            float term = 0.0f;
            if (live && k < nt) {
                const int t = t0 + k;
                const int8_t *xb = x.q + (size_t)t * x.cols + b * 32;
                const int4 xl = ld_i4(xb), xh = ld_i4(xb + 16);
                int dot = 0;
                dot = dp4a(nib_lo(qv.x), xl.x, dot);
                dot = dp4a(nib_lo(qv.y), xl.y, dot);
                dot = dp4a(nib_lo(qv.z), xl.z, dot);
                dot = dp4a(nib_lo(qv.w), xl.w, dot);
                dot = dp4a(nib_hi(qv.x), xh.x, dot);
                dot = dp4a(nib_hi(qv.y), xh.y, dot);
                dot = dp4a(nib_hi(qv.z), xh.z, dot);
                dot = dp4a(nib_hi(qv.w), xh.w, dot);
                const int sum = __ldg(x.s + (size_t)t * x.sstride + b);
                term = fmul(fmul(d, __ldg(x.d + (size_t)t * x.dstride + b)), (float)(dot - 8 * sum));
            }
            const int lim = min(32, nb - b0);
            for (int g = 0; g < lim; g++) acc[k] = fadd(acc[k], __shfl_sync(0xffffffffu, term, g));
        }
    }
}

// ---- Q4_1 / Q5_1 (matvecQ41Int :1242): one lane per block ------------------------------
// dot over the unsigned (5-bit) quants, the min folded out as m * sum(xq):
// term = xd * (d*dot + m*sum). Q5_1's fifth bits: value i < 16 takes bit i of
// qh, value 16 + i bit 16 + i; spread4 moves four bits to bit 4 of four bytes.
__device__ __forceinline__ uint32_t spread4(uint32_t b) {
    return ((b & 1u) << 4) | ((b & 2u) << 11) | ((b & 4u) << 18) | ((b & 8u) << 25);
}

template <int TY, int NT>
__device__ __forceinline__ void rowdot_q41(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                           float (&acc)[NT], int lane) {
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        const bool live = b < nb;
        uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
        float d = 0.0f, m = 0.0f;
        if (live) {
            const uint64_t gb = gb0 + b;
            const uint4 qv = ld_stream_v4(w.q + gb * 16);
            const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
            uint32_t qh = 0;
            if (TY == T_Q5_1) qh = __ldg(reinterpret_cast<const uint32_t *>(w.sc) + gb);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                lo[k] = (qw[k] & 0x0F0F0F0Fu) | (TY == T_Q5_1 ? spread4((qh >> (4 * k)) & 0xF) : 0u);
                hi[k] = ((qw[k] >> 4) & 0x0F0F0F0Fu) | (TY == T_Q5_1 ? spread4((qh >> (16 + 4 * k)) & 0xF) : 0u);
            }
            d = f16_to_f32(__ldg(w.d + 2 * gb));
            m = f16_to_f32(__ldg(w.d + 2 * gb + 1));
        }
#pragma unroll
        for (int k = 0; k < NT; k++) {
            float term = 0.0f;
            if (live && k < nt) {
                const int t = t0 + k;
                const int8_t *xb = x.q + (size_t)t * x.cols + b * 32;
                const int4 xl = ld_i4(xb), xh = ld_i4(xb + 16);
                int dot = 0;
                dot = dp4a((int)lo[0], xl.x, dot);
                dot = dp4a((int)lo[1], xl.y, dot);
                dot = dp4a((int)lo[2], xl.z, dot);
                dot = dp4a((int)lo[3], xl.w, dot);
                dot = dp4a((int)hi[0], xh.x, dot);
                dot = dp4a((int)hi[1], xh.y, dot);
                dot = dp4a((int)hi[2], xh.z, dot);
                dot = dp4a((int)hi[3], xh.w, dot);
                const int sum = __ldg(x.s + (size_t)t * x.sstride + b);
                const float xd = __ldg(x.d + (size_t)t * x.dstride + b);
                term = fmul(xd, fadd(fmul(d, (float)dot), fmul(m, (float)sum)));
            }
            const int lim = min(32, nb - b0);
            for (int g = 0; g < lim; g++) acc[k] = fadd(acc[k], __shfl_sync(0xffffffffu, term, g));
        }
    }
}

// ---- F32 (dotF32 order) ------------------------------------------------------------
// Lane j is accumulator lane j of dotF32's four 8-wide vectors (acc(j/8)[j%8]).
__device__ __forceinline__ float rowdot_f32(const float *__restrict__ row, const float *__restrict__ xv, int n,
                                            int lane) {
    float a = 0.0f;
    int i = 0;
#pragma unroll 8
    for (; i + 32 <= n; i += 32) a = fadd(a, fmul(__ldg(row + i + lane), __ldg(xv + i + lane)));
    for (; i + 8 <= n; i += 8)
        if (lane < 8) a = fadd(a, fmul(__ldg(row + i + lane), __ldg(xv + i + lane)));
    const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
    const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
    const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
    const float v = fadd(fadd(fadd(a, a8), a16), a24);  // meaningful in lanes 0..7
    float r = __shfl_sync(0xffffffffu, v, 0);
#pragma unroll
    for (int jj = 1; jj < 8; jj++) r = fadd(r, __shfl_sync(0xffffffffu, v, jj));
    for (; i < n; i++) r = fadd(r, fmul(__ldg(row + i), __ldg(xv + i)));
    return r;
}

// ---- Q2_K / Q3_K / Q5_K: the uniform K-quant decode (ggml.zig kDecode :882) --------
// Eight lanes per super-block, lane g holding weight group g (values 32g ..
// 32g+31, per-16 sub-blocks 2g and 2g+1), four super-blocks per pass:
//   Q5_K  nibble of qs[32 (g/2) + l] (low for even g) | bit g of qh[l] << 4
//   Q2_K  (qs[32 (g/4) + l] >> 2 (g%4)) & 3, per-16 scale / min nibbles
//   Q3_K  ((qs[32 (g/4) + l] >> 2 (g%4)) & 3) | bit g of hmask[l] << 2, minus 4
//         (as sum u x - 4 bsum, an integer identity), per-16 scales q3kScales - 32
// then kBlockDot :1002: I = sum_j sc_j (w.x)_j, M = sum_j mn_j bsum_j,
// term = xd*(d*I - dmin*M) (Q2_K, Q5_K) or (xd*d)*I (Q3_K), blocks in order.
template <int TY, int NT>
__device__ __forceinline__ void rowdot_kq(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                          float (&acc)[NT], int lane) {
    const int g = lane & 7, grp = lane >> 3;
    for (int b0 = 0; b0 < nb; b0 += 4) {
        const int b = b0 + grp;
        const bool live = b < nb;
        uint32_t wv[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // the group's 32 weights as int8 (Q3_K: u = q + 4)
        int sc0 = 0, sc1 = 0, mn0 = 0, mn1 = 0;
        float d = 0.0f, dmin = 0.0f;
        if (live) {
            const uint64_t gb = gb0 + b;
            if (TY == T_Q5_K) {
                const uint8_t *blk = w.q + gb * 176;
                const uint4 hdr = ld_stream_v4(blk);
                const uint4 h0 = ld_stream_v4(blk + 16), h1 = ld_stream_v4(blk + 32);
                const uint4 q0 = ld_stream_v4(blk + 48 + 32 * (g >> 1)), q1 = ld_stream_v4(blk + 64 + 32 * (g >> 1));
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
                for (int k = 0; k < 8; k++)
                    wv[k] = ((g & 1) ? (qw[k] >> 4) & 0x0F0F0F0Fu : qw[k] & 0x0F0F0F0Fu) | (((hw[k] >> g) & 0x01010101u) << 4);
                uint8_t s[12];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    s[i] = (hdr.y >> (8 * i)) & 0xFF;
                    s[4 + i] = (hdr.z >> (8 * i)) & 0xFF;
                    s[8 + i] = (hdr.w >> (8 * i)) & 0xFF;
                }
                scale_min_k4(g, s, sc0, mn0);
                sc1 = sc0;
                mn1 = mn0;
                d = f16_to_f32((uint16_t)(hdr.x & 0xFFFF));
                dmin = f16_to_f32((uint16_t)(hdr.x >> 16));
            } else if (TY == T_Q2_K) {
                const uint8_t *qb = w.q + gb * 80;
                const uint4 sv = ld_stream_v4(qb);
                const uint4 q0 = ld_stream_v4(qb + 16 + 32 * (g >> 2)), q1 = ld_stream_v4(qb + 32 + 32 * (g >> 2));
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int k = 0; k < 8; k++) wv[k] = (qw[k] >> (2 * (g & 3))) & 0x03030303u;
                const uint32_t s4[4] = {sv.x, sv.y, sv.z, sv.w};
                const uint32_t sb0 = (s4[g >> 1] >> (16 * (g & 1))) & 0xFF, sb1 = (s4[g >> 1] >> (16 * (g & 1) + 8)) & 0xFF;
                sc0 = (int)(sb0 & 0xF);
                mn0 = (int)(sb0 >> 4);
                sc1 = (int)(sb1 & 0xF);
                mn1 = (int)(sb1 >> 4);
                d = f16_to_f32(__ldg(w.d + 2 * gb));
                dmin = f16_to_f32(__ldg(w.d + 2 * gb + 1));
            } else {  // T_Q3_K
                const uint8_t *qb = w.q + gb * 96;
                const uint4 h0 = ld_stream_v4(qb), h1 = ld_stream_v4(qb + 16);
                const uint4 q0 = ld_stream_v4(qb + 32 + 32 * (g >> 2)), q1 = ld_stream_v4(qb + 48 + 32 * (g >> 2));
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
                for (int k = 0; k < 8; k++)
                    wv[k] = ((qw[k] >> (2 * (g & 3))) & 0x03030303u) | (((hw[k] >> g) & 0x01010101u) << 2);
                const uint4 sv = ld_stream_v4(w.sc + gb * 16);
                uint8_t p[12];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    p[i] = (sv.x >> (8 * i)) & 0xFF;
                    p[4 + i] = (sv.y >> (8 * i)) & 0xFF;
                    p[8 + i] = (sv.z >> (8 * i)) & 0xFF;
                }
                sc0 = q3k_scale(p, 2 * g) - 32;
                sc1 = q3k_scale(p, 2 * g + 1) - 32;
                d = f16_to_f32(__ldg(w.d + gb));
            }
        }
#pragma unroll
        for (int k = 0; k < NT; k++) {
            int I = 0, M = 0;
            if (live && k < nt) {
                const int t = t0 + k;
                const int8_t *xb = x.q + (size_t)t * x.cols + b * 256 + 32 * g;
                const int4 xl = ld_i4(xb), xh = ld_i4(xb + 16);
                int dl = 0, dh = 0;
                dl = dp4a((int)wv[0], xl.x, dl);
                dl = dp4a((int)wv[1], xl.y, dl);
                dl = dp4a((int)wv[2], xl.z, dl);
                dl = dp4a((int)wv[3], xl.w, dl);
                dh = dp4a((int)wv[4], xh.x, dh);
                dh = dp4a((int)wv[5], xh.y, dh);
                dh = dp4a((int)wv[6], xh.z, dh);
                dh = dp4a((int)wv[7], xh.w, dh);
                const int32_t *bs = x.s + (size_t)t * x.sstride + b * 16 + 2 * g;
                if (TY == T_Q3_K) {
                    dl -= 4 * __ldg(bs);
                    dh -= 4 * __ldg(bs + 1);
                } else {
                    M = mn0 * __ldg(bs) + mn1 * __ldg(bs + 1);
                }
                I = sc0 * dl + sc1 * dh;
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                I += __shfl_xor_sync(0xffffffffu, I, o);
                if (TY != T_Q3_K) M += __shfl_xor_sync(0xffffffffu, M, o);
            }
            float term = 0.0f;
            if (live && k < nt) {
                const float xd = __ldg(x.d + (size_t)(t0 + k) * x.dstride + b);
                term = TY == T_Q3_K ? fmul(fmul(xd, d), (float)I) : fmul(xd, fsub(fmul(d, (float)I), fmul(dmin, (float)M)));
            }
#pragma unroll
            for (int gg = 0; gg < 4; gg++) {
                const float tg = __shfl_sync(0xffffffffu, term, 8 * gg);
                if (b0 + gg < nb) acc[k] = fadd(acc[k], tg);
            }
        }
    }
}

// Dispatch on the (warp-uniform) block type. acc must start at 0.
template <int NT>
__device__ __forceinline__ void rowdot(const WDev &w, uint64_t gb0, int nb, const XQ &x, int t0, int nt,
                                       float (&acc)[NT], int lane) {
    switch (w.type) {
        case T_Q4_K: rowdot_q4k<NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q6_K: rowdot_q6k<NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q8_0: rowdot_q80<NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q4_0: rowdot_q40<NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q5_K: rowdot_kq<T_Q5_K, NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q4_1: rowdot_q41<T_Q4_1, NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q5_1: rowdot_q41<T_Q5_1, NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q2_K: rowdot_kq<T_Q2_K, NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        case T_Q3_K: rowdot_kq<T_Q3_K, NT>(w, gb0, nb, x, t0, nt, acc, lane); break;
        default: break;
    }
}

}  // namespace loom
