// warpdot.cuh -- the warp-level dot engine of the decode kernels.
//
// One warp computes up to S "streams" (a stream = one weight row against one
// int8 activation vector) of NB blocks each. Work is cut into units
// (stream, block); a unit is served by LPB lanes (Q4_K 8, Q6_K 4, Q8_0 2,
// Q4_0 1), so a warp serves G = 32/LPB units per step. ALL weight loads of the
// warp are issued before any is consumed (the fragments live in registers),
// which is what keeps enough bytes in flight to stream HBM.
//
// Numerics are those of rowdot.cuh (ggml.zig kBlockDot :1002, matvecQ40Int
// :1196, matvecQ80Int :1277): exact integer partials, one IEEE rounding per
// float operation, and each stream's block terms added in block order, so the
// results are bit-identical to the CPU reference.
#pragma once
#include "common.cuh"

namespace loom {

// Activation view for one stream: block b's int8 values at q + b*BE, its scale
// at d[b], its sums at s + b*(BE == 256 ? 16 : 1). Plain (generic) loads: the
// view may point at shared or global memory.
struct XV {
    const int8_t *q;
    const float *d;
    const int32_t *s;
};

template <int TY> struct QT;

template <> struct QT<T_Q4_K> {
    static constexpr int LPB = 8, BE = 256, SPB = 16;
    struct Frag {
        uint4 h, q;
    };
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int sub) {
        const uint8_t *blk = w.q + gb * 144;
        return Frag{ld_stream_v4(blk), ld_stream_v4(blk + 16 + 16 * sub)};
    }
    __device__ __forceinline__ static void part(const Frag &f, int sub, const int8_t *xq, const int32_t *xs, int &I,
                                                int &M) {
        const int j = sub >> 1, h = sub & 1;
        const int4 xl = *reinterpret_cast<const int4 *>(xq + 64 * j + 16 * h);
        const int4 xh = *reinterpret_cast<const int4 *>(xq + 64 * j + 32 + 16 * h);
        int dl = 0, dh = 0;
        dl = dp4a((int)(f.q.x & 0x0F0F0F0Fu), xl.x, dl);
        dl = dp4a((int)(f.q.y & 0x0F0F0F0Fu), xl.y, dl);
        dl = dp4a((int)(f.q.z & 0x0F0F0F0Fu), xl.z, dl);
        dl = dp4a((int)(f.q.w & 0x0F0F0F0Fu), xl.w, dl);
        dh = dp4a((int)((f.q.x >> 4) & 0x0F0F0F0Fu), xh.x, dh);
        dh = dp4a((int)((f.q.y >> 4) & 0x0F0F0F0Fu), xh.y, dh);
        dh = dp4a((int)((f.q.z >> 4) & 0x0F0F0F0Fu), xh.z, dh);
        dh = dp4a((int)((f.q.w >> 4) & 0x0F0F0F0Fu), xh.w, dh);
        // scaleMinK4 (ggml.zig:1332) for sub-blocks 2j and 2j+1 from the 12
        // scale bytes held in h.y (bytes 0-3), h.z (4-7), h.w (8-11)
        int sc0, mn0, sc1, mn1;
        if (j < 2) {
            const uint32_t a = f.h.y >> (16 * j), b = f.h.z >> (16 * j);
            sc0 = a & 63;
            sc1 = (a >> 8) & 63;
            mn0 = b & 63;
            mn1 = (b >> 8) & 63;
        } else {
            const int jj = j - 2;                    // sub-blocks 4+2jj, 5+2jj
            const uint32_t lo = f.h.w >> (16 * jj);  // scales[8+2jj], scales[9+2jj]
            const uint32_t hs = f.h.y >> (16 * jj);  // scales[2jj], scales[2jj+1]  (top 2 bits -> sc)
            const uint32_t hm = f.h.z >> (16 * jj);  // scales[4+2jj], scales[5+2jj] (top 2 bits -> mn)
            sc0 = (lo & 0xF) | (((hs >> 6) & 3) << 4);
            mn0 = ((lo >> 4) & 0xF) | (((hm >> 6) & 3) << 4);
            sc1 = ((lo >> 8) & 0xF) | (((hs >> 14) & 3) << 4);
            mn1 = ((lo >> 12) & 0xF) | (((hm >> 14) & 3) << 4);
        }
        I = sc0 * dl + sc1 * dh;
        M = mn0 * xs[4 * j + h] + mn1 * xs[4 * j + 2 + h];
    }
    __device__ __forceinline__ static float term(const Frag &f, int I, int M, float xd) {
        const float d = f16_to_f32((uint16_t)(f.h.x & 0xFFFF));
        const float dmin = f16_to_f32((uint16_t)(f.h.x >> 16));
        return fmul(xd, fsub(fmul(d, (float)I), fmul(dmin, (float)M)));
    }
};

// Q4_K with 32 bytes of nibbles per lane (4 lanes per super-block): half the
// reduction and bookkeeping instructions per weight byte of the 8-lane form.
// Used where the unit mapping allows G = 8.
constexpr int T_Q4_KW = 112;

template <> struct QT<T_Q4_KW> {
    static constexpr int LPB = 4, BE = 256, SPB = 16;
    struct Frag {
        uint4 h, q0, q1;
    };
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int sub) {
        const uint8_t *blk = w.q + gb * 144;
        return Frag{ld_stream_v4(blk), ld_stream_v4(blk + 16 + 32 * sub), ld_stream_v4(blk + 32 + 32 * sub)};
    }
    __device__ __forceinline__ static void part(const Frag &f, int j, const int8_t *xq, const int32_t *xs, int &I,
                                                int &M) {
        const int4 *x4 = reinterpret_cast<const int4 *>(xq + 64 * j);
        const int4 l0 = x4[0], l1 = x4[1], h0 = x4[2], h1 = x4[3];
        int dl = 0, dh = 0;
        dl = dp4a((int)(f.q0.x & 0x0F0F0F0Fu), l0.x, dl);
        dl = dp4a((int)(f.q0.y & 0x0F0F0F0Fu), l0.y, dl);
        dl = dp4a((int)(f.q0.z & 0x0F0F0F0Fu), l0.z, dl);
        dl = dp4a((int)(f.q0.w & 0x0F0F0F0Fu), l0.w, dl);
        dl = dp4a((int)(f.q1.x & 0x0F0F0F0Fu), l1.x, dl);
        dl = dp4a((int)(f.q1.y & 0x0F0F0F0Fu), l1.y, dl);
        dl = dp4a((int)(f.q1.z & 0x0F0F0F0Fu), l1.z, dl);
        dl = dp4a((int)(f.q1.w & 0x0F0F0F0Fu), l1.w, dl);
        dh = dp4a((int)((f.q0.x >> 4) & 0x0F0F0F0Fu), h0.x, dh);
        dh = dp4a((int)((f.q0.y >> 4) & 0x0F0F0F0Fu), h0.y, dh);
        dh = dp4a((int)((f.q0.z >> 4) & 0x0F0F0F0Fu), h0.z, dh);
        dh = dp4a((int)((f.q0.w >> 4) & 0x0F0F0F0Fu), h0.w, dh);
        dh = dp4a((int)((f.q1.x >> 4) & 0x0F0F0F0Fu), h1.x, dh);
        dh = dp4a((int)((f.q1.y >> 4) & 0x0F0F0F0Fu), h1.y, dh);
        dh = dp4a((int)((f.q1.z >> 4) & 0x0F0F0F0Fu), h1.z, dh);
        dh = dp4a((int)((f.q1.w >> 4) & 0x0F0F0F0Fu), h1.w, dh);
        // scaleMinK4 (ggml.zig:1332) for sub-blocks 2j, 2j+1, without divergence
        const int sh = 16 * (j & 1);
        const uint32_t a = f.h.y >> sh, b = f.h.z >> sh, lo = f.h.w >> sh;
        const bool low = j < 2;
        const int sc0 = low ? (a & 63) : ((lo & 0xF) | (((a >> 6) & 3) << 4));
        const int mn0 = low ? (b & 63) : (((lo >> 4) & 0xF) | (((b >> 6) & 3) << 4));
        const int sc1 = low ? ((a >> 8) & 63) : (((lo >> 8) & 0xF) | (((a >> 14) & 3) << 4));
        const int mn1 = low ? ((b >> 8) & 63) : (((lo >> 12) & 0xF) | (((b >> 14) & 3) << 4));
        const int4 bs = *reinterpret_cast<const int4 *>(xs + 4 * j);
        I = sc0 * dl + sc1 * dh;
        M = mn0 * (bs.x + bs.y) + mn1 * (bs.z + bs.w);
    }
    __device__ __forceinline__ static float term(const Frag &f, int I, int M, float xd) {
        const float d = f16_to_f32((uint16_t)(f.h.x & 0xFFFF));
        const float dmin = f16_to_f32((uint16_t)(f.h.x >> 16));
        return fmul(xd, fsub(fmul(d, (float)I), fmul(dmin, (float)M)));
    }
};

template <> struct QT<T_Q6_K> {
    static constexpr int LPB = 4, BE = 256, SPB = 16;
    struct Frag {
        uint4 a, b, h, s;
        uint32_t d;
    };
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int sub) {
        const int n = sub >> 1, hh = sub & 1;
        const uint8_t *qb = w.q + gb * 192;
        Frag f;
        f.a = ld_stream_v4(qb + 64 * n + 16 * hh);
        f.b = ld_stream_v4(qb + 64 * n + 32 + 16 * hh);
        f.h = ld_stream_v4(qb + 128 + 32 * n + 16 * hh);
        f.s = ld_stream_v4(w.sc + gb * 16);
        f.d = __ldg(w.d + gb);
        return f;
    }
    __device__ __forceinline__ static void part(const Frag &f, int sub, const int8_t *xq, const int32_t *xs, int &I,
                                                int &M) {
        const int n = sub >> 1, hh = sub & 1;
        const int8_t *xb = xq + 128 * n + 16 * hh;
        const int4 x0 = *reinterpret_cast<const int4 *>(xb), x1 = *reinterpret_cast<const int4 *>(xb + 32);
        const int4 x2 = *reinterpret_cast<const int4 *>(xb + 64), x3 = *reinterpret_cast<const int4 *>(xb + 96);
        const uint32_t A[4] = {f.a.x, f.a.y, f.a.z, f.a.w}, B[4] = {f.b.x, f.b.y, f.b.z, f.b.w};
        const uint32_t H[4] = {f.h.x, f.h.y, f.h.z, f.h.w};
        const int X0[4] = {x0.x, x0.y, x0.z, x0.w}, X1[4] = {x1.x, x1.y, x1.z, x1.w};
        const int X2[4] = {x2.x, x2.y, x2.z, x2.w}, X3[4] = {x3.x, x3.y, x3.z, x3.w};
        int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t a = A[k], b = B[k], h = H[k];
            d0 = dp4a((int)((a & 0x0F0F0F0Fu) | ((h & 0x03030303u) << 4)), X0[k], d0);
            d1 = dp4a((int)((b & 0x0F0F0F0Fu) | (((h >> 2) & 0x03030303u) << 4)), X1[k], d1);
            d2 = dp4a((int)(((a >> 4) & 0x0F0F0F0Fu) | (((h >> 4) & 0x03030303u) << 4)), X2[k], d2);
            d3 = dp4a((int)(((b >> 4) & 0x0F0F0F0Fu) | (((h >> 6) & 0x03030303u) << 4)), X3[k], d3);
        }
        // int8 scales sc[8n + 2g + hh], g = 0..3: byte (8n + hh + 2g) of f.s
        const uint32_t sw0 = n ? f.s.z : f.s.x, sw1 = n ? f.s.w : f.s.y;
        const int s0 = (int)(int8_t)(sw0 >> (8 * hh)), s1 = (int)(int8_t)(sw0 >> (8 * (hh + 2)));
        const int s2 = (int)(int8_t)(sw1 >> (8 * hh)), s3 = (int)(int8_t)(sw1 >> (8 * (hh + 2)));
        const int32_t *bs = xs + 8 * n + hh;
        // (q - 32) . x = q . x - 32 * sum(x)
        I = s0 * (d0 - 32 * bs[0]) + s1 * (d1 - 32 * bs[2]) + s2 * (d2 - 32 * bs[4]) + s3 * (d3 - 32 * bs[6]);
        M = 0;
    }
    __device__ __forceinline__ static float term(const Frag &f, int I, int, float xd) {
        return fmul(fmul(xd, f16_to_f32((uint16_t)f.d)), (float)I);
    }
};

// Q4_KW and Q6_K read from shared memory (tiles staged there by bulk copies):
// same fragments and arithmetic, plain loads instead of streaming global
// loads, and the int8 activations in a padded shared-memory layout that keeps
// a quarter-warp's 16-byte loads on distinct banks:
//   Q4_KW_S  block stride 320 bytes, 64-value chunk j at 80*j
//   Q6_K_S   block stride 320 bytes, 128-value half n at 160*n
constexpr int T_Q4_KW_S = 113;
constexpr int T_Q6_K_S = 114;
constexpr int XPAD_BLOCK = 320;

__device__ __forceinline__ int xpad_q4kw(int i) { return (i >> 8) * XPAD_BLOCK + ((i & 255) >> 6) * 80 + (i & 63); }
__device__ __forceinline__ int xpad_q6k(int i) { return (i >> 8) * XPAD_BLOCK + ((i & 255) >> 7) * 160 + (i & 127); }

template <> struct QT<T_Q4_KW_S> : QT<T_Q4_KW> {
    static constexpr int BE = XPAD_BLOCK;  // activation block stride (bytes)
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int sub) {
        const uint8_t *blk = w.q + gb * 144;
        return Frag{*reinterpret_cast<const uint4 *>(blk), *reinterpret_cast<const uint4 *>(blk + 16 + 32 * sub),
                    *reinterpret_cast<const uint4 *>(blk + 32 + 32 * sub)};
    }
    __device__ __forceinline__ static void part(const Frag &f, int j, const int8_t *xq, const int32_t *xs, int &I,
                                                int &M) {
        QT<T_Q4_KW>::part(f, j, xq + 16 * j, xs, I, M);  // chunk j at 80*j
    }
};

template <> struct QT<T_Q6_K_S> : QT<T_Q6_K> {
    static constexpr int BE = XPAD_BLOCK;
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int sub) {
        const int n = sub >> 1, hh = sub & 1;
        const uint8_t *qb = w.q + gb * 192;
        Frag f;
        f.a = *reinterpret_cast<const uint4 *>(qb + 64 * n + 16 * hh);
        f.b = *reinterpret_cast<const uint4 *>(qb + 64 * n + 32 + 16 * hh);
        f.h = *reinterpret_cast<const uint4 *>(qb + 128 + 32 * n + 16 * hh);
        f.s = *reinterpret_cast<const uint4 *>(w.sc + gb * 16);
        f.d = w.d[gb];
        return f;
    }
    __device__ __forceinline__ static void part(const Frag &f, int sub, const int8_t *xq, const int32_t *xs, int &I,
                                                int &M) {
        QT<T_Q6_K>::part(f, sub, xq + 32 * (sub >> 1), xs, I, M);  // half n at 160*n
    }
};

// dp4a with unsigned bytes in a and signed bytes in b (dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One group of the T = 1 gate/up phase from shared memory: NR rows of gate
// and NR rows of up (2*NR "streams", NB Q4_K blocks each, the NR rows of a
// matrix consecutive in the tile) against one int8 activation vector in the
// xpad_q4kw layout. Lane (b = lane/4, j = lane%4) takes block b and sub-block
// pair j of every stream, so its activation fragment is loaded once; the two
// nibble halves go through dp4a directly (the high half unshifted, as 16x the
// nibble through the unsigned form, divided back exactly). Each stream's block
// terms are then added in block order from +0 through a per-warp shared
// transpose `tt` (2*NR*NB floats), leaving stream s's dot in lane s.
// Numerics are QT<T_Q4_KW>'s exactly (integer partials, same float tail).
template <int NR, int NB>
__device__ __forceinline__ float q4k_group_dot_smem(const uint8_t *tile_g, const uint8_t *tile_u, const int8_t *xq,
                                                    const float *xd, const int32_t *xs, float *tt, int lane) {
    static_assert(NB == 8, "one lane group per block");
    constexpr int S = 2 * NR;
    const int b = lane >> 2, j = lane & 3;
    const int4 *x4 = reinterpret_cast<const int4 *>(xq + b * XPAD_BLOCK + 80 * j);
    const int4 l0 = x4[0], l1 = x4[1], h0 = x4[2], h1 = x4[3];
    const int4 bs = *reinterpret_cast<const int4 *>(xs + b * 16 + 4 * j);
    const float xdb = xd[b];
    const int ms0 = bs.x + bs.y, ms1 = bs.z + bs.w;
    const int sh = 16 * (j & 1);
    const bool low = j < 2;
    // straight-line per stream (no branch, no shuffle): the streams' chains interleave
    int I[S], M[S];
    uint32_t hx[S];
#pragma unroll
    for (int s = 0; s < S; s++) {
        const uint8_t *blk = (s < NR ? tile_g + (size_t)s * NB * 144 : tile_u + (size_t)(s - NR) * NB * 144) + b * 144;
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * j);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * j);
        int dla = dp4a((int)(q0.x & 0x0F0F0F0Fu), l0.x, 0), dlb = dp4a((int)(q0.y & 0x0F0F0F0Fu), l0.y, 0);
        dla = dp4a((int)(q0.z & 0x0F0F0F0Fu), l0.z, dla);
        dlb = dp4a((int)(q0.w & 0x0F0F0F0Fu), l0.w, dlb);
        dla = dp4a((int)(q1.x & 0x0F0F0F0Fu), l1.x, dla);
        dlb = dp4a((int)(q1.y & 0x0F0F0F0Fu), l1.y, dlb);
        dla = dp4a((int)(q1.z & 0x0F0F0F0Fu), l1.z, dla);
        dlb = dp4a((int)(q1.w & 0x0F0F0F0Fu), l1.w, dlb);
        int dha = dp4a_us(q0.x & 0xF0F0F0F0u, h0.x, 0), dhb = dp4a_us(q0.y & 0xF0F0F0F0u, h0.y, 0);
        dha = dp4a_us(q0.z & 0xF0F0F0F0u, h0.z, dha);
        dhb = dp4a_us(q0.w & 0xF0F0F0F0u, h0.w, dhb);
        dha = dp4a_us(q1.x & 0xF0F0F0F0u, h1.x, dha);
        dhb = dp4a_us(q1.y & 0xF0F0F0F0u, h1.y, dhb);
        dha = dp4a_us(q1.z & 0xF0F0F0F0u, h1.z, dha);
        dhb = dp4a_us(q1.w & 0xF0F0F0F0u, h1.w, dhb);
        const int dl = dla + dlb, dh = (dha + dhb) >> 4;  // exact: a multiple of 16
        // scaleMinK4 (ggml.zig:1332) for sub-blocks 2j, 2j+1
        const uint32_t a = h.y >> sh, bb = h.z >> sh, lo = h.w >> sh;
        const int sc0 = low ? (a & 63) : ((lo & 0xF) | (((a >> 6) & 3) << 4));
        const int mn0 = low ? (bb & 63) : (((lo >> 4) & 0xF) | (((bb >> 6) & 3) << 4));
        const int sc1 = low ? ((a >> 8) & 63) : (((lo >> 8) & 0xF) | (((a >> 14) & 3) << 4));
        const int mn1 = low ? ((bb >> 8) & 63) : (((lo >> 12) & 0xF) | (((bb >> 14) & 3) << 4));
        I[s] = sc0 * dl + sc1 * dh;
        M[s] = mn0 * ms0 + mn1 * ms1;
        hx[s] = h.x;
    }
    // the block's four lanes: integer sums (exact, any order)
#pragma unroll
    for (int s = 0; s < S; s++) {
        I[s] += __shfl_xor_sync(0xffffffffu, I[s], 1);
        M[s] += __shfl_xor_sync(0xffffffffu, M[s], 1);
    }
#pragma unroll
    for (int s = 0; s < S; s++) {
        I[s] += __shfl_xor_sync(0xffffffffu, I[s], 2);
        M[s] += __shfl_xor_sync(0xffffffffu, M[s], 2);
    }
    if (j == 0) {
#pragma unroll
        for (int s = 0; s < S; s++) {
            const float d = f16_to_f32((uint16_t)(hx[s] & 0xFFFF)), dmin = f16_to_f32((uint16_t)(hx[s] >> 16));
            tt[s * NB + b] = fmul(xdb, fsub(fmul(d, (float)I[s]), fmul(dmin, (float)M[s])));
        }
    }
    __syncwarp();
    float acc = 0.0f;
    if (lane < S) {
#pragma unroll
        for (int bb = 0; bb < NB; bb++) acc = fadd(acc, tt[lane * NB + bb]);
    }
    __syncwarp();
    return acc;
}

// SC consecutive rows of a staged Q6_K tile (row r's NB blocks at block index
// (row0 + r) * NB; rows past nvalid repeat row0) against one int8 activation
// vector in the xpad_q6k layout (one scale per 256-block, sums per 16). Lane
// group g = lane/4 takes row g and, lane sub = lane%4, a quarter of every
// block; each row's block terms are then added in block order from +0 inside
// the group's own lanes (no transpose). Returns row (lane/4)'s dot on every
// lane of its group. Numerics are QT<T_Q6_K>'s exactly.
template <int SC, int NB>
__device__ __forceinline__ float q6k_rows_dot_smem(const WDev &w, int row0, int nvalid, const int8_t *aq,
                                                   const float *ad, const int32_t *as, int lane) {
    static_assert(SC == 8, "one lane group per row");
    const int g = lane >> 2, sub = lane & 3;
    const uint64_t gb0 = (uint64_t)(row0 + (g < nvalid ? g : 0)) * NB;
    int I[NB];
    uint32_t dw[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
        const typename QT<T_Q6_K_S>::Frag f = QT<T_Q6_K_S>::load(w, gb0 + b, sub);
        int Ib, Mb;
        QT<T_Q6_K_S>::part(f, sub, aq + b * XPAD_BLOCK, as + b * 16, Ib, Mb);
        I[b] = Ib;
        dw[b] = f.d;
    }
#pragma unroll
    for (int b = 0; b < NB; b++) I[b] += __shfl_xor_sync(0xffffffffu, I[b], 1);
#pragma unroll
    for (int b = 0; b < NB; b++) I[b] += __shfl_xor_sync(0xffffffffu, I[b], 2);
    float acc = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; b++)
        acc = fadd(acc, fmul(fmul(ad[b], f16_to_f32((uint16_t)dw[b])), (float)I[b]));
    return acc;
}

template <> struct QT<T_Q8_0> {
    static constexpr int LPB = 2, BE = 32, SPB = 1;
    struct Frag {
        uint4 q;
        uint32_t d;
    };
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int sub) {
        return Frag{ld_stream_v4(w.q + gb * 32 + 16 * sub), (uint32_t)__ldg(w.d + gb)};
    }
    __device__ __forceinline__ static void part(const Frag &f, int sub, const int8_t *xq, const int32_t *, int &I,
                                                int &M) {
        const int4 x = *reinterpret_cast<const int4 *>(xq + 16 * sub);
        int dot = 0;
        dot = dp4a((int)f.q.x, x.x, dot);
        dot = dp4a((int)f.q.y, x.y, dot);
        dot = dp4a((int)f.q.z, x.z, dot);
        dot = dp4a((int)f.q.w, x.w, dot);
        I = dot;
        M = 0;
    }
    __device__ __forceinline__ static float term(const Frag &f, int I, int, float xd) {
        return fmul(fmul(f16_to_f32((uint16_t)f.d), xd), (float)I);
    }
};

template <> struct QT<T_Q4_0> {
    static constexpr int LPB = 1, BE = 32, SPB = 1;
    struct Frag {
        uint4 q;
        uint32_t d;
    };
    __device__ __forceinline__ static Frag load(const WDev &w, uint64_t gb, int) {
        return Frag{ld_stream_v4(w.q + gb * 16), (uint32_t)__ldg(w.d + gb)};
    }
    __device__ __forceinline__ static void part(const Frag &f, int, const int8_t *xq, const int32_t *xs, int &I, int &M) {
        const int4 xl = *reinterpret_cast<const int4 *>(xq), xh = *reinterpret_cast<const int4 *>(xq + 16);
        int dot = 0;
        dot = dp4a((int)(f.q.x & 0x0F0F0F0Fu), xl.x, dot);
        dot = dp4a((int)(f.q.y & 0x0F0F0F0Fu), xl.y, dot);
        dot = dp4a((int)(f.q.z & 0x0F0F0F0Fu), xl.z, dot);
        dot = dp4a((int)(f.q.w & 0x0F0F0F0Fu), xl.w, dot);
        dot = dp4a((int)((f.q.x >> 4) & 0x0F0F0F0Fu), xh.x, dot);
        dot = dp4a((int)((f.q.y >> 4) & 0x0F0F0F0Fu), xh.y, dot);
        dot = dp4a((int)((f.q.z >> 4) & 0x0F0F0F0Fu), xh.z, dot);
        dot = dp4a((int)((f.q.w >> 4) & 0x0F0F0F0Fu), xh.w, dot);
        I = dot - 8 * xs[0];
        M = 0;
    }
    __device__ __forceinline__ static float term(const Frag &f, int I, int, float xd) {
        return fmul(fmul(f16_to_f32((uint16_t)f.d), xd), (float)I);
    }
};

// Streams: a functor `at(s, w, gb, xv)` giving stream s's weight tensor, first
// block, and activation view (s < nS <= S always).
//
// The engine is split so a kernel can issue its weight loads, then wait for
// the producer of its activations (programmatic dependent launch), then
// finish: wd_load issues every load of the warp; wd_finish forms the terms and
// adds each stream's terms in block order into acc[0..nS). NB (blocks per
// stream) and nS (streams in use, <= S) are runtime values with
// nS*NB <= MAXU*G.
template <int TY, int MAXU> struct WFrags {
    typename QT<TY>::Frag f[MAXU];
};

template <int TY, int S, int MAXU, class Streams>
__device__ __forceinline__ void wd_load(const Streams &st, int NB, int nS, WFrags<TY, MAXU> &fr, int lane) {
    using Q = QT<TY>;
    constexpr int G = 32 / Q::LPB;
    const int U = nS * NB;
    const int grp = lane / Q::LPB, sub = lane % Q::LPB;
#pragma unroll
    for (int j = 0; j < MAXU; j++) {
        const int u = j * G + grp;
        if (u < U) {
            const int s = u / NB, b = u - s * NB;
            WDev w;
            uint64_t gb;
            XV xv;
            st.at(s, w, gb, xv);
            fr.f[j] = Q::load(w, gb + b, sub);
        }
    }
}

template <int TY, int S, int MAXU, class Streams>
__device__ __forceinline__ void wd_finish(const Streams &st, int NB, int nS, const WFrags<TY, MAXU> &fr,
                                          float (&acc)[S], int lane) {
    using Q = QT<TY>;
    constexpr int G = 32 / Q::LPB;
    const int U = nS * NB;
    const int grp = lane / Q::LPB, sub = lane % Q::LPB;
    float term[MAXU];
#pragma unroll
    for (int j = 0; j < MAXU; j++) {
        const int u = j * G + grp;
        int I = 0, M = 0;
        float xd = 0.0f;
        if (u < U) {
            const int s = u / NB, b = u - s * NB;
            WDev w;
            uint64_t gb;
            XV xv;
            st.at(s, w, gb, xv);
            Q::part(fr.f[j], sub, xv.q + b * Q::BE, xv.s + b * Q::SPB, I, M);
            xd = xv.d[b];
        }
#pragma unroll
        for (int o = 1; o < Q::LPB; o <<= 1) {
            I += __shfl_xor_sync(0xffffffffu, I, o);
            M += __shfl_xor_sync(0xffffffffu, M, o);
        }
        term[j] = u < U ? Q::term(fr.f[j], I, M, xd) : 0.0f;
    }
    // units are numbered stream-major, so walking them in order visits every
    // stream's blocks in block order
    float a = 0.0f;
#pragma unroll
    for (int j = 0; j < MAXU; j++) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            const int u = j * G + g;
            const float t = __shfl_sync(0xffffffffu, term[j], g * Q::LPB);
            if (u < U) {
                const int s = u / NB, b = u - s * NB;
                a = fadd(b == 0 ? 0.0f : a, t);  // the CPU accumulator starts at +0
                if (b == NB - 1) {
#pragma unroll
                    for (int ss = 0; ss < S; ss++)
                        if (ss == s) acc[ss] = a;
                }
            }
        }
    }
}

}  // namespace loom

namespace loom {

// ---- compile-time engine ------------------------------------------------------------
// Same arithmetic as wd_load/wd_finish, with S streams of NB blocks fixed at
// compile time and a unit order that makes every stream/block index a
// constant or a lane offset (no division at run time):
//   stream-major  (NB % G == 0): unit j*G + grp is stream (j*G)/NB, block (j*G)%NB + grp
//   block-major   (S  % G == 0): unit j*G + grp is block (j*G)/S,  stream (j*G)%S + grp
// The Streams functor takes the (possibly lane-dependent) stream index.
template <int TY, int S, int NB> struct CEng {
    using Q = QT<TY>;
    static constexpr int G = 32 / Q::LPB;
    static constexpr bool SM = NB % G == 0;
    static constexpr bool BM = !SM && S % G == 0;
    static constexpr bool OK = SM || BM;
    static constexpr int MAXU = (S * NB) / G;
    using Frags = WFrags<TY, MAXU>;  // shared with the run-time engine for partial chunks
    __device__ __forceinline__ static void unit(int j, int grp, int &s, int &b) {
        if constexpr (SM) {
            s = (j * G) / NB;
            b = (j * G) % NB + grp;
        } else {
            b = (j * G) / S;
            s = (j * G) % S + grp;
        }
    }
    template <class Streams>
    __device__ __forceinline__ static void load(const Streams &st, Frags &fr, int lane) {
        const int grp = lane / Q::LPB, sub = lane % Q::LPB;
#pragma unroll
        for (int j = 0; j < MAXU; j++) {
            int s, b;
            unit(j, grp, s, b);
            fr.f[j] = Q::load(st.w(s), st.gb(s) + b, sub);
        }
    }
    template <class Streams>
    __device__ __forceinline__ static void finish(const Streams &st, const Frags &fr, float (&acc)[S], int lane) {
        const int grp = lane / Q::LPB, sub = lane % Q::LPB;
        float term[MAXU];
#pragma unroll
        for (int j = 0; j < MAXU; j++) {
            int s, b;
            unit(j, grp, s, b);
            const XV xv = st.x(s);
            int I, M;
            Q::part(fr.f[j], sub, xv.q + b * Q::BE, xv.s + b * Q::SPB, I, M);
#pragma unroll
            for (int o = 1; o < Q::LPB; o <<= 1) {
                I += __shfl_xor_sync(0xffffffffu, I, o);
                if constexpr (TY == T_Q4_K || TY == T_Q4_KW || TY == T_Q4_KW_S) M += __shfl_xor_sync(0xffffffffu, M, o);
            }
            term[j] = Q::term(fr.f[j], I, M, xv.d[b]);
        }
        sum_terms(term, acc);
    }
    // load + finish in one pass for operands in shared memory (no fragment
    // array held across the loads)
    template <class Streams>
    __device__ __forceinline__ static void run(const Streams &st, float (&acc)[S], int lane) {
        const int grp = lane / Q::LPB, sub = lane % Q::LPB;
        float term[MAXU];
#pragma unroll
        for (int j = 0; j < MAXU; j++) {
            int s, b;
            unit(j, grp, s, b);
            const typename Q::Frag f = Q::load(st.w(s), st.gb(s) + b, sub);
            const XV xv = st.x(s);
            int I, M;
            Q::part(f, sub, xv.q + b * Q::BE, xv.s + b * Q::SPB, I, M);
#pragma unroll
            for (int o = 1; o < Q::LPB; o <<= 1) {
                I += __shfl_xor_sync(0xffffffffu, I, o);
                if constexpr (TY == T_Q4_K || TY == T_Q4_KW || TY == T_Q4_KW_S) M += __shfl_xor_sync(0xffffffffu, M, o);
            }
            term[j] = Q::term(f, I, M, xv.d[b]);
        }
        sum_terms(term, acc);
    }
    // each stream's block terms added in block order from +0
    __device__ __forceinline__ static void sum_terms(const float (&term)[MAXU], float (&acc)[S]) {
#pragma unroll
        for (int s = 0; s < S; s++) {
            float a = 0.0f;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                const int u = SM ? s * NB + b : b * S + s;
                a = fadd(a, __shfl_sync(0xffffffffu, term[u / G], (u % G) * Q::LPB));
            }
            acc[s] = a;
        }
    }
};

}  // namespace loom
