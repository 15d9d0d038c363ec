// common.cuh -- block formats, device layouts and small device helpers shared
// by every kernel of the CUDA backend.
//
// GGUF block formats (ch4r10t33r/loom src/gguf/ggml.zig:87-99):
//   Q4_0  18 B: f16 d, 16 B nibbles (lane i low, lane i+16 high)
//   Q8_0  34 B: f16 d, 32 x int8
//   Q4_K 144 B: f16 d, f16 dmin, 12 B packed 6-bit scales/mins, 128 B nibbles
//   Q6_K 210 B: 128 B ql, 64 B qh, 16 x int8 scales, f16 d
//
// Device layouts (chosen so every quant load is a 16-byte aligned, coalesced
// 128-bit load; the values they decode to are unchanged):
//   F32   row-major floats
//   Q4_K  the GGUF blocks as they are (144 = 9 x 16 B)
//   Q6_K  three regions: quants [nblk][192] (ql then qh), scales [nblk][16],
//         d [nblk] (u16)
//   Q8_0  quants [nblk][32], d [nblk]
//   Q4_0  quants [nblk][16], d [nblk]
// Regions start on 256-byte boundaries. Block index = global block number in
// the tensor, so a 3D expert tensor's plane e, row r, block b is block
// (e*rows + r)*blocks_per_row + b in every layout.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace loom {

enum GgmlType : int {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12,
    T_Q5_K = 13, T_Q6_K = 14
};
__host__ __device__ constexpr bool is_kquant(int t) {
    return t == T_Q2_K || t == T_Q3_K || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

constexpr int QK_0 = 32;
constexpr int QK_K = 256;

__host__ __device__ constexpr int block_elems(int t) {
    return t == T_F32 ? 1 : (t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0) ? QK_0
         : is_kquant(t) ? QK_K : 0;
}
__host__ __device__ constexpr int block_bytes(int t) {
    return t == T_F32 ? 4 : t == T_Q4_0 ? 18 : t == T_Q8_0 ? 34 : t == T_Q4_K ? 144 : t == T_Q6_K ? 210
         : t == T_Q2_K ? 84 : t == T_Q3_K ? 110 : t == T_Q5_K ? 176 : t == T_Q4_1 ? 20 : t == T_Q5_1 ? 24 : t == T_Q5_0 ? 22 : 0;
}
// bytes of the quant region per block in the device layout (Q2_K: scales +
// quants; Q3_K: high-bit mask + quants; Q4_K / Q5_K: the whole block)
__host__ __device__ constexpr int layout_qbytes(int t) {
    return t == T_F32 ? 4 : t == T_Q4_0 ? 16 : t == T_Q8_0 ? 32 : t == T_Q4_K ? 144 : t == T_Q6_K ? 192
         : t == T_Q2_K ? 80 : t == T_Q3_K ? 96 : t == T_Q5_K ? 176 : (t == T_Q4_1 || t == T_Q5_1 || t == T_Q5_0) ? 16 : 0;
}
// true when a type's activation is quantized per 256 (Q8_K style) rather than per 32
__host__ __device__ constexpr bool act256(int t) { return is_kquant(t) || t == 112; }

// A device-resident weight tensor in its device layout.
struct WDev {
    const uint8_t *q;   // quants (or the Q4_K blocks, or floats)
    const uint8_t *sc;  // Q6_K scales region, else null
    const uint16_t *d;  // f16 scales region (Q6_K/Q8_0/Q4_0), else null
    int type;
    int pad_;           // flags (WDEV_*)
};
// Q6_K tensor whose int8 sub-block scales all satisfy |sc| <= 32: then
// |sc * (q - 32)| <= 1024 is an integer fp16 holds exactly, and 128 of them
// times int8 activations sum to less than 2^24 (exact in an f32 accumulator):
// the tensor-core path's condition
constexpr int WDEV_Q6K_SMALL_SCALES = 1;

// Quantized activations for a batch of vectors, each `cols` wide:
//   q[t*cols + i]        int8
//   d[t*dstride + b]     f32 scale per 256 (K types) or 32 (Q4_0/Q8_0) block
//   s[t*sstride + j]     i32 per-16 sums (K types) or per-32 sums
struct XQ {
    const int8_t *q;
    const float *d;
    const int32_t *s;
    int cols;
    int dstride;
    int sstride;
    int kind256;
};

// ---- loads -------------------------------------------------------------------

// Streamed weight load: read-only path, do not allocate in L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_v4(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ int4 ld_i4(const void *p) { return __ldg(reinterpret_cast<const int4 *>(p)); }

__device__ __forceinline__ float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// ---- exact scalar helpers (one IEEE rounding per op; never contracted) ----------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// e^x in f32 for the softmax, sigmoid and SiLU (tensor.zig:18-35): the double
// precision exp rounded once to f32. That is the correctly rounded result
// except within ~2^-29 of a rounding boundary; the reference's f32 exp
// (within ~0.5 ulp) agrees with it nearly everywhere, CUDA's single-precision
// expf (within 2 ulp) often does not, and one ulp there can move an int8
// activation of the next matvec.
__device__ __forceinline__ float exp_f(float x) { return (float)exp((double)x); }

// ggml.zig:1067-1074 toI8Saturating
__device__ __forceinline__ int to_i8_sat(float v) {
    if (!isfinite(v)) return 0;
    float r = roundf(v);  // half away from zero, as Zig's @round
    if (r >= 127.0f) return 127;
    if (r <= -127.0f) return -127;
    return (int)r;
}

// ggml.zig:1332-1340 scaleMinK4, on the 12 scale bytes held as three words
// q3kScales (ggml.zig:1173-1191): six-bit scale j (0..15) of the 12 packed
// bytes p (low four bits from bytes 0-7, high two bits from bytes 8-11)
__host__ __device__ __forceinline__ int q3k_scale(const uint8_t *p, int j) {
    const int lo = j < 8 ? (p[j] & 0x0F) : (p[j - 8] >> 4);
    const int hi = (p[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
    return lo | (hi << 4);
}

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *s, int &sc, int &mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace loom
