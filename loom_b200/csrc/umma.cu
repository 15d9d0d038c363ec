// umma.cu -- tensor-core (tcgen05) kernels: the bf16 GEMM building block and
// its self-test entry point.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "umma.cuh"
#include "warpdot.cuh"

namespace loom {

constexpr uint32_t UMMA_POLLS = 1u << 22;  // bounded wait on an MMA completion barrier

// D[M][N] (f32, row-major) = A[M][K] . B[N][K]^T (bf16, K contiguous), one
// 128-row tile per CTA, 128 threads, N a multiple of 16 in [16, 256], K a
// multiple of 64. K steps of 64 are staged into shared memory in the
// K-major core-matrix layout and fed to four M=128 x N x K=16 MMAs.
__global__ void __launch_bounds__(128) k_umma_selftest(const uint16_t *A, const uint16_t *B, float *D, int M, int N,
                                                       int K, int *err) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t *sA = sm;                   // [8][128][16 B]
    uint8_t *sB = sm + 8 * 128 * 16;    // [8][N][16 B]
    __shared__ __align__(8) uint64_t mbar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_ok;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int m0 = blockIdx.x * 128;
    uint32_t ncols = 32;
    while ((int)ncols < N) ncols <<= 1;
    if (warp == 0) tmem_alloc(&s_tmem, ncols);
    if (t == 0) {
        mbar_init(&mbar, 1);
        s_ok = 1;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const uint32_t idesc = umma_idesc_bf16_f32(128, N);
    uint32_t phase = 0;
    for (int k0 = 0; k0 < K && s_ok; k0 += 64) {
        for (int kc = 0; kc < 8; kc++) {
            if (m0 + t < M)
                *reinterpret_cast<uint4 *>(sA + (kc * 128 + t) * 16) =
                    *reinterpret_cast<const uint4 *>(A + (size_t)(m0 + t) * K + k0 + 8 * kc);
            for (int n = t; n < N; n += 128)
                *reinterpret_cast<uint4 *>(sB + ((size_t)kc * N + n) * 16) =
                    *reinterpret_cast<const uint4 *>(B + (size_t)n * K + k0 + 8 * kc);
        }
        fence_async_smem();
        __syncthreads();
        if (t == 0) {
            tc_fence_after();
#pragma unroll
            for (int s = 0; s < 4; s++)
                umma_bf16(tmem, umma_desc_kmajor(sA + 2 * s * 128 * 16, 128),
                          umma_desc_kmajor(sB + (size_t)2 * s * N * 16, (uint32_t)N), idesc, k0 > 0 || s > 0);
            umma_commit(&mbar);
            if (!mbar_wait(&mbar, phase, UMMA_POLLS)) {
                atomicOr(err, 1);
                mbar_wait(&mbar, phase, UMMA_POLLS);  // let the MMAs finish before the shared memory is reused
                s_ok = 0;
            }
        }
        phase ^= 1;
        __syncthreads();
    }
    tc_fence_after();
    if (s_ok) {
        for (int c0 = 0; c0 < N; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, r);
            const int row = m0 + 32 * warp + lane;
            if (row < M)
                for (int i = 0; i < 16; i++) D[(size_t)row * N + c0 + i] = __uint_as_float(r[i]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_free(tmem, ncols);
}

}  // namespace loom

using namespace loom;

extern "C" int loom_cuda_umma_selftest(const uint16_t *A, const uint16_t *B, float *D, int M, int N, int K);

// Diagnostic entry (no counterpart in the reference): runs the bf16 tcgen05
// GEMM on host arrays; returns 0, 1 on bad arguments, 2 on a CUDA error, 3 if
// an MMA completion wait gave up.
int loom_cuda_umma_selftest(const uint16_t *A, const uint16_t *B, float *D, int M, int N, int K) {
    if (M <= 0 || M % 128 || N < 16 || N > 256 || N % 16 || K <= 0 || K % 64) return 1;
    uint16_t *dA = nullptr, *dB = nullptr;
    float *dD = nullptr;
    int *derr = nullptr, herr = 0;
    int rc = 0;
    const size_t smem = 8 * 128 * 16 + (size_t)8 * N * 16;
    if (cudaMalloc(&dA, (size_t)M * K * 2) || cudaMalloc(&dB, (size_t)N * K * 2) || cudaMalloc(&dD, (size_t)M * N * 4) ||
        cudaMalloc(&derr, 4)) {
        rc = 2;
    } else if (cudaMemcpy(dA, A, (size_t)M * K * 2, cudaMemcpyHostToDevice) ||
               cudaMemcpy(dB, B, (size_t)N * K * 2, cudaMemcpyHostToDevice) || cudaMemset(derr, 0, 4) ||
               cudaFuncSetAttribute(k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) {
        rc = 2;
    } else {
        k_umma_selftest<<<M / 128, 128, smem>>>(dA, dB, dD, M, N, K, derr);
        if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost) ||
            cudaMemcpy(D, dD, (size_t)M * N * 4, cudaMemcpyDeviceToHost))
            rc = 2;
        else if (herr)
            rc = 3;
    }
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dD);
    cudaFree(derr);
    return rc;
}

// ==== expert FFN on the tensor cores (batched prefill) ==================================
// For T tokens with about 16 or more per expert, gate/up and down run per
// expert as tcgen05 MMAs (kind::f16, f32 accumulators in TMEM) that carry the
// reference's INTEGER arithmetic (ggml.zig kBlockDot :1002):
//   A = the weight's integer sub-block products, folded per value:
//         Q4_K  sc * q          (6-bit scale x 4-bit quant  <= 945)
//         Q6_K  sc * (q - 32)   (int8 scale x 6-bit quant)
//   B = the int8 activations of quantizeX256 (ggml.zig:776), per token.
// Both are integers exactly representable in fp16, every product is exact in
// f32, and each MMA group sums 128 of them (half a super-block), so every
// partial sum is an integer below 2^24: the accumulator holds the exact
// integer dot. The epilogue forms the reference's float tail per super-block
// and adds the blocks in block order from +0, so the results are the CPU's
// bit for bit (for Q6_K scales |sc| <= 64, where sc*(q-32) stays within
// fp16's exact integers; larger scales round the fold).

#include "decode.cuh"

namespace loom {

static inline unsigned cdivu(uint64_t a, uint64_t b) { return (unsigned)((a + b - 1) / b); }

// scaleMinK4 (ggml.zig:1332-1340) with the 12 scale bytes in three words
__device__ __forceinline__ void scale_min_k4w(int j, uint32_t y, uint32_t z, uint32_t w, int &sc, int &mn) {
    auto byte = [&](int i) -> int { return (int)(((i < 4 ? y : i < 8 ? z : w) >> (8 * (i & 3))) & 0xFF); };
    if (j < 4) {
        sc = byte(j) & 63;
        mn = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
        mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

__device__ __forceinline__ void umma_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// two small integers -> packed fp16 pair (exact for |v| <= 2048)
__device__ __forceinline__ uint32_t h2i(int a, int b) {
    return (uint32_t)__half_as_ushort(__int2half_rn(a)) | ((uint32_t)__half_as_ushort(__int2half_rn(b)) << 16);
}
// 8 int8 (two words) -> 8 fp16 as one 16-byte chunk
__device__ __forceinline__ uint4 h8_from_i8(uint32_t lo, uint32_t hi) {
    auto sb = [](uint32_t w, int i) { return (int)(int8_t)(w >> (8 * i)); };
    return make_uint4(h2i(sb(lo, 0), sb(lo, 1)), h2i(sb(lo, 2), sb(lo, 3)), h2i(sb(hi, 0), sb(hi, 1)),
                      h2i(sb(hi, 2), sb(hi, 3)));
}

// Exact small-integer -> fp16 conversions through the fp16 "magic" 1024:
// 0x6400 | v is 1024 + v for 0 <= v < 1024, and one fused HFMA2 / HSUB2 of
// exactly representable operands with an exactly representable result is
// exact.
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Q4_K: 4 bytes of nibbles -> low nibbles (4 values, scale sl) and high
// nibbles (4 values, scale sh) as fp16 pairs: sc * q, exact (<= 945)
__device__ __forceinline__ void q4_word_to_h(uint32_t w, __half2 sl2, __half2 offl, __half2 sh16, __half2 offh,
                                             uint32_t &lo01, uint32_t &lo23, uint32_t &hi01, uint32_t &hi23) {
    const uint32_t p01 = __byte_perm(w, 0, 0x4140), p23 = __byte_perm(w, 0, 0x4342);
    lo01 = h2u(__hfma2(u2h((p01 & 0x000F000Fu) | 0x64006400u), sl2, offl));  // (1024 + q) * sc - 1024 sc
    lo23 = h2u(__hfma2(u2h((p23 & 0x000F000Fu) | 0x64006400u), sl2, offl));
    hi01 = h2u(__hfma2(u2h((p01 & 0x00F000F0u) | 0x64006400u), sh16, offh));  // (1024 + 16q) * sc/16 - 64 sc
    hi23 = h2u(__hfma2(u2h((p23 & 0x00F000F0u) | 0x64006400u), sh16, offh));
}

// 8 int8 (two words) -> 8 fp16, exact: (1024 + (v + 128)) - 1152
__device__ __forceinline__ uint4 h8_from_i8_fast(uint32_t lo, uint32_t hi) {
    const __half2 k = u2h(0x64806480u);  // 1152, 1152
    lo ^= 0x80808080u;
    hi ^= 0x80808080u;
    return make_uint4(h2u(__hsub2(u2h(__byte_perm(lo, 0x64646464u, 0x7170) ), k)),
                      h2u(__hsub2(u2h(__byte_perm(lo, 0x64646464u, 0x7372)), k)),
                      h2u(__hsub2(u2h(__byte_perm(hi, 0x64646464u, 0x7170)), k)),
                      h2u(__hsub2(u2h(__byte_perm(hi, 0x64646464u, 0x7372)), k)));
}

// Instruction descriptor of kind::f16 with fp16 A and B, f32 accumulator
// (formats 0 = F16 in bits [7,10) and [10,13)).
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

constexpr int MMA_THREADS = 512;  // 16 warps: TMEM row quarter = warp % 4, token group = warp / 4
constexpr int MMA_NP = 64;        // tokens per pass (the MMA's N)

struct MmaCtl {
    uint64_t mbar[2];
    uint32_t tmem;
    int ok;
};

// thread 0 waits (bounded) for the MMAs committed on mbar[b] (use `parity`);
// the verdict is shared.
__device__ __forceinline__ bool mma_wait(MmaCtl &S, int b, uint32_t parity, int *err) {
    if (threadIdx.x == 0 && S.ok && !mbar_wait(&S.mbar[b], parity, UMMA_POLLS)) {
        if (err) atomicOr(err, 32);
        mbar_wait(&S.mbar[b], parity, UMMA_POLLS);  // let the MMAs finish before the memory is reused
        S.ok = 0;
    }
    __syncthreads();
    return S.ok != 0;
}

// one warp: 16 f32 accumulator columns of TMEM row quarter q -> exact ints
__device__ __forceinline__ void tmem_ints16(uint32_t tmem, int q, uint32_t col, int (&v)[16]) {
    uint32_t r[16];
    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + col, r);
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __float2int_rn(__uint_as_float(r[i]));
}

// raw Q4_K words thread t needs at gate/up step ks: the super-block header and
// the 32 nibble bytes of its sub-block pair
template <int NBG>
__device__ __forceinline__ void gu_fetch_t(uint4 (&pw)[3], const WDev &wg, const WDev &wu, uint64_t plane, int row0,
                                           int ffn, int ks, int t) {
    const int mat = t >> 8, jj = (t >> 7) & 1, r = t & 127, row = row0 + r;
    if (row >= ffn) return;
    const uint8_t *bp = (mat ? wu : wg).q + (plane + (uint64_t)row * NBG + (ks >> 1)) * 144;
    const int j = 2 * (ks & 1) + jj;
    pw[0] = ld_stream_v4(bp);
    pw[1] = ld_stream_v4(bp + 16 + 32 * j);
    pw[2] = ld_stream_v4(bp + 32 + 32 * j);
}
#define gu_fetch gu_fetch_t<NBG>

// ---- gate/up (Q4_K): act[slot][row] = silu(gate . x) * (up . x) ----------------------------
// Expert blockIdx.y (n_local = the shared expert), rows [128*blockIdx.x, +128).
template <int NBG>
__global__ void __launch_bounds__(MMA_THREADS, 1) k_gu_mma(DecodeArgs A) {
    constexpr int dim = NBG * 256, KSTEPS = NBG * 2;
    constexpr size_t A_BYTES = (size_t)2 * 16 * 128 * 16;  // gate | up: [16 chunks][128 rows][16 B]
    constexpr size_t B_BYTES = (size_t)16 * MMA_NP * 16;   // [16 chunks][NP tokens][16 B]
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ MmaCtl S;
    // per block parity: weight rows' d, dmin, mins (8 x 6 bits in 2 words) and the tokens' xd, per-32 sums
    __shared__ float s_d[2][2][128], s_dmin[2][2][128];
    __shared__ uint32_t s_mn[2][2][128][2];
    __shared__ float s_xd[2][MMA_NP];
    __shared__ uint4 s_bsp[2][MMA_NP];  // per token: per-32 sums of the block as low bytes | signed high bytes
    __shared__ const int8_t *s_tok[MMA_NP];
    umma_pdl_wait();
    const int e = blockIdx.y;
    const bool shared = e == A.n_local;
    const int n = shared ? A.T : A.grp_cnt[e];
    const int ffn = shared ? A.shexp_ffn : A.ffn;
    const int row0 = blockIdx.x * 128;
    if (n == 0 || row0 >= ffn) return;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, q = warp & 3, tg = warp >> 2;
    const int *list = shared ? nullptr : A.grp_list + A.grp_off[e];
    const WDev wg = shared ? A.sg : A.g, wu = shared ? A.su : A.u;
    const uint64_t plane = shared ? 0 : (uint64_t)e * ffn * NBG;
    const uint32_t ncols = 2 * 2 * MMA_NP;  // two buffers of gate | up
    if (warp == 0) tmem_alloc(&S.tmem, ncols);
    if (t == 0) {
        mbar_init(&S.mbar[0], 1);
        mbar_init(&S.mbar[1], 1);
        S.ok = 1;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;
    uint32_t gstep = 0;  // MMA steps committed (buffer = step & 1, its use count = step >> 1)
    for (int c0 = 0; c0 < n && S.ok; c0 += MMA_NP) {
        const int nc = n - c0 < MMA_NP ? n - c0 : MMA_NP, N = (nc + 15) / 16 * 16;
        const uint32_t idesc = umma_idesc_f16_f32(128, N);
        const int tok0 = 16 * tg;  // this warp's tokens in the pass
        int Ig[16], Iu[16];
        float ag[16], au[16];
#pragma unroll
        for (int i = 0; i < 16; i++) ag[i] = au[i] = 0.0f;
        const uint32_t step0 = gstep;
        for (int i = t; i < nc; i += MMA_THREADS) {  // this pass's tokens' int8 rows
            const int slot = shared ? A.T * A.n_used + c0 + i : list[c0 + i];
            s_tok[i] = A.x256.q + (size_t)(shared ? c0 + i : slot / A.n_used) * dim;
        }
        __syncthreads();
        uint4 pw[3];  // this thread's raw weight words of the next step (header, two nibble quarters)
        gu_fetch(pw, wg, wu, plane, row0, ffn, 0, t);
        uint2 px[2];  // this thread's token words of the next step
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int it = t + u * MMA_THREADS;
            if (it < N * 16 && (it >> 4) < nc) px[u] = *reinterpret_cast<const uint2 *>(s_tok[it >> 4] + (it & 15) * 8);
        }
        for (int ks = 0; ks <= KSTEPS; ks++) {
            if (ks < KSTEPS) {  // ---- stage step ks into buffer gstep & 1 (its previous MMAs were awaited below)
                const int b = gstep & 1, blk = ks >> 1, h = ks & 1, pb = blk & 1;
                uint8_t *tA = sm + (size_t)b * (A_BYTES + B_BYTES), *tB = tA + A_BYTES;
                {   // weights (prefetched one step ahead): thread -> (matrix, sub-block pair jj of this half, row);
                    // a warp stores 32 consecutive rows of one chunk (no bank conflicts)
                    const int mat = t >> 8, jj = (t >> 7) & 1, r = t & 127, row = row0 + r;
                    uint8_t *tile = tA + (size_t)mat * 16 * 128 * 16;
                    const uint4 hd = pw[0], q0 = pw[1], q1 = pw[2];
                    if (ks + 1 < KSTEPS) gu_fetch(pw, wg, wu, plane, row0, ffn, ks + 1, t);
                    if (row < ffn) {
                        const int j = 2 * h + jj;  // warp-uniform
                        int sl, ml, sh, mh;
                        scale_min_k4w(2 * j, hd.y, hd.z, hd.w, sl, ml);
                        scale_min_k4w(2 * j + 1, hd.y, hd.z, hd.w, sh, mh);
                        const __half2 sl2 = __half2half2(__int2half_rn(sl)), offl = __half2half2(__int2half_rn(-1024 * sl));
                        const __half2 sh16 = __half2half2(__float2half_rn((float)sh * 0.0625f)),
                                      offh = __half2half2(__int2half_rn(-64 * sh));
                        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                        for (int c = 0; c < 4; c++) {  // chunk 8jj + c: low nibbles of bytes 8c..8c+7, 8jj + 4 + c: high
                            uint32_t a0, a1, b0, b1, c0_, c1_, d0, d1;
                            q4_word_to_h(w[2 * c], sl2, offl, sh16, offh, a0, a1, b0, b1);
                            q4_word_to_h(w[2 * c + 1], sl2, offl, sh16, offh, c0_, c1_, d0, d1);
                            *reinterpret_cast<uint4 *>(tile + ((size_t)(8 * jj + c) * 128 + r) * 16) = make_uint4(a0, a1, c0_, c1_);
                            *reinterpret_cast<uint4 *>(tile + ((size_t)(8 * jj + 4 + c) * 128 + r) * 16) = make_uint4(b0, b1, d0, d1);
                        }
                        if (h == 0 && jj == 0) {  // the super-block's float scales and its 8 mins
                            s_d[pb][mat][r] = f16_to_f32((uint16_t)(hd.x & 0xFFFF));
                            s_dmin[pb][mat][r] = f16_to_f32((uint16_t)(hd.x >> 16));
                            // mins: bytes 4..7 & 63 (sub-blocks 0-3); sub-blocks 4-7: (byte 8+i >> 4) | (byte 4+i >> 6) << 4
                            const uint32_t m0 = hd.z & 0x3F3F3F3Fu;
                            const uint32_t m1 = ((hd.w >> 4) & 0x0F0F0F0Fu) | (((hd.z >> 6) & 0x03030303u) << 4);
                            s_mn[pb][mat][r][0] = m0;
                            s_mn[pb][mat][r][1] = m1;
                        }
                    } else {
                        for (int kc = 8 * jj; kc < 8 * jj + 8; kc++)
                            *reinterpret_cast<uint4 *>(tile + ((size_t)kc * 128 + r) * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
#pragma unroll
                for (int u = 0; u < 2; u++) {  // tokens (prefetched one step ahead): int8 activations -> fp16
                    const int it = t + u * MMA_THREADS;
                    if (it < N * 16) {
                        const int i = it >> 4, kc = it & 15;
                        *reinterpret_cast<uint4 *>(tB + ((size_t)kc * N + i) * 16) =
                            i < nc ? h8_from_i8_fast(px[u].x, px[u].y) : make_uint4(0, 0, 0, 0);
                        if (ks + 1 < KSTEPS && i < nc)
                            px[u] = *reinterpret_cast<const uint2 *>(s_tok[i] + ((ks + 1) >> 1) * 256 + ((ks + 1) & 1) * 128 + kc * 8);
                    }
                }
                if (h == 0)
                    for (int i = t; i < nc; i += MMA_THREADS) {  // tokens' xd and per-32 sums of block blk
                        const int tok = (int)((s_tok[i] - A.x256.q) / dim);
                        s_xd[pb][i] = A.x256.d[(size_t)tok * NBG + blk];
                        const int4 *ss = reinterpret_cast<const int4 *>(A.x256.s + ((size_t)tok * NBG + blk) * 16);
                        uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
                        for (int k4 = 0; k4 < 4; k4++) {  // per-32 sum bs = 256*hi + lo (lo unsigned byte, hi signed)
                            const int4 v = ss[k4];
                            const int b0 = v.x + v.y, b1 = v.z + v.w, k = 2 * k4;
                            lo[k >> 2] |= (uint32_t)(b0 & 0xFF) << (8 * (k & 3));
                            hi[k >> 2] |= (uint32_t)((b0 >> 8) & 0xFF) << (8 * (k & 3));
                            lo[(k + 1) >> 2] |= (uint32_t)(b1 & 0xFF) << (8 * ((k + 1) & 3));
                            hi[(k + 1) >> 2] |= (uint32_t)((b1 >> 8) & 0xFF) << (8 * ((k + 1) & 3));
                        }
                        s_bsp[pb][i] = make_uint4(lo[0], lo[1], hi[0], hi[1]);
                    }
                fence_async_smem();
                __syncthreads();
                if (t == 0) {
                    tc_fence_after();
                    const uint32_t dcol = (uint32_t)b * 2 * MMA_NP;
                    // K step s: the start address field (16-byte units) advances by 2 chunks
                    const uint64_t ag = umma_desc_kmajor(tA, 128), au = umma_desc_kmajor(tA + 16 * 128 * 16, 128);
                    const uint64_t bd = umma_desc_kmajor(tB, (uint32_t)N);
#pragma unroll
                    for (int s = 0; s < 8; s++) {
                        const uint64_t bs = bd + (uint64_t)(2 * s * N);
                        umma_bf16(tmem + dcol, ag + (uint64_t)(256 * s), bs, idesc, s > 0);
                        umma_bf16(tmem + dcol + MMA_NP, au + (uint64_t)(256 * s), bs, idesc, s > 0);
                    }
                    umma_commit(&S.mbar[b]);
                }
                gstep++;
            }
            if (ks >= 1) {  // ---- epilogue of step ks - 1 (its MMAs done), overlapping step ks's MMAs
                const uint32_t ps = gstep - (ks < KSTEPS ? 2 : 1);  // the step to finish
                const int pbuf = ps & 1;
                if (!mma_wait(S, pbuf, (ps >> 1) & 1, A.err)) break;
                tc_fence_after();
                const int pks = (int)(ps - step0), pblk = pks >> 1, ph = pks & 1, pb = pblk & 1;
                if (tok0 < N) {
                    int vg[16], vu[16];
                    const uint32_t dcol = (uint32_t)pbuf * 2 * MMA_NP + (uint32_t)tok0;
                    tmem_ints16(tmem, q, dcol, vg);
                    tmem_ints16(tmem, q, dcol + MMA_NP, vu);
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        Ig[i] = ph ? Ig[i] + vg[i] : vg[i];
                        Iu[i] = ph ? Iu[i] + vu[i] : vu[i];
                    }
                    if (ph == 1) {  // block pblk complete: the reference's float tail, blocks in order
                        const int r = 32 * q + lane;
                        const float dg = s_d[pb][0][r], dmg = s_dmin[pb][0][r];
                        const float du = s_d[pb][1][r], dmu = s_dmin[pb][1][r];
                        const uint32_t mg0 = s_mn[pb][0][r][0], mg1 = s_mn[pb][0][r][1];
                        const uint32_t mu0 = s_mn[pb][1][r][0], mu1 = s_mn[pb][1][r][1];
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const int ti = tok0 + i;
                            if (ti < nc) {
                                // mins term M = sum_sub mn * bs through dp4a on bs = 256*hi + lo (exact)
                                const uint4 bp = s_bsp[pb][ti];
                                const int Mg = (int)__dp4a(mg0, bp.x, __dp4a(mg1, bp.y, 0u)) +
                                               256 * dp4a_us(mg0, (int)bp.z, dp4a_us(mg1, (int)bp.w, 0));
                                const int Mu = (int)__dp4a(mu0, bp.x, __dp4a(mu1, bp.y, 0u)) +
                                               256 * dp4a_us(mu0, (int)bp.z, dp4a_us(mu1, (int)bp.w, 0));
                                const float xd = s_xd[pb][ti];
                                ag[i] = fadd(ag[i], fmul(xd, fsub(fmul(dg, (float)Ig[i]), fmul(dmg, (float)Mg))));
                                au[i] = fadd(au[i], fmul(xd, fsub(fmul(du, (float)Iu[i]), fmul(dmu, (float)Mu))));
                            }
                        }
                    }
                }
                tc_fence_before();
            }
        }
        if (!S.ok) break;
        if (tok0 < nc) {  // act = silu(gate) * up for this warp's tokens of row 32q + lane
            const int row = row0 + 32 * q + lane;
            if (row < ffn)
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    if (tok0 + i >= nc) break;
                    const int slot = shared ? A.T * A.n_used + c0 + tok0 + i : list[c0 + tok0 + i];
                    A.act[(size_t)slot * A.act_stride + row] = fmul(fdiv(ag[i], fadd(1.0f, expf(-ag[i]))), au[i]);
                }
        }
        __syncthreads();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_free(tmem, ncols);
}

constexpr int GU_NP = 32;  // tokens per pass of the pipelined down kernel

__device__ __forceinline__ bool mbar_wait_err(uint64_t *bar, uint32_t parity, int *ok, int *err) {
    if (!*reinterpret_cast<volatile int *>(ok)) return false;
    if (mbar_wait(bar, parity, UMMA_POLLS)) return true;
    if (err) atomicOr(err, 32);
    *reinterpret_cast<volatile int *>(ok) = 0;
    return false;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// ---- down (Q6_K): y[slot][row] = W_down[row] . act[slot] ------------------------------------
// act quantized per slot by quantizeX256 (aq / ad); expert blockIdx.y, output
// rows [128*blockIdx.x, +128). The same two-group pipeline as k_gu_mma. A
// fill thread takes row tf & 127 and the value groups gp and gp + 2 of the
// half super-block (gp = tf >> 7), which share their ql bytes (low and high
// nibbles): A = sc * (q - 32).
template <int NBD>
__device__ __forceinline__ void dn_fetch_w(uint4 (&pq)[4], uint32_t &scw, float &d, const WDev &wd, uint64_t plane,
                                           int row0, int dim, int ks, int tf) {
    const int r = tf & 127, gp = tf >> 7, row = row0 + r, h = ks & 1;
    if (row >= dim) return;
    const uint64_t gb = plane + (uint64_t)row * NBD + (ks >> 1);
    const uint8_t *qb = wd.q + gb * 192;
    pq[0] = ld_stream_v4(qb + 64 * h + 32 * gp);
    pq[1] = ld_stream_v4(qb + 64 * h + 32 * gp + 16);
    pq[2] = ld_stream_v4(qb + 128 + 32 * h);
    pq[3] = ld_stream_v4(qb + 128 + 32 * h + 16);
    const uint8_t *scb = wd.sc + gb * 16 + 8 * h;  // groups g: scales scb[2g] (l < 16), scb[2g + 1]
    scw = (uint32_t)scb[2 * gp] | ((uint32_t)scb[2 * gp + 1] << 8) | ((uint32_t)scb[2 * gp + 4] << 16) |
          ((uint32_t)scb[2 * gp + 5] << 24);
    d = f16_to_f32(wd.d[gb]);
}

template <int NBD>
__global__ void __launch_bounds__(MMA_THREADS, 1) k_dn_mma(DecodeArgs A) {
    constexpr int KSTEPS = NBD * 2;
    constexpr size_t A_BYTES = (size_t)16 * 128 * 16, B_BYTES = (size_t)16 * GU_NP * 16;
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t full[2], done[2], sfree[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_ok;
    __shared__ float s_d[2][128], s_xd[2][GU_NP];
    __shared__ const int8_t *s_act[GU_NP];
    umma_pdl_wait();
    const int e = blockIdx.y;
    const bool shared = e == A.n_local;
    const int n = shared ? A.T : A.grp_cnt[e];
    const int row0 = blockIdx.x * 128;
    if (n == 0 || row0 >= A.dim) return;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const bool fillg = warp < 8;
    const int *list = shared ? nullptr : A.grp_list + A.grp_off[e];
    const WDev wd = shared ? A.sdn : A.dn;
    const uint64_t plane = shared ? 0 : (uint64_t)e * A.dim * NBD;
    const int stride = A.act_stride;
    const uint32_t ncols = 2 * GU_NP;
    if (warp == 0) tmem_alloc(&s_tmem, ncols);
    if (t == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&done[i], 1);
            mbar_init(&sfree[i], 1);
        }
        s_ok = 1;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    uint32_t g0 = 0;
    for (int c0 = 0; c0 < n; c0 += GU_NP) {
        const int nc = n - c0 < GU_NP ? n - c0 : GU_NP, N = (nc + 15) / 16 * 16;
        const uint32_t idesc = umma_idesc_f16_f32(128, N);
        for (int i = t; i < nc; i += MMA_THREADS) {
            const int slot = shared ? A.T * A.n_used + c0 + i : list[c0 + i];
            s_act[i] = A.aq + (size_t)slot * stride;
        }
        __syncthreads();
        if (fillg) {
            const int tf = t, r = tf & 127, gp = tf >> 7, row = row0 + r;
            uint4 pq[4];
            uint32_t pscw = 0;
            float pd = 0.0f;
            dn_fetch_w<NBD>(pq, pscw, pd, wd, plane, row0, A.dim, 0, tf);
            uint2 px[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int it = tf + u * 256;
                if (it < N * 16 && (it >> 4) < nc) px[u] = *reinterpret_cast<const uint2 *>(s_act[it >> 4] + (it & 15) * 8);
            }
            const __half2 k1056 = u2h(0x64206420u);  // 1056 = 1024 + 32
            for (int ks = 0; ks < KSTEPS; ks++) {
                const uint32_t g = g0 + ks;
                const int b = g & 1, blk = ks >> 1, h = ks & 1, pb = blk & 1;
                if (g >= 2 && tf == 0) mbar_wait_err(&sfree[b], ((g >> 1) - 1) & 1, &s_ok, A.err);
                named_sync(1, 256);
                uint8_t *tA = sm + (size_t)b * (A_BYTES + B_BYTES), *tB = tA + A_BYTES;
                const uint4 ql0 = pq[0], ql1 = pq[1], qh0 = pq[2], qh1 = pq[3];
                const uint32_t scw = pscw;
                const float dcur = pd;
                if (ks + 1 < KSTEPS) dn_fetch_w<NBD>(pq, pscw, pd, wd, plane, row0, A.dim, ks + 1, tf);
                if (row < A.dim) {
                    const uint32_t qlw[8] = {ql0.x, ql0.y, ql0.z, ql0.w, ql1.x, ql1.y, ql1.z, ql1.w};
                    const uint32_t qhw[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
#pragma unroll
                    for (int gi = 0; gi < 2; gi++) {  // group g = gp + 2 gi: low (gi 0) or high (gi 1) nibbles
                        const int gg = gp + 2 * gi;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const int sc = (int)(int8_t)((scw >> (16 * gi + 8 * (c >> 1))) & 0xFF);
                            const __half2 sc2 = __half2half2(__int2half_rn(sc));
                            uint32_t o[4];
#pragma unroll
                            for (int wi = 0; wi < 2; wi++) {
                                const uint32_t lw = qlw[2 * c + wi], hw = qhw[2 * c + wi];
                                const uint32_t lo4 = (gi ? lw >> 4 : lw) & 0x0F0F0F0Fu;
                                const uint32_t qb = lo4 | (((hw >> (2 * gg)) & 0x03030303u) << 4);
                                o[2 * wi] = h2u(__hmul2(__hsub2(u2h(__byte_perm(qb, 0x64646464u, 0x7170)), k1056), sc2));
                                o[2 * wi + 1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(qb, 0x64646464u, 0x7372)), k1056), sc2));
                            }
                            *reinterpret_cast<uint4 *>(tA + ((size_t)(4 * gg + c) * 128 + r) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                    if (h == 0 && gp == 0) s_d[pb][r] = dcur;
                } else {
                    for (int gi = 0; gi < 2; gi++)
                        for (int c = 0; c < 4; c++)
                            *reinterpret_cast<uint4 *>(tA + ((size_t)(4 * (gp + 2 * gi) + c) * 128 + r) * 16) = make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < 2; u++) {  // activations (prefetched one step ahead): int8 -> fp16
                    const int it = tf + u * 256;
                    if (it < N * 16) {
                        const int i = it >> 4, kc = it & 15;
                        *reinterpret_cast<uint4 *>(tB + ((size_t)kc * N + i) * 16) =
                            i < nc ? h8_from_i8_fast(px[u].x, px[u].y) : make_uint4(0, 0, 0, 0);
                        if (ks + 1 < KSTEPS && i < nc)
                            px[u] = *reinterpret_cast<const uint2 *>(s_act[i] + ((ks + 1) >> 1) * 256 + ((ks + 1) & 1) * 128 + kc * 8);
                    }
                }
                if (h == 0)
                    for (int i = tf; i < nc; i += 256) {
                        const size_t slot = (size_t)(s_act[i] - A.aq) / stride;
                        s_xd[pb][i] = A.ad[slot * (stride / 32) + blk];
                    }
                fence_async_smem();
                named_sync(1, 256);
                if (tf == 0) mbar_arrive(&full[b]);
            }
        } else {
            const int we = warp - 8, q = we & 3, tok0 = 16 * (we >> 2);
            const bool lead = t == 256;
            int I[16];
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; i++) acc[i] = 0.0f;
            auto issue = [&](uint32_t g) {
                const int b = g & 1;
                if (!mbar_wait_err(&full[b], (g >> 1) & 1, &s_ok, A.err)) return;
                tc_fence_after();
                uint8_t *tA = sm + (size_t)b * (A_BYTES + B_BYTES), *tB = tA + A_BYTES;
                const uint64_t ad = umma_desc_kmajor(tA, 128), bd = umma_desc_kmajor(tB, (uint32_t)N);
#pragma unroll
                for (int s2 = 0; s2 < 8; s2++)
                    umma_bf16(tmem + (uint32_t)b * GU_NP, ad + (uint64_t)(256 * s2), bd + (uint64_t)(2 * s2 * N), idesc,
                              s2 > 0);
                umma_commit(&done[b]);
            };
            if (lead) issue(g0);
            for (int ks = 0; ks < KSTEPS; ks++) {
                const uint32_t g = g0 + ks;
                const int b = g & 1, blk = ks >> 1, h = ks & 1, pb = blk & 1;
                if (lead) {
                    if (ks + 1 < KSTEPS) issue(g + 1);
                    if (mbar_wait_err(&done[b], (g >> 1) & 1, &s_ok, A.err)) mbar_arrive(&sfree[b]);
                }
                named_sync(2, 256);
                tc_fence_after();
                if (tok0 < N) {
                    int v[16];
                    tmem_ints16(tmem, q, (uint32_t)b * GU_NP + (uint32_t)tok0, v);
#pragma unroll
                    for (int i = 0; i < 16; i++) I[i] = h ? I[i] + v[i] : v[i];
                }
                tc_fence_before();
                named_sync(2, 256);
                if (h == 1 && tok0 < N) {
                    const float d = s_d[pb][32 * q + lane];
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        if (tok0 + i < nc) acc[i] = fadd(acc[i], fmul(fmul(s_xd[pb][tok0 + i], d), (float)I[i]));
                }
            }
            if (s_ok && tok0 < nc) {
                const int row = row0 + 32 * q + lane;
                if (row < A.dim)
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        if (tok0 + i >= nc) break;
                        const int slot = shared ? A.T * A.n_used + c0 + tok0 + i : list[c0 + tok0 + i];
                        A.y[(size_t)slot * A.dim + row] = acc[i];
                    }
            }
        }
        g0 += KSTEPS;
        __syncthreads();
        if (!s_ok) break;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_free(tmem, ncols);
}

using MmaFn = void (*)(DecodeArgs);

static MmaFn gu_mma_fn(int nbg) {
    switch (nbg) {
        case 4: return k_gu_mma<4>;
        case 8: return k_gu_mma<8>;
        case 16: return k_gu_mma<16>;
        case 28: return k_gu_mma<28>;
    }
    return nullptr;
}
static MmaFn dn_mma_fn(int nbd) {
    switch (nbd) {
        case 2: return k_dn_mma<2>;
        case 3: return k_dn_mma<3>;
        case 4: return k_dn_mma<4>;
        case 8: return k_dn_mma<8>;
    }
    return nullptr;
}

static constexpr size_t GU_MMA_SMEM = (size_t)2 * ((size_t)2 * 16 * 128 * 16 + (size_t)16 * MMA_NP * 16);
static constexpr size_t DN_MMA_SMEM = (size_t)2 * ((size_t)16 * 128 * 16 + (size_t)16 * GU_NP * 16);

bool moe_mma_supported(const DecodeArgs &A) {
    if (A.g.type != T_Q4_K || A.u.type != T_Q4_K || A.dn.type != T_Q6_K) return false;
    if (A.dim % 256 || A.ffn % 256) return false;
    if (!gu_mma_fn(A.dim / 256) || !dn_mma_fn(A.ffn / 256)) return false;
    if (A.has_shared && (A.sg.type != T_Q4_K || A.su.type != T_Q4_K || A.sdn.type != T_Q6_K || A.shexp_ffn != A.ffn))
        return false;
    return true;
}

// gate/up on the tensor cores, the activations' quantization, down on the
// tensor cores: after the grouping kernel, before the combine.
cudaError_t launch_moe_mma(const DecodeArgs &A, cudaStream_t st, cudaError_t (*quant)(const DecodeArgs &, cudaStream_t)) {
    const int nexp = A.n_local + (A.has_shared ? 1 : 0);
    const int mffn = A.has_shared && A.shexp_ffn > A.ffn ? A.shexp_ffn : A.ffn;
    MmaFn gf = gu_mma_fn(A.dim / 256), df = dn_mma_fn(A.ffn / 256);
    cudaError_t e = cudaFuncSetAttribute(gf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GU_MMA_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(df, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DN_MMA_SMEM);
    if (e != cudaSuccess) return e;
    count_launch();
    gf<<<dim3(cdivu(mffn, 128), (unsigned)nexp), MMA_THREADS, GU_MMA_SMEM, st>>>(A);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = quant(A, st)) != cudaSuccess) return e;
    count_launch();
    df<<<dim3(cdivu(A.dim, 128), (unsigned)nexp), MMA_THREADS, DN_MMA_SMEM, st>>>(A);
    return cudaGetLastError();
}

}  // namespace loom
