// umma.cu -- tensor-core (tcgen05) kernels: the bf16 GEMM building block and
// its self-test entry point.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "umma.cuh"

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
    __shared__ int s_bs[2][MMA_NP][8];
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
        for (int ks = 0; ks <= KSTEPS; ks++) {
            if (ks < KSTEPS) {  // ---- stage step ks into buffer gstep & 1 (its previous MMAs were awaited below)
                const int b = gstep & 1, blk = ks >> 1, h = ks & 1, pb = blk & 1;
                uint8_t *tA = sm + (size_t)b * (A_BYTES + B_BYTES), *tB = tA + A_BYTES;
                {   // weights: thread -> (matrix, row, sub-block pair jj of this half)
                    const int mat = t >> 8, r = (t >> 1) & 127, jj = t & 1, row = row0 + r;
                    uint8_t *tile = tA + (size_t)mat * 16 * 128 * 16;
                    if (row < ffn) {
                        const uint8_t *bp = (mat ? wu : wg).q + (plane + (uint64_t)row * NBG + blk) * 144;
                        const uint4 hd = *reinterpret_cast<const uint4 *>(bp);
                        const int j = 2 * h + jj;
                        const uint4 q0 = *reinterpret_cast<const uint4 *>(bp + 16 + 32 * j);
                        const uint4 q1 = *reinterpret_cast<const uint4 *>(bp + 32 + 32 * j);
                        int sl, ml, sh, mh;
                        scale_min_k4w(2 * j, hd.y, hd.z, hd.w, sl, ml);
                        scale_min_k4w(2 * j + 1, hd.y, hd.z, hd.w, sh, mh);
                        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                        for (int c = 0; c < 4; c++) {  // chunk 8jj + c: low nibbles, 8jj + 4 + c: high
                            const uint32_t a = w[2 * c], bb = w[2 * c + 1];
                            auto nb = [](uint32_t x, int i, int sh4) { return (int)((x >> (8 * i + sh4)) & 0xF); };
                            *reinterpret_cast<uint4 *>(tile + ((size_t)(8 * jj + c) * 128 + r) * 16) =
                                make_uint4(h2i(sl * nb(a, 0, 0), sl * nb(a, 1, 0)), h2i(sl * nb(a, 2, 0), sl * nb(a, 3, 0)),
                                           h2i(sl * nb(bb, 0, 0), sl * nb(bb, 1, 0)), h2i(sl * nb(bb, 2, 0), sl * nb(bb, 3, 0)));
                            *reinterpret_cast<uint4 *>(tile + ((size_t)(8 * jj + 4 + c) * 128 + r) * 16) =
                                make_uint4(h2i(sh * nb(a, 0, 4), sh * nb(a, 1, 4)), h2i(sh * nb(a, 2, 4), sh * nb(a, 3, 4)),
                                           h2i(sh * nb(bb, 0, 4), sh * nb(bb, 1, 4)), h2i(sh * nb(bb, 2, 4), sh * nb(bb, 3, 4)));
                        }
                        if (h == 0 && jj == 0) {  // the super-block's float scales and its 8 mins
                            s_d[pb][mat][r] = f16_to_f32((uint16_t)(hd.x & 0xFFFF));
                            s_dmin[pb][mat][r] = f16_to_f32((uint16_t)(hd.x >> 16));
                            uint32_t m0 = 0, m1 = 0;
#pragma unroll
                            for (int sbk = 0; sbk < 8; sbk++) {
                                int sc_, mn_;
                                scale_min_k4w(sbk, hd.y, hd.z, hd.w, sc_, mn_);
                                if (sbk < 4) m0 |= (uint32_t)mn_ << (8 * sbk);
                                else m1 |= (uint32_t)mn_ << (8 * (sbk - 4));
                            }
                            s_mn[pb][mat][r][0] = m0;
                            s_mn[pb][mat][r][1] = m1;
                        }
                    } else {
                        for (int kc = 8 * jj; kc < 8 * jj + 8; kc++)
                            *reinterpret_cast<uint4 *>(tile + ((size_t)kc * 128 + r) * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                for (int it = t; it < N * 16; it += MMA_THREADS) {  // tokens: int8 activations -> fp16
                    const int i = it >> 4, kc = it & 15;
                    uint4 v4 = make_uint4(0, 0, 0, 0);
                    if (i < nc) {
                        const int slot = shared ? A.T * A.n_used + c0 + i : list[c0 + i];
                        const int tok = shared ? c0 + i : slot / A.n_used;
                        const uint2 x8 = *reinterpret_cast<const uint2 *>(A.x256.q + (size_t)tok * dim + blk * 256 +
                                                                          h * 128 + kc * 8);
                        v4 = h8_from_i8(x8.x, x8.y);
                    }
                    *reinterpret_cast<uint4 *>(tB + ((size_t)kc * N + i) * 16) = v4;
                }
                if (h == 0)
                    for (int it = t; it < nc * 9; it += MMA_THREADS) {  // tokens' xd and per-32 sums of block blk
                        const int i = it / 9, k = it % 9;
                        const int slot = shared ? A.T * A.n_used + c0 + i : list[c0 + i];
                        const int tok = shared ? c0 + i : slot / A.n_used;
                        if (k == 8) s_xd[pb][i] = A.x256.d[(size_t)tok * NBG + blk];
                        else {
                            const int32_t *ss = A.x256.s + ((size_t)tok * NBG + blk) * 16 + 2 * k;
                            s_bs[pb][i][k] = ss[0] + ss[1];
                        }
                    }
                fence_async_smem();
                __syncthreads();
                if (t == 0) {
                    tc_fence_after();
                    const uint32_t dcol = (uint32_t)b * 2 * MMA_NP;
#pragma unroll
                    for (int s = 0; s < 8; s++) {
                        const uint64_t bd = umma_desc_kmajor(tB + (size_t)2 * s * N * 16, (uint32_t)N);
                        umma_bf16(tmem + dcol, umma_desc_kmajor(tA + 2 * s * 128 * 16, 128), bd, idesc, s > 0);
                        umma_bf16(tmem + dcol + MMA_NP, umma_desc_kmajor(tA + 16 * 128 * 16 + 2 * s * 128 * 16, 128),
                                  bd, idesc, s > 0);
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
                                int Mg = 0, Mu = 0;
#pragma unroll
                                for (int sb = 0; sb < 8; sb++) {
                                    const int bs = s_bs[pb][ti][sb];
                                    Mg += (int)(((sb < 4 ? mg0 : mg1) >> (8 * (sb & 3))) & 0xFF) * bs;
                                    Mu += (int)(((sb < 4 ? mu0 : mu1) >> (8 * (sb & 3))) & 0xFF) * bs;
                                }
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

// ---- down (Q6_K): y[slot][row] = W_down[row] . act[slot] ------------------------------------
// act quantized per slot by quantizeX256 (aq / ad); expert blockIdx.y, output
// rows [128*blockIdx.x, +128).
template <int NBD>
__global__ void __launch_bounds__(MMA_THREADS, 1) k_dn_mma(DecodeArgs A) {
    constexpr int KSTEPS = NBD * 2;
    constexpr size_t A_BYTES = (size_t)16 * 128 * 16, B_BYTES = (size_t)16 * MMA_NP * 16;
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ MmaCtl S;
    __shared__ float s_d[2][128], s_xd[2][MMA_NP];
    umma_pdl_wait();
    const int e = blockIdx.y;
    const bool shared = e == A.n_local;
    const int n = shared ? A.T : A.grp_cnt[e];
    const int row0 = blockIdx.x * 128;
    if (n == 0 || row0 >= A.dim) return;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, q = warp & 3, tg = warp >> 2;
    const int *list = shared ? nullptr : A.grp_list + A.grp_off[e];
    const WDev wd = shared ? A.sdn : A.dn;
    const uint64_t plane = shared ? 0 : (uint64_t)e * A.dim * NBD;
    const int stride = A.act_stride;
    const uint32_t ncols = 2 * MMA_NP;
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
    uint32_t gstep = 0;
    for (int c0 = 0; c0 < n && S.ok; c0 += MMA_NP) {
        const int nc = n - c0 < MMA_NP ? n - c0 : MMA_NP, N = (nc + 15) / 16 * 16;
        const uint32_t idesc = umma_idesc_f16_f32(128, N);
        const int tok0 = 16 * tg;
        int I[16];
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; i++) acc[i] = 0.0f;
        const uint32_t step0 = gstep;
        for (int ks = 0; ks <= KSTEPS; ks++) {
            if (ks < KSTEPS) {
                const int b = gstep & 1, blk = ks >> 1, h = ks & 1, pb = blk & 1;
                uint8_t *tA = sm + (size_t)b * (A_BYTES + B_BYTES), *tB = tA + A_BYTES;
                {   // weights: thread -> (row, group g of the half): values 32g + l, l < 32 -> chunks 4g .. 4g+3
                    const int r = t >> 2, g = t & 3, row = row0 + r;
                    if (row < A.dim) {
                        const uint64_t gb = plane + (uint64_t)row * NBD + blk;
                        const uint8_t *qb = wd.q + gb * 192;
                        const int8_t *scb = reinterpret_cast<const int8_t *>(wd.sc + gb * 16) + 8 * h;
                        const int s0 = scb[2 * g], s1 = scb[2 * g + 1];  // l < 16, l >= 16
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint2 qlw = *reinterpret_cast<const uint2 *>(qb + 64 * h + 32 * (g & 1) + 8 * c);
                            const uint2 qhw = *reinterpret_cast<const uint2 *>(qb + 128 + 32 * h + 8 * c);
                            const int sc = c < 2 ? s0 : s1;
                            int v[8];
#pragma unroll
                            for (int i = 0; i < 8; i++) {
                                const uint32_t lw = i < 4 ? qlw.x : qlw.y, hw = i < 4 ? qhw.x : qhw.y;
                                const uint32_t lb = (lw >> (8 * (i & 3))) & 0xFF, hb = (hw >> (8 * (i & 3))) & 0xFF;
                                const int qv = (int)((g >= 2 ? lb >> 4 : lb & 0xF) | (((hb >> (2 * g)) & 3) << 4));
                                v[i] = sc * (qv - 32);
                            }
                            *reinterpret_cast<uint4 *>(tA + ((size_t)(4 * g + c) * 128 + r) * 16) =
                                make_uint4(h2i(v[0], v[1]), h2i(v[2], v[3]), h2i(v[4], v[5]), h2i(v[6], v[7]));
                        }
                        if (h == 0 && g == 0) s_d[pb][r] = f16_to_f32(wd.d[gb]);
                    } else {
                        for (int kc = 4 * g; kc < 4 * g + 4; kc++)
                            *reinterpret_cast<uint4 *>(tA + ((size_t)kc * 128 + r) * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                for (int it = t; it < N * 16; it += MMA_THREADS) {  // int8 activations -> fp16
                    const int i = it >> 4, kc = it & 15;
                    uint4 v4 = make_uint4(0, 0, 0, 0);
                    if (i < nc) {
                        const int slot = shared ? A.T * A.n_used + c0 + i : list[c0 + i];
                        const uint2 x8 =
                            *reinterpret_cast<const uint2 *>(A.aq + (size_t)slot * stride + blk * 256 + h * 128 + kc * 8);
                        v4 = h8_from_i8(x8.x, x8.y);
                    }
                    *reinterpret_cast<uint4 *>(tB + ((size_t)kc * N + i) * 16) = v4;
                }
                if (h == 0)
                    for (int i = t; i < nc; i += MMA_THREADS) {
                        const int slot = shared ? A.T * A.n_used + c0 + i : list[c0 + i];
                        s_xd[pb][i] = A.ad[(size_t)slot * (stride / 32) + blk];
                    }
                fence_async_smem();
                __syncthreads();
                if (t == 0) {
                    tc_fence_after();
                    const uint32_t dcol = (uint32_t)b * MMA_NP;
#pragma unroll
                    for (int s = 0; s < 8; s++)
                        umma_bf16(tmem + dcol, umma_desc_kmajor(tA + 2 * s * 128 * 16, 128),
                                  umma_desc_kmajor(tB + (size_t)2 * s * N * 16, (uint32_t)N), idesc, s > 0);
                    umma_commit(&S.mbar[b]);
                }
                gstep++;
            }
            if (ks >= 1) {
                const uint32_t ps = gstep - (ks < KSTEPS ? 2 : 1);
                const int pbuf = ps & 1;
                if (!mma_wait(S, pbuf, (ps >> 1) & 1, A.err)) break;
                tc_fence_after();
                const int pks = (int)(ps - step0), pblk = pks >> 1, ph = pks & 1, pb = pblk & 1;
                if (tok0 < N) {
                    int v[16];
                    tmem_ints16(tmem, q, (uint32_t)pbuf * MMA_NP + (uint32_t)tok0, v);
#pragma unroll
                    for (int i = 0; i < 16; i++) I[i] = ph ? I[i] + v[i] : v[i];
                    if (ph == 1) {
                        const float d = s_d[pb][32 * q + lane];
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if (tok0 + i < nc) acc[i] = fadd(acc[i], fmul(fmul(s_xd[pb][tok0 + i], d), (float)I[i]));
                    }
                }
                tc_fence_before();
            }
        }
        if (!S.ok) break;
        if (tok0 < nc) {
            const int row = row0 + 32 * q + lane;
            if (row < A.dim)
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    if (tok0 + i >= nc) break;
                    const int slot = shared ? A.T * A.n_used + c0 + tok0 + i : list[c0 + tok0 + i];
                    A.y[(size_t)slot * A.dim + row] = acc[i];
                }
        }
        __syncthreads();
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
static constexpr size_t DN_MMA_SMEM = (size_t)2 * ((size_t)16 * 128 * 16 + (size_t)16 * MMA_NP * 16);

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
