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
