// gemv.cuh -- one-token matvec (ggml.matvec, ggml.zig:602) for the model
// step: out[r] = W[r] . x for the quantized activations x of one vector.
#pragma once
#include "kernels.cuh"

namespace loom {

// True when the warp engine takes this type and width (Q4_K, Q6_K, Q8_0,
// Q4_0 with at most 32 / 64 blocks per row); otherwise the caller uses launch_mm.
bool gemv_supported(int type, int cols);
// Launched with programmatic dependent launch: the weight loads are issued
// before the wait for the kernel that wrote x. Bit-identical to launch_mm.
cudaError_t launch_gemv(const WDev &w, int rows, int cols, const XQ &x, float *out, cudaStream_t st);
// Large matrices (>= 4096 rows, Q4_K or Q6_K with nb % 8 == 0, up to 128 blocks
// a row): tiles streamed through shared memory by bulk copies, one CTA per SM.
// Bit-identical to launch_gemv / launch_mm.
// res (optional): out[r] = res[r] + W[r] . x (the residual add, llama.zig's x + ffn).
bool gemv_stream_supported(int type, int rows, int cols);
bool gemv_stream_shape_ok(int type, int cols);  // any row count
cudaError_t launch_gemv_stream(const WDev &w, int rows, int cols, const XQ &x, float *out, cudaStream_t st,
                               const float *res = nullptr);

}  // namespace loom
