// attn_block.cuh -- the attention half of a decoder layer as one cooperative
// launch (attn_block.cu).
#pragma once
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace loom {

constexpr int MAX_AB_HD = 256;

struct AttnBlockArgs {
    float *x;                  // [dim] residual stream: x += W_o . attention (in place)
    float *normed;             // [dim] out: RMSNorm(x) * ffn_norm, the FFN's input; null: not computed
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
    float eps;
    int serial;                // RMSNorm sum of squares in the reference's serial order
    WDev wq, wk, wv, wo;
    int dim, n_heads, n_kv, hd, rope_dim, neox;
    const float *rope;         // [ctx][rope_dim / 2] (cos, sin)
    float scale;
    const uint32_t *pos;
    int ctx;
    float *kc, *vc;            // this layer's cache [ctx][n_kv * hd]
    float *q, *k, *v, *part;   // scratch
    int nsplit;
    int8_t *aq;                // quantized attention output (the output projection's input)
    float *ad;
    int32_t *as;
    unsigned long long *bar;   // zeroed 32 bytes: arrival counter, epoch + exit count, error word
    unsigned long long *trace; // optional [8]: %globaltimer ns of CTA 0 at the phase boundaries (diagnostic)
    // set by attn_block_plan
    int groups, so, ta, tv, to;
    int merge_bulk;             // the merge CTAs bulk-copy their heads' partial records into shared memory
    size_t smem, off_o, off_u;  // dynamic shared memory: total, staged output-projection rows, union area
};

// Fills the plan fields; 0 when the fused kernel does not take these types or
// shapes (the caller then runs the separate kernels).
int attn_block_plan(AttnBlockArgs &A, int type_q, int type_k, int type_v, int type_o, size_t ctx);
cudaError_t launch_attn_block(const AttnBlockArgs &A, cudaStream_t st);

}  // namespace loom
