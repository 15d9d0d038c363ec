// model_kernel.cuh -- every layer of a decode step in ONE persistent
// cooperative launch (model_kernel.cu): the attention half of each layer as in
// attn_block.cu, then its routed MoE FFN (router, route, gate/up + SwiGLU,
// down + ordered combine + residual), the layers in sequence inside the
// kernel. The code and the grid stay resident for the whole token.
#pragma once
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace loom {

// One decoder layer as the persistent kernel reads it (device array).
struct MkLayer {
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
    WDev wq, wk, wv, wo;
    float *kc, *vc;         // this layer's cache [ctx][n_kv * hd]
    const float *router;    // f32 [n_expert][dim]
    const float *bias;      // selection bias [n_expert] or null
    WDev g, u, dn;          // gate/up [n_expert][ffn][dim], down [n_expert][dim][ffn]
};

struct MkArgs {
    const MkLayer *layers;  // device array [n_layers]
    int n_layers;
    int dim, n_heads, n_kv, hd, rope_dim, neox;
    const float *rope;      // [ctx][rope_dim / 2] (cos, sin)
    float scale, eps;
    int serial;             // RMSNorm sums in the reference's serial order
    const uint32_t *pos;
    int ctx;
    int n_expert, n_used, ffn, gating, weights_norm;
    float weights_scale;
    float *x;               // [dim] in: the token's embedding row; out: the residual stream after the last layer
    float *q, *k, *v, *part;
    int nsplit;
    int8_t *aq;             // quantized attention output
    float *ad;
    int32_t *as;
    float *logits;          // [n_expert]
    float *act;             // [n_used][ffn] SwiGLU activations
    uint32_t *ids_out;      // optional [n_layers][n_used] routing
    unsigned long long *bar;  // zeroed 32 words: arrival counter, epoch + exit count, error word
    unsigned long long *trace;  // optional diagnostic timestamps (CTA 0), or null
    // set by model_kernel_plan
    int groups, so;
    size_t smem, off_r1, off_r2;
};

// 0 when the persistent kernel does not take this model (types, shapes,
// shared memory); the caller then launches per layer.
int model_kernel_plan(MkArgs &A, int type_q, int type_k, int type_v, int type_o, int type_g, int type_u,
                      int type_d);
cudaError_t launch_model_kernel(const MkArgs &A, cudaStream_t st);

}  // namespace loom
