// decode.cuh -- arguments of the fused MoE decode path (decode.cu).
#pragma once
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace loom {

struct XQW {  // writable quantized-activation buffers
    int8_t *q;
    float *d;
    int32_t *s;
};

struct DecodeArgs {
    int T, dim, ffn, n_expert, n_used;
    int gating, weights_norm;
    float weights_scale;
    int n_group, topk_group; // group-limited selection (1, 1: plain top-k)
    int expert0, n_local;
    const float *router;     // f32 [n_expert][dim], or null when logits_in is given
    const float *bias;       // selection bias [n_expert] or null
    const float *logits_in;  // caller logits [T][n_expert] (router == null)
    const int *ids_in;       // optional routing decided elsewhere [T][n_used] (then no router, no route) ...
    const float *gates_in;   // ... with these gates (null: 1.0)
    const float *x;          // [T][dim]
    const float *prenorm_w;  // T = 1 router kernels: x is the raw residual stream, normed in the
    float prenorm_eps;       // prologue as RMSNorm(x) * prenorm_w (null: x is already the FFN input)
    float *out;              // [T][dim]
    const float *residual;   // [T][dim] or null
    float *logits;           // scratch [T][n_expert]
    int *ids;                // scratch [T][n_used]
    float *gates;            // scratch [T][n_used]
    uint32_t *ids_out;       // optional copy of ids for the caller
    int *cnt_tok;            // zeroed counters [T]
    int *cnt_slot;           // zeroed counters [n_slots]
    XQW x256, x32;
    int need256, need32;
    WDev g, u, dn;
    int has_shared;
    WDev sg, su, sdn;
    int shexp_ffn;
    float *act;              // [n_slots][act_stride]
    int8_t *aq;              // [n_slots][act_stride]
    float *ad;               // [n_slots][act_stride/32]
    int32_t *as;             // [n_slots][act_stride/16]
    int act_stride;          // multiple of 256
    // expert-major batch path (launch_batch): tokens grouped per local expert
    int *grp_cnt;            // [n_local] slots per local expert
    int *grp_off;            // [n_local] first position in grp_list
    int *grp_list;           // [T*n_used] routed slots, grouped by expert, slot order within a group
    int *tc_pre;             // [n_local + 2] tiled expert kernels: chunks of tc_chunk slots before each expert
    int tc_chunk;            // slots per tile of the tiled expert kernels (0: none)
    float *y;                // [n_slots][dim] per-slot down outputs
    int trace_reg;           // test hook: use the register-staged router instead of the TMA one
    int *err;                // device error word (bounded waits that timed out), or null
    const uint8_t *next_router;   // optional: the next layer's router weights, prefetched into L2
    size_t next_router_bytes;
    unsigned long long *trace;  // optional [2*k] (first start, last end) globaltimer ns per kernel, or null
    int trace_slot;             // this layer's first kernel index in `trace`
};

// True when the fused decode kernels cover this layer's types and shapes.
bool decode_supported(const DecodeArgs &A);
// Enqueue the three PDL-chained kernels of one layer.
cudaError_t launch_decode(const DecodeArgs &A, cudaStream_t st);
// Expert-major batch path (any T): router, grouping, gate/up per expert with
// every token of the expert against one read of its rows, activation
// quantization, down per expert, ordered combine.
bool batch_supported(const DecodeArgs &A);
// path: BATCH_GRP the int8 dot kernels per expert, BATCH_MMA gate/up and down
// on the tensor cores (moe_mma_supported), BATCH_DP4A the tiled dp4a kernels
// (moe_dp4a_supported)
enum { BATCH_GRP = 2, BATCH_MMA = 3, BATCH_DP4A = 4 };
cudaError_t launch_batch(const DecodeArgs &A, int path, cudaStream_t st);
bool moe_mma_supported(const DecodeArgs &A);
extern int g_tc_exact;  // tensor-core arithmetic: 1 integer-exact, 0 dequantized fp16 (default)
bool moe_dp4a_supported(const DecodeArgs &A);
constexpr int MOE_DP_CH = 16;  // slots per dp4a tile
cudaError_t launch_moe_dp4a(const DecodeArgs &A, cudaStream_t st,
                            cudaError_t (*quant)(const DecodeArgs &, cudaStream_t));
constexpr int MOE_TC_N = 64;  // slots per tensor-core tile
// Largest |scale| of a Q6_K scales region (nblk x 16 int8); synchronises st. -1 on error.
int q6k_max_scale(const uint8_t *sc, uint64_t nblk, int *d_tmp, cudaStream_t st);
cudaError_t launch_moe_mma(const DecodeArgs &A, cudaStream_t st,
                           cudaError_t (*quant)(const DecodeArgs &, cudaStream_t));

}  // namespace loom

namespace loom {

// One decode step (T = 1) through a stack of MoE layers in ONE persistent
// cooperative kernel: x_{l+1} = x_l + MoE_l(x_l), phases separated by grid
// barriers instead of kernel boundaries.
struct StackLayer {
    const float *router;  // f32 [n_expert][dim]
    WDev g, u, dn;        // [n_expert][ffn][dim], [n_expert][dim][ffn]
};

struct StackArgs {
    const StackLayer *layers;  // device array [n_layers]
    int n_layers;
    int dim, ffn, n_expert, n_used;
    int gating, weights_norm;
    float weights_scale;
    const float *x_in;
    const float *residual;     // optional: the last layer's output adds its experts to this instead of its x
    float *part;               // [2][n_used][dim] gate-weighted expert outputs (by layer parity)
    float *out;                // [dim] output of the last layer
    unsigned long long *logits; // [LOGIT_REPLICAS][n_expert + 32] tagged words (float bits | layer tag << 32)
    unsigned long long *act;   // [n_used][act_stride] tagged words
    uint32_t *ids_out;         // optional [n_layers][n_used]
    unsigned *bar;             // zeroed 256 bytes: [8,12) err, [16,20) launch epoch, [24,28) exit count,
                               // [32,48) parts arrival counters (u64) by layer parity
    int *err;                  // device error word (2: a grid barrier gave up, 4: router staging timed out)
    int act_stride;
    unsigned long long *trace; // optional [n_layers][STACK_TRACE_SLOTS] %globaltimer ns (zeroed; max-reduced)
};
constexpr int LOGIT_REPLICAS = 16;  // copies of the router logits (stride n_expert + 32): every CTA reads them
constexpr int STACK_TRACE_SLOTS = 12;
// After the 12 timer slots of a layer: STACK_CYC_SECTIONS pairs (max over
// CTAs, sum over CTAs) of thread 0's clock64 cycles spent in each section.
constexpr int STACK_CYC_SECTIONS = 16;
constexpr int STACK_TRACE_WORDS = STACK_TRACE_SLOTS + 2 * STACK_CYC_SECTIONS;

bool stack_supported(const StackArgs &S, int g_type, int dn_type);
cudaError_t launch_stack(const StackArgs &S, int g_type, int dn_type, cudaStream_t st);

}  // namespace loom
