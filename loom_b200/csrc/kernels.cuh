// kernels.cuh -- device kernels of the CUDA backend and their host launchers.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace loom {

// One routed (or host-listed) expert applied to one token: the unit the MoE
// kernels iterate over. Mirrors the seam's ExpertRef (src/compute/cpu.zig:23)
// plus the token it serves and where its activation lives in scratch.
struct Slot {
    WDev g, u, dn;        // gate [ffn x dim], up [ffn x dim], down [dim x ffn]
    uint64_t gb_g, gb_u, gb_dn;  // first block of this expert's plane in each tensor
    int ffn;
    int token;
    float weight;
    int act_off;          // element offset of this slot's activation in scratch (multiple of 256)
};

// Routed-layer description the device-side router expands into slots.
struct RoutedLayerDev {
    WDev g, u, dn;
    uint64_t plane_blk_g, plane_blk_u, plane_blk_dn;  // blocks per expert plane
    int ffn, dim;
    int n_expert, n_used;
    int gating;           // 1 softmax, 2 sigmoid, 3 softmax_topk
    int weights_norm;
    float weights_scale;
    int n_group, topk_group;  // group-limited selection (1, 1: plain top-k)
    int has_shared;
    WDev sg, su, sdn;     // shared expert (gb offsets 0)
    int shexp_ffn;
    int expert0;          // first expert id held by this rank (expert parallelism); 0 otherwise
    int n_local;          // experts held locally; n_expert when not sharded
};

// launchers (all asynchronous on `st`)
void launch_synth(int type, uint8_t *raw, uint64_t blk0, uint64_t nblk, uint64_t seed, float sigma, cudaStream_t st);
void launch_repack(int type, const uint8_t *raw, uint8_t *q, uint8_t *sc, uint16_t *d, uint64_t nblk, cudaStream_t st);
void launch_unpack(int type, const WDev &w, uint8_t *raw, uint64_t nblk, cudaStream_t st);
void launch_dequant(const WDev &w, uint64_t gb0, uint64_t nblk, float *out, cudaStream_t st);
// MLA (deepseek.zig attnLayer): W_k absorbed into q per head, qa [n_heads][kvr];
// and W_v applied per head to head h's quantized activation (token h of x), out [n_heads][vd]
void launch_mla_absorb(const WDev &w, int kvr, int nope, int vd, int kd, int n_heads, const float *q, float *qa,
                       cudaStream_t st);
void launch_mla_wv(const WDev &w, int kvr, int nope, int vd, int n_heads, const XQ &x, float *out, cudaStream_t st);
// row tok[i] of a [vocab][dim] tensor into x + i * dim, i < ntok (embedding lookup)
void launch_embed(const WDev &w, int dim, const uint32_t *tok, int vocab, float *x, cudaStream_t st, int ntok = 1);
// act[i] = silu(g[i]) * u[i]
void launch_swiglu(const float *g, const float *u, int n, float *act, cudaStream_t st);
void launch_quant_act(const float *x, int ntok, int cols, int xstride, int kind256, int8_t *q, float *d,
                      int32_t *s, int dstride, int sstride, cudaStream_t st);
void launch_mm(const WDev &w, uint64_t gb_base, int rows, int cols, const XQ &x, int ntok, float *out,
               cudaStream_t st);
void launch_mm_f32(const float *W, int rows, int cols, const float *xs, int ntok, float *out, cudaStream_t st);
// launch_mm for many token rows (prefill.cu): weight and token tiles staged in shared memory;
// Q4_K / Q6_K / Q8_0 / Q4_0 only (false: not launched, use launch_mm). Bit-identical to launch_mm.
bool launch_mm_tiled(const WDev &w, int rows, int cols, const XQ &x, int ntok, float *out, cudaStream_t st);
// Q5_0 on f32 activations (matvecQ50, ggml.zig:1673), out[k*rows + r]
void launch_mm_q50(const WDev &w, uint64_t gb_base, int rows, int cols, const float *xs, int ntok, float *out,
                   cudaStream_t st);
void launch_route(const float *logits, const float *bias, int T, int n_expert, int n_used, int gating,
                  int weights_norm, float weights_scale, int *ids, float *gates, cudaStream_t st,
                  int n_group = 1, int topk_group = 1);
// Expert phase (gate/up + SwiGLU, activation quantization, down + weighted
// combine) for a host-built slot array (one token) or for a routed layer whose
// router already wrote ids/gates [T][n_used].
void launch_experts_host(const Slot *slots, int n, int max_ffn, int dim, const XQ &x256, const XQ &x32, float *act,
                         int8_t *aq, float *ad, int32_t *as, float *out, cudaStream_t st);
void launch_experts_routed(const RoutedLayerDev &L, const int *ids, const float *gates, int T, int act_stride,
                           const XQ &x256, const XQ &x32, float *act, int8_t *aq, float *ad, int32_t *as, float *out,
                           const float *residual, cudaStream_t st);

// sampler.zig:7-15 argmax of v[0..n) into *out; slot / count: 16 zeroed bytes
// of device scratch that the kernel leaves zeroed again
void launch_argmax(const float *v, int n, unsigned long long *slot, unsigned *count, uint32_t *out, cudaStream_t st);

// number of kernel launches issued by this library (host-side count)
uint64_t launches();
void count_launch();
void count_launches(uint64_t n);

}  // namespace loom
