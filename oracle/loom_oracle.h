/*
 * loom_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement, in plain C++, of the reference's CPU kernels for the
 * quantized MoE forward path (ch4r10t33r/loom, Zig). It is the checker the
 * CUDA backend is compared against and the timed CPU baseline; it is never
 * linked into, called by or shipped with the product library.
 *
 * Every function cites the reference file:line it restates. Floating-point
 * operations follow the Zig source one rounding at a time (the build uses
 * -ffp-contract=off: Zig does not contract a*b-c into an FMA).
 *
 * Parity is pinned against the reference's own known-answer tests
 * (src/gguf/ggml.zig:1906-2210, src/gguf/moe.zig:210-262), which the CPU test
 * suite replays against this library.
 */
#ifndef LOOM_ORACLE_H
#define LOOM_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, src/gguf/ggml.zig:23-45 */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7, OR_Q8_0 = 8, OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14 };

size_t or_row_bytes(int type, size_t n);          /* ggml.zig:103 rowBytes */
size_t or_block_elems(int type);                  /* ggml.zig:128 blockElems */
size_t or_block_bytes(int type);                  /* ggml.zig:157 blockBytes */

/* worker pool, ggml.zig:279-398 (parallelBegin/parallelEnd) */
void or_parallel_begin(int n);
void or_parallel_end(void);
int or_pool_workers(void);

/* kernels */
int or_dequant_row(int type, float *out, const uint8_t *data, size_t r, size_t cols);      /* ggml.zig:1739 */
int or_matvec(int type, float *out, const uint8_t *data, const float *x, size_t rows, size_t cols); /* ggml.zig:602 */
int or_matmul(int type, float *out, const uint8_t *data, const float *xs, size_t n, size_t rows, size_t cols); /* ggml.zig:504 */
float or_dot_f32(const float *a, const float *b, size_t n);                               /* ggml.zig:198 dotF32 */

/* activation quantizers. ggml.zig:776 quantizeX256: q[cols], d[cols/256], bsum[cols/16];
 * ggml.zig:1077 quantizeX: q[cols], d[cols/32], sum[cols/32] */
void or_quantize_x256(const float *x, size_t cols, int8_t *q, float *d, int32_t *bsum);
void or_quantize_x32(const float *x, size_t cols, int8_t *q, float *d, int32_t *sum);

/* elementwise, src/core/tensor.zig:9-57 */
void or_softmax(float *x, size_t n);
float or_silu(float x);
float or_sigmoid(float x);
void or_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps);

/* router, src/gguf/moe.zig:106-158. gating: 1 softmax, 2 sigmoid, 3 softmax_topk */
int or_route(const float *logits, const float *bias, size_t n_expert, size_t n_used, int gating,
             int weights_norm, float weights_scale, uint32_t *ids, float *gates);
/* sampler.zig:7-15 argmax: strict '>' from -inf, so the first maximum wins,
 * NaN is never taken, and an input with nothing above -inf gives 0. */
size_t or_argmax(const float *logits, size_t n);
/* or_route with DeepSeek-V3's group-limited selection (n_group groups of
 * n_expert / n_group consecutive experts, the topk_group best by the sum of
 * their two largest biased choices kept); n_group = 1 is or_route. No
 * counterpart in the reference: restated from the published routing. */
int or_route_grouped(const float *logits, const float *bias, size_t n_expert, size_t n_used, int gating,
                     int weights_norm, float weights_scale, size_t n_group, size_t topk_group, uint32_t *ids,
                     float *gates);

/* One expert as the seam's ExpertRef (src/compute/cpu.zig:23). */
typedef struct {
    int gate_type, up_type, down_type;
    const uint8_t *gate, *up, *down;
    float weight;
    size_t ffn;
} or_expert;

/* moeFfnBlock semantics: out = sum_k weight_k * FFN_k(normed), in list order
 * (src/gguf/llama.zig:1363-1398 denseFFN + acc loop; deepseek.zig:1405-1442). */
int or_moe_ffn_block(const float *normed, size_t dim, const or_expert *experts, size_t n, float *out);

/* moeFfnBlockRouted semantics (deepseek.zig:1340-1380 with cpu route +
 * the host loop): route(logits, bias) -> per selected expert plane FFN ->
 * weighted sum in selection order -> + shared expert (plain add).
 * 3D tensors are n_expert contiguous planes. */
int or_moe_ffn_routed(const float *normed, size_t dim, const float *logits, const float *bias,
                      int gate_type, const uint8_t *gate3d, int up_type, const uint8_t *up3d,
                      int down_type, const uint8_t *down3d, size_t ffn,
                      const int *shexp_types, const uint8_t *const *shexp, size_t shexp_ffn,
                      size_t n_expert, size_t n_used, int gating_sigmoid, int weights_norm,
                      float weights_scale, float *out);

/* A whole MoE layer at T tokens (src/gguf/llama.zig:1262-1272 moeLayer):
 * logits = matvec(f32 router, x_t); route; experts; out_t. Router f32 [n_expert][dim]. */
int or_moe_layer(const float *x, size_t T, size_t dim, const float *router_w, int gate_type,
                 const uint8_t *gate3d, int up_type, const uint8_t *up3d, int down_type,
                 const uint8_t *down3d, size_t ffn, size_t n_expert, size_t n_used, int gating,
                 int weights_norm, float weights_scale, float *out, uint32_t *ids_out);

/* One decoder layer of llama.zig's model (Model.layers, llama.zig:136-200):
 * attention weights, optional per-head Q/K RMSNorm weights (qwen3moe), and
 * either a dense SwiGLU FFN (router == NULL) or a routed MoE FFN whose f32
 * router is [n_expert][dim] and whose gate/up/down are 3D expert tensors. */
typedef struct {
    const float *attn_norm, *ffn_norm;   /* f32 [dim] */
    int wq_type, wk_type, wv_type, wo_type;
    const uint8_t *wq, *wk, *wv, *wo;    /* [n_heads*hd][dim], [n_kv*hd][dim] x2, [dim][n_heads*hd] */
    const float *q_norm, *k_norm;        /* f32 [hd] or NULL */
    int gate_type, up_type, down_type;
    const uint8_t *gate, *up, *down;     /* dense [ffn][dim].. or 3D [n_expert][ffn][dim].. */
    size_t ffn;
    const float *router;                 /* f32 [n_expert][dim]; NULL = dense FFN */
} or_llama_layer;
typedef struct {
    size_t dim, n_layers, n_heads, n_kv_heads, head_dim, rope_dim, vocab, ctx_len;
    float eps, rope_base, attn_logit_mul;
    int rope_neox;                        /* 1: ropeNeox (qwen3moe), 0: ropeNorm (llama) */
    size_t n_expert, n_used;              /* routed layers */
    int gating, weights_norm;
    float weights_scale;
    int embd_type;
    const uint8_t *token_embd;            /* [vocab][dim] */
    const float *output_norm;             /* f32 [dim] */
    int output_type;
    const uint8_t *output;                /* [vocab][dim] */
    const or_llama_layer *layers;
} or_llama_model;
/* llama.zig:1111-1228 step (the per-operation path, no frame): embedding
 * row, per layer RMSNorm -> q/k/v matvecs -> headNorm (:938) -> RoPE (:830-858)
 * -> KV append -> per-head softmax attention over positions 0..pos (dotF32,
 * softmax, axpy) -> output projection -> residual; RMSNorm -> dense FFN or
 * moeLayer -> residual; final RMSNorm -> output head. k_cache / v_cache:
 * f32 [n_layers][ctx_len][n_kv*hd], the caller's. logits: f32 [vocab]. */
int or_llama_step(const or_llama_model *m, float *k_cache, float *v_cache, uint32_t token, size_t pos,
                  float *logits);

/* One DeepSeek-V2/V3 decoder layer (deepseek.zig Model.layers): MLA attention
 * weights (q either from wq, or q_a -> RMSNorm(q_a_norm) -> q_b when
 * q_lora_rank > 0), then a dense FFN (router == NULL) or a routed MoE with
 * optional bias and optional shared expert (shexp_gate != NULL). */
typedef struct {
    const float *attn_norm, *ffn_norm;
    int wq_type; const uint8_t *wq;                 /* [n_heads*(nope+rope)][dim] (q_lora_rank == 0) */
    int q_a_type; const uint8_t *q_a; const float *q_a_norm;  /* [q_lora][dim], f32 [q_lora] */
    int q_b_type; const uint8_t *q_b;               /* [n_heads*(nope+rope)][q_lora] */
    int kv_a_type; const uint8_t *kv_a;             /* [kv_lora+rope][dim] (attn_kv_a_mqa) */
    const float *kv_a_norm;                         /* f32 [kv_lora] */
    int kv_b_type; const uint8_t *kv_b;             /* [n_heads*(nope+v_head)][kv_lora] */
    int wo_type; const uint8_t *wo;                 /* [dim][n_heads*v_head] */
    int gate_type, up_type, down_type;
    const uint8_t *gate, *up, *down;                /* dense or 3D expert tensors */
    size_t ffn;
    const float *router, *router_bias;              /* f32 [n_expert][dim], [n_expert] or NULL */
    int sh_gate_type, sh_up_type, sh_down_type;
    const uint8_t *sh_gate, *sh_up, *sh_down;       /* shared expert or NULL */
    size_t sh_ffn;
} or_ds_layer;
typedef struct {
    size_t dim, n_layers, n_heads, nope, rope, kv_lora, q_lora, v_head, vocab, ctx_len;
    float eps, rope_base, attn_scale;
    size_t n_expert, n_used;
    int gating_sigmoid, weights_norm;
    float weights_scale;
    int embd_type; const uint8_t *token_embd;
    const float *output_norm;
    int output_type; const uint8_t *output;
    const or_ds_layer *layers;
    size_t n_group, topk_group;   /* DeepSeek-V3 group-limited routing (1, 1: moe.zig route) */
} or_ds_model;
/* deepseek.zig:1275-1537 step (host path) with attnLayer (:851-1049):
 * c_cache f32 [n_layers][ctx][kv_lora], r_cache f32 [n_layers][ctx][rope]. */
int or_deepseek_step(const or_ds_model *m, float *c_cache, float *r_cache, uint32_t token, size_t pos,
                     float *logits);

/* Seeded synthetic tensors (counter-based, the same generator the CUDA backend
 * runs on the device): blocks [blk0, blk0+nblk) of a tensor of `type`. For
 * OR_F32, "blocks" are elements ~ sigma * IrwinHall12. */
void or_synth(int type, void *out, uint64_t blk0, uint64_t nblk, uint64_t seed, float sigma);
uint16_t or_f32_to_f16_rne(float f);
float or_f16_to_f32(uint16_t h);

#ifdef __cplusplus
}
#endif
#endif
