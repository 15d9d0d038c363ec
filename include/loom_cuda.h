/*
 * loom_cuda.h -- C ABI of the B200 (sm_100a) CUDA compute backend for Loom's
 * quantized Mixture-of-Experts forward path.
 *
 * The backend slots in behind Loom's comptime backend seam
 * (src/compute/backend.zig:28-49) as a `cuda` arm, next to cpu/metal/vulkan.
 * Each seam entry below cites the reference declaration it replaces.
 *
 * Conventions (the seam's, src/compute/backend.zig and src/vulkan/backend.zig):
 *  - Host slices are borrowed for the duration of the call; `out` is written
 *    completely before a call returns LOOM_CUDA_OK.
 *  - Weights are immutable host byte ranges (GGUF blocks, typically views into
 *    an mmap). The backend keeps a device copy in its own layout, keyed by the
 *    host pointer, byte length and type, or addressed inside a registered arena.
 *  - Status codes: LOOM_CUDA_OK = done; LOOM_CUDA_DECLINED = the backend did
 *    nothing (unsupported type/shape, not initialised) and the caller runs its
 *    CPU path -- the seam's "return false"; LOOM_CUDA_ERROR = a CUDA error (the
 *    message is in loom_cuda_last_error). No CPU fallback exists inside the
 *    backend.
 *  - One generation thread calls the backend; it is not reentrant.
 *  - Streams: entries that take `void *stream` run on that cudaStream_t. NULL
 *    means the backend's own stream, a blocking stream: it is ordered after
 *    and before work on the legacy default stream (stream 0), but not with
 *    other non-blocking streams -- a caller that queues inputs on its own
 *    stream passes that stream.
 *
 * ggml type ids (src/gguf/ggml.zig:23-45): F32 0, Q4_0 2, Q8_0 8, Q4_K 12, Q6_K 14.
 */
#ifndef LOOM_CUDA_H
#define LOOM_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LOOM_CUDA_OK 0
#define LOOM_CUDA_DECLINED 1
#define LOOM_CUDA_ERROR 2

enum {
    LOOM_F32 = 0,
    LOOM_Q4_0 = 2,
    LOOM_Q4_1 = 3,
    LOOM_Q5_0 = 6,
    LOOM_Q5_1 = 7,
    LOOM_Q8_0 = 8,
    LOOM_Q2_K = 10,
    LOOM_Q3_K = 11,
    LOOM_Q4_K = 12,
    LOOM_Q5_K = 13,
    LOOM_Q6_K = 14
};

/* WeightRef, src/compute/cpu.zig:21: a weight tensor as the fused entries take it. */
typedef struct {
    int ggml_type;
    const void *data;
    size_t bytes;
} loom_weight;

/* ExpertRef, src/compute/cpu.zig:23: one expert of a MoE layer. */
typedef struct {
    loom_weight gate, up, down;
    float weight;
    size_t ffn;
} loom_expert;

/* RoutedCfg, src/compute/cpu.zig:61. */
typedef struct {
    size_t n_expert;
    size_t n_used;
    int gating_sigmoid;
    int weights_norm;
    float weights_scale;
} loom_routed_cfg;

/* ---- lifecycle ------------------------------------------------------------ */

/* Select the device, create the backend's stream and scratch. Replaces the
 * device bring-up the GPU backends do inside parallelBegin
 * (src/compute/backend.zig:225-226, src/vulkan/backend.zig parallelBegin). */
int loom_cuda_init(int device);
void loom_cuda_shutdown(void);
/* parallelBegin/parallelEnd (src/compute/backend.zig:225-226): init on first
 * begin; end is a no-op (the device stays up for the process). */
void loom_cuda_parallel_begin(size_t n);
void loom_cuda_parallel_end(void);
/* MAX_BATCH (src/compute/backend.zig:229): the largest matmul batch taken. */
size_t loom_cuda_max_batch(void);

/* registerArena (src/compute/backend.zig:98): remember a host mapping; false
 * (DECLINED) when not initialised. Tensors inside it are then addressed by
 * offset once materialised. */
int loom_cuda_register_arena(const void *mem, size_t bytes);
/* materializeArenas (src/compute/backend.zig:104): copy every registered
 * mapping to the device; returns the bytes made resident (0 on failure, with
 * the reason in loom_cuda_arena_error). */
size_t loom_cuda_materialize_arenas(void);
/* arena_error (src/compute/backend.zig:118). NULL when none. */
const char *loom_cuda_arena_error(void);

/* ---- GGUF tensor table (host side, no device needed) -----------------------
 *
 * gguf.parse (src/gguf/gguf.zig:251-325) over a file image, and the engine's
 * checked tensor resolve (src/gguf/llama.zig:259-273, sizes by
 * src/gguf/ggml.zig:143-153). A failed call leaves the reference's error name
 * in loom_gguf_error(): NotGguf, UnsupportedGgufVersion, TruncatedGguf,
 * BadTensorDims, BadAlignment, ArrayNestingTooDeep, UnknownValueType;
 * resolve adds MissingTensor, UnsupportedTensorType, BadTensorShape. Names,
 * strings and tensor data are views into the image, which must outlive the
 * handle. */
typedef struct loom_gguf loom_gguf;

enum {
    LOOM_GGUF_META_INT = 1,
    LOOM_GGUF_META_UINT = 2,
    LOOM_GGUF_META_FLOAT = 3,
    LOOM_GGUF_META_BOOL = 4,
    LOOM_GGUF_META_STRING = 5,
    LOOM_GGUF_META_ARRAY_STR = 6,  /* `array` -> first string's u64 length */
    LOOM_GGUF_META_ARRAY_F32 = 7,  /* `array` -> count little-endian f32 */
    LOOM_GGUF_META_ARRAY_I32 = 8,
    LOOM_GGUF_META_ARRAY = 9       /* other element types: only type and count kept */
};

/* TensorInfo (src/gguf/gguf.zig:36-47); dims past n_dims read 1. */
typedef struct {
    const char *name;
    size_t name_len;
    uint32_t n_dims;
    uint64_t dims[8];
    uint32_t ggml_type;
    uint64_t offset; /* relative to the data section */
} loom_gguf_tensor;

/* MetaKV / MetaValue (src/gguf/gguf.zig:49-72). */
typedef struct {
    const char *key;
    size_t key_len;
    int kind;
    int64_t i;
    uint64_t u; /* UINT, and BOOL as 0/1 */
    double f;
    const char *str;
    size_t str_len;
    uint32_t elem_type;
    uint64_t count;
    const void *array;
    uint64_t span_start, span_end; /* byte span of the whole pair in the file */
} loom_gguf_value;

/* Model.resolve's Tensor (src/gguf/llama.zig:259-273): a checked byte view. */
typedef struct {
    int ggml_type;
    const void *data;
    size_t bytes;
    uint64_t ne0, ne1, ne2;
} loom_gguf_view;

loom_gguf *loom_gguf_parse(const void *image, size_t bytes);
/* parse of a file mapped read-only (the mapping is released by close). */
loom_gguf *loom_gguf_open(const char *path);
const char *loom_gguf_error(void);
void loom_gguf_close(loom_gguf *g);
uint32_t loom_gguf_version(const loom_gguf *g);
uint64_t loom_gguf_alignment(const loom_gguf *g);
uint64_t loom_gguf_data_offset(const loom_gguf *g);
uint64_t loom_gguf_file_size(const loom_gguf *g);
const void *loom_gguf_image(const loom_gguf *g);
size_t loom_gguf_n_tensors(const loom_gguf *g);
size_t loom_gguf_n_meta(const loom_gguf *g);
int loom_gguf_tensor_info(const loom_gguf *g, size_t i, loom_gguf_tensor *out);
/* findTensor / findMeta (src/gguf/gguf.zig:92,120): DECLINED when absent. */
int loom_gguf_find_tensor(const loom_gguf *g, const char *name, loom_gguf_tensor *out);
int loom_gguf_meta(const loom_gguf *g, size_t i, loom_gguf_value *out);
int loom_gguf_find_meta(const loom_gguf *g, const char *key, loom_gguf_value *out);
/* getUint / getFloat / getString / getBool (src/gguf/gguf.zig:99-126),
 * with the same kind conversions; DECLINED where the reference gives null. */
int loom_gguf_get_uint(const loom_gguf *g, const char *key, uint64_t *out);
int loom_gguf_get_float(const loom_gguf *g, const char *key, double *out);
int loom_gguf_get_string(const loom_gguf *g, const char *key, const char **s, size_t *len);
int loom_gguf_get_bool(const loom_gguf *g, const char *key, int *out);
int loom_gguf_resolve(const loom_gguf *g, const char *name, loom_gguf_view *out);

/* ---- verified upload ---------------------------------------------------------
 *
 * A content-addressed shard: the host byte ranges of one block of weights (an
 * expert's gate, up and down planes) in order, and the SHA-256 of their
 * concatenation -- the digest the reference keeps per range and checks
 * before any read (src/core/hash.zig:12-23, src/p2p/weights.zig:862-879).
 * Each extent must lie inside one weight tensor the backend holds (or it is
 * uploaded as its own tensor) and start on a block boundary of it. */
typedef struct {
    loom_weight ext[4];
    int n_ext;
    uint8_t digest[32];
} loom_shard;

/* Compute each shard's SHA-256 on the device over the bytes the kernels will
 * read (the device copy, its GGUF bytes rebuilt from the layout repack) and
 * compare with `digest`. bad[i] (optional) = 1 on mismatch. A mismatching
 * shard's tensors are dropped from the weight cache, so the next use uploads
 * them again from the host -- the reference clears the range's holding bit
 * (src/p2p/weights.zig:873-876). Returns OK and the mismatch count in
 * *n_bad; DECLINED for an extent the backend cannot place. */
int loom_cuda_verify_shards(const loom_shard *shards, size_t n, uint8_t *bad, size_t *n_bad);
/* SHA-256 of device bytes (a test and manifest helper). */
int loom_cuda_sha256_device(const void *d_bytes, size_t bytes, uint8_t digest[32]);
/* SHA-256 of blocks [blk0, blk0 + nblk) of a device tensor, over their GGUF
 * bytes (the layout repack undone). */
int loom_cuda_tensor_sha256(uint64_t t, uint64_t blk0, uint64_t nblk, uint8_t digest[32]);
/* takeCmdBufCount (src/compute/backend.zig:112): seam submissions since the
 * last call, then reset. */
size_t loom_cuda_take_cmdbuf_count(void);
/* Kernel launches issued by this library since load (never reset). */
uint64_t loom_cuda_kernel_launches(void);
/* Copy the last error message into buf (NUL-terminated); returns its length. */
size_t loom_cuda_last_error(char *buf, size_t len);
/* Drop every cached device copy of host weights (the Vulkan backend's
 * clearWeightCache, src/vulkan/backend.zig:159-168). */
void loom_cuda_clear_weight_cache(void);

/* ---- seam ops (host buffers) ------------------------------------------------ */

/* matvec (src/compute/backend.zig:62 -> cpu.zig:17 ggml.matvec, ggml.zig:602):
 * out[r] = W[r] . x with int8-quantized activations, bit-identical to the CPU
 * kernels for Q4_0/Q8_0/Q4_K/Q6_K and to dotF32 for F32. */
int loom_cuda_matvec(int ggml_type, float *out, const void *w, size_t w_bytes, const float *x, size_t rows,
                     size_t cols);
/* matmul (src/compute/backend.zig:66 -> ggml.zig:504): out[k*rows + r],
 * bit-identical to n matvecs. */
int loom_cuda_matmul(int ggml_type, float *out, const void *w, size_t w_bytes, const float *xs, size_t n, size_t rows,
                     size_t cols);
/* dequantRow (src/compute/backend.zig:69 -> ggml.zig:1739), bit-exact. */
int loom_cuda_dequant_row(int ggml_type, float *out, const void *w, size_t w_bytes, size_t r, size_t cols);
/* moeRoute (src/compute/backend.zig:183 -> cpu.zig:86; moe.zig:106 route):
 * ids_out/gates_out hold n_used entries. */
int loom_cuda_moe_route(const float *logits, const float *bias, size_t n_expert, uint32_t *ids_out, float *gates_out,
                        size_t n_used, int gating_sigmoid, int weights_norm, float weights_scale);
/* moeFfnBlock (src/compute/backend.zig:104 -> cpu.zig:27): out = sum_k
 * experts[k].weight * FFN_k(normed), in list order (llama.zig:1363-1398). */
int loom_cuda_moe_ffn_block(const float *normed, size_t dim, const loom_expert *experts, size_t n_experts, float *out);
/* moeFfnBlockRouted (src/compute/backend.zig:189 -> cpu.zig:68): route from
 * logits, run the selected planes of the 3D tensors, weighted sum in selection
 * order, plus the shared expert (shexp3 = NULL when absent), as ONE submission
 * (deepseek.zig:1340-1380). */
int loom_cuda_moe_ffn_routed(const float *normed, size_t dim, const float *logits, const float *bias,
                             loom_weight gate, loom_weight up, loom_weight down, const loom_weight *shexp3, size_t ffn,
                             size_t shexp_ffn, loom_routed_cfg cfg, float *out);

/* ---- device-resident API (no counterpart in the reference's seam: the
 * engine-side layer that keeps a whole model on the device) ---------------- */

typedef uint64_t loom_tensor; /* handle to a device-resident tensor in the backend's layout; 0 = none */

/* Upload host GGUF bytes (ggml_type blocks) into a device tensor. */
int loom_cuda_tensor_upload(int ggml_type, const void *data, size_t bytes, loom_tensor *out);
/* Create a tensor of nblocks blocks from the seeded counter-based generator
 * (the synthetic-weight generator the benchmarks use; sigma is the f32
 * standard deviation). */
int loom_cuda_tensor_synth(int ggml_type, uint64_t nblocks, uint64_t seed, float sigma, loom_tensor *out);
/* The same generator for blocks [blk0, blk0 + nblocks) of a larger tensor
 * (an expert-parallel rank's slice of a 3D expert tensor). */
int loom_cuda_tensor_synth_range(int ggml_type, uint64_t blk0, uint64_t nblocks, uint64_t seed, float sigma,
                                 loom_tensor *out);
/* Read a tensor back as GGUF bytes (bytes = nblocks * block bytes). */
int loom_cuda_tensor_download(loom_tensor t, void *dst, size_t bytes);
int loom_cuda_tensor_free(loom_tensor t);
/* Device bytes a tensor occupies. */
size_t loom_cuda_tensor_device_bytes(loom_tensor t);

/* One MoE layer over device-resident tensors. router: f32 [n_expert][dim]
 * (0 = logits are supplied by the caller); gate/up: [n_local][ffn][dim];
 * down: [n_local][dim][ffn]; shexp: 0 = none. For expert parallelism this rank
 * holds experts [expert0, expert0 + n_local). */
typedef struct {
    size_t dim, ffn, n_expert, n_used;
    int gating;        /* 1 softmax, 2 sigmoid, 3 softmax_topk (moe.zig:35-42) */
    int weights_norm;
    float weights_scale;
    loom_tensor router, router_bias;
    loom_tensor gate, up, down;
    loom_tensor shexp_gate, shexp_up, shexp_down;
    size_t shexp_ffn;
    size_t expert0, n_local;
    /* optional hint: the next layer's router (f32 [n_expert][dim]); its weights
     * are prefetched into L2 while this layer's experts stream */
    loom_tensor next_router;
    /* DeepSeek-V3 group-limited routing (no counterpart in the reference):
     * the experts form n_group groups of n_expert / n_group consecutive ids,
     * only the topk_group groups with the largest sum of their two best
     * biased scores are eligible for the top-n_used. n_group 0 or 1 = plain
     * moe.zig:106 route. */
    size_t n_group, topk_group;
} loom_moe_desc;

/* d_x: device f32 [T][dim]; d_out: device f32 [T][dim] (d_out = d_residual +
 * MoE(d_x) when d_residual is non-NULL). d_logits: optional device f32
 * [T][n_expert] supplied by the caller instead of the router. d_ids: optional
 * device u32 [T][n_used] that receives the routing. stream: a cudaStream_t or
 * NULL for the backend's own stream. Asynchronous; launches only (no
 * allocation) once loom_cuda_reserve covered T. */
int loom_cuda_moe_forward(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out,
                          const float *d_residual, const float *d_logits, uint32_t *d_ids, void *stream);
/* Size the scratch for layers up to (dim, ffn, n_expert, n_used) at T tokens so
 * later forwards never allocate (required before CUDA-graph capture). */
int loom_cuda_reserve(size_t T, size_t dim, size_t ffn, size_t n_expert, size_t n_used);
/* Allocation-free variant of loom_cuda_moe_forward. No counterpart in the
 * reference: it exists for callers that must not allocate device memory while
 * they run (code inside someone else's CUDA stream capture, engines with a
 * fixed memory budget, processes sharing a GPU under a fixed allocation).
 * The layer's scratch is a fixed 1 MiB array (LOOM_CUDA_NOALLOC_SCRATCH_BYTES)
 * that every GPU loading this library holds until the process exits; no
 * cudaMalloc/cudaFree is ever called. Covers the fused decode shapes (T <= 16,
 * the layer's scratch <= 1 MiB, router on the device); anything larger is
 * declined with a message. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture. All calls share the one array and it keeps the last call's
 * contents (nothing in it needs to start at zero): calls that overlap on the
 * GPU (different streams, no ordering) race and must not be issued. */
#define LOOM_CUDA_NOALLOC_SCRATCH_BYTES (1u << 20)
int loom_cuda_moe_forward_noalloc(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out,
                                  const float *d_residual, void *stream);
/* ---- whole-model decode on the device ----------------------------------------
 * The reference's decode step (llama.zig:1111-1228 `step`; the seam's frame
 * path beginFrame/layerBlock/endFrame, src/compute/backend.zig:146-156, with
 * attnInit/kvAppend/attnHeads, :121-160) kept on the device for a whole token:
 * embedding row (dequantRow), then per layer RMSNorm -> q/k/v matvecs ->
 * per-head Q/K RMSNorm when given (headNorm, :938) -> RoPE (ropeNorm or
 * ropeNeox, :830-858) -> append to the f32 KV cache [layer][ctx][n_kv*hd] ->
 * softmax attention of every query head over positions 0..pos (GQA) -> output
 * projection -> residual add -> RMSNorm -> dense SwiGLU FFN or routed MoE
 * layer -> residual add; final RMSNorm -> output head -> argmax (sampler.zig:7).
 * The residual stream never leaves the device. Every tensor is a device tensor
 * (loom_tensor); norms are f32. */
typedef struct {
    loom_tensor attn_norm;            /* f32 [dim] */
    loom_tensor wq, wk, wv, wo;       /* [n_heads*hd][dim], [n_kv*hd][dim] (x2), [dim][n_heads*hd] */
    loom_tensor q_norm, k_norm;       /* f32 [hd] each, or 0 (no per-head norm) */
    loom_tensor ffn_norm;             /* f32 [dim] */
    /* FFN: routed when moe.n_expert > 0 (moe.dim must equal the model's dim),
     * else dense: ffn_gate/ffn_up [ffn][dim], ffn_down [dim][ffn] */
    loom_tensor ffn_gate, ffn_up, ffn_down;
    size_t ffn;
    loom_moe_desc moe;
    /* multi-head latent attention (desc.mla = 1; deepseek.zig:851-1049), in place
     * of wq/wk/wv: q = wq . x (q_lora_rank 0) or q_b . RMSNorm(q_a . x) *
     * q_a_norm; kv_a [kv_lora + rope][dim] (attn_kv_a_mqa); kv_a_norm f32
     * [kv_lora]; kv_b [n_heads*(nope + v_head)][kv_lora]; wo [dim][n_heads*v_head] */
    loom_tensor q_a, q_a_norm, q_b, kv_a, kv_a_norm, kv_b;
} loom_model_layer;
typedef struct {
    size_t dim, n_layers, n_heads, n_kv_heads, head_dim, rope_dim, vocab, ctx_len;
    float eps, rope_base, attn_logit_mul; /* scores = q.k * attn_logit_mul / sqrt(head_dim) */
    int rope_neox;                        /* 1 ropeNeox (qwen3moe, qwen2moe), 0 ropeNorm (llama) */
    /* 1: keep the reference's summation order at every width -- RMSNorm's
     * serial sum of squares (a few microseconds per norm at dim 2048) and the
     * ordered attention at any context; 0: tree sums for RMSNorm wider than
     * 1024 and split attention beyond 512 positions (faster, within rounding) */
    int exact_order;
    loom_tensor token_embd;               /* [vocab][dim], any supported type */
    loom_tensor output_norm;              /* f32 [dim] */
    loom_tensor output;                   /* [vocab][dim] */
    const loom_model_layer *layers;       /* [n_layers], copied by create */
    /* multi-head latent attention (DeepSeek-V2/V3): head_dim = nope + rope_dim
     * per query head; the cache holds [ctx][kv_lora] compressed rows and
     * [ctx][rope_dim] rope rows per layer; scores scale by mla_scale
     * (deepseek.zig:360: mscale^2 / sqrt(nope + rope)). n_kv_heads is ignored. */
    int mla;
    size_t kv_lora, q_lora, nope, v_head;
    float mla_scale;
} loom_model_desc;
/* Build the model: checks every tensor's type and size, allocates the KV
 * cache (2 x n_layers x ctx_len x n_kv*hd f32), the RoPE table and the step's
 * buffers. Limits: head_dim even and <= 256, rope_dim <= head_dim, n_heads a
 * multiple of n_kv_heads with at most 16 query heads per KV head, ctx_len up
 * to 32768 with exact_order. Contexts up to 512 positions (any, with
 * exact_order) use the attention kernel that keeps the reference's operation
 * order (dotF32 scores, serial softmax sum, axpy in position order); longer
 * contexts split the positions across CTAs and merge. */
int loom_cuda_model_create(const loom_model_desc *desc, uint64_t *handle);
/* One decode step on device memory (graph-capturable after the first call):
 * d_token / d_pos: device u32 [1] (the token at position pos < ctx_len);
 * d_logits: optional device f32 [vocab]; d_next: optional device u32 [1]
 * receiving the greedy token. The caller keeps token < vocab and
 * pos < ctx_len; out-of-range values only stay inside the model's buffers
 * (the token is clamped, a position >= ctx_len skips the cache write and the
 * attention) and give a meaningless result. */
int loom_cuda_model_step(uint64_t handle, const uint32_t *d_token, const uint32_t *d_pos, float *d_logits,
                         uint32_t *d_next, void *stream);
/* The same step with host values: one host->device copy of (token, pos), the
 * step replayed from a CUDA graph (captured on the second call), one
 * device->host copy of the greedy token (and of the logits when logits !=
 * NULL), then a wait for completion. */
int loom_cuda_model_decode(uint64_t handle, uint32_t token, size_t pos, float *logits, uint32_t *next);
/* Batched prefill (llama.zig:1698-1825 stepBatch): the n host token ids at
 * positions pos_base .. pos_base + n - 1 through every layer, each layer over
 * all n rows before the next (matmuls bit-identical to per-token matvecs,
 * each token attending causally to cache rows 0..its position in the
 * reference's order, the FFN on the expert-major batch path), their K/V rows
 * appended to the cache; then the last token's logits (host, vocab f32, or
 * NULL) and greedy next token (or NULL). Synchronous. Declines MLA models and
 * positions beyond the context; allocates its row buffers on first use of a
 * larger n (not for use inside a stream capture). */
int loom_cuda_model_prefill(uint64_t handle, const uint32_t *tokens, size_t n, size_t pos_base, float *logits,
                            uint32_t *next);
/* Batched decode of B sequences (llama.zig:1939 decodeBatch): row b is
 * sequence b's token at position positions[b], with its own KV cache (B
 * caches, zeroed, allocated by the first call, which fixes the largest B;
 * separate from the single-sequence cache of loom_cuda_model_decode). Every
 * row's logits (host [B][vocab] f32, or NULL) and greedy next token (host
 * [B], or NULL). Synchronous. Declines MLA models. */
int loom_cuda_model_decode_batch(uint64_t handle, const uint32_t *tokens, const uint32_t *positions, size_t B,
                                 float *logits, uint32_t *next);
/* Copy one cache row (layer, pos) of keys and values (n_kv*hd f32 each; with
 * MLA the compressed row, kv_lora f32, and the rope row, rope_dim f32) to the
 * host -- the read-back that keeps a host copy authoritative (mlaReadCache,
 * backend.zig:191). */
int loom_cuda_model_read_kv(uint64_t handle, size_t layer, size_t pos, float *k, float *v);
/* The device error word of the model's cooperative attention kernel (1 = a
 * grid barrier gave up waiting; the kernel left without finishing the step);
 * synchronizes, and re-arms the barrier counters after an error. 0 when
 * none, -1 on an unknown handle or a failed stream. */
int loom_cuda_model_error(uint64_t handle);
int loom_cuda_model_free(uint64_t handle);
/* Diagnostic (no counterpart in the reference; the spirit of LOOM_PROFILE,
 * deepseek.zig:705-850): layer >= 0 makes that layer's fused attention
 * launch record %globaltimer ns of CTA 0 at its phase boundaries (zeroed
 * now); layer < 0 copies min(n, 32) recorded words to out. */
int loom_cuda_model_trace(uint64_t handle, int layer, unsigned long long *out, size_t n);

/* A decode step (one token) through a whole stack of MoE layers as ONE
 * persistent cooperative kernel: x_{l+1} = x_l + MoE_l(x_l) for every layer,
 * the phases of each layer separated by grid barriers instead of kernel
 * launches. The layers share one shape and routing configuration (plain
 * routed layers: no bias, shared expert or expert sharding). prepare uploads
 * the layer table (outside any stream capture); forward only launches, so it
 * can be captured in a CUDA graph. Output is bit-identical to running
 * loom_cuda_moe_forward layer by layer with the residual. d_ids (optional)
 * receives [n_layers][n_used] expert ids. Engine-level API: no counterpart
 * in the reference's seam. */
int loom_cuda_stack_prepare(const loom_moe_desc *descs, size_t n_layers, uint64_t *handle);
int loom_cuda_stack_forward(uint64_t handle, const float *d_x, float *d_out, uint32_t *d_ids, void *stream);
/* The same launch, the last layer adding its experts to d_residual instead of
 * its own input: for a one-layer stack, d_out = d_residual + MoE(d_x) -- a
 * decoder layer's FFN on its normed input (llama.zig:1222-1225). */
int loom_cuda_stack_forward_residual(uint64_t handle, const float *d_x, const float *d_residual, float *d_out,
                                     uint32_t *d_ids, void *stream);
/* The stack kernel's device error word (2 = a grid barrier gave up waiting);
 * synchronizes, and re-arms the barrier after an error. -1 on an unknown handle or a failed stream. */
int loom_cuda_stack_error(uint64_t handle);
int loom_cuda_stack_free(uint64_t handle);
/* Phase trace of the stack kernel: enable=1 arms it for the following
 * launches (outside stream capture); enable=0 synchronizes, copies up to n
 * words into out and disarms it. Per layer 44 words: 12 %globaltimer ns
 * points (layer start, router rows done, route barrier exit, route done,
 * gate/up done, gate/up barrier exit, activations quantized, down rows done,
 * unused, gate/up tiles landed, down tiles landed, unused), then for 13
 * sections of thread 0's work (x load, router dot, barrier, route, tile
 * requests, gate/up tile wait, gate/up compute, barrier, activation load,
 * activation quantization, down tile wait, down compute, barrier, then
 * within the gate/up compute: the dots, the activation stores, unused) the
 * max and the sum over CTAs of its clock64 cycles. */
int loom_cuda_stack_trace(uint64_t handle, int enable, uint64_t *out, size_t n);

/* ---- expert parallelism (no counterpart in the reference: its experts never
 * leave one node's CPU/GPU; this is the north star's expert-parallel mode over
 * NVLink) -------------------------------------------------------------------
 * One process per GPU. Rank 0 creates an id, every rank passes it to
 * loom_cuda_ep_init. After that, loom_cuda_moe_forward on a descriptor whose
 * expert range [expert0, expert0+n_local) is a strict subset of the experts
 * computes this rank's partial output and sums the ranks' partials with an
 * NCCL all-reduce on the same stream (the residual is added on rank 0 only),
 * so every rank ends with the full layer output. */
int loom_cuda_ep_unique_id(void *out, size_t bytes);
int loom_cuda_ep_init(int nranks, int rank, const void *id, size_t bytes);
void loom_cuda_ep_shutdown(void);
int loom_cuda_ep_rank(void);
int loom_cuda_ep_size(void);
/* 1 when the combine of small partials (T x dim <= 16384 floats) runs as the
 * one-shot peer-memory kernel (every rank stores its partial into every rank's
 * slot over NVLink, flags with release/acquire at system scope, rank-ordered
 * sum: identical bits on every rank), 0 when it is NCCL's all-reduce
 * (LOOM_CUDA_EP_NCCL set, more than 8 ranks, or setup failed on any rank).
 * No counterpart in the reference (its experts stay on one host). */
int loom_cuda_ep_peer_combine(void);
/* The peer combine's error word (1 = a wait for a peer's flag gave up; the
 * combine was skipped); synchronizes. After an error the backend stays on
 * NCCL. 0 when none, -1 on a failed device. */
int loom_cuda_ep_error(void);
/* All-to-all form (token-sharded attention): each rank passes ITS OWN T
 * tokens (T may differ between ranks, and may be 0) and a descriptor of its
 * contiguous shard [r*E/R, (r+1)*E/R). The rank routes its tokens, sends each
 * routed row to the expert's owner (grouped ncclSend/ncclRecv), runs the rows
 * that arrive through its experts, receives the outputs back and combines
 * them in selection order with its tokens' shared expert: d_out is
 * bit-identical to the unsharded layer on those tokens. Collective: every
 * rank calls it for every layer. Synchronises the stream once (the receive
 * counts go to the host). Without loom_cuda_ep_init it runs as one rank. */
int loom_cuda_ep_a2a_forward(const loom_moe_desc *desc, const float *d_x, size_t T, float *d_out,
                             const float *d_residual, const float *d_logits, uint32_t *d_ids, void *stream);
/* The same layer with fixed-capacity exchanges: every rank passes the same
 * t_cap >= its T, and every rank sends every other rank a run of exactly
 * t_cap * n_used rows (the unused entries carry no expert and are skipped).
 * No size depends on the routing, so nothing goes to the host and the call
 * can be captured in a CUDA graph with the NCCL exchanges (after one eager
 * call has sized the buffers). Output bit-identical to
 * loom_cuda_ep_a2a_forward. The exchange carries world * t_cap * n_used rows
 * each way, so size t_cap to the decode batch, not to a prefill. Engine-level
 * API: no counterpart in the reference's seam. */
int loom_cuda_ep_a2a_forward_cap(const loom_moe_desc *desc, const float *d_x, size_t T, size_t t_cap, float *d_out,
                                 const float *d_residual, const float *d_logits, uint32_t *d_ids, void *stream);
/* Greedy sampling (sampler.zig:7-15 argmax) of device logits into *d_index
 * (device u32): the first maximum; NaN never taken; 0 when nothing is above
 * -inf. Asynchronous on `stream`; calls on one device share a 16-byte scratch,
 * so they must not run concurrently on different streams. */
int loom_cuda_argmax(const float *d_logits, size_t n, uint32_t *d_index, void *stream);
/* The output head of one token and its greedy sample (llama.zig:1225-1226,
 * sampler.zig:7-15): logits[vocab] = W[vocab][dim] . x with the tensor's
 * bit-exact matvec, then their argmax. d_logits may be NULL (library
 * scratch). */
int loom_cuda_lm_head_argmax(loom_tensor w, size_t vocab, size_t dim, const float *d_x, float *d_logits,
                             uint32_t *d_index, void *stream);
/* Device matvec/matmul on a device tensor: out[k*rows + r], device buffers. */
int loom_cuda_tensor_matmul(loom_tensor w, size_t rows, size_t cols, const float *d_xs, size_t n, float *d_out,
                            void *stream);
/* Test hook selecting the MoE kernel family: 0 automatic (fused decode
 * kernels for T <= 2, expert-major batch kernels above, on the tensor cores
 * once the experts average >= 16 tokens), 1 the general slot kernels, 2 the
 * expert-major batch kernels at any T, 3 the expert-major batch kernels on
 * the tensor cores at any T (Q4_K gate/up with Q6_K down, any scales;
 * other layers fall back to 2). Every family computes the same
 * numbers bit for bit, except the tensor cores in their default
 * dequantized form (loom_cuda_tc_exact). Returns the previous setting. */
int loom_cuda_force_generic(int on);
/* Arithmetic of the tensor-core expert kernels (batched prefill, no
 * counterpart in the reference's seam; its tensor-core path is specified by
 * tolerance): 0 (default) dequantized fp16 weight tiles (Q4_K (d sc) q -
 * dmin m, Q6_K (d sc)(q - 32)) against the int8 activations of
 * quantizeX256 dequantized to fp16, f32 accumulation over the whole row,
 * within 2e-3 relative L2 of the reference; 1 the integer-exact kernels,
 * bit-identical to the CPU (ggml.zig:1002-1021), slower. Returns the previous
 * setting. */
int loom_cuda_tc_exact(int on);
/* Kernel family the last routed layer ran: 0 fused decode, 1 slot kernels,
 * 2 expert-major int8 batch kernels, 3 tensor cores; -1 before the first. */
int loom_cuda_last_path(void);
/* Phase tracing of the fused decode kernels (the counterpart of the
 * reference's LOOM_PROFILE phase timers, deepseek.zig:705-850): with room for
 * n_kernels traced launches, each decode kernel records its first CTA start
 * and last CTA end (GPU globaltimer, ns). Kernels are assigned trace entries
 * in launch order, twelve per layer: router, gate/up, down (first CTA start,
 * last CTA end), the router's post-wait span up to its cluster barrier, the
 * first post-wait instants of gate/up and down, (route done, activation
 * quantized) in the router, then SM-cycle counts (max over CTAs) of the
 * router's copy wait and dots, its route tail, gate/up's staging and dots,
 * and down's quantization and dots. n_kernels = 0
 * turns tracing off. */
int loom_cuda_trace_enable(size_t n_kernels);
/* Clear the recorded times (keeps the entry assignment of captured graphs). */
int loom_cuda_trace_reset(void);
/* Copy (start, end) pairs of the first n entries; returns entries copied. */
size_t loom_cuda_trace_read(uint64_t *out, size_t n_kernels);
/* Bitwise OR of the device error words the kernels raise instead of trapping
 * (1 = a bounded wait on an asynchronous copy gave up); 0 when none, -1 when
 * the stream itself is in error. Synchronizes the backend's stream. */
int loom_cuda_device_error(void);
/* Synchronize the backend's stream. */
int loom_cuda_sync(void);
/* The backend's stream (cudaStream_t). */
void *loom_cuda_stream(void);
/* Diagnostic (no counterpart in the reference): enable >= 0 turns the
 * tensor-core kernels' cycle profile of CTA 0 on (1) or off (0) and zeroes it;
 * enable < 0 synchronizes the device and copies min(n, 32) counters (gate/up
 * then down, 16 each) to out. */
int loom_cuda_tc_profile(int enable, unsigned long long *out, size_t n);
/* Diagnostic (no counterpart in the reference): a bf16 tcgen05 GEMM
 * D[M][N] = A[M][K] . B[N][K]^T on host arrays (bf16 bit patterns in, f32
 * out). M a multiple of 128, N in 16..256 in steps of 16, K a multiple of 64.
 * 0 ok, 1 bad arguments, 2 CUDA error, 3 an MMA completion wait gave up. */
int loom_cuda_umma_selftest(const uint16_t *A, const uint16_t *B, float *D, int M, int N, int K);

#ifdef __cplusplus
}
#endif
#endif
