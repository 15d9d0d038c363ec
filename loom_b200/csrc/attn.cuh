// attn.cuh -- the attention half of a decoder layer on the device (attn.cu):
// RMSNorm with the activation quantization fused in, per-head Q/K norm + RoPE
// + KV-cache append, and softmax attention over an f32 cache.
#pragma once
#include <cuda_runtime.h>

#include "decode.cuh"

namespace loom {

// x (+)= add (when add != null, written back to x); normed = rmsnorm(x) * w
// (tensor.zig:9-15); then normed quantized per 256 (q256.q != null, dim a
// multiple of 256) and/or per 32 (q32.q != null) for the matvecs that read it.
// The sum of squares is the reference's serial sum when `serial`, else a
// tree sum.
constexpr int RN_SERIAL_MAX = 1024;  // default: serial up to this width
// rows > 1: rows consecutive vectors (x, add, normed and the quantized forms
// advance by one row each), one CTA per row.
void launch_rmsnorm_q(float *x, const float *add, const float *w, int dim, float eps, float *normed, XQW q256,
                      XQW q32, bool serial, cudaStream_t st, int rows = 1);

// Per head: optional RMSNorm over head_dim (headNorm, llama.zig:938-950, serial
// sum), then RoPE at position *pos (ropeNeox / ropeNorm, llama.zig:830-858)
// with the (cos, sin) of pair j at rope[(pos * rope_dim / 2 + j) * 2], in
// place on q [n_heads][hd] and k [n_kv][hd]; k and v are stored at row *pos of
// this layer's caches kc / vc ([ctx][n_kv*hd]). Nothing is written when
// *pos >= ctx.
// ntok > 1: token i of a batch (q, k, v advance by one token's heads) at
// position *pos + i; with pos_rows, token i is sequence i at position pos[i]
// with its own cache rows at kc / vc + i * cache_stride (the same for the
// attention launchers below).
void launch_qk_rope(float *q, float *k, const float *v, const float *qn, const float *kn, int n_heads, int n_kv,
                    int hd, int rope_dim, int neox, const float *rope, float eps, const uint32_t *pos, int ctx,
                    float *kc, float *vc, cudaStream_t st, int ntok = 1, int pos_rows = 0, size_t cache_stride = 0);
// The ordered attention for a batch of ntok tokens at positions *pos + i
// (llama.zig:1749-1774 stepBatch: token i sees cache rows 0..*pos + i only),
// q and out [ntok][n_heads * hd]; one CTA per (query head, token).
// The same batch in another summation order (fused multiply-adds, tree sums),
// one CTA per (KV head, token) with one warp per query head: false when the
// shape does not fit (query heads per KV head > 16, hd not a multiple of 4, or
// scores of the context beyond 200 KB of shared memory).
// max_pos: the batch's last position (host-side bound of the scores' room).
bool launch_attention_prefill_rows(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd,
                                   float scale, const uint32_t *pos, int ctx, float *out, int ntok, int max_pos,
                                   cudaStream_t st, int pos_rows = 0, size_t cache_stride = 0);
// The split form (k_attn_part + k_attn_merge) for nrows sequences: row i at
// position pos[i] of its own cache (kc / vc + i * cache_stride); part holds
// nrows * attn_part_floats(...) floats; out [nrows][n_heads * hd], not quantized.
void launch_attention_split_rows(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd,
                                 float scale, const uint32_t *pos, int ctx, float *part, float *out, int nrows,
                                 size_t cache_stride, cudaStream_t st);
void launch_attention_ordered_rows(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd,
                                   float scale, const uint32_t *pos, int ctx, float *out, int ntok, cudaStream_t st,
                                   int pos_rows = 0, size_t cache_stride = 0);

// Softmax attention of every query head over cache rows 0..*pos
// (llama.zig:1171-1191), out [n_heads][hd].
// Ordered form (`ordered`): one CTA per query head keeps the
// reference's order of operations (dotF32 scores times the scale, serial
// softmax sum and 1/sum, axpy over positions in order).
// Split form: the rows are split in chunks of ATT_CH across CTAs (one CTA
// per KV head and chunk, all its query heads against one read of each row),
// each with a running maximum and sum; a merge kernel combines the chunks.
// `part` holds attn_part_floats(...) floats (split form only). With the split
// form the merge also quantizes the output (q256 / q32 non-null) when
// attn_merge_quantizes(); otherwise the caller quantizes `out` itself.
constexpr int ATT_CH = 32;
constexpr int ATT_ORDERED_MAX = 512;      // default: ordered up to this context
constexpr int ATT_ORDERED_LIMIT = 32768;  // largest context of the ordered form
size_t attn_part_floats(int n_heads, int n_kv, int hd, int ctx);
// Split-position MLA attention (contexts past the ordered limit, not exact_order):
// records [n_heads][ctx / 16][kvr + 4] in `part` (mla_part_floats), then c_acc.
// err (optional) gets bit 4 when a chunk's bulk copies time out.
size_t mla_part_floats(int n_heads, int kvr, int ctx);
bool mla_split_supported(int kvr, int rope);
void launch_mla_split(const float *qa, const float *q, int kvr, int rope, int kd, int nope, int n_heads, float scale,
                      const uint32_t *pos, int ctx, const float *c_cache, const float *r_cache, float *part,
                      float *c_acc, int *err, cudaStream_t st);
bool attn_merge_quantizes(int n_heads, int hd, int ctx);
void launch_attention(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd, float scale,
                      const uint32_t *pos, int ctx, float *part, float *out, bool ordered, XQW q256, XQW q32,
                      cudaStream_t st);

// MLA (deepseek.zig:851-1049). front: the compressed and rope cache rows at
// *pos from kv_a [kvr + rope] (RMSNorm with kv_norm; RoPE adjacent pairs) and
// the RoPE of every head's q rope part (q [n_heads][kd], rope part at nope).
void launch_mla_front(const float *kv_a, const float *kv_norm, int kvr, int rope, float eps, float *q, int n_heads,
                      int kd, int nope, const float *rope_tab, const uint32_t *pos, int ctx, float *c_cache,
                      float *r_cache, cudaStream_t st);
// attention in compressed space over rows 0..*pos: c_acc [n_heads][kvr]
// (ctx <= ATT_ORDERED_LIMIT)
void launch_mla_attn(const float *qa, const float *q, int kvr, int rope, int kd, int nope, int n_heads, float scale,
                     const uint32_t *pos, int ctx, const float *c_cache, const float *r_cache, float *c_acc,
                     cudaStream_t st);

}  // namespace loom
