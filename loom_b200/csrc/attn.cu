// attn.cu -- the attention half of a decoder layer (llama.zig:1138-1195) on
// the device: RMSNorm + activation quantization, Q/K head norm + RoPE + KV
// append, and softmax attention over the f32 KV cache.
//
// Every elementwise step is the reference's arithmetic with one rounding per
// multiply or add (no contraction). The reductions follow the reference's
// order where that is cheap (RMSNorm up to 1024 wide, head norms, the
// ordered attention: dotF32 scores, serial softmax sum, axpy in position
// order); the wide RMSNorm and the split attention use tree / chunked sums.
#include <cstdlib>

#include "attn.cuh"
#include "devutil.cuh"
#include "pdl.cuh"
#include "tma.cuh"

namespace loom {

namespace {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ggml.zig:198-217 dotF32 of a and b (n floats) by one thread: four 8-lane
// accumulators over 32-wide steps, an 8-wide tail into the first, the four
// added lane by lane ((a0 + a1) + a2) + a3, lanes 0..7 added in order, then a
// scalar tail.
__device__ __forceinline__ float dot_f32_ordered(const float *a, const float *b, int n) {
    float acc[4][8];
#pragma unroll
    for (int k = 0; k < 4; k++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[k][j] = 0.0f;
    int i = 0;
    for (; i + 32 <= n; i += 32)
#pragma unroll
        for (int k = 0; k < 4; k++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[k][j] = fadd(acc[k][j], fmul(a[i + 8 * k + j], b[i + 8 * k + j]));
    for (; i + 8 <= n; i += 8)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[0][j] = fadd(acc[0][j], fmul(a[i + j], b[i + j]));
    float r = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float v = fadd(fadd(fadd(acc[0][j], acc[1][j]), acc[2][j]), acc[3][j]);
        r = j == 0 ? v : fadd(r, v);
    }
    for (; i < n; i++) r = fadd(r, fmul(a[i], b[i]));
    return r;
}

// ---- RMSNorm (+ residual add) + quantization ---------------------------------------

constexpr int RN_THREADS = 1024;

__global__ void __launch_bounds__(RN_THREADS) k_rmsnorm_q(float *x, const float *add, const float *w, int dim,
                                                          float eps, float *normed, XQW q256, XQW q32,
                                                          int serial) {
    extern __shared__ float sx[];  // [dim]
    __shared__ float red[RN_THREADS / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (blockIdx.y) {  // row blockIdx.y of a batch: every vector advances by its row
        const size_t y = blockIdx.y;
        x += y * dim;
        if (add) add += y * dim;
        normed += y * dim;
        if (q256.q) {
            q256.q += y * dim;
            q256.d += y * (dim / 256);
            q256.s += y * (dim / 16);
        }
        if (q32.q) {
            q32.q += y * dim;
            q32.d += y * (dim / 32);
            q32.s += y * (dim / 32);
        }
    }
    pdl_wait_();
    pdl_trigger_();
    float ss = 0.0f;
    for (int i = tid; i < dim; i += RN_THREADS) {
        float v = x[i];
        if (add) {
            v = fadd(v, add[i]);  // tensor.zig:48 add
            x[i] = v;
        }
        sx[i] = v;
        if (!serial) ss = fadd(ss, fmul(v, v));
    }
    if (serial) {
        __syncthreads();
        if (tid == 0) {  // tensor.zig:11: for (x) |v| ss += v * v
            float s = 0.0f;
            for (int i = 0; i < dim; i++) s = fadd(s, fmul(sx[i], sx[i]));
            red[0] = s;
        }
    } else {
        ss = warp_sum_f(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float t = lane < RN_THREADS / 32 ? red[lane] : 0.0f;
            t = warp_sum_f(t);
            if (lane == 0) red[0] = t;
        }
    }
    __syncthreads();
    // tensor.zig:12-13: scale = 1 / sqrt(ss / n + eps); out = v * scale * w
    const float scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(red[0], (float)dim), eps)));
    for (int i = tid; i < dim; i += RN_THREADS) {
        const float nv = fmul(fmul(sx[i], scale), w[i]);
        normed[i] = nv;
        sx[i] = nv;
    }
    __syncthreads();
    const int nwarps = RN_THREADS / 32;
    if (q256.q) {
        for (int b = warp; b < dim / 256; b += nwarps) {
            const int off = b * 256 + lane * 8;
            quant_lane8(sx + off, true, 32, q256.q + off, q256.d + b, q256.s + b * 16 + lane / 2, nullptr, lane);
        }
    }
    if (q32.q) {
        const int nb = dim / 32, ng = (nb + 7) / 8;
        for (int g = warp; g < ng; g += nwarps) {
            const int b = g * 8 + lane / 4;
            const bool live = b < nb;
            const int off = b * 32 + (lane & 3) * 8;
            quant_lane8(sx + (live ? off : 0), live, 4, q32.q + off, q32.d + b, nullptr, q32.s + b, lane);
        }
    }
}

// ---- head norm + RoPE + cache append -----------------------------------------------

constexpr int QR_WARPS = 8;
constexpr int MAX_HD = 256;

__global__ void __launch_bounds__(QR_WARPS * 32) k_qk_rope(float *q, float *k, const float *v, const float *qn,
                                                          const float *kn, int n_heads, int n_kv, int hd,
                                                          int rope_dim, int neox, const float *rope, float eps,
                                                          const uint32_t *pos_p, int ctx, float *kc, float *vc,
                                                          int pos_rows, size_t cache_stride) {
    __shared__ float hv_all[QR_WARPS][MAX_HD];
    __shared__ float inv_all[QR_WARPS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int head = blockIdx.x * QR_WARPS + warp;
    // token blockIdx.y of a batch at position *pos_p + blockIdx.y
    q += (size_t)blockIdx.y * n_heads * hd;
    k += (size_t)blockIdx.y * n_kv * hd;
    v += (size_t)blockIdx.y * n_kv * hd;
    kc += blockIdx.y * cache_stride;
    vc += blockIdx.y * cache_stride;
    pdl_wait_();
    pdl_trigger_();
    if (head >= n_heads + n_kv) return;
    // row blockIdx.y: position pos_p[y] of its own cache (a batch of sequences, pos_rows) or *pos_p + y
    const int pos = pos_rows ? (int)pos_p[blockIdx.y] : (int)*pos_p + (int)blockIdx.y;
    if (pos >= ctx) return;
    const bool isk = head >= n_heads;
    const int kh = head - n_heads;
    float *vec = isk ? k + (size_t)kh * hd : q + (size_t)head * hd;
    const float *g = isk ? kn : qn;
    float *hv = hv_all[warp];
    for (int i = lane; i < hd; i += 32) hv[i] = vec[i];
    __syncwarp();
    if (g) {  // headNorm: serial ss; inv = 1 / sqrt(ss / hd + eps); v * inv * g
        if (lane == 0) {
            float ss = 0.0f;
            for (int i = 0; i < hd; i++) ss = fadd(ss, fmul(hv[i], hv[i]));
            inv_all[warp] = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)hd), eps)));
        }
        __syncwarp();
        const float inv = inv_all[warp];
        for (int i = lane; i < hd; i += 32) hv[i] = fmul(fmul(hv[i], inv), g[i]);
        __syncwarp();
    }
    const float *cs = rope + (size_t)pos * rope_dim;  // (cos, sin) of the pairs at this position
    const int half = rope_dim / 2;
    for (int j = lane; j < half; j += 32) {
        const int ia = neox ? j : 2 * j, ib = neox ? j + half : 2 * j + 1;
        const float c = cs[2 * j], s = cs[2 * j + 1];
        const float a = hv[ia], b = hv[ib];
        hv[ia] = fsub(fmul(a, c), fmul(b, s));
        hv[ib] = fadd(fmul(a, s), fmul(b, c));
    }
    __syncwarp();
    for (int i = lane; i < hd; i += 32) vec[i] = hv[i];
    if (isk) {  // llama.zig:1157-1159 cache append
        const size_t row = (size_t)pos * n_kv * hd + (size_t)kh * hd;
        for (int i = lane; i < hd; i += 32) {
            kc[row + i] = hv[i];
            vc[row + i] = v[(size_t)kh * hd + i];
        }
    }
}

// ---- attention ------------------------------------------------------------------------

constexpr int AT_THREADS = 128, AT_WARPS = AT_THREADS / 32;
constexpr int MAX_GQA = 16;

// Ordered form: one CTA per query head.
__global__ void __launch_bounds__(AT_THREADS) k_attn_ordered(const float *q, const float *kc, const float *vc,
                                                            int n_heads, int n_kv, int hd, float scale,
                                                            const uint32_t *pos_p, int ctx, float *out, int pos_rows,
                                                            size_t cache_stride) {
    __shared__ float qs[MAX_HD];
    extern __shared__ float sc[];  // [ctx]
    __shared__ float inv_s;
    const int h = blockIdx.x, tid = threadIdx.x;
    // token blockIdx.y of a batch at position *pos_p + blockIdx.y: causal, it sees rows 0..its position
    q += (size_t)blockIdx.y * n_heads * hd;
    out += (size_t)blockIdx.y * n_heads * hd;
    kc += blockIdx.y * cache_stride;
    vc += blockIdx.y * cache_stride;
    pdl_wait_();
    pdl_trigger_();
    // row blockIdx.y: position pos_p[y] of its own cache (a batch of sequences, pos_rows) or *pos_p + y
    const int pos = pos_rows ? (int)pos_p[blockIdx.y] : (int)*pos_p + (int)blockIdx.y;
    if (pos >= ctx) return;
    const int seq = pos + 1, kvd = n_kv * hd;
    const int kvh = h / (n_heads / n_kv);
    for (int i = tid; i < hd; i += AT_THREADS) qs[i] = q[(size_t)h * hd + i];
    __syncthreads();
    for (int t = tid; t < seq; t += AT_THREADS)  // llama.zig:1175: dotF32(qh, kt) * scale
        sc[t] = fmul(dot_f32_ordered(qs, kc + (size_t)t * kvd + (size_t)kvh * hd, hd), scale);
    __syncthreads();
    if (tid < 32) {  // tensor.zig:18-28 softmax: max, exp(v - m), serial sum, inv = 1 / sum
        float m = -INFINITY;
        for (int t = tid; t < seq; t += 32) m = fmaxf(m, sc[t]);
        m = warp_max(m);
        for (int t = tid; t < seq; t += 32) sc[t] = exp_f(fsub(sc[t], m));
        __syncwarp();
        if (tid == 0) {
            float sum = 0.0f;
            for (int t = 0; t < seq; t++) sum = fadd(sum, sc[t]);
            inv_s = fdiv(1.0f, sum);
        }
        __syncwarp();
        const float inv = inv_s;
        for (int t = tid; t < seq; t += 32) sc[t] = fmul(sc[t], inv);
    }
    __syncthreads();
    for (int d = tid; d < hd; d += AT_THREADS) {  // ggml.zig:222 axpy per position, in order, from 0
        float o = 0.0f;
        const float *vp = vc + (size_t)kvh * hd + d;
        for (int t = 0; t < seq; t++) o = fadd(o, fmul(sc[t], vp[(size_t)t * kvd]));
        out[(size_t)h * hd + d] = o;
    }
}

// Prefill form (batched causal attention, llama.zig:1759-1774 in another
// order): one CTA per (KV head, token), one warp per query head of the group.
// Each lane scores keys lane, lane + 32, ... (float4 rows from L2, fused
// multiply-adds), the warp takes the maximum and the sum of e^(s - max), then
// lane l accumulates dims 4l..4l+3 of sum_t p_t v_t over the positions. The
// group's warps read the same key and value rows (L1 hits after the first).
// HD > 0: the head width at compile time (loops unrolled, loads in flight together); 0: hd.
constexpr int AP_MAX_GQ = 16;
template <int HD>
__global__ void __launch_bounds__(AP_MAX_GQ * 32) k_attn_prefill(const float *q, const float *kc, const float *vc,
                                                                 int n_heads, int n_kv, int hd_, float scale,
                                                                 const uint32_t *pos_p, int ctx, float *out,
                                                                 int smax, int pos_rows, size_t cache_stride) {
    extern __shared__ float ap_sm[];  // per warp: the query head [hd], the scores [smax]
    const int hd = HD > 0 ? HD : hd_;
    const int g = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int GQ = n_heads / n_kv, h = g * GQ + w, kvd = n_kv * hd;
    q += (size_t)blockIdx.y * n_heads * hd;
    out += (size_t)blockIdx.y * n_heads * hd;
    kc += blockIdx.y * cache_stride;
    vc += blockIdx.y * cache_stride;
    pdl_wait_();
    pdl_trigger_();
    // row blockIdx.y: position pos_p[y] of its own cache (a batch of sequences, pos_rows) or *pos_p + y
    const int pos = pos_rows ? (int)pos_p[blockIdx.y] : (int)*pos_p + (int)blockIdx.y;
    if (pos >= ctx || w >= GQ) return;
    const int seq = pos + 1;
    if (seq > smax) return;  // (the launch sized the scores for the batch's last position)
    float *qs = ap_sm + (size_t)w * (hd + smax), *sc = qs + hd;
    for (int i = lane; i < hd; i += 32) qs[i] = q[(size_t)h * hd + i];
    __syncwarp();
    const float *kb = kc + (size_t)g * hd, *vb = vc + (size_t)g * hd;
    float m = -INFINITY;
    // scores of 512 keys at a time, key lane + 32 k in acc[k]; the query read from shared memory
    // once per 32 dims (a broadcast) into registers, not once per key
    for (int tb = 0; tb < seq; tb += 512) {
        float acc[16];
#pragma unroll
        for (int k = 0; k < 16; k++) acc[k] = 0.0f;
        for (int c = 0; c < hd; c += 32) {
            const int cw = min(32, hd - c);
            float4 qr[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                qr[i] = 4 * i < cw ? *reinterpret_cast<const float4 *>(qs + c + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int t = tb + lane + 32 * k;
                if (t < seq) {
                    const float4 *kr = reinterpret_cast<const float4 *>(kb + (size_t)t * kvd + c);
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        if (4 * i < cw) {
                            const float4 k4 = __ldg(kr + i);
                            acc[k] = fmaf(k4.x, qr[i].x, acc[k]);
                            acc[k] = fmaf(k4.y, qr[i].y, acc[k]);
                            acc[k] = fmaf(k4.z, qr[i].z, acc[k]);
                            acc[k] = fmaf(k4.w, qr[i].w, acc[k]);
                        }
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const int t = tb + lane + 32 * k;
            if (t < seq) {
                const float s2 = acc[k] * scale;
                sc[t] = s2;
                m = fmaxf(m, s2);
            }
        }
    }
    m = warp_max(m);
    float sum = 0.0f;
    for (int t = lane; t < seq; t += 32) {
        const float e = exp_f(sc[t] - m);
        sc[t] = e;
        sum += e;
    }
    sum = warp_sum_f(sum);
    __syncwarp();
    const float inv = 1.0f / sum;
    for (int d4 = lane; d4 < hd / 4; d4 += 32) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        const int seq4 = seq & ~3;
#pragma unroll 2
        for (int t = 0; t < seq4; t += 4) {  // four weights per shared-memory read
            const float4 p4 = *reinterpret_cast<const float4 *>(sc + t);
            const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float4 v4 = __ldg(reinterpret_cast<const float4 *>(vb + (size_t)(t + u) * kvd) + d4);
                o.x = fmaf(pp[u], v4.x, o.x);
                o.y = fmaf(pp[u], v4.y, o.y);
                o.z = fmaf(pp[u], v4.z, o.z);
                o.w = fmaf(pp[u], v4.w, o.w);
            }
        }
        for (int t = seq4; t < seq; t++) {
            const float p = sc[t];
            const float4 v4 = __ldg(reinterpret_cast<const float4 *>(vb + (size_t)t * kvd) + d4);
            o.x = fmaf(p, v4.x, o.x);
            o.y = fmaf(p, v4.y, o.y);
            o.z = fmaf(p, v4.z, o.z);
            o.w = fmaf(p, v4.w, o.w);
        }
        reinterpret_cast<float4 *>(out + (size_t)h * hd)[d4] = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    }
}

// Prefill form for GQA groups of 8 heads of 128 (the Qwen3 shape), tiled:
// one CTA per (KV head, 8 consecutive tokens), warp w = token t0 + w with all
// 8 query heads of the group. Key and value rows go through shared memory in
// chunks of 32 positions, read once for the tile's 64 query rows (instead of
// once per warp of every token); per query row a running maximum and sum
// (online softmax) and the output dims 4l..4l+3 of every head in lane l.
constexpr int APT_TOK = 8, APT_GQ = 8, APT_HD = 128, APT_CH = 32, APT_KS = APT_HD + 4;
constexpr size_t APT_SMEM = (size_t)(APT_CH * APT_KS + APT_CH * APT_HD + APT_TOK * APT_GQ * APT_HD + APT_TOK * APT_GQ * APT_CH) * 4;
__global__ void __launch_bounds__(APT_TOK * 32) k_attn_prefill_tile(const float *q, const float *kc, const float *vc,
                                                                    int n_heads, int n_kv, float scale,
                                                                    const uint32_t *pos_p, int ctx, int ntok, float *out) {
    extern __shared__ __align__(16) float apt[];
    float *sK = apt, *sV = sK + APT_CH * APT_KS, *sQ = sV + APT_CH * APT_HD, *sP = sQ + APT_TOK * APT_GQ * APT_HD;
    const int g = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int kvd = n_kv * APT_HD, t0 = blockIdx.y * APT_TOK;
    pdl_wait_();
    pdl_trigger_();
    const int pos0 = (int)*pos_p;
    const int tok = t0 + w, p = pos0 + tok;  // this warp's token and position
    const bool live = tok < ntok && p < ctx;
    const int last = min(pos0 + min(t0 + APT_TOK, ntok) - 1, ctx - 1);  // the tile's last position
    // the tile's query rows: token t, head hh at sQ[(t * 8 + hh) * 128]
    for (int i = tid; i < APT_TOK * APT_GQ * APT_HD / 4; i += APT_TOK * 32) {
        const int t = i / (APT_GQ * APT_HD / 4), r = i - t * (APT_GQ * APT_HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + t < ntok)
            v = reinterpret_cast<const float4 *>(q + (size_t)(t0 + t) * n_heads * APT_HD + (size_t)g * APT_GQ * APT_HD)[r];
        reinterpret_cast<float4 *>(sQ)[i] = v;
    }
    float m[APT_GQ], l[APT_GQ];
    float4 o[APT_GQ];
#pragma unroll
    for (int h = 0; h < APT_GQ; h++) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
        o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float *qw = sQ + (size_t)w * APT_GQ * APT_HD;
    float *pw = sP + (size_t)w * APT_GQ * APT_CH;
    for (int c0 = 0; c0 <= last; c0 += APT_CH) {
        __syncthreads();  // the previous chunk's rows are no longer read
        for (int i = tid; i < APT_CH * APT_HD / 4; i += APT_TOK * 32) {
            const int j = i / (APT_HD / 4), d4 = i - j * (APT_HD / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (c0 + j <= last) {
                kv = __ldg(reinterpret_cast<const float4 *>(kc + (size_t)(c0 + j) * kvd + (size_t)g * APT_HD) + d4);
                vv = __ldg(reinterpret_cast<const float4 *>(vc + (size_t)(c0 + j) * kvd + (size_t)g * APT_HD) + d4);
            }
            *reinterpret_cast<float4 *>(sK + j * APT_KS + 4 * d4) = kv;
            reinterpret_cast<float4 *>(sV)[i] = vv;
        }
        __syncthreads();
        if (!live || c0 > p) continue;  // warp-uniform: every key of the chunk is past this token
        // scores: lane = key c0 + lane, all 8 heads
        float sc[APT_GQ];
#pragma unroll
        for (int h = 0; h < APT_GQ; h++) sc[h] = 0.0f;
        const float *kr = sK + lane * APT_KS;
#pragma unroll 4
        for (int d = 0; d < APT_HD; d += 4) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
#pragma unroll
            for (int h = 0; h < APT_GQ; h++) {
                const float4 q4 = *reinterpret_cast<const float4 *>(qw + h * APT_HD + d);
                sc[h] = fmaf(k4.x, q4.x, fmaf(k4.y, q4.y, fmaf(k4.z, q4.z, fmaf(k4.w, q4.w, sc[h]))));
            }
        }
        const bool valid = c0 + lane <= p;
#pragma unroll
        for (int h = 0; h < APT_GQ; h++) {
            const float s2 = valid ? sc[h] * scale : -INFINITY;
            const float mc = warp_max(s2), mn = fmaxf(m[h], mc);
            const float e = valid ? exp_f(s2 - mn) : 0.0f;
            const float corr = m[h] == -INFINITY ? 0.0f : exp_f(m[h] - mn);
            l[h] = l[h] * corr + warp_sum_f(e);
            o[h].x *= corr;
            o[h].y *= corr;
            o[h].z *= corr;
            o[h].w *= corr;
            m[h] = mn;
            pw[h * APT_CH + lane] = e;
        }
        __syncwarp();
        // o[h] += sum_j e[h][j] v_j, dims 4 lane .. 4 lane + 3
        const int jn = min(APT_CH, p - c0 + 1);
        for (int j = 0; j < jn; j++) {
            const float4 v4 = reinterpret_cast<const float4 *>(sV + j * APT_HD)[lane];
#pragma unroll
            for (int h = 0; h < APT_GQ; h++) {
                const float e = pw[h * APT_CH + j];
                o[h].x = fmaf(e, v4.x, o[h].x);
                o[h].y = fmaf(e, v4.y, o[h].y);
                o[h].z = fmaf(e, v4.z, o[h].z);
                o[h].w = fmaf(e, v4.w, o[h].w);
            }
        }
        __syncwarp();
    }
    if (!live) return;
#pragma unroll
    for (int h = 0; h < APT_GQ; h++) {
        const float inv = 1.0f / l[h];
        reinterpret_cast<float4 *>(out + (size_t)tok * n_heads * APT_HD + (size_t)(g * APT_GQ + h) * APT_HD)[lane] =
            make_float4(o[h].x * inv, o[h].y * inv, o[h].z * inv, o[h].w * inv);
    }
}

// Split form: one CTA per (KV head g, chunk sp of ATT_CH cache rows). The
// chunk's key and value rows are staged into shared memory with cp.async (all
// of them in flight at once; keys at a padded row stride so a warp's rows fall
// on distinct banks), then each thread scores one row against two query heads
// of the group. Partial record per query head: o[hd] = sum_t e^(s_t - m) v_t,
// then m and l = sum_t e^(s_t - m). The split form does not follow the
// reference's summation order, so it uses fused multiply-adds.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

__host__ __device__ constexpr int att_kstride(int hd) { return hd + 4; }

__global__ void __launch_bounds__(AT_THREADS) k_attn_part(const float *q, const float *kc, const float *vc,
                                                         int n_heads, int n_kv, int hd, float scale,
                                                         const uint32_t *pos_p, int ctx, int nsplit, float *part,
                                                         int pos_rows, size_t cache_stride, size_t part_stride) {
    extern __shared__ __align__(16) float sm[];
    const int G = n_heads / n_kv, kvd = n_kv * hd, KS = att_kstride(hd);
    // row blockIdx.z of a batch of sequences (pos_rows): its query, its cache, its records
    q += (size_t)blockIdx.z * n_heads * hd;
    kc += blockIdx.z * cache_stride;
    vc += blockIdx.z * cache_stride;
    part += blockIdx.z * part_stride;
    float *sK = sm;                      // [ATT_CH][KS]
    float *sV = sK + ATT_CH * KS;        // [ATT_CH][hd]
    float *qs = sV + ATT_CH * hd;        // [G][hd]
    float *sc = qs + G * hd;             // [G][ATT_CH]
    const int g = blockIdx.x, sp = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait_();
    pdl_trigger_();
    const int pos = pos_rows ? (int)pos_p[blockIdx.z] : (int)*pos_p;
    if (pos >= ctx) return;
    const int seq = pos + 1, t0 = sp * ATT_CH;
    if (t0 >= seq) return;
    const int n = min(ATT_CH, seq - t0);
    const float *kb = kc + (size_t)t0 * kvd + (size_t)g * hd, *vb = vc + (size_t)t0 * kvd + (size_t)g * hd;
    const bool vec4 = (hd & 3) == 0;
    if (vec4) {
        const int q4 = hd / 4;
        for (int i = tid; i < n * q4; i += AT_THREADS) {
            const int j = i / q4, c = (i % q4) * 4;
            cp_async16(sK + j * KS + c, kb + (size_t)j * kvd + c);
            cp_async16(sV + j * hd + c, vb + (size_t)j * kvd + c);
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    } else {
#pragma unroll 4
        for (int i = tid; i < n * hd; i += AT_THREADS) {
            const int j = i / hd, c = i % hd;
            sK[j * KS + c] = kb[(size_t)j * kvd + c];
            sV[i] = vb[(size_t)j * kvd + c];
        }
    }
    for (int i = tid; i < G * hd; i += AT_THREADS) qs[i] = q[(size_t)g * G * hd + i];
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    // scores: lane = cache row, warp = pair of query heads
    const int HP = (G + 1) / 2;
    for (int hp = warp; hp < HP; hp += AT_WARPS) {
        const int j = lane, ha = 2 * hp, hb = min(2 * hp + 1, G - 1);
        if (j < n) {
            const float *kr = sK + j * KS, *qa = qs + ha * hd, *qb = qs + hb * hd;
            float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
            if (vec4) {
                for (int d = 0; d < hd; d += 4) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
                    const float4 x4 = *reinterpret_cast<const float4 *>(qa + d);
                    const float4 y4 = *reinterpret_cast<const float4 *>(qb + d);
                    a0 = fmaf(k4.x, x4.x, a0); a1 = fmaf(k4.y, x4.y, a1);
                    a0 = fmaf(k4.z, x4.z, a0); a1 = fmaf(k4.w, x4.w, a1);
                    b0 = fmaf(k4.x, y4.x, b0); b1 = fmaf(k4.y, y4.y, b1);
                    b0 = fmaf(k4.z, y4.z, b0); b1 = fmaf(k4.w, y4.w, b1);
                }
            } else {
                for (int d = 0; d < hd; d++) {
                    a0 = fmaf(kr[d], qa[d], a0);
                    b0 = fmaf(kr[d], qb[d], b0);
                }
            }
            sc[ha * ATT_CH + j] = (a0 + a1) * scale;
            sc[hb * ATT_CH + j] = (b0 + b1) * scale;
        }
    }
    __syncthreads();
    float *rec = part + ((size_t)g * nsplit + sp) * G * (hd + 2);
    for (int hh = warp; hh < G; hh += AT_WARPS) {  // chunk max, exponentials, sum (one row per lane)
        const float v = lane < n ? sc[hh * ATT_CH + lane] : -INFINITY;
        const float m = warp_max(v);
        const float e = lane < n ? exp_f(v - m) : 0.0f;
        if (lane < n) sc[hh * ATT_CH + lane] = e;
        const float l = warp_sum_f(e);
        if (lane == 0) {
            rec[hh * (hd + 2) + hd] = m;
            rec[hh * (hd + 2) + hd + 1] = l;
        }
    }
    __syncthreads();
    for (int d = tid; d < hd; d += AT_THREADS) {  // o = sum_t e_t v_t
        float acc[MAX_GQA];
#pragma unroll
        for (int hh = 0; hh < MAX_GQA; hh++) acc[hh] = 0.0f;
        for (int j = 0; j < n; j++) {
            const float vv = sV[j * hd + d];
#pragma unroll
            for (int hh = 0; hh < MAX_GQA; hh++)
                if (hh < G) acc[hh] = fmaf(sc[hh * ATT_CH + j], vv, acc[hh]);
        }
#pragma unroll
        for (int hh = 0; hh < MAX_GQA; hh++)
            if (hh < G) rec[hh * (hd + 2) + d] = acc[hh];
    }
}

// Merge: one CTA per 256 consecutive outputs (ATT_MG_HEADS query heads of
// 256 / ATT_MG_HEADS values): out = (sum_s o_s e^(m_s - M)) / (sum_s l_s
// e^(m_s - M)), the weights e^(m_s - M) computed once per head and split;
// then, when q256 / q32 are given, the 256 outputs are quantized for the
// output projection (quantizeX256 / quantizeX), so no separate pass reads them.
__global__ void __launch_bounds__(256) k_attn_merge(const float *part, int n_heads, int n_kv, int hd,
                                                   const uint32_t *pos_p, int ctx, int nsplit, float *out, XQW q256,
                                                   XQW q32, int pos_rows, size_t part_stride) {
    extern __shared__ float wsm[];  // [heads in CTA][nsplit] weights
    __shared__ float Ls[40];  // heads per CTA <= 256 / 8 + 1 (head_dim >= 8)
    __shared__ __align__(16) float val[256];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait_();
    pdl_trigger_();
    part += blockIdx.z * part_stride;  // row blockIdx.z of a batch of sequences (pos_rows)
    out += (size_t)blockIdx.z * n_heads * hd;
    const int pos = pos_rows ? (int)pos_p[blockIdx.z] : (int)*pos_p;
    if (pos >= ctx) return;
    const int G = n_heads / n_kv, qd = n_heads * hd;
    const int live = (pos + 1 + ATT_CH - 1) / ATT_CH;
    const size_t stride = (size_t)G * (hd + 2);
    const int e0 = blockIdx.x * 256;
    const int h0 = e0 / hd, h1 = min((e0 + 256 - 1) / hd, n_heads - 1);
    // per head of this CTA (one warp each): M, weights, L (splits in order)
    for (int lh = warp; lh <= h1 - h0; lh += 8) {  // per-head smem: (h1 - h0 + 1) x nsplit floats
        const int h = h0 + lh, g = h / G, hh = h % G;
        const float *rec = part + (size_t)g * nsplit * stride + (size_t)hh * (hd + 2);
        float *w = wsm + (size_t)lh * nsplit;
        float M = -INFINITY;
        for (int s = lane; s < live; s += 32) M = fmaxf(M, rec[s * stride + hd]);
        M = warp_max(M);
        float L = 0.0f;
        for (int s = lane; s < live; s += 32) {
            const float ws = exp_f(rec[s * stride + hd] - M);
            w[s] = ws;
            L = fmaf(rec[s * stride + hd + 1], ws, L);
        }
        L = warp_sum_f(L);
        if (lane == 0) Ls[lh] = L;
    }
    __syncthreads();
    const int e = e0 + tid;
    float o = 0.0f;
    if (e < qd) {
        const int h = e / hd, d = e % hd, g = h / G, hh = h % G, lh = h - h0;
        const float *rec = part + (size_t)g * nsplit * stride + (size_t)hh * (hd + 2) + d;
        const float *w = wsm + (size_t)lh * nsplit;
#pragma unroll 8
        for (int s = 0; s < live; s++) o = fmaf(rec[s * stride], w[s], o);
        o = o / Ls[lh];
        out[e] = o;
    }
    val[tid] = o;
    __syncthreads();
    if (q256.q && warp == 0 && e0 + 256 <= qd) {
        const int off = lane * 8;
        quant_lane8(val + off, true, 32, q256.q + e0 + off, q256.d + blockIdx.x, q256.s + e0 / 16 + lane / 2,
                    nullptr, lane);
    }
    if (q32.q && warp == 0) {
        const int b = e0 / 32 + lane / 4, nb = qd / 32;
        const bool live_b = b < nb;
        const int off = (lane / 4) * 32 + (lane & 3) * 8;
        quant_lane8(val + (live_b ? off : 0), live_b, 4, q32.q + e0 + off, q32.d + b, nullptr, q32.s + b, lane);
    }
}

// ---- MLA (deepseek.zig:851-1049) --------------------------------------------------------

// CTA 0: the compressed row c = RMSNorm(kv_a[0..kvr]) * kv_a_norm (serial sum
// of squares) and the rope row (kv_a[kvr..], RoPE at pos) into the caches.
// CTAs 1..: one warp per head, RoPE of the head's q rope part in place.
__global__ void __launch_bounds__(256) k_mla_front(const float *kv_a, const float *kv_norm, int kvr, int rope,
                                                  float eps, float *q, int n_heads, int kd, int nope,
                                                  const float *rope_tab, const uint32_t *pos_p, int ctx,
                                                  float *c_cache, float *r_cache) {
    __shared__ float red;
    extern __shared__ float kva_s[];  // [kvr] the compressed row, loaded by every thread at once
    pdl_wait_();
    pdl_trigger_();
    const int pos = (int)*pos_p;
    if (pos >= ctx) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *cs = rope_tab + (size_t)pos * rope;
    if (blockIdx.x == 0) {
        for (int i = tid; i < kvr; i += blockDim.x) kva_s[i] = kv_a[i];
        __syncthreads();
        if (tid == 0) {  // serial sum of squares (the reference's order), from shared memory
            float ss = 0.0f;
            for (int i = 0; i < kvr; i++) ss = fadd(ss, fmul(kva_s[i], kva_s[i]));
            red = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)kvr), eps)));
        }
        __syncthreads();
        float *c = c_cache + (size_t)pos * kvr;
        for (int i = tid; i < kvr; i += blockDim.x) c[i] = fmul(fmul(kva_s[i], red), kv_norm[i]);
        float *r = r_cache + (size_t)pos * rope;
        for (int j = tid; 2 * j + 1 < rope; j += blockDim.x) {  // ropeNormPlain: adjacent pairs
            const float a = kv_a[kvr + 2 * j], b = kv_a[kvr + 2 * j + 1], co = cs[2 * j], si = cs[2 * j + 1];
            r[2 * j] = fsub(fmul(a, co), fmul(b, si));
            r[2 * j + 1] = fadd(fmul(a, si), fmul(b, co));
        }
        return;
    }
    const int h = (blockIdx.x - 1) * (blockDim.x >> 5) + warp;
    if (h >= n_heads) return;
    float *v = q + (size_t)h * kd + nope;
    for (int j = lane; 2 * j + 1 < rope; j += 32) {
        const float a = v[2 * j], b = v[2 * j + 1], co = cs[2 * j], si = cs[2 * j + 1];
        v[2 * j] = fsub(fmul(a, co), fmul(b, si));
        v[2 * j + 1] = fadd(fmul(a, si), fmul(b, co));
    }
}

// One CTA per head, the reference's order: score_t = (dotF32(qa, c_t) +
// dotF32(q_rope, r_t)) * scale, softmax (max, exp, serial sum, 1/sum), then
// c_acc = sum_t p_t c_t in position order from +0 (axpy).
__global__ void __launch_bounds__(AT_THREADS) k_mla_attn(const float *qa, const float *q, int kvr, int rope, int kd,
                                                        int nope, float scale, const uint32_t *pos_p, int ctx,
                                                        const float *c_cache, const float *r_cache, float *c_acc) {
    extern __shared__ float sc[];  // [ctx]
    __shared__ float inv_s;
    const int h = blockIdx.x, tid = threadIdx.x;
    pdl_wait_();
    pdl_trigger_();
    const int pos = (int)*pos_p;
    if (pos >= ctx) return;
    const int seq = pos + 1;
    const float *qh = qa + (size_t)h * kvr, *qr = q + (size_t)h * kd + nope;
    for (int t = tid; t < seq; t += AT_THREADS)
        sc[t] = fmul(fadd(dot_f32_ordered(qh, c_cache + (size_t)t * kvr, kvr),
                          dot_f32_ordered(qr, r_cache + (size_t)t * rope, rope)),
                     scale);
    __syncthreads();
    if (tid < 32) {
        float m = -INFINITY;
        for (int t = tid; t < seq; t += 32) m = fmaxf(m, sc[t]);
        m = warp_max(m);
        for (int t = tid; t < seq; t += 32) sc[t] = exp_f(fsub(sc[t], m));
        __syncwarp();
        if (tid == 0) {
            float sum = 0.0f;
            for (int t = 0; t < seq; t++) sum = fadd(sum, sc[t]);
            inv_s = fdiv(1.0f, sum);
        }
        __syncwarp();
        const float inv = inv_s;
        for (int t = tid; t < seq; t += 32) sc[t] = fmul(sc[t], inv);
    }
    __syncthreads();
    for (int j = tid; j < kvr; j += AT_THREADS) {
        float o = 0.0f;
        for (int t = 0; t < seq; t++) o = fadd(o, fmul(sc[t], c_cache[(size_t)t * kvr + j]));
        c_acc[(size_t)h * kvr + j] = o;
    }
}

// Split-position MLA attention (the fast form; contexts past the ordered
// limit): CTA (s, hg) takes positions [s*MLA_CH, +MLA_CH) for heads
// [16 hg, +16). The chunk's compressed and rope rows and the heads' absorbed
// queries come in by bulk copies; scores (warp per (head, position), lanes over
// the 576 columns), the chunk's softmax max / sum per head, then the
// chunk-weighted rows per head into a head-major record [head][split][REC]:
// kvr outputs, running max, sum. k_mla_merge rescales and sums the records.
constexpr int MLA_CH = 16, MLA_HG = 16, MLA_THREADS = 512;
constexpr uint32_t MLA_POLLS = 1u << 22;

__global__ void __launch_bounds__(MLA_THREADS) k_mla_part(const float *qa, const float *q, int kvr, int rope, int kd,
                                                         int nope, int n_heads, float scale, const uint32_t *pos_p,
                                                         int ctx, const float *c_cache, const float *r_cache,
                                                         float *part, int nsplit, int *err) {
    extern __shared__ __align__(16) float ms[];
    __shared__ __align__(8) uint64_t bar;
    pdl_wait_();
    pdl_trigger_();
    const int pos = (int)*pos_p;
    const int s = blockIdx.x, h0 = blockIdx.y * MLA_HG;
    const int t0 = s * MLA_CH;
    if (pos >= ctx || t0 > pos) return;
    const int n = min(MLA_CH, pos + 1 - t0), nh = min(MLA_HG, n_heads - h0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int REC = kvr + 4;
    float *sc_c = ms;                               // [MLA_CH][kvr]
    float *sc_r = sc_c + MLA_CH * kvr;              // [MLA_CH][rope]
    float *sq = sc_r + MLA_CH * rope;               // [MLA_HG][kvr]
    float *sqr = sq + MLA_HG * kvr;                 // [MLA_HG][rope]
    float *sp = sqr + MLA_HG * rope;                // [MLA_HG][MLA_CH] scores, then weights
    if (tid == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const uint32_t bytes = (uint32_t)(n * kvr + n * rope + nh * kvr) * 4;
        mbar_expect_tx(&bar, bytes);
        bulk_g2s(sc_c, c_cache + (size_t)t0 * kvr, (uint32_t)(n * kvr * 4), &bar);
        bulk_g2s(sc_r, r_cache + (size_t)t0 * rope, (uint32_t)(n * rope * 4), &bar);
        bulk_g2s(sq, qa + (size_t)h0 * kvr, (uint32_t)(nh * kvr * 4), &bar);
    }
    for (int i = tid; i < nh * rope; i += MLA_THREADS) {  // the heads' rope parts (strided rows)
        const int hh = i / rope, j = i - hh * rope;
        sqr[i] = __ldg(q + (size_t)(h0 + hh) * kd + nope + j);
    }
    __syncthreads();
    if (!mbar_wait(&bar, 0, MLA_POLLS)) {
        if (tid == 0 && err) atomicOr(err, 4);
        return;
    }
    // scores: warp per (head, position)
    for (int pr = warp; pr < nh * n; pr += MLA_THREADS / 32) {
        const int hh = pr / n, t = pr - hh * n;
        const float *qh = sq + hh * kvr, *ct = sc_c + t * kvr, *qr = sqr + hh * rope, *rt = sc_r + t * rope;
        float a = 0.0f;
        for (int j = lane; j < kvr; j += 32) a = fmaf(qh[j], ct[j], a);
        for (int j = lane; j < rope; j += 32) a = fmaf(qr[j], rt[j], a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) sp[hh * MLA_CH + t] = a * scale;
    }
    __syncthreads();
    if (warp < nh) {  // chunk max and sum per head
        const float v = lane < n ? sp[warp * MLA_CH + lane] : -INFINITY;
        const float m = warp_max(v);
        const float e = lane < n ? exp_f(v - m) : 0.0f;
        if (lane < n) sp[warp * MLA_CH + lane] = e;
        float l = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            float *rec = part + ((size_t)(h0 + warp) * nsplit + s) * REC;
            rec[kvr] = m;
            rec[kvr + 1] = l;
        }
    }
    __syncthreads();
    for (int j = tid; j < kvr; j += MLA_THREADS) {  // weighted rows: column j for every head
        float cv[MLA_CH];
#pragma unroll
        for (int t = 0; t < MLA_CH; t++) cv[t] = t < n ? sc_c[t * kvr + j] : 0.0f;
        for (int hh = 0; hh < nh; hh++) {
            float o = 0.0f;
#pragma unroll
            for (int t = 0; t < MLA_CH; t++) o = fmaf(sp[hh * MLA_CH + t], cv[t], o);
            part[((size_t)(h0 + hh) * nsplit + s) * REC + j] = o;
        }
    }
}

// c_acc[h][j] = sum_s rec_s[j] * exp(m_s - M) / sum_s l_s * exp(m_s - M), one
// CTA per head (columns across threads: each split's record row is read once
// and coalesced).
__global__ void __launch_bounds__(MLA_THREADS) k_mla_merge(int kvr, const uint32_t *pos_p, int ctx, const float *part,
                                                          int nsplit, float *c_acc) {
    extern __shared__ float wts[];  // [live] weights
    __shared__ float inv_l;
    pdl_wait_();
    pdl_trigger_();
    const int pos = (int)*pos_p;
    if (pos >= ctx) return;
    const int h = blockIdx.x, tid = threadIdx.x, REC = kvr + 4;
    const int live = (pos + 1 + MLA_CH - 1) / MLA_CH;
    const float *rec = part + (size_t)h * nsplit * REC;
    if (tid < 32) {
        float M = -INFINITY;
        for (int s2 = tid; s2 < live; s2 += 32) M = fmaxf(M, __ldcg(rec + (size_t)s2 * REC + kvr));
        M = warp_max(M);
        float L = 0.0f;
        for (int s2 = tid; s2 < live; s2 += 32) {
            const float w = exp_f(__ldcg(rec + (size_t)s2 * REC + kvr) - M);
            wts[s2] = w;
            L = fmaf(__ldcg(rec + (size_t)s2 * REC + kvr + 1), w, L);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (tid == 0) inv_l = 1.0f / L;
    }
    __syncthreads();
    for (int j = tid; j < kvr; j += MLA_THREADS) {
        float o = 0.0f;
        int s2 = 0;
        for (; s2 + 32 <= live; s2 += 32) {  // 32 record loads in flight, then added in order
            float v[32];
#pragma unroll
            for (int k = 0; k < 32; k++) v[k] = __ldcg(rec + (size_t)(s2 + k) * REC + j);
#pragma unroll
            for (int k = 0; k < 32; k++) o = fmaf(v[k], wts[s2 + k], o);
        }
        for (; s2 < live; s2++) o = fmaf(__ldcg(rec + (size_t)s2 * REC + j), wts[s2], o);
        c_acc[(size_t)h * kvr + j] = o * inv_l;
    }
}

unsigned cdiv_u(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

}  // namespace

void launch_rmsnorm_q(float *x, const float *add, const float *w, int dim, float eps, float *normed, XQW q256,
                      XQW q32, bool serial, cudaStream_t st, int rows) {
    launch_pdl_(k_rmsnorm_q, dim3(1, rows), dim3(RN_THREADS), (size_t)dim * 4, st, x, add, w, dim, eps, normed, q256,
                q32, (int)serial);
}

void launch_qk_rope(float *q, float *k, const float *v, const float *qn, const float *kn, int n_heads, int n_kv,
                    int hd, int rope_dim, int neox, const float *rope, float eps, const uint32_t *pos, int ctx,
                    float *kc, float *vc, cudaStream_t st, int ntok, int pos_rows, size_t cache_stride) {
    launch_pdl_(k_qk_rope, dim3(cdiv_u(n_heads + n_kv, QR_WARPS), ntok), dim3(QR_WARPS * 32), 0, st, q, k, v, qn, kn,
                n_heads, n_kv, hd, rope_dim, neox, rope, eps, pos, ctx, kc, vc, pos_rows, cache_stride);
}

bool launch_attention_prefill_rows(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd,
                                   float scale, const uint32_t *pos, int ctx, float *out, int ntok, int max_pos,
                                   cudaStream_t st, int pos_rows, size_t cache_stride) {
    const int gq = n_heads / n_kv;
    if (!pos_rows && gq == APT_GQ && hd == APT_HD && !getenv("LOOM_CUDA_NO_ATT_TILE")) {
        static bool set = false;
        if (!set) {
            cudaFuncSetAttribute(k_attn_prefill_tile, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)APT_SMEM);
            set = true;
        }
        return launch_pdl_(k_attn_prefill_tile, dim3(n_kv, cdiv_u(ntok, APT_TOK)), dim3(APT_TOK * 32), APT_SMEM, st, q,
                           kc, vc, n_heads, n_kv, scale, pos, ctx, ntok, out) == cudaSuccess;
    }
    const int smax = ((max_pos + 1 < ctx ? max_pos + 1 : ctx) + 3) & ~3;  // scores of the batch's last position at most
    const size_t smem = (size_t)gq * (hd + smax) * 4;
    if (gq > AP_MAX_GQ || hd % 4 || smem > 200 * 1024) return false;
    static bool smem_set = false;
    if (!smem_set) {
        cudaFuncSetAttribute(k_attn_prefill<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(k_attn_prefill<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        smem_set = true;
    }
    return launch_pdl_(hd == 128 ? k_attn_prefill<128> : k_attn_prefill<0>, dim3(n_kv, ntok), dim3(gq * 32), smem, st,
                       q, kc, vc, n_heads, n_kv, hd, scale, pos, ctx, out, smax, pos_rows, cache_stride) == cudaSuccess;
}

void launch_attention_ordered_rows(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd,
                                   float scale, const uint32_t *pos, int ctx, float *out, int ntok, cudaStream_t st,
                                   int pos_rows, size_t cache_stride) {
    static bool smem_set = false;
    if (!smem_set) {
        cudaFuncSetAttribute(k_attn_ordered, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_ORDERED_LIMIT * 4);
        smem_set = true;
    }
    launch_pdl_(k_attn_ordered, dim3(n_heads, ntok), dim3(AT_THREADS), (size_t)ctx * 4, st, q, kc, vc, n_heads, n_kv,
                hd, scale, pos, ctx, out, pos_rows, cache_stride);
}

void launch_mla_front(const float *kv_a, const float *kv_norm, int kvr, int rope, float eps, float *q, int n_heads,
                      int kd, int nope, const float *rope_tab, const uint32_t *pos, int ctx, float *c_cache,
                      float *r_cache, cudaStream_t st) {
    if (kvr * 4 > 48 * 1024) cudaFuncSetAttribute(k_mla_front, cudaFuncAttributeMaxDynamicSharedMemorySize, kvr * 4);
    launch_pdl_(k_mla_front, dim3(1 + cdiv_u(n_heads, 8)), dim3(256), (size_t)kvr * 4, st, kv_a, kv_norm, kvr, rope, eps, q,
                n_heads, kd, nope, rope_tab, pos, ctx, c_cache, r_cache);
}

void launch_mla_attn(const float *qa, const float *q, int kvr, int rope, int kd, int nope, int n_heads, float scale,
                     const uint32_t *pos, int ctx, const float *c_cache, const float *r_cache, float *c_acc,
                     cudaStream_t st) {
    static bool smem_set = false;
    if (!smem_set) {
        cudaFuncSetAttribute(k_mla_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_ORDERED_LIMIT * 4);
        smem_set = true;
    }
    launch_pdl_(k_mla_attn, dim3(n_heads), dim3(AT_THREADS), (size_t)ctx * 4, st, qa, q, kvr, rope, kd, nope, scale,
                pos, ctx, c_cache, r_cache, c_acc);
}

size_t mla_part_floats(int n_heads, int kvr, int ctx) {
    return (size_t)n_heads * ((ctx + MLA_CH - 1) / MLA_CH) * (kvr + 4);
}

bool mla_split_supported(int kvr, int rope) {
    const size_t smem = ((size_t)MLA_CH * (kvr + rope) + (size_t)MLA_HG * (kvr + rope) + MLA_HG * MLA_CH) * 4;
    return kvr % 4 == 0 && rope % 4 == 0 && kvr <= 1024 && smem <= 200 * 1024;
}

void launch_mla_split(const float *qa, const float *q, int kvr, int rope, int kd, int nope, int n_heads, float scale,
                      const uint32_t *pos, int ctx, const float *c_cache, const float *r_cache, float *part,
                      float *c_acc, int *err, cudaStream_t st) {
    const int nsplit = (ctx + MLA_CH - 1) / MLA_CH;
    const size_t smem = ((size_t)MLA_CH * (kvr + rope) + (size_t)MLA_HG * (kvr + rope) + MLA_HG * MLA_CH) * 4;
    static size_t set = 0;
    if (smem > set) {
        cudaFuncSetAttribute(k_mla_part, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(k_mla_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, nsplit * 4 > 48 * 1024 ? nsplit * 4 : 48 * 1024);
        set = smem;
    }
    launch_pdl_(k_mla_part, dim3(nsplit, cdiv_u(n_heads, MLA_HG)), dim3(MLA_THREADS), smem, st, qa, q, kvr, rope, kd,
                nope, n_heads, scale, pos, ctx, c_cache, r_cache, part, nsplit, err);
    launch_pdl_(k_mla_merge, dim3(n_heads), dim3(MLA_THREADS), (size_t)nsplit * 4, st, kvr, pos, ctx, part, nsplit, c_acc);
}

size_t attn_part_floats(int n_heads, int n_kv, int hd, int ctx) {
    const size_t nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    return (size_t)n_kv * nsplit * (n_heads / n_kv) * (hd + 4);  // records of hd + 2 floats, or hd + 4 (16-byte rows)
}

bool attn_merge_quantizes(int n_heads, int hd, int ctx) {
    const int qd = n_heads * hd, nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    return qd % 256 == 0 && (256 % hd == 0 || hd % 256 == 0) && (size_t)(256 / hd + 1) * nsplit * 4 <= 96 * 1024;
}

void launch_attention(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd, float scale,
                      const uint32_t *pos, int ctx, float *part, float *out, bool ordered, XQW q256, XQW q32,
                      cudaStream_t st) {
    if (ordered) {
        static bool smem_set = false;  // the scores of up to ATT_ORDERED_LIMIT positions
        if (!smem_set) {
            cudaFuncSetAttribute(k_attn_ordered, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_ORDERED_LIMIT * 4);
            smem_set = true;
        }
        launch_pdl_(k_attn_ordered, dim3(n_heads), dim3(AT_THREADS), (size_t)ctx * 4, st, q, kc, vc, n_heads, n_kv,
                    hd, scale, pos, ctx, out, 0, (size_t)0);
        return;
    }
    const int nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    const int G = n_heads / n_kv;
    const size_t smem = ((size_t)ATT_CH * att_kstride(hd) + (size_t)ATT_CH * hd + (size_t)G * hd + (size_t)G * ATT_CH) * 4;
    static bool part_smem_set = false;
    if (!part_smem_set) {
        cudaFuncSetAttribute(k_attn_part, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (ATT_CH * att_kstride(MAX_HD) + ATT_CH * MAX_HD + MAX_GQA * MAX_HD + MAX_GQA * ATT_CH) * 4);
        cudaFuncSetAttribute(k_attn_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        part_smem_set = true;
    }
    launch_pdl_(k_attn_part, dim3(n_kv, nsplit), dim3(AT_THREADS), smem, st, q, kc, vc, n_heads, n_kv, hd, scale, pos,
                ctx, nsplit, part, 0, (size_t)0, (size_t)0);
    const int qd = n_heads * hd;
    const int heads_per_cta = 256 / hd + 1 < n_heads ? 256 / hd + 1 : n_heads;
    launch_pdl_(k_attn_merge, dim3(cdiv_u(qd, 256)), dim3(256), (size_t)heads_per_cta * nsplit * 4, st, part, n_heads,
                n_kv, hd, pos, ctx, nsplit, out, q256, q32, 0, (size_t)0);
}

void launch_attention_split_rows(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd,
                                 float scale, const uint32_t *pos, int ctx, float *part, float *out, int nrows,
                                 size_t cache_stride, cudaStream_t st) {
    const int nsplit = (int)cdiv_u(ctx, ATT_CH), G = n_heads / n_kv;
    const size_t smem = ((size_t)ATT_CH * att_kstride(hd) + (size_t)ATT_CH * hd + (size_t)G * hd + (size_t)G * ATT_CH) * 4;
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(k_attn_part, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (ATT_CH * att_kstride(MAX_HD) + ATT_CH * MAX_HD + MAX_GQA * MAX_HD + MAX_GQA * ATT_CH) * 4);
        cudaFuncSetAttribute(k_attn_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        set = true;
    }
    const size_t part_stride = attn_part_floats(n_heads, n_kv, hd, ctx);
    launch_pdl_(k_attn_part, dim3(n_kv, nsplit, nrows), dim3(AT_THREADS), smem, st, q, kc, vc, n_heads, n_kv, hd, scale,
                pos, ctx, nsplit, part, 1, cache_stride, part_stride);
    const int qd = n_heads * hd;
    const int heads_per_cta = 256 / hd + 1 < n_heads ? 256 / hd + 1 : n_heads;
    launch_pdl_(k_attn_merge, dim3(cdiv_u(qd, 256), 1, nrows), dim3(256), (size_t)heads_per_cta * nsplit * 4, st, part,
                n_heads, n_kv, hd, pos, ctx, nsplit, out, XQW{}, XQW{}, 1, part_stride);
}

}  // namespace loom
