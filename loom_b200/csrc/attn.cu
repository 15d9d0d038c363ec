// attn.cu -- the attention half of a decoder layer (llama.zig:1138-1195) on
// the device: RMSNorm + activation quantization, Q/K head norm + RoPE + KV
// append, and softmax attention over the f32 KV cache.
//
// Every elementwise step is the reference's arithmetic with one rounding per
// multiply or add (no contraction). The reductions follow the reference's
// order where that is cheap (RMSNorm up to 1024 wide, head norms, the
// ordered attention: dotF32 scores, serial softmax sum, axpy in position
// order); the wide RMSNorm and the split attention use tree / chunked sums.
#include "attn.cuh"
#include "devutil.cuh"

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
                                                          const uint32_t *pos_p, int ctx, float *kc, float *vc) {
    __shared__ float hv_all[QR_WARPS][MAX_HD];
    __shared__ float inv_all[QR_WARPS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int head = blockIdx.x * QR_WARPS + warp;
    if (head >= n_heads + n_kv) return;
    const int pos = (int)*pos_p;
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
                                                            const uint32_t *pos_p, int ctx, float *out) {
    __shared__ float qs[MAX_HD];
    extern __shared__ float sc[];  // [ctx]
    __shared__ float inv_s;
    const int h = blockIdx.x, tid = threadIdx.x;
    const int pos = (int)*pos_p;
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

// Split form: one CTA per (KV head g, chunk sp of ATT_CH cache rows). Partial
// record per query head: o[hd] = sum_t e^(s_t - m) v_t, then m, l = sum_t e^(s_t - m).
__global__ void __launch_bounds__(AT_THREADS) k_attn_part(const float *q, const float *kc, const float *vc,
                                                         int n_heads, int n_kv, int hd, float scale,
                                                         const uint32_t *pos_p, int ctx, int nsplit, float *part) {
    extern __shared__ float sm[];
    const int G = n_heads / n_kv, kvd = n_kv * hd;
    float *qs = sm;             // [G][hd]
    float *sc = sm + G * hd;    // [G][ATT_CH]
    const int g = blockIdx.x, sp = blockIdx.y;
    const int pos = (int)*pos_p;
    if (pos >= ctx) return;
    const int seq = pos + 1, t0 = sp * ATT_CH;
    if (t0 >= seq) return;
    const int n = min(ATT_CH, seq - t0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < G * hd; i += AT_THREADS) qs[i] = q[(size_t)g * G * hd + i];
    __syncthreads();
    // scores: one warp per cache row, every query head of the group against one read of the key
    for (int j = warp; j < n; j += AT_WARPS) {
        const float *kr = kc + (size_t)(t0 + j) * kvd + (size_t)g * hd;
        float kv[MAX_HD / 32];
#pragma unroll
        for (int c = 0; c < MAX_HD / 32; c++) {
            const int d = lane + 32 * c;
            kv[c] = d < hd ? kr[d] : 0.0f;
        }
        for (int hh = 0; hh < G; hh++) {
            float p = 0.0f;
#pragma unroll
            for (int c = 0; c < MAX_HD / 32; c++) {
                const int d = lane + 32 * c;
                if (d < hd) p = fadd(p, fmul(qs[hh * hd + d], kv[c]));
            }
            p = warp_sum_f(p);
            if (lane == 0) sc[hh * ATT_CH + j] = fmul(p, scale);
        }
    }
    __syncthreads();
    float *rec = part + ((size_t)g * nsplit + sp) * G * (hd + 2);
    for (int hh = warp; hh < G; hh += AT_WARPS) {  // chunk max, exponentials, sum
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[hh * ATT_CH + j]);
        m = warp_max(m);
        float l = 0.0f;
        for (int j = lane; j < n; j += 32) {
            const float e = exp_f(fsub(sc[hh * ATT_CH + j], m));
            sc[hh * ATT_CH + j] = e;
            l = fadd(l, e);
        }
        l = warp_sum_f(l);
        if (lane == 0) {
            rec[hh * (hd + 2) + hd] = m;
            rec[hh * (hd + 2) + hd + 1] = l;
        }
    }
    __syncthreads();
    for (int d = tid; d < hd; d += AT_THREADS) {  // o = sum_t e_t v_t, one read of each value row
        float acc[MAX_GQA];
#pragma unroll
        for (int hh = 0; hh < MAX_GQA; hh++) acc[hh] = 0.0f;
        for (int j = 0; j < n; j++) {
            const float vv = vc[(size_t)(t0 + j) * kvd + (size_t)g * hd + d];
#pragma unroll
            for (int hh = 0; hh < MAX_GQA; hh++)
                if (hh < G) acc[hh] = fadd(acc[hh], fmul(sc[hh * ATT_CH + j], vv));
        }
#pragma unroll
        for (int hh = 0; hh < MAX_GQA; hh++)
            if (hh < G) rec[hh * (hd + 2) + d] = acc[hh];
    }
}

// One CTA per query head: out = (sum_s o_s e^(m_s - M)) / (sum_s l_s e^(m_s - M)).
__global__ void __launch_bounds__(AT_THREADS) k_attn_merge(const float *part, int n_heads, int n_kv, int hd,
                                                          const uint32_t *pos_p, int ctx, int nsplit, float *out) {
    const int h = blockIdx.x, G = n_heads / n_kv, g = h / G, hh = h % G;
    const int pos = (int)*pos_p;
    if (pos >= ctx) return;
    const int live = (pos + 1 + ATT_CH - 1) / ATT_CH;
    const size_t stride = (size_t)G * (hd + 2);
    const float *rec = part + (size_t)g * nsplit * stride + (size_t)hh * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < live; s++) M = fmaxf(M, rec[s * stride + hd]);
    float L = 0.0f;
    for (int s = 0; s < live; s++) L = fadd(L, fmul(rec[s * stride + hd + 1], exp_f(fsub(rec[s * stride + hd], M))));
    for (int d = threadIdx.x; d < hd; d += AT_THREADS) {
        float o = 0.0f;
        for (int s = 0; s < live; s++) o = fadd(o, fmul(rec[s * stride + d], exp_f(fsub(rec[s * stride + hd], M))));
        out[(size_t)h * hd + d] = fdiv(o, L);
    }
}

unsigned cdiv_u(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

}  // namespace

void launch_rmsnorm_q(float *x, const float *add, const float *w, int dim, float eps, float *normed, XQW q256,
                      XQW q32, bool serial, cudaStream_t st) {
    k_rmsnorm_q<<<1, RN_THREADS, (size_t)dim * 4, st>>>(x, add, w, dim, eps, normed, q256, q32, (int)serial);
    count_launch();
}

void launch_qk_rope(float *q, float *k, const float *v, const float *qn, const float *kn, int n_heads, int n_kv,
                    int hd, int rope_dim, int neox, const float *rope, float eps, const uint32_t *pos, int ctx,
                    float *kc, float *vc, cudaStream_t st) {
    k_qk_rope<<<cdiv_u(n_heads + n_kv, QR_WARPS), QR_WARPS * 32, 0, st>>>(q, k, v, qn, kn, n_heads, n_kv, hd,
                                                                          rope_dim, neox, rope, eps, pos, ctx, kc, vc);
    count_launch();
}

size_t attn_part_floats(int n_heads, int n_kv, int hd, int ctx) {
    const size_t nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    return (size_t)n_kv * nsplit * (n_heads / n_kv) * (hd + 2);
}

void launch_attention(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd, float scale,
                      const uint32_t *pos, int ctx, float *part, float *out, bool ordered, cudaStream_t st) {
    if (ordered) {
        static bool smem_set = false;  // the scores of up to ATT_ORDERED_LIMIT positions
        if (!smem_set) {
            cudaFuncSetAttribute(k_attn_ordered, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_ORDERED_LIMIT * 4);
            smem_set = true;
        }
        k_attn_ordered<<<n_heads, AT_THREADS, (size_t)ctx * 4, st>>>(q, kc, vc, n_heads, n_kv, hd, scale, pos, ctx,
                                                                      out);
        count_launch();
        return;
    }
    const int nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    const int G = n_heads / n_kv;
    const size_t smem = ((size_t)G * hd + (size_t)G * ATT_CH) * 4;
    k_attn_part<<<dim3(n_kv, nsplit), AT_THREADS, smem, st>>>(q, kc, vc, n_heads, n_kv, hd, scale, pos, ctx, nsplit,
                                                               part);
    k_attn_merge<<<n_heads, AT_THREADS, 0, st>>>(part, n_heads, n_kv, hd, pos, ctx, nsplit, out);
    count_launches(2);
}

}  // namespace loom
