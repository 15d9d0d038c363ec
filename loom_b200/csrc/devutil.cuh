// devutil.cuh -- device helpers shared by the kernel files: the activation
// quantizer lane step and the warp router.
#pragma once
#include "common.cuh"

namespace loom {

// Activation quantization (ggml.zig:776 quantizeX256 / :1077 quantizeX): each
// lane holds 8 consecutive values of a block that spans `group_lanes` lanes
// (32 for a 256-wide block, 4 for a 32-wide one). d = amax/127 (IEEE divide),
// q = round-half-away(v * (1/d)) saturated to +-127, non-finite -> 0.
__device__ __forceinline__ void quant_vals8(const float (&v)[8], bool live, int group_lanes, int8_t *qdst,
                                            float *ddst, int32_t *sdst_pairs, int32_t *sdst_group, int lane) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++)
        if (live && isfinite(v[i])) amax = fmaxf(amax, fabsf(v[i]));
    if (group_lanes == 32)  // amax >= 0: its bits order as unsigned integers
        amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
    else
        for (int o = 1; o < group_lanes; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = fdiv(amax, 127.0f);
    const float inv = (d != 0.0f && isfinite(d)) ? fdiv(1.0f, d) : 0.0f;
    int sum = 0;
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int q = to_i8_sat(fmul(v[i], inv));
        sum += q;
        if (i < 4) lo |= ((uint32_t)(q & 0xFF)) << (8 * i);
        else hi |= ((uint32_t)(q & 0xFF)) << (8 * (i - 4));
    }
    if (live) *reinterpret_cast<uint2 *>(qdst) = make_uint2(lo, hi);
    const int pair = sum + __shfl_xor_sync(0xffffffffu, sum, 1);
    if (sdst_pairs && live && (lane & 1) == 0) *sdst_pairs = pair;
    if (sdst_group) {
        int gs = sum;
        if (group_lanes == 32)
            gs = __reduce_add_sync(0xffffffffu, gs);
        else
            for (int o = 1; o < group_lanes; o <<= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
        if (live && (lane % group_lanes) == 0) *sdst_group = gs;
    }
    if (live && (lane % group_lanes) == 0) *ddst = isfinite(d) ? d : 0.0f;
}

__device__ __forceinline__ void quant_lane8(const float *src, bool live, int group_lanes, int8_t *qdst, float *ddst,
                                            int32_t *sdst_pairs, int32_t *sdst_group, int lane) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = live ? src[i] : 0.0f;
    quant_vals8(v, live, group_lanes, qdst, ddst, sdst_pairs, sdst_group, lane);
}


// moe.zig:106-158 route. Scores and the biased choice live in shared memory.
// The route in three phases so a whole CTA can share the ranking:
//   route_scores  (one warp)  scores = softmax / sigmoid / raw logits, choice =
//                 scores + bias; returns whether every choice is > -inf
//   route_rank    (any threads) the rank of e is the number of experts the
//                 serial scan takes before it (greater value, or equal value
//                 and lower index); with every value > -inf this is exactly the
//                 serial first-max order, so rank < k selects slot `rank`
//   route_finish  (one warp)  the serial k-round scan when some value is NaN or
//                 -inf, then softmax_topk / renormalisation / scale, and the
//                 copy to ids_out/gates_out
// scores/choice: ne floats of shared memory; ids/gates: nk words of shared memory.
__device__ __forceinline__ bool route_scores(const float *logits, const float *bias, int ne, int gating,
                                             float *scores, float *choice, int lane) {
    if (gating == 2) {
        for (int e = lane; e < ne; e += 32) scores[e] = fdiv(1.0f, fadd(1.0f, exp_f(-logits[e])));
    } else if (gating == 1) {
        float m = -INFINITY;
        for (int e = lane; e < ne; e += 32) m = fmaxf(m, logits[e]);
        m = warp_max(m);
        float sum = 0.0f;
        for (int e = lane; e < ne; e += 32) {
            const float v = exp_f(fsub(logits[e], m));
            scores[e] = v;
            sum = fadd(sum, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum = fadd(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        const float inv = fdiv(1.0f, sum);
        for (int e = lane; e < ne; e += 32) scores[e] = fmul(scores[e], inv);
    } else {
        for (int e = lane; e < ne; e += 32) scores[e] = logits[e];
    }
    bool all_finite = true;
    for (int e = lane; e < ne; e += 32) {
        const float c = bias ? fadd(scores[e], bias[e]) : scores[e];
        choice[e] = c;
        all_finite &= c > -INFINITY;
    }
    return __all_sync(0xffffffffu, all_finite);
}

__device__ __forceinline__ void route_rank(const float *scores, const float *choice, int ne, int nk, int *ids,
                                           float *gates, int tid, int nthreads) {
    for (int e = tid; e < ne; e += nthreads) {
        const float c = choice[e];
        int rank = 0;
        for (int j = 0; j < ne; j++) {
            const float cj = choice[j];
            rank += (cj > c) | ((cj == c) & (j < e));
        }
        if (rank < nk) {
            ids[rank] = e;
            gates[rank] = scores[e];
        }
    }
}

// The serial k-round first-max scan (the cold path of route_finish: some
// value is NaN or -inf). Out of line to keep the kernels that inline the
// route small.
static __device__ __noinline__ void route_scan_serial(int ne, int nk, const float *scores, float *choice, int *ids,
                                                      float *gates, int lane) {
    for (int k = 0; k < nk; k++) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < ne; e += 32) {
            const float c = choice[e];
            if (c > bv) {  // strict: first maximum in this lane's (ascending) run
                bv = c;
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi == 0x7fffffff) bi = 0;  // nothing beats -inf: the serial scan keeps index 0
        if (lane == 0) {
            ids[k] = bi;
            gates[k] = scores[bi];
            choice[bi] = -INFINITY;  // used
        }
        __syncwarp();
    }
}

// DeepSeek-V3's group-limited selection by one warp (no counterpart in the
// reference; restated from the published routing): ne experts in n_group
// (<= 32) groups of ne / n_group consecutive ids; lane g scores group g as the
// sum of its two largest choices (its one choice when a group holds one
// expert); the topk_group best groups are kept by a serial first-max scan
// (lowest group index on ties), every lane running the same scan over the
// shuffled scores; choices outside the kept groups become -inf.
static __device__ __noinline__ void route_group_mask(float *choice, int ne, int n_group, int topk_group, int lane) {
    const int gs = ne / n_group;
    float gsc = -INFINITY;
    if (lane < n_group) {
        float top1 = -INFINITY, top2 = -INFINITY;
        for (int e = lane * gs; e < (lane + 1) * gs; e++) {
            const float c = choice[e];
            if (c > top1) {
                top2 = top1;
                top1 = c;
            } else if (c > top2) {
                top2 = c;
            }
        }
        gsc = gs == 1 ? top1 : fadd(top1, top2);
    }
    uint32_t keep = 0;
    for (int k = 0; k < topk_group; k++) {
        int best = -1;
        float bv = -INFINITY;
        for (int g = 0; g < n_group; g++) {
            const float v = __shfl_sync(0xffffffffu, gsc, g);
            if (!(keep >> g & 1u) && (best < 0 || v > bv)) {
                best = g;
                bv = v;
            }
        }
        keep |= 1u << best;
    }
    __syncwarp();
    for (int e = lane; e < ne; e += 32)
        if (!(keep >> (e / gs) & 1u)) choice[e] = -INFINITY;
    __syncwarp();
}

__device__ __forceinline__ void route_finish(bool ranked, int ne, int nk, int gating, int weights_norm,
                                             float weights_scale, const float *scores, float *choice, int *ids,
                                             float *gates, int *ids_out, float *gates_out, int lane) {
    if (!ranked) route_scan_serial(ne, nk, scores, choice, ids, gates, lane);
    if (gating == 3 && lane == 0) {  // softmax over the selected k (tensor.zig:18 softmax)
        float m = -INFINITY;
        for (int k = 0; k < nk; k++) m = fmaxf(m, gates[k]);
        float sum = 0.0f;
        for (int k = 0; k < nk; k++) {
            gates[k] = exp_f(fsub(gates[k], m));
            sum = fadd(sum, gates[k]);
        }
        const float inv = fdiv(1.0f, sum);
        for (int k = 0; k < nk; k++) gates[k] = fmul(gates[k], inv);
    }
    __syncwarp();
    float denom = 1.0f;
    if (weights_norm) {  // the sum runs in selection order, as the serial loop does
        float sum = 0.0f;
        for (int k = 0; k < nk; k++) sum = fadd(sum, gates[k]);
        denom = fmaxf(sum, 6.103515625e-5f);
    }
    __syncwarp();  // every lane has read the gates before they are rewritten
    for (int k = lane; k < nk; k += 32) {
        float g = gates[k];
        if (weights_norm) g = fdiv(g, denom);
        if (weights_scale != 1.0f) g = fmul(g, weights_scale);
        ids_out[k] = ids[k];
        gates_out[k] = g;
        gates[k] = g;
    }
    __syncwarp();
}

// Order-preserving 32-bit key of a float (+0 and -0 map to the same key):
// a > b  <=>  key(a) > key(b) for non-NaN a, b.
__device__ __forceinline__ uint32_t f32_order_key(float x) {
    const uint32_t u = x == 0.0f ? 0u : __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// moe.zig:106-158 route by ONE warp with the expert values in registers
// (lane l holds experts l, l+32, ..., ne <= 32*RW_MAX), bit-identical to
// route_block: the softmax sum runs in route_block's order (per 128-thread
// stride, then per warp, then the four warp partials in order), and top-k
// takes k rounds of a warp arg-max on (value, lowest index) keys, which is the
// serial first-max order when every value is > -inf; otherwise the serial scan
// of route_finish runs on scores/choice in shared memory. ids/gates: shared
// memory (nk words); logits may be global memory written by other CTAs of the
// grid (read with ld.global.cg) or shared memory.
constexpr int RW_MAX = 8;

// Scores of the route on logits in registers (v[t] = logit of expert
// lane + 32t, -inf past ne): sigmoid, softmax (its sum in route_block's order:
// per 128-thread stride, then per warp, then the four warp partials in order)
// or the raw logits.
template <int RW>
__device__ __forceinline__ void route_warp_sc(const float (&v)[RW], int ne, int gating, float (&sc)[RW], int lane) {
    if (gating == 2) {
#pragma unroll
        for (int t = 0; t < RW; t++) sc[t] = fdiv(1.0f, fadd(1.0f, exp_f(-v[t])));
    } else if (gating == 1) {
        float m = -INFINITY;  // fmaxf skips NaN, so the lane maximum is never NaN
#pragma unroll
        for (int t = 0; t < RW; t++)
            if (lane + 32 * t < ne) m = fmaxf(m, v[t]);
        {
            const uint32_t km = __reduce_max_sync(0xffffffffu, f32_order_key(m));
            m = __uint_as_float((km & 0x80000000u) ? (km & 0x7fffffffu) : ~km);
        }
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // route_block's warp w sums experts 32w + l + 128j
#pragma unroll
        for (int t = 0; t < RW; t++) {
            sc[t] = exp_f(fsub(v[t], m));
            if (lane + 32 * t < ne) part[t & 3] = fadd(part[t & 3], sc[t]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int w = 0; w < 4; w++) part[w] = fadd(part[w], __shfl_xor_sync(0xffffffffu, part[w], o));
        const float tot = fadd(fadd(fadd(part[0], part[1]), part[2]), part[3]);
        const float inv = fdiv(1.0f, tot);
#pragma unroll
        for (int t = 0; t < RW; t++) sc[t] = fmul(sc[t], inv);
    } else {
#pragma unroll
        for (int t = 0; t < RW; t++) sc[t] = v[t];
    }
}

// The route on logits already in registers: v[t] = logit of expert lane + 32t
// (-inf past ne).
template <int RW>
__device__ __forceinline__ void route_warp_vals(float (&v)[RW], const float *bias, int ne, int nk, int gating,
                                                int weights_norm, float weights_scale, float *scores, float *choice,
                                                int *ids, float *gates, int *ids_out, float *gates_out, int lane) {
    float sc[RW];
    route_warp_sc<RW>(v, ne, gating, sc, lane);
    bool fin = true;
    uint32_t key[RW];
    int ei[RW];
#pragma unroll
    for (int t = 0; t < RW; t++) {
        const int e = lane + 32 * t;
        const float c = bias && e < ne ? fadd(sc[t], bias[e]) : sc[t];
        if (e < ne) fin &= c > -INFINITY;
        key[t] = e < ne ? f32_order_key(c) : 0u;  // 0: below every real key (exhausted / absent)
        ei[t] = e;
        v[t] = c;
    }
    fin = __all_sync(0xffffffffu, fin);
    if (fin) {
        // sort the lane's candidates by (value desc, index asc), then take k
        // rounds of the warp maximum of the lanes' current heads
        float sv[RW];
#pragma unroll
        for (int t = 0; t < RW; t++) sv[t] = sc[t];
#pragma unroll
        for (int i = 0; i < RW; i++)
#pragma unroll
            for (int j = RW - 1; j > i; j--) {
                const bool sw = key[j] > key[j - 1] || (key[j] == key[j - 1] && ei[j] < ei[j - 1]);
                if (sw) {
                    const uint32_t tk = key[j]; key[j] = key[j - 1]; key[j - 1] = tk;
                    const int te = ei[j]; ei[j] = ei[j - 1]; ei[j - 1] = te;
                    const float ts = sv[j]; sv[j] = sv[j - 1]; sv[j - 1] = ts;
                }
            }
        // k rounds; the winner's value and index reach every lane by shuffle (off the
        // rounds' dependency chain) and lane k keeps pick k in registers, while
        // the renormalisation sum runs in selection order as the picks arrive
        int my_id = 0;
        float my_g = 0.0f, sum = 0.0f;
        for (int k = 0; k < nk; k++) {
            const uint32_t kmax = __reduce_max_sync(0xffffffffu, key[0]);
            const bool mine = key[0] == kmax;
            const uint32_t ball = __ballot_sync(0xffffffffu, mine);
            int wl = __ffs(ball) - 1;
            if (__popc(ball) > 1) {  // equal values: the lowest index wins
                const uint32_t emin = __reduce_min_sync(0xffffffffu, mine ? (uint32_t)ei[0] : 0xffffffffu);
                wl = __ffs(__ballot_sync(0xffffffffu, mine && (uint32_t)ei[0] == emin)) - 1;
            }
            const float gk = __shfl_sync(0xffffffffu, sv[0], wl);
            const int ik = __shfl_sync(0xffffffffu, ei[0], wl);
            if (lane == wl) {
#pragma unroll
                for (int t = 0; t + 1 < RW; t++) {
                    key[t] = key[t + 1];
                    ei[t] = ei[t + 1];
                    sv[t] = sv[t + 1];
                }
                key[RW - 1] = 0u;
            }
            if (k < 32 && lane == k) {
                my_id = ik;
                my_g = gk;
            }
            if (gating != 3) sum = fadd(sum, gk);
            if (k >= 32 || gating == 3) {  // the general tail keeps the picks in shared memory
                if (lane == 0) {
                    ids[k] = ik;
                    gates[k] = gk;
                }
            }
        }
        if (gating != 3 && nk <= 32) {  // the tail of route_finish (moe.zig:149-157), lane k for pick k
            const float denom = fmaxf(sum, 6.103515625e-5f);
            if (lane < nk) {
                float g = my_g;
                if (weights_norm) g = fdiv(g, denom);
                if (weights_scale != 1.0f) g = fmul(g, weights_scale);
                ids_out[lane] = my_id;
                gates_out[lane] = g;
                ids[lane] = my_id;
                gates[lane] = g;
            }
            __syncwarp();
            return;
        }
        if (lane < nk && lane < 32) {
            ids[lane] = my_id;
            gates[lane] = my_g;
        }
    } else {
#pragma unroll
        for (int t = 0; t < RW; t++) {
            const int e = lane + 32 * t;
            if (e < ne) {
                scores[e] = sc[t];
                choice[e] = v[t];
            }
        }
    }
    __syncwarp();
    route_finish(fin, ne, nk, gating, weights_norm, weights_scale, scores, choice, ids, gates, ids_out, gates_out,
                 lane);
}

template <bool GLOBAL_CG, int RW = RW_MAX>
__device__ __forceinline__ void route_warp_regs(const float *logits, const float *bias, int ne, int nk, int gating,
                                                int weights_norm, float weights_scale, float *scores, float *choice,
                                                int *ids, float *gates, int *ids_out, float *gates_out, int lane) {
    float v[RW];
#pragma unroll
    for (int t = 0; t < RW; t++) {
        const int e = lane + 32 * t;
        v[t] = e < ne ? (GLOBAL_CG ? __ldcg(logits + e) : logits[e]) : -INFINITY;
    }
    route_warp_vals<RW>(v, bias, ne, nk, gating, weights_norm, weights_scale, scores, choice, ids, gates, ids_out,
                        gates_out, lane);
}

// moe.zig:106-158 route by the first ROUTE_THREADS threads of a CTA (the
// other warps may run other work meanwhile: this code synchronizes with named
// barrier 1 over these threads only). logits may alias choice. red: 8 floats
// of shared memory.
constexpr int ROUTE_THREADS = 128;

__device__ __forceinline__ void route_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void route_block(const float *logits, const float *bias, int ne, int nk, int gating,
                                            int weights_norm, float weights_scale, float *scores, float *choice,
                                            int *ids, float *gates, float *red, int *ids_out, float *gates_out,
                                            int n_group = 1, int topk_group = 1) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = ROUTE_THREADS / 32;
    if (gating == 2) {
        for (int e = tid; e < ne; e += ROUTE_THREADS) scores[e] = fdiv(1.0f, fadd(1.0f, exp_f(-logits[e])));
    } else if (gating == 1) {
        float m = -INFINITY;
        for (int e = tid; e < ne; e += ROUTE_THREADS) m = fmaxf(m, logits[e]);
        m = warp_max(m);
        if (lane == 0) red[warp] = m;
        route_bar();
        m = red[0];
#pragma unroll
        for (int w = 1; w < NW; w++) m = fmaxf(m, red[w]);
        float sum = 0.0f;
        for (int e = tid; e < ne; e += ROUTE_THREADS) {
            const float v = exp_f(fsub(logits[e], m));
            scores[e] = v;
            sum = fadd(sum, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum = fadd(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        route_bar();  // everyone has read red[] as the max
        if (lane == 0) red[warp] = sum;
        route_bar();
        float tot = red[0];
#pragma unroll
        for (int w = 1; w < NW; w++) tot = fadd(tot, red[w]);
        const float inv = fdiv(1.0f, tot);
        for (int e = tid; e < ne; e += ROUTE_THREADS) scores[e] = fmul(scores[e], inv);
    } else {
        for (int e = tid; e < ne; e += ROUTE_THREADS) scores[e] = logits[e];
    }
    bool fin = true;
    for (int e = tid; e < ne; e += ROUTE_THREADS) {
        const float c = bias ? fadd(scores[e], bias[e]) : scores[e];
        choice[e] = c;
        fin &= c > -INFINITY;
    }
    if (n_group > 1 && topk_group < n_group) {  // masked experts are -inf: the serial scan picks
        route_bar();
        if (warp == 0) route_group_mask(choice, ne, n_group, topk_group, lane);
        fin = false;
    }
    fin = __all_sync(0xffffffffu, fin);
    route_bar();  // red[] free again, choice complete
    if (lane == 0) red[warp] = fin ? 1.0f : 0.0f;
    route_bar();
    bool ranked = ne % 4 == 0;
#pragma unroll
    for (int w = 0; w < NW; w++) ranked &= red[w] != 0.0f;
    if (ranked) {
        // the rank of e is the number of experts the serial scan takes before
        // it (greater value, or equal value and lower index); with every value
        // > -inf this is exactly the serial first-max order
        const float4 *c4 = reinterpret_cast<const float4 *>(choice);
        for (int e = tid; e < ne; e += ROUTE_THREADS) {
            const float c = choice[e];
            int rank = 0;
#pragma unroll 8
            for (int j4 = 0; j4 < ne / 4; j4++) {
                const float4 v = c4[j4];
                const int j = 4 * j4;
                rank += (v.x > c) | ((v.x == c) & (j < e));
                rank += (v.y > c) | ((v.y == c) & (j + 1 < e));
                rank += (v.z > c) | ((v.z == c) & (j + 2 < e));
                rank += (v.w > c) | ((v.w == c) & (j + 3 < e));
            }
            if (rank < nk) {
                ids[rank] = e;
                gates[rank] = scores[e];
            }
        }
    }
    route_bar();
    if (warp == 0)
        route_finish(ranked, ne, nk, gating, weights_norm, weights_scale, scores, choice, ids, gates, ids_out,
                     gates_out, lane);
    route_bar();
}

}  // namespace loom
