// model_kernel.cu -- a whole decode step's layers in ONE persistent cooperative
// launch (llama.zig:1132-1225 for every layer of the token). One CTA per SM,
// 12 warps, the layers in sequence; per layer eight bounded grid barriers:
//   A1  x -> attention RMSNorm -> int8 (every CTA, shared memory); this CTA's
//       q/k/v rows and output-projection rows bulk-copied into shared memory
//       at the phase start; the q/k/v dots.                              | B
//   A2  headNorm + RoPE, k/v appended to the cache (one warp per head).  | B
//   A3  split-position attention chunks (groups of 4 warps).             | B
//   A4  merge + quantization of the attention output (256 per CTA).      | B
//   A5  output-projection rows from shared memory: x[r] += W_o[r] . att. | B
//   M1  x -> FFN RMSNorm -> int8 (every CTA); router logits (dotF32
//       order, one warp per expert).                                     | B
//   M2  the route (moe.zig:106, every CTA the same from the same logits);
//       this CTA's gate/up rows of the selected experts and its down rows
//       bulk-copied at once; gate/up dots + SwiGLU -> act.               | B
//   M3  act quantized (every CTA); down rows of every selected expert
//       for this CTA's output rows, ordered combine (acc += g_k y_k),
//       x[r] += acc.                                                     | B
// Every wait is bounded (grid barriers, bulk-copy mbarriers); a time-out
// raises a bit of the error word and the kernel leaves.
// The arithmetic is that of the per-layer kernels (attn_block.cu, decode.cu):
// integer block dots bit-identical to the CPU reference, the reference's
// combine order, RMSNorm serial or tree as configured.
#include "attn_block.cuh"
#include "model_kernel.cuh"
#include "step_dev.cuh"

#include <algorithm>

namespace loom {

namespace {

constexpr int MK_NBAR = 8;      // grid barriers per layer
constexpr int MK_MAX_USED = 16; // routed slots the kernel stages
constexpr int MK_MAX_EXPERT = 1024;

// dotF32 (ggml.zig:198) of a router row in global memory and x in shared
// memory by one warp, in rowdot_f32's lane order (lane j accumulates lane j
// of dotF32's four 8-wide vectors).
__device__ __forceinline__ float mk_dot_f32(const float *row, const float *xs, int n, int lane) {
    float a = 0.0f;
    int i = 0;
#pragma unroll 4
    for (; i + 32 <= n; i += 32) a = fadd(a, fmul(__ldg(row + i + lane), xs[i + lane]));
    for (; i + 8 <= n; i += 8)
        if (lane < 8) a = fadd(a, fmul(__ldg(row + i + lane), xs[i + lane]));
    const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
    const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
    const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
    const float v = fadd(fadd(fadd(a, a8), a16), a24);
    float r = __shfl_sync(0xffffffffu, v, 0);
#pragma unroll
    for (int jj = 1; jj < 8; jj++) r = fadd(r, __shfl_sync(0xffffffffu, v, jj));
    for (; i < n; i++) r = fadd(r, fmul(__ldg(row + i), xs[i]));
    return r;
}

// One output row r (local to the staged slices) of every routed slot's down
// projection: stream s = slot s, its own staged slice ds[s], against slot s's
// quantized activation (aq + s*ffn, ad + s*ffn/BE, as + s*ffn/16). Lane s
// returns y_s (block terms added in block order from +0).
template <int TY>
__device__ __noinline__ float mk_down_row(const AbStage *ds, int nslot, int r, const int8_t *aq, const float *ad,
                                          const int32_t *as, int ffn, float *tsm, int lane) {
    using Q = QT<TY>;
    constexpr int GG = 32 / Q::LPB;
    const int NB = ds[0].nb, U = nslot * NB, grp = lane / Q::LPB, sub = lane % Q::LPB;
#pragma unroll 4
    for (int u0 = 0; u0 < U; u0 += GG) {
        const int u = u0 + grp;
        int I = 0, M = 0;
        float xdv = 0.0f;
        typename Q::Frag f{};
        if (u < U) {
            const int s2 = u / NB, b = u - s2 * NB;
            f = ab_frag<TY>(ds[s2], r * NB + b, sub);
            Q::part(f, sub, aq + (size_t)s2 * ffn + b * Q::BE, as + (size_t)s2 * (ffn / 16) + b * Q::SPB, I, M);
            xdv = ad[(size_t)s2 * (ffn / Q::BE) + b];
        }
#pragma unroll
        for (int o = 1; o < Q::LPB; o <<= 1) {
            I += __shfl_xor_sync(0xffffffffu, I, o);
            M += __shfl_xor_sync(0xffffffffu, M, o);
        }
        if (u < U && sub == 0) tsm[u] = Q::term(f, I, M, xdv);
    }
    __syncwarp();
    float a = 0.0f;
    if (lane < nslot) {
#pragma unroll 1
        for (int b = 0; b < NB; b++) a = fadd(b == 0 ? 0.0f : a, tsm[lane * NB + b]);
    }
    __syncwarp();
    return a;
}

// Carve a slice's regions (quants, Q6_K scales, f16 scales) out of a bump pointer.
__device__ __forceinline__ void mk_carve(AbStage &st, const WDev &w, int ra, int rb, int nb, uint8_t *&p) {
    const size_t n = (size_t)(rb - ra) * nb;
    st.ra = ra;
    st.rb = rb;
    st.nb = nb;
    st.q = p;
    p += ab_al128(n * layout_qbytes(w.type));
    st.sc = p;
    if (w.sc) p += ab_al128(n * 16);
    st.d = reinterpret_cast<const uint16_t *>(p);
    if (w.d) p += ab_al128(n * 2);
}
__device__ __forceinline__ uint32_t mk_stage_bytes(const WDev &w, int ra, int rb, int nb) {
    const size_t n = (size_t)(rb - ra) * nb;
    return (uint32_t)(n * layout_qbytes(w.type) + (w.sc ? n * 16 : 0));
}

__device__ __forceinline__ void mk_mark(const MkArgs &A, int i) {
    if (A.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        A.trace[i] = t;
    }
}

template <int TA, int TV, int TO, int SO, int TG, int TD>
__global__ void __launch_bounds__(AB_THREADS, 1) k_model(MkArgs A) {
    extern __shared__ __align__(128) uint8_t ab_smem[];
    __shared__ float red[AB_WARPS];
    __shared__ float Ls[40];
    __shared__ __align__(8) uint64_t mb[2];  // [0] q/k/v then gate/up rows; [1] output-projection then down rows
    __shared__ float tsm_all[AB_WARPS][64];  // per-warp unit terms of the compact row dots
    // route buffers: route_block reads `choice` as float4 (16-byte alignment required)
    __shared__ __align__(16) float r_scores[MK_MAX_EXPERT];
    __shared__ __align__(16) float r_choice[MK_MAX_EXPERT];
    __shared__ float r_red[8], r_gates[64], sel_g[MK_MAX_USED];
    __shared__ int r_ids[64], sel_ids[MK_MAX_USED], gu_rr[2], gu_k[2], n_gu;
    __shared__ AbStage gp[2], upc[2], dsl[MK_MAX_USED];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x, gw = c * AB_WARPS + warp, W = G * AB_WARPS;
    const int dim = A.dim, nh = A.n_heads, nkv = A.n_kv, hd = A.hd, qd = nh * hd, kvd = nkv * hd;
    const int GQ = nh / nkv;
    const int ne = A.n_expert, nk = A.n_used, ffn = A.ffn;
    float *tsm = tsm_all[warp];
    unsigned long long *ctr = A.bar;
    unsigned *ep = reinterpret_cast<unsigned *>(A.bar + 1);
    unsigned *err = reinterpret_cast<unsigned *>(A.bar + 2);
    const unsigned long long base =
        (unsigned long long)G * MK_NBAR * A.n_layers * *reinterpret_cast<volatile unsigned *>(ep);
    int nbar = 0;
    mk_mark(A, 0);
    const int pos = (int)*A.pos;
    const bool pos_ok = pos < A.ctx;
    float *sx = reinterpret_cast<float *>(ab_smem);
    int8_t *xq = reinterpret_cast<int8_t *>(ab_smem + ab_al16((size_t)dim * 4));
    float *xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xq) + ab_al16(dim));
    int32_t *xs = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(xd) + ab_al16((size_t)dim / 32 * 4));
    if (tid == 0) {
        mbar_init(&mb[0], 1);
        mbar_init(&mb[1], 1);
    }
    __syncthreads();
#pragma unroll 1
    for (int l = 0; l < A.n_layers; l++) {
    const MkLayer L = A.layers[l];
    uint8_t *o_stage = ab_smem + A.off_r1;
    uint8_t *u_area = ab_smem + A.off_r2;
    float *att_sm = reinterpret_cast<float *>(u_area);
        // ---- this CTA's row slices -------------------------------------------------------
        const int nbA = dim / QT<TA>::BE, nbV = dim / QT<TV>::BE, nbO = qd / QT<TO>::BE;
        const int qa = qd * c / G, qb = qd * (c + 1) / G, ka = kvd * c / G, kb = kvd * (c + 1) / G;
        const int oa = dim * c / G, ob = dim * (c + 1) / G;
        AbStage sq, sk, sv, so;
        {
            uint8_t *p = u_area;
            auto carve = [&](AbStage &st, const WDev &w, int ra, int rb, int nb) -> uint8_t * {
                const size_t n = (size_t)(rb - ra) * nb;
                st.ra = ra;
                st.rb = rb;
                st.nb = nb;
                st.q = p;
                p += ab_al128(n * layout_qbytes(w.type));
                st.sc = p;
                if (w.sc) p += ab_al128(n * 16);
                st.d = reinterpret_cast<const uint16_t *>(p);
                if (w.d) p += ab_al128(n * 2);
                return p;
            };
            carve(sq, L.wq, qa, qb, nbA);
            carve(sk, L.wk, ka, kb, nbA);
            carve(sv, L.wv, ka, kb, nbV);
            p = o_stage;
            carve(so, L.wo, oa, ob, nbO);
        }
        if (tid == 0) {  // every weight byte of the layer this CTA needs, in flight at once
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier generic accesses of the regions
            const uint32_t bq = (uint32_t)((size_t)(qb - qa) * nbA * layout_qbytes(TA) + (size_t)(kb - ka) * nbA * layout_qbytes(TA) +
                                           (size_t)(kb - ka) * nbV * (layout_qbytes(TV) + (L.wv.sc ? 16 : 0)) +
                                           (size_t)(qb - qa + kb - ka) * nbA * (L.wq.sc ? 16 : 0));
            mbar_expect_tx(&mb[0], bq);
            ab_stage_bulk(L.wq, qa, qb, nbA, const_cast<uint8_t *>(sq.q), const_cast<uint8_t *>(sq.sc), &mb[0]);
            ab_stage_bulk(L.wk, ka, kb, nbA, const_cast<uint8_t *>(sk.q), const_cast<uint8_t *>(sk.sc), &mb[0]);
            ab_stage_bulk(L.wv, ka, kb, nbV, const_cast<uint8_t *>(sv.q), const_cast<uint8_t *>(sv.sc), &mb[0]);
            const uint32_t bo = (uint32_t)((size_t)(ob - oa) * nbO * (layout_qbytes(TO) + (L.wo.sc ? 16 : 0)));
            mbar_expect_tx(&mb[1], bo);
            ab_stage_bulk(L.wo, oa, ob, nbO, const_cast<uint8_t *>(so.q), const_cast<uint8_t *>(so.sc), &mb[1]);
        }
        ab_stage_d(L.wq, qa, qb, nbA, const_cast<uint16_t *>(sq.d));
        ab_stage_d(L.wk, ka, kb, nbA, const_cast<uint16_t *>(sk.d));
        ab_stage_d(L.wv, ka, kb, nbV, const_cast<uint16_t *>(sv.d));
        ab_stage_d(L.wo, oa, ob, nbO, const_cast<uint16_t *>(so.d));
        if (pos_ok) {  // this layer's cache rows, requested into L2 for the attention phase
            const size_t gt = (size_t)c * AB_THREADS + tid, nt = (size_t)G * AB_THREADS;
            ab_prefetch(L.kc, (size_t)pos * kvd * 4, gt, nt);
            ab_prefetch(L.vc, (size_t)pos * kvd * 4, gt, nt);
        }

        // ---- P1: RMSNorm + quantization, then the q/k/v rows from shared memory ---------------
        ab_rmsnorm(A.x, L.attn_norm, dim, A.eps, A.serial, sx, red);  // (its barriers publish mb init and d regions)
        {
            bool staged = mbar_wait(&mb[0], 0, STAGE_POLLS_AB);
            if (!staged && lane == 0) atomicOr(err, 2u);
            const bool k256A = QT<TA>::BE == 256, k256V = QT<TV>::BE == 256;
            const XV xv{xq, xd, xs};
            constexpr int SA = 4;
            const int cq = (qb - qa + SA - 1) / SA, ck = (kb - ka + SA - 1) / SA;
            const int nchunk = cq + 2 * ck;
            for (int pass = 0; pass < 2; pass++) {
                const bool k256 = pass == 0;
                if (k256 ? !(k256A || k256V) : (k256A && k256V)) continue;
                __syncthreads();
                ab_quant(sx, dim, k256, xq, xd, xs);
                __syncthreads();
                for (int ch = warp; ch < nchunk && staged; ch += AB_WARPS) {
                    const int m = ch < cq ? 0 : ch < cq + ck ? 1 : 2;
                    const int lc = m == 0 ? ch : m == 1 ? ch - cq : ch - cq - ck;
                    const AbStage &st = m == 0 ? sq : m == 1 ? sk : sv;
                    if ((m <= 1 ? k256A : k256V) != k256) continue;
                    const int r0 = lc * SA, nS = min(SA, st.rb - st.ra - r0);
                    const float a = m <= 1 ? ab_rows<TA>(st, r0, nS, xv, tsm, lane) : ab_rows<TV>(st, r0, nS, xv, tsm, lane);
                    float *dst = (m == 0 ? A.q : m == 1 ? A.k : A.v) + st.ra + r0;
                    if (lane < nS) dst[lane] = a;
                }
            }
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;

        // ---- P2: head norm + RoPE + append (one warp per head, in shared memory) -------------
        for (int head = gw; head < nh + nkv && pos_ok; head += W) {
            const bool isk = head >= nh;
            const int kh = head - nh;
            float *vec = isk ? A.k + (size_t)kh * hd : A.q + (size_t)head * hd;
            const float *g = isk ? L.k_norm : L.q_norm;
            float *hv = att_sm + warp * MAX_AB_HD;
            const float *cs = A.rope + (size_t)pos * A.rope_dim;
            const int half = A.rope_dim / 2;
            float cj[MAX_AB_HD / 64][2], vv[MAX_AB_HD / 32], gg[MAX_AB_HD / 32];
    #pragma unroll
            for (int t = 0; t < MAX_AB_HD / 64; t++) {  // (cos, sin) of the pairs this lane rotates
                const int j = lane + 32 * t;
                cj[t][0] = j < half ? cs[2 * j] : 0.0f;
                cj[t][1] = j < half ? cs[2 * j + 1] : 0.0f;
            }
    #pragma unroll
            for (int t = 0; t < MAX_AB_HD / 32; t++) {
                const int i = lane + 32 * t;
                vv[t] = isk && i < hd ? A.v[(size_t)kh * hd + i] : 0.0f;
                gg[t] = g && i < hd ? g[i] : 0.0f;
                if (i < hd) hv[i] = vec[i];
            }
            __syncwarp();
            if (g) {  // headNorm (llama.zig:938): serial sum of squares, inv = 1 / sqrt(ss / hd + eps)
                float inv = 0.0f;
                if (lane == 0) {
                    float ss = 0.0f;
                    for (int i = 0; i < hd; i++) ss = fadd(ss, fmul(hv[i], hv[i]));
                    inv = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)hd), A.eps)));
                }
                inv = __shfl_sync(0xffffffffu, inv, 0);
    #pragma unroll
                for (int t = 0; t < MAX_AB_HD / 32; t++) {
                    const int i = lane + 32 * t;
                    if (i < hd) hv[i] = fmul(fmul(hv[i], inv), gg[t]);
                }
                __syncwarp();
            }
    #pragma unroll
            for (int t = 0; t < MAX_AB_HD / 64; t++) {  // RoPE (llama.zig:830-858) on the pairs
                const int j = lane + 32 * t;
                if (j < half) {
                    const int ia = A.neox ? j : 2 * j, ib = A.neox ? j + half : 2 * j + 1;
                    const float a = hv[ia], b = hv[ib];
                    hv[ia] = fsub(fmul(a, cj[t][0]), fmul(b, cj[t][1]));
                    hv[ib] = fadd(fmul(a, cj[t][1]), fmul(b, cj[t][0]));
                }
            }
            __syncwarp();
            const size_t row = (size_t)pos * kvd + (size_t)kh * hd;
    #pragma unroll
            for (int t = 0; t < MAX_AB_HD / 32; t++) {
                const int i = lane + 32 * t;
                if (i < hd) {
                    vec[i] = hv[i];
                    if (isk) {  // llama.zig:1157-1159 cache append
                        L.kc[row + i] = hv[i];
                        L.vc[row + i] = vv[t];
                    }
                }
            }
            __syncwarp();
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;

        // ---- P3: attention chunks ------------------------------------------------------------
        if (pos_ok) {
            const int grp = warp / AB_GRP_WARPS, gl = tid % (AB_GRP_WARPS * 32), gwarp = warp % AB_GRP_WARPS;
            const int ngrp = A.groups;  // groups per CTA that fit in shared memory
            const int KS = hd + 4;
            const size_t per = (size_t)ATT_CH * KS + (size_t)ATT_CH * hd + (size_t)GQ * hd + (size_t)GQ * ATT_CH;
            const int live = (pos + 1 + ATT_CH - 1) / ATT_CH, items = nkv * live;
            if (grp < ngrp) {
                float *sK = att_sm + grp * per, *sV = sK + ATT_CH * KS, *qs = sV + ATT_CH * hd, *sc = qs + GQ * hd;
                for (int it = c * ngrp + grp; it < items; it += G * ngrp) {
                    const int g = it / live, sp = it % live;
                    const int t0 = sp * ATT_CH, n = min(ATT_CH, pos + 1 - t0);
                    const float *kb = L.kc + (size_t)t0 * kvd + (size_t)g * hd;
                    const float *vb = L.vc + (size_t)t0 * kvd + (size_t)g * hd;
                    const int q4 = hd / 4;
                    for (int i = gl; i < n * q4; i += AB_GRP_WARPS * 32) {
                        const int j = i / q4, c4 = (i % q4) * 4;
                        ab_cp16(sK + j * KS + c4, kb + (size_t)j * kvd + c4);
                        ab_cp16(sV + j * hd + c4, vb + (size_t)j * kvd + c4);
                    }
                    asm volatile("cp.async.commit_group;\n" ::: "memory");
                    for (int i = gl; i < GQ * hd; i += AB_GRP_WARPS * 32) qs[i] = A.q[(size_t)g * GQ * hd + i];
                    asm volatile("cp.async.wait_all;\n" ::: "memory");
                    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                    const int HP = (GQ + 1) / 2;
                    for (int hp = gwarp; hp < HP; hp += AB_GRP_WARPS) {
                        const int j = lane, ha = 2 * hp, hb = min(2 * hp + 1, GQ - 1);
                        if (j < n) {
                            const float *kr = sK + j * KS, *qa = qs + ha * hd, *qb = qs + hb * hd;
                            float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
                            for (int d = 0; d < hd; d += 4) {
                                const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
                                const float4 x4 = *reinterpret_cast<const float4 *>(qa + d);
                                const float4 y4 = *reinterpret_cast<const float4 *>(qb + d);
                                a0 = fmaf(k4.x, x4.x, a0); a1 = fmaf(k4.y, x4.y, a1);
                                a0 = fmaf(k4.z, x4.z, a0); a1 = fmaf(k4.w, x4.w, a1);
                                b0 = fmaf(k4.x, y4.x, b0); b1 = fmaf(k4.y, y4.y, b1);
                                b0 = fmaf(k4.z, y4.z, b0); b1 = fmaf(k4.w, y4.w, b1);
                            }
                            sc[ha * ATT_CH + j] = (a0 + a1) * A.scale;
                            sc[hb * ATT_CH + j] = (b0 + b1) * A.scale;
                        }
                    }
                    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                    float *rec = A.part + ((size_t)g * A.nsplit + sp) * GQ * (hd + 2);
                    for (int hh = gwarp; hh < GQ; hh += AB_GRP_WARPS) {
                        const float v = lane < n ? sc[hh * ATT_CH + lane] : -INFINITY;
                        const float m = warp_max(v);
                        const float e = lane < n ? exp_f(v - m) : 0.0f;
                        if (lane < n) sc[hh * ATT_CH + lane] = e;
                        const float l = ab_warp_sum(e);
                        if (lane == 0) {
                            rec[hh * (hd + 2) + hd] = m;
                            rec[hh * (hd + 2) + hd + 1] = l;
                        }
                    }
                    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                    for (int d = gl; d < hd; d += AB_GRP_WARPS * 32) {
                        float acc[16];
    #pragma unroll
                        for (int hh = 0; hh < 16; hh++) acc[hh] = 0.0f;
                        for (int j = 0; j < n; j++) {
                            const float vv = sV[j * hd + d];
    #pragma unroll
                            for (int hh = 0; hh < 16; hh++)
                                if (hh < GQ) acc[hh] = fmaf(sc[hh * ATT_CH + j], vv, acc[hh]);
                        }
    #pragma unroll
                        for (int hh = 0; hh < 16; hh++)
                            if (hh < GQ) rec[hh * (hd + 2) + d] = acc[hh];
                    }
                    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                }
            }
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;

        {
            // ---- P4: merge + quantization ----------------------------------------------------
            const bool k256O = QT<TO>::BE == 256;
            if (pos_ok && c < (qd + 255) / 256) {
                const int live = (pos + 1 + ATT_CH - 1) / ATT_CH;
                const size_t stride = (size_t)GQ * (hd + 2);
                const int e0 = c * 256, h0 = e0 / hd, h1 = min((e0 + 255) / hd, nh - 1);
                float *wsm = att_sm;                         // [heads][live]
                float *val = att_sm + (h1 - h0 + 1) * live;  // [256]
                for (int lh = warp; lh <= h1 - h0; lh += AB_WARPS) {
                    const int h = h0 + lh, g = h / GQ, hh = h % GQ;
                    const float *rec = A.part + (size_t)g * A.nsplit * stride + (size_t)hh * (hd + 2);
                    float *w = wsm + lh * live;
                    float M = -INFINITY;
                    for (int s2 = lane; s2 < live; s2 += 32) M = fmaxf(M, rec[s2 * stride + hd]);
                    M = warp_max(M);
                    float L = 0.0f;
                    for (int s2 = lane; s2 < live; s2 += 32) {
                        const float ws = exp_f(rec[s2 * stride + hd] - M);
                        w[s2] = ws;
                        L = fmaf(rec[s2 * stride + hd + 1], ws, L);
                    }
                    L = ab_warp_sum(L);
                    if (lane == 0) Ls[lh] = L;
                }
                __syncthreads();
                if (tid < 256) {
                    const int e = e0 + tid;
                    float o = 0.0f;
                    if (e < qd) {
                        const int h = e / hd, d = e % hd, g = h / GQ, hh = h % GQ, lh = h - h0;
                        const float *rec = A.part + (size_t)g * A.nsplit * stride + (size_t)hh * (hd + 2) + d;
                        const float *w = wsm + lh * live;
    #pragma unroll 32
                        for (int s2 = 0; s2 < live; s2++) o = fmaf(rec[s2 * stride], w[s2], o);
                        o = o / Ls[lh];
                    }
                    val[tid] = o;
                }
                __syncthreads();
                if (warp == 0) {
                    if (k256O) {
                        const int off = lane * 8;
                        quant_lane8(val + off, true, 32, A.aq + e0 + off, A.ad + c, A.as + e0 / 16 + lane / 2, nullptr,
                                    lane);
                    } else {
                        const int b = e0 / 32 + lane / 4, nb = qd / 32;
                        const bool lb = b < nb;
                        const int off = (lane / 4) * 32 + (lane & 3) * 8;
                        quant_lane8(val + (lb ? off : 0), lb, 4, A.aq + e0 + off, A.ad + b, nullptr, A.as + b, lane);
                    }
                }
            }
            if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;

            // ---- P5: output projection from the staged rows + residual ------------------------
            const bool staged = mbar_wait(&mb[1], 0, STAGE_POLLS_AB);
            if (!staged && lane == 0) atomicOr(err, 2u);
            const XV av{A.aq, A.ad, A.as};
            const int nco = (ob - oa + SO - 1) / SO;
            for (int ch = warp; ch < nco && staged; ch += AB_WARPS) {
                const int r0 = ch * SO, nS = min(SO, ob - oa - r0);
                const float a = ab_rows<TO>(so, r0, nS, av, tsm, lane);
                if (lane < nS) A.x[oa + r0 + lane] = fadd(A.x[oa + r0 + lane], a);  // llama.zig:1195 add
            }
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;


        // ---- M1: FFN RMSNorm -> int8 (every CTA); router logits ---------------------------
        ab_rmsnorm(A.x, L.ffn_norm, dim, A.eps, A.serial, sx, red);
        ab_quant(sx, dim, QT<TG>::BE == 256, xq, xd, xs);  // gate/up activations, kept for M2
        for (int e = gw; e < ne; e += W) {  // moeLayer's router matvec (llama.zig:1264)
            const float lg = mk_dot_f32(L.router + (size_t)e * dim, sx, dim, lane);
            if (lane == 0) A.logits[e] = lg;
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;

        {
            // ---- M2: route, stage the selected experts' rows, gate/up + SwiGLU ----------------
            if (tid < ROUTE_THREADS) {
                for (int e = tid; e < ne; e += ROUTE_THREADS) r_choice[e] = __ldcg(A.logits + e);
                asm volatile("bar.sync 1, %0;" ::"r"(ROUTE_THREADS) : "memory");
                route_block(r_choice, L.bias, ne, nk, A.gating, A.weights_norm, A.weights_scale, r_scores, r_choice,
                            r_ids, r_gates, r_red, sel_ids, sel_g);
            }
            __syncthreads();
            if (A.ids_out && c == 0 && tid < nk) A.ids_out[(size_t)l * nk + tid] = (uint32_t)sel_ids[tid];
            const int nbG = dim / QT<TG>::BE, nbD = ffn / QT<TD>::BE;
            const int P = nk * ffn, pa = (int)((long long)P * c / G), pb = (int)((long long)P * (c + 1) / G);
            const int da = dim * c / G, db = dim * (c + 1) / G;
            const int qn = nk * ffn;  // act-quant region at the head of R1: [qn] int8, [qn/256] f32, [qn/16] i32
            uint8_t *aq_sm = ab_smem + A.off_r1;
            float *ad_sm = reinterpret_cast<float *>(aq_sm + ab_al128(qn));
            int32_t *as_sm = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(ad_sm) + ab_al128((size_t)qn / 256 * 4));
            if (tid == 0) {  // this CTA's slices: gate/up pairs [pa, pb) of (slot, row), down rows [da, db) of every slot
                uint8_t *p2 = u_area;
                int n = 0;
                for (int k = pa / ffn; k < nk && k * ffn < pb && n < 2; k++, n++) {
                    const int e = sel_ids[k], ra = max(pa - k * ffn, 0), rb = min(pb - k * ffn, ffn);
                    mk_carve(gp[n], L.g, e * ffn + ra, e * ffn + rb, nbG, p2);
                    mk_carve(upc[n], L.u, e * ffn + ra, e * ffn + rb, nbG, p2);
                    gu_rr[n] = ra;
                    gu_k[n] = k;
                }
                n_gu = n;
                uint8_t *p1 = reinterpret_cast<uint8_t *>(as_sm) + ab_al128((size_t)qn / 16 * 4);
                for (int k = 0; k < nk; k++) mk_carve(dsl[k], L.dn, sel_ids[k] * dim + da, sel_ids[k] * dim + db, nbD, p1);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                uint32_t bg = 0;
                for (int i = 0; i < n; i++)
                    bg += mk_stage_bytes(L.g, gp[i].ra, gp[i].rb, nbG) + mk_stage_bytes(L.u, upc[i].ra, upc[i].rb, nbG);
                mbar_expect_tx(&mb[0], bg);
                for (int i = 0; i < n; i++) {
                    ab_stage_bulk(L.g, gp[i].ra, gp[i].rb, nbG, const_cast<uint8_t *>(gp[i].q), const_cast<uint8_t *>(gp[i].sc),
                                  &mb[0]);
                    ab_stage_bulk(L.u, upc[i].ra, upc[i].rb, nbG, const_cast<uint8_t *>(upc[i].q),
                                  const_cast<uint8_t *>(upc[i].sc), &mb[0]);
                }
                uint32_t bd = 0;
                for (int k = 0; k < nk; k++) bd += mk_stage_bytes(L.dn, dsl[k].ra, dsl[k].rb, nbD);
                mbar_expect_tx(&mb[1], bd);
                for (int k = 0; k < nk; k++)
                    ab_stage_bulk(L.dn, dsl[k].ra, dsl[k].rb, nbD, const_cast<uint8_t *>(dsl[k].q),
                                  const_cast<uint8_t *>(dsl[k].sc), &mb[1]);
            }
            __syncthreads();
            for (int i = 0; i < n_gu; i++) {
                ab_stage_d(L.g, gp[i].ra, gp[i].rb, nbG, const_cast<uint16_t *>(gp[i].d));
                ab_stage_d(L.u, upc[i].ra, upc[i].rb, nbG, const_cast<uint16_t *>(upc[i].d));
            }
            if (L.dn.d) {  // every slot's f16 scales in one pass (one round trip, not one per slot)
                const int nd = (db - da) * nbD;
                for (int i = tid; i < nk * nd; i += AB_THREADS) {
                    const int k = i / nd, j = i - k * nd;
                    const_cast<uint16_t *>(dsl[k].d)[j] = __ldg(L.dn.d + (size_t)dsl[k].ra * nbD + j);
                }
            }
            __syncthreads();
            const bool staged = mbar_wait(&mb[0], 1, STAGE_POLLS_AB);
            if (!staged && lane == 0) atomicOr(err, 2u);
            const XV xv{xq, xd, xs};
            constexpr int SG = 4;
            const int c0 = n_gu > 0 ? (gp[0].rb - gp[0].ra + SG - 1) / SG : 0;
            const int c1 = n_gu > 1 ? (gp[1].rb - gp[1].ra + SG - 1) / SG : 0;
            for (int ch = warp; ch < c0 + c1 && staged; ch += AB_WARPS) {
                const int i = ch < c0 ? 0 : 1, r0 = (ch < c0 ? ch : ch - c0) * SG;
                const int nS = min(SG, gp[i].rb - gp[i].ra - r0);
                const float g = ab_rows<TG>(gp[i], r0, nS, xv, tsm, lane);
                const float u = ab_rows<TG>(upc[i], r0, nS, xv, tsm, lane);
                if (lane < nS)  // silu(g) * u (tensor.zig:30,53)
                    A.act[(size_t)gu_k[i] * ffn + gu_rr[i] + r0 + lane] = fmul(fdiv(g, fadd(1.0f, exp_f(-g))), u);
            }
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;

        {
            // ---- M3: act quantized (every CTA), down rows, ordered combine + residual ----------
            const int qn = nk * ffn;
            int8_t *aq_sm = reinterpret_cast<int8_t *>(ab_smem + A.off_r1);
            float *ad_sm = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(aq_sm) + ab_al128(qn));
            int32_t *as_sm = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(ad_sm) + ab_al128((size_t)qn / 256 * 4));
            for (int b = warp; b < qn / 256; b += AB_WARPS) {  // quantizeX256 of every slot's activation
                const int off = b * 256 + lane * 8;
                float v8[8];
                const float4 lo = __ldcg(reinterpret_cast<const float4 *>(A.act + off));
                const float4 hi = __ldcg(reinterpret_cast<const float4 *>(A.act + off + 4));
                v8[0] = lo.x; v8[1] = lo.y; v8[2] = lo.z; v8[3] = lo.w;
                v8[4] = hi.x; v8[5] = hi.y; v8[6] = hi.z; v8[7] = hi.w;
                quant_vals8(v8, true, 32, aq_sm + off, ad_sm + b, as_sm + b * 16 + lane / 2, nullptr, lane);
            }
            __syncthreads();
            const bool staged = mbar_wait(&mb[1], 1, STAGE_POLLS_AB);
            if (!staged && lane == 0) atomicOr(err, 2u);
            const int da = dim * c / G, db = dim * (c + 1) / G;
            for (int r = warp; r < db - da && staged; r += AB_WARPS) {
                const float y = mk_down_row<TD>(dsl, nk, r, aq_sm, ad_sm, as_sm, ffn, tsm, lane);
                float acc = 0.0f;
                for (int k = 0; k < nk; k++)  // moeRun: acc += gate * out in selection order (llama.zig:1397)
                    acc = fadd(acc, fmul(sel_g[k], __shfl_sync(0xffffffffu, y, k)));
                if (lane == 0) A.x[da + r] = fadd(A.x[da + r], acc);  // add(x, moe_acc)
            }
        }
        if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;
    }
out:
    mk_mark(A, 1);
    __syncthreads();
    if (tid == 0) {  // the last CTA out advances the epoch
        __threadfence();
        unsigned *ex = ep + 1;
        if (atomicAdd(ex, 1u) == (unsigned)G - 1) {
            *ex = 0;
            __threadfence();
            atomicAdd(ep, 1u);
        }
    }
}

using MkFn = void (*)(MkArgs);

MkFn mk_fn(int ta, int tv, int to, int tg, int td, int so) {
    if (ta == T_Q4_K && tv == T_Q6_K && to == T_Q4_K && tg == T_Q4_K && td == T_Q6_K)
        return so == 4 ? k_model<T_Q4_K, T_Q6_K, T_Q4_K, 4, T_Q4_K, T_Q6_K>
             : so == 2 ? k_model<T_Q4_K, T_Q6_K, T_Q4_K, 2, T_Q4_K, T_Q6_K>
             : so == 1 ? k_model<T_Q4_K, T_Q6_K, T_Q4_K, 1, T_Q4_K, T_Q6_K> : nullptr;
    return nullptr;
}

size_t mk_slice(int type, size_t rows, int nb) {  // a slice's staging bytes (quants, Q6_K scales, f16 scales)
    const size_t n = rows * nb;
    const bool sc = type == T_Q6_K, d = type == T_Q6_K || type == T_Q8_0 || type == T_Q4_0;
    return ab_al128(n * layout_qbytes(type)) + (sc ? ab_al128(n * 16) : 0) + (d ? ab_al128(n * 2) : 0);
}

int mk_units(int t) { return t == T_Q4_K ? 32 : t == T_Q6_K ? 32 : t == T_Q8_0 ? 64 : t == T_Q4_0 ? 64 : 0; }

int mk_sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace

int model_kernel_plan(MkArgs &A, int ta, int tk, int tv, int to, int tg, int tu, int td) {
    if (ta != tk || tg != tu) return 0;
    const int qd = A.n_heads * A.hd, kvd = A.n_kv * A.hd, GQ = A.n_heads / A.n_kv;
    const int nbO = qd / block_elems(to);
    const int so = nbO * 4 <= mk_units(to) ? 4 : nbO * 2 <= mk_units(to) ? 2 : nbO <= mk_units(to) ? 1 : 0;
    if (!so || !mk_fn(ta, tv, to, tg, td, so)) return 0;
    if (A.hd % 4 || A.hd > MAX_AB_HD || GQ > 16 || qd % 256 || kvd % 4 || A.dim % 256) return 0;
    if ((A.dim / 256) * 4 > mk_units(ta) || (A.dim / 256) * 4 > mk_units(tv) || (A.dim / 256) * 4 > mk_units(tg)) return 0;
    if (A.ffn % 256 || A.n_used > MK_MAX_USED || A.n_expert > MK_MAX_EXPERT || A.n_used > A.n_expert) return 0;
    if ((A.ffn / 256) * A.n_used > 64) return 0;  // the down row's units in the per-warp term buffer
    if (A.gating < 1 || A.gating > 3) return 0;
    const int G = mk_sm_count();
    if (A.n_used > G || A.n_heads + A.n_kv > G * AB_WARPS || qd / 256 > G) return 0;
    const int nbA = A.dim / 256, nbV = A.dim / 256, nbG = A.dim / 256, nbD = A.ffn / 256;
    const size_t rq = (qd + G - 1) / G + 1, rk = (kvd + G - 1) / G + 1, ro = (A.dim + G - 1) / G + 1;
    const size_t qkv = mk_slice(ta, rq, nbA) + mk_slice(ta, rk, nbA) + mk_slice(tv, rk, nbV);
    const size_t ost = mk_slice(to, ro, nbO);
    const size_t pairs = ((size_t)A.n_used * A.ffn + G - 1) / G + 1;
    const size_t gu = 2 * (mk_slice(tg, pairs, nbG) + 256);  // two pieces at most, each padded
    const size_t qn = (size_t)A.n_used * A.ffn;
    const size_t actq = ab_al128(qn) + ab_al128(qn / 256 * 4) + ab_al128(qn / 16 * 4);
    const size_t down = (size_t)A.n_used * mk_slice(td, ro, nbD);
    const size_t per = ((size_t)ATT_CH * (A.hd + 4) + (size_t)ATT_CH * A.hd + (size_t)GQ * A.hd + (size_t)GQ * ATT_CH) * 4;
    const size_t nsplit = (A.ctx + ATT_CH - 1) / ATT_CH;
    const size_t merge = ((size_t)(256 / A.hd + 2) * nsplit + 256) * 4;
    const size_t fixed = ab_al128(ab_al16((size_t)A.dim * 4) + ab_al16(A.dim) + ab_al16((size_t)A.dim / 32 * 4) +
                                  ab_al16((size_t)A.dim / 16 * 4));
    const size_t r1 = std::max(ost, actq + down);
    const size_t limit = 212 * 1024;  // dynamic shared memory next to ~13 KB of static
    const size_t base2 = std::max(std::max(qkv, gu), std::max(merge, (size_t)AB_WARPS * MAX_AB_HD * 4));
    if (fixed + r1 + base2 > limit) return 0;
    const int groups = (int)std::min<size_t>(AB_WARPS / AB_GRP_WARPS, (limit - fixed - r1) / per);
    if (groups < 1) return 0;
    A.groups = groups;
    A.so = so;
    A.off_r1 = fixed;
    A.off_r2 = fixed + r1;
    A.smem = A.off_r2 + std::max(base2, (size_t)groups * per);
    return 1;
}

cudaError_t launch_model_kernel(const MkArgs &A, cudaStream_t st) {
    // the instantiation is the plan's: types are fixed (Q4_K_M mix) and only the rows per warp vary
    MkFn fn = mk_fn(T_Q4_K, T_Q6_K, T_Q4_K, T_Q4_K, T_Q6_K, A.so);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)A.smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, AB_THREADS, A.smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mk_sm_count());
    cfg.blockDim = dim3(AB_THREADS);
    cfg.dynamicSmemBytes = A.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, fn, A);
}

}  // namespace loom
