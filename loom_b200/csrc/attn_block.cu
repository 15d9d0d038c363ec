// attn_block.cu -- the attention half of one decoder layer (llama.zig:1138-1216)
// as ONE cooperative launch: RMSNorm -> q/k/v matvecs -> headNorm + RoPE + KV
// append -> split-position softmax attention -> merge + quantization -> output
// projection + residual -> FFN RMSNorm, the phases separated by bounded grid
// barriers instead of kernel boundaries (the separate-kernel path of
// model.cu costs ~8 launches of a few microseconds each per layer at batch 1).
//
// One CTA per SM, 16 warps. Phases (W = all warps of the grid):
//   P1  every CTA: x -> RMSNorm -> int8 quantization into shared memory (each
//       CTA its own copy); warps hold 4 q/k/v rows each, their weight loads
//       issued before the norm (warp engine, warpdot.cuh), then the
//       reference's integer block dots; q, k, v rows to global.      barrier
//   P2  one warp per head: headNorm + RoPE; k, v appended to the cache. barrier
//   P3  groups of 4 warps: one (KV head, 32-row chunk) each, rows staged by
//       cp.async, running max / sum per query head (as k_attn_part). barrier
//   P4  CTA c < q_dim/256: merge of 256 outputs + their quantization; the
//       output-projection warps issue their weight loads first.      barrier
//   P5  output-projection rows (2 or 4 per warp): x[r] += W_o[r] . att. barrier
//   P6  CTA 0: FFN RMSNorm of the new x -> normed (the MoE layer's input).
// Every wait is bounded; on a time-out the kernel raises a bit of the error
// word and leaves (the host re-arms the counters). The arrival counter is
// monotonic: launch e of the kernel expects G * (5e + b) arrivals at barrier
// b, e being the epoch the last CTA to exit advances.
#include "attn_block.cuh"
#include "step_dev.cuh"

#include <algorithm>

namespace loom {

namespace {

template <int TA, int TV, int TO, int SO>
__global__ void __launch_bounds__(AB_THREADS, 1) k_attn_block(AttnBlockArgs A) {
    extern __shared__ __align__(128) uint8_t ab_smem[];
    __shared__ float red[AB_WARPS];
    __shared__ float Ls[40];
    __shared__ __align__(8) uint64_t mb[2];  // staged q/k/v rows, staged output-projection rows
    __shared__ float tsm_all[AB_WARPS][64];  // per-warp unit terms of ab_rows (<= 4 rows x 16 blocks)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x, gw = c * AB_WARPS + warp, W = G * AB_WARPS;
    const int dim = A.dim, nh = A.n_heads, nkv = A.n_kv, hd = A.hd, qd = nh * hd, kvd = nkv * hd;
    const int GQ = nh / nkv;
    float *tsm = tsm_all[threadIdx.x >> 5];
    unsigned long long *ctr = A.bar;
    unsigned *ep = reinterpret_cast<unsigned *>(A.bar + 1);
    unsigned *err = reinterpret_cast<unsigned *>(A.bar + 2);
    const unsigned long long base = (unsigned long long)G * AB_NBAR * *reinterpret_cast<volatile unsigned *>(ep);
    int nbar = 0;
    auto mark = [&](int i) {
        if (A.trace && c == 0 && tid == 0) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            A.trace[i] = t;
        }
    };
    mark(0);
    const int pos = (int)*A.pos;
    const bool pos_ok = pos < A.ctx;

    // ---- shared memory map (offsets from attn_block_plan, 128-byte aligned) -----------
    float *sx = reinterpret_cast<float *>(ab_smem);
    int8_t *xq = reinterpret_cast<int8_t *>(ab_smem + ab_al16((size_t)dim * 4));
    float *xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xq) + ab_al16(dim));
    int32_t *xs = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(xd) + ab_al16((size_t)dim / 32 * 4));
    uint8_t *o_stage = ab_smem + A.off_o;       // output-projection rows (live until P5)
    uint8_t *u_area = ab_smem + A.off_u;        // q/k/v rows (P1), then head scratch, attention, merge
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
        carve(sq, A.wq, qa, qb, nbA);
        carve(sk, A.wk, ka, kb, nbA);
        carve(sv, A.wv, ka, kb, nbV);
        p = o_stage;
        carve(so, A.wo, oa, ob, nbO);
    }
    if (tid == 0) {  // every weight byte of the layer this CTA needs, in flight at once
        mbar_init(&mb[0], 1);
        mbar_init(&mb[1], 1);
        const uint32_t bq = (uint32_t)((size_t)(qb - qa) * nbA * layout_qbytes(TA) + (size_t)(kb - ka) * nbA * layout_qbytes(TA) +
                                       (size_t)(kb - ka) * nbV * (layout_qbytes(TV) + (A.wv.sc ? 16 : 0)) +
                                       (size_t)(qb - qa + kb - ka) * nbA * (A.wq.sc ? 16 : 0));
        mbar_expect_tx(&mb[0], bq);
        ab_stage_bulk(A.wq, qa, qb, nbA, const_cast<uint8_t *>(sq.q), const_cast<uint8_t *>(sq.sc), &mb[0]);
        ab_stage_bulk(A.wk, ka, kb, nbA, const_cast<uint8_t *>(sk.q), const_cast<uint8_t *>(sk.sc), &mb[0]);
        ab_stage_bulk(A.wv, ka, kb, nbV, const_cast<uint8_t *>(sv.q), const_cast<uint8_t *>(sv.sc), &mb[0]);
        const uint32_t bo = (uint32_t)((size_t)(ob - oa) * nbO * (layout_qbytes(TO) + (A.wo.sc ? 16 : 0)));
        mbar_expect_tx(&mb[1], bo);
        ab_stage_bulk(A.wo, oa, ob, nbO, const_cast<uint8_t *>(so.q), const_cast<uint8_t *>(so.sc), &mb[1]);
    }
    ab_stage_d(A.wq, qa, qb, nbA, const_cast<uint16_t *>(sq.d));
    ab_stage_d(A.wk, ka, kb, nbA, const_cast<uint16_t *>(sk.d));
    ab_stage_d(A.wv, ka, kb, nbV, const_cast<uint16_t *>(sv.d));
    ab_stage_d(A.wo, oa, ob, nbO, const_cast<uint16_t *>(so.d));
    if (pos_ok) {  // this layer's cache rows, requested into L2 for the attention phase
        const size_t gt = (size_t)c * AB_THREADS + tid, nt = (size_t)G * AB_THREADS;
        ab_prefetch(A.kc, (size_t)pos * kvd * 4, gt, nt);
        ab_prefetch(A.vc, (size_t)pos * kvd * 4, gt, nt);
    }

    // ---- P1: RMSNorm + quantization, then the q/k/v rows from shared memory ---------------
    mark(8);
    ab_rmsnorm(A.x, A.attn_norm, dim, A.eps, A.serial, sx, red);  // (its barriers publish mb init and d regions)
    mark(9);
    {
        bool staged = mbar_wait(&mb[0], 0, STAGE_POLLS_AB);
        if (!staged && lane == 0) atomicOr(err, 2u);
        mark(11);
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
    mark(10);
    if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;
    mark(1);

    // ---- P2: head norm + RoPE + append (one warp per head, in shared memory) -------------
    for (int head = gw; head < nh + nkv && pos_ok; head += W) {
        const bool isk = head >= nh;
        const int kh = head - nh;
        float *vec = isk ? A.k + (size_t)kh * hd : A.q + (size_t)head * hd;
        const float *g = isk ? A.k_norm : A.q_norm;
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
                    A.kc[row + i] = hv[i];
                    A.vc[row + i] = vv[t];
                }
            }
        }
        __syncwarp();
    }
    if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;
    mark(2);

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
                const float *kb = A.kc + (size_t)t0 * kvd + (size_t)g * hd;
                const float *vb = A.vc + (size_t)t0 * kvd + (size_t)g * hd;
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
    mark(3);

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
        mark(4);

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
    mark(5);

    // ---- P6: FFN RMSNorm -> the MoE layer's input ----------------------------------------
    if (c == 0) {
        ab_rmsnorm(A.x, A.ffn_norm, dim, A.eps, A.serial, sx, red);
        for (int i = tid; i < dim; i += AB_THREADS) A.normed[i] = sx[i];
    }
out:
    mark(7);
    __syncthreads();
    if (tid == 0) {  // the last CTA out advances the epoch (counters stay consistent only without errors)
        __threadfence();
        unsigned *ex = ep + 1;
        if (atomicAdd(ex, 1u) == (unsigned)G - 1) {
            *ex = 0;
            __threadfence();
            atomicAdd(ep, 1u);
        }
    }
}

using AbFn = void (*)(AttnBlockArgs);

template <int TA, int TV, int TO> AbFn ab_pick(int so) {
    return so == 4 ? k_attn_block<TA, TV, TO, 4> : so == 2 ? k_attn_block<TA, TV, TO, 2> : k_attn_block<TA, TV, TO, 1>;
}

AbFn ab_fn(int ta, int tv, int to, int so) {
    if (ta == T_Q4_K && tv == T_Q6_K && to == T_Q4_K) return ab_pick<T_Q4_K, T_Q6_K, T_Q4_K>(so);
    if (ta == T_Q4_K && tv == T_Q4_K && to == T_Q4_K) return ab_pick<T_Q4_K, T_Q4_K, T_Q4_K>(so);
    if (ta == T_Q4_0 && tv == T_Q4_0 && to == T_Q4_0) return ab_pick<T_Q4_0, T_Q4_0, T_Q4_0>(so);
    if (ta == T_Q8_0 && tv == T_Q8_0 && to == T_Q8_0) return ab_pick<T_Q8_0, T_Q8_0, T_Q8_0>(so);
    return nullptr;
}

int ab_units(int t) { return t == T_Q4_K ? 32 : t == T_Q6_K ? 32 : t == T_Q8_0 ? 64 : t == T_Q4_0 ? 64 : 0; }

int ab_so(int to, int qd) {  // output-projection rows per warp
    const int nb = qd / block_elems(to), u = ab_units(to);
    return nb * 4 <= u ? 4 : nb * 2 <= u ? 2 : nb <= u ? 1 : 0;
}

size_t ab_fixed_smem(int dim) {
    return ab_al16((size_t)dim * 4) + ab_al16(dim) + ab_al16((size_t)dim / 32 * 4) + ab_al16((size_t)dim / 16 * 4);
}

int sm_count_ab() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace

// bytes a CTA's slice of `rows` rows (nb blocks each) of a type takes in the staging area
static size_t ab_stage_bytes(int type, size_t rows, int nb, bool sc, bool d) {
    const size_t n = rows * nb;
    return ab_al128(n * layout_qbytes(type)) + (sc ? ab_al128(n * 16) : 0) + (d ? ab_al128(n * 2) : 0);
}

int attn_block_plan(AttnBlockArgs &A, int ta, int tk, int tv, int to, size_t ctx) {
    if (ta != tk) return 0;
    const int qd = A.n_heads * A.hd, kvd = A.n_kv * A.hd, GQ = A.n_heads / A.n_kv;
    const int so = ab_so(to, qd);
    if (!ab_fn(ta, tv, to, so) || so == 0) return 0;
    if (A.hd % 4 || A.hd > MAX_AB_HD || GQ > 16 || qd % 4 || kvd % 4 || A.dim % 4) return 0;
    if (A.dim % block_elems(ta) || A.dim % block_elems(tv) || qd % block_elems(to)) return 0;
    if ((A.dim / block_elems(ta)) * 4 > ab_units(ta) || (A.dim / block_elems(tv)) * 4 > ab_units(tv)) return 0;
    if (block_elems(to) == 256 && qd % 256) return 0;
    const int G = sm_count_ab();
    if (A.n_heads + A.n_kv > G * AB_WARPS || (qd + 255) / 256 > G) return 0;
    auto has_sc = [](int t) { return t == T_Q6_K; };
    auto has_d = [](int t) { return t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0; };
    const int nbA = A.dim / block_elems(ta), nbV = A.dim / block_elems(tv), nbO = qd / block_elems(to);
    const size_t rq = (qd + G - 1) / G, rk = (kvd + G - 1) / G, ro = (A.dim + G - 1) / G;
    const size_t qkv = ab_stage_bytes(ta, rq, nbA, has_sc(ta), has_d(ta)) + ab_stage_bytes(ta, rk, nbA, has_sc(ta), has_d(ta)) +
                       ab_stage_bytes(tv, rk, nbV, has_sc(tv), has_d(tv));
    const size_t ost = ab_stage_bytes(to, ro, nbO, has_sc(to), has_d(to));
    const size_t per = ((size_t)ATT_CH * (A.hd + 4) + (size_t)ATT_CH * A.hd + (size_t)GQ * A.hd + (size_t)GQ * ATT_CH) * 4;
    const size_t nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    const size_t merge = ((size_t)(256 / A.hd + 2) * nsplit + 256) * 4;
    const size_t fixed = ab_al128(ab_fixed_smem(A.dim));
    const size_t limit = 225 * 1024;
    if (fixed + ost + std::max(qkv, merge) > limit) return 0;
    const size_t room = limit - fixed - ost;
    const int groups = (int)std::min<size_t>(AB_WARPS / AB_GRP_WARPS, room / per);
    if (groups < 1) return 0;
    A.groups = groups;
    A.off_o = fixed;
    A.off_u = fixed + ost;
    A.smem = A.off_u + std::max(std::max(qkv, (size_t)groups * per), std::max(merge, (size_t)AB_WARPS * MAX_AB_HD * 4));
    A.so = so;
    A.ta = ta;
    A.tv = tv;
    A.to = to;
    return 1;
}

cudaError_t launch_attn_block(const AttnBlockArgs &A, cudaStream_t st) {
    AbFn fn = ab_fn(A.ta, A.tv, A.to, A.so);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)A.smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, AB_THREADS, A.smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count_ab());
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
