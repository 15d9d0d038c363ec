// attn_block.cu -- the attention half of one decoder layer (llama.zig:1138-1216)
// as ONE cooperative launch: RMSNorm -> q/k/v matvecs -> headNorm + RoPE + KV
// append -> split-position softmax attention -> merge + quantization -> output
// projection + residual -> FFN RMSNorm, the phases separated by bounded grid
// barriers instead of kernel boundaries (the separate-kernel path of
// model.cu costs ~8 launches of a few microseconds each per layer at batch 1).
//
// One CTA per SM, 12 warps. Phases (W = all warps of the grid):
//   P1  every CTA: x -> RMSNorm -> int8 quantization into shared memory (each
//       CTA its own copy); warps hold 4 q/k/v rows each, their weight loads
//       issued before the norm (warp engine, warpdot.cuh), then the
//       reference's integer block dots; q, k, v rows to global.      barrier
//   P3  groups of 4 warps: one (KV head, 32-row chunk) each, rows staged by
//       cp.async; meanwhile the group's query heads get headNorm + RoPE in
//       shared memory, and the chunk holding the new position makes its key
//       (headNorm + RoPE) and value rows and appends them to the cache; then
//       running max / sum per query head (as k_attn_part).          barrier
//   P4  CTA c < q_dim/256: merge of 256 outputs + their quantization; the
//       output-projection warps issue their weight loads first.      barrier
//   P5  output-projection rows (2 or 4 per warp): x[r] += W_o[r] . att. barrier
//   P6  CTA 0: FFN RMSNorm of the new x -> normed (the MoE layer's input);
//       skipped with its barrier when `normed` is null: the MoE layer's
//       router kernel then normalizes the residual row in its prologue.
// Every wait is bounded; on a time-out the kernel raises a bit of the error
// word and leaves (the host re-arms the counters). The arrival counter is
// monotonic: launch e of the kernel expects G * (n e + b) arrivals at barrier
// b (n = 4 barriers per launch, 3 without P6), e being the epoch the last CTA
// to exit advances.
#include "attn_block.cuh"
#include "step_dev.cuh"

#include <algorithm>

namespace loom {

namespace {

#ifndef AB_HEAD_COMPACT
#define AB_HEAD_COMPACT 1
#endif

template <int TA, int TV, int TO, int SO>
__global__ void __launch_bounds__(AB_THREADS, 1) k_attn_block(AttnBlockArgs A) {
    extern __shared__ __align__(128) uint8_t ab_smem[];
    __shared__ float red[AB_WARPS];
    __shared__ float Ls[40];
    __shared__ __align__(8) uint64_t mb[2];  // staged q/k/v rows, staged output-projection rows
    __shared__ __align__(8) uint64_t mbh[AB_WARPS / AB_GRP_WARPS];  // per attention group: its head rows
    __shared__ __align__(8) uint64_t mbkv[AB_WARPS / AB_GRP_WARPS];  // per attention group: its cache rows
    __shared__ __align__(8) uint64_t mbm[3];  // merge records; output-projection input; the residual row
    __shared__ float tsm_all[AB_WARPS][64];  // per-warp unit terms of ab_rows (<= 4 rows x 16 blocks)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int dim = A.dim, nh = A.n_heads, nkv = A.n_kv, hd = A.hd, qd = nh * hd, kvd = nkv * hd;
    const int GQ = nh / nkv;
    const int RS = hd + 4;  // floats of a partial record: hd outputs, running max, sum, 2 pad (16-byte rows)
    float *tsm = tsm_all[threadIdx.x >> 5];
    unsigned long long *ctr = A.bar;
    unsigned *ep = reinterpret_cast<unsigned *>(A.bar + 1);
    unsigned *err = reinterpret_cast<unsigned *>(A.bar + 2);
    // grid barriers per launch: five, or four when the FFN norm is left to the MoE layer (normed == null)
    const int nbar_launch = A.normed ? AB_NBAR : AB_NBAR - 1;

    const unsigned long long base = (unsigned long long)G * nbar_launch * *reinterpret_cast<volatile unsigned *>(ep);
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
    // the normed activation in the padded layout (ab_quant_pad)
    int8_t *xq = reinterpret_cast<int8_t *>(ab_smem + ab_al16((size_t)dim * 4));
    float *xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xq) + ab_al16(ab_pad_qbytes(dim)));
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
        mbar_init_nf(&mb[0], 1);
        mbar_init_nf(&mb[1], 1);
        for (int i = 0; i < AB_WARPS / AB_GRP_WARPS; i++) {
            mbar_init_nf(&mbh[i], 1);
            mbar_init_nf(&mbkv[i], 1);
        }
        for (int i = 0; i < 3; i++) mbar_init_nf(&mbm[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t bq = (uint32_t)((size_t)(qb - qa) * nbA * layout_qbytes(TA) + (size_t)(kb - ka) * nbA * layout_qbytes(TA) +
                                       (size_t)(kb - ka) * nbV * (layout_qbytes(TV) + (A.wv.sc ? 16 : 0)) +
                                       (size_t)(qb - qa + kb - ka) * nbA * (A.wq.sc ? 16 : 0));
        mbar_expect_tx(&mb[0], bq);
        ab_stage_bulk(A.wq, qa, qb, nbA, const_cast<uint8_t *>(sq.q), const_cast<uint8_t *>(sq.sc), &mb[0]);
        ab_stage_bulk(A.wk, ka, kb, nbA, const_cast<uint8_t *>(sk.q), const_cast<uint8_t *>(sk.sc), &mb[0]);
        ab_stage_bulk(A.wv, ka, kb, nbV, const_cast<uint8_t *>(sv.q), const_cast<uint8_t *>(sv.sc), &mb[0]);
    }
    // The weights do not depend on the previous kernel: they were requested above, before
    // the wait for it (programmatic dependent launch; a no-op when launched without it).
    // The residual row does: requested after.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0) {
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_expect_tx(&mbm[2], (uint32_t)dim * 4);
        bulk_g2s(sx, A.x, (uint32_t)dim * 4, &mbm[2]);
    }

    // ---- P1: RMSNorm + quantization, then the q/k/v rows from shared memory ---------------
    mark(8);
    __syncthreads();  // publishes the mbarrier init
    if (!mbar_wait(&mbm[2], 0, STAGE_POLLS_AB) && lane == 0) atomicOr(err, 2u);
    // this CTA's output rows of the residual, kept for the output projection's add
    constexpr int XRES = 64;
    __shared__ float xres[XRES];
    const bool xres_ok = ob - oa <= XRES;
    if (xres_ok && tid < ob - oa) xres[tid] = sx[oa + tid];
    ab_rmsnorm_sx(A.attn_norm, dim, A.eps, A.serial, sx, red);
    mark(9);
    // the f16 scale regions (published by the barriers before the dots and before P5)
    ab_stage_d(A.wq, qa, qb, nbA, const_cast<uint16_t *>(sq.d));
    ab_stage_d(A.wk, ka, kb, nbA, const_cast<uint16_t *>(sk.d));
    ab_stage_d(A.wv, ka, kb, nbV, const_cast<uint16_t *>(sv.d));
    ab_stage_d(A.wo, oa, ob, nbO, const_cast<uint16_t *>(so.d));
    {
        bool staged = mbar_wait(&mb[0], 0, STAGE_POLLS_AB);
        if (!staged && lane == 0) atomicOr(err, 2u);
        mark(11);
        // the q/k/v rows are in: now the output-projection rows and this layer's cache rows
        // (they would otherwise share HBM with the rows the first phase waits for)
        if (tid == 0) {
            const uint32_t bo = (uint32_t)((size_t)(ob - oa) * nbO * (layout_qbytes(TO) + (A.wo.sc ? 16 : 0)));
            mbar_expect_tx(&mb[1], bo);
            ab_stage_bulk(A.wo, oa, ob, nbO, const_cast<uint8_t *>(so.q), const_cast<uint8_t *>(so.sc), &mb[1]);
        }
        if (pos_ok) {
            const size_t gt = (size_t)c * AB_THREADS + tid, nt = (size_t)G * AB_THREADS;
            ab_prefetch(A.kc, (size_t)pos * kvd * 4, gt, nt);
            ab_prefetch(A.vc, (size_t)pos * kvd * 4, gt, nt);
        }
        const bool k256A = QT<TA>::BE == 256, k256V = QT<TV>::BE == 256;
        const XV xv{xq, xd, xs};
        constexpr int SA = 4;
        const int cq = (qb - qa + SA - 1) / SA, ck = (kb - ka + SA - 1) / SA;
        const int nchunk = cq + 2 * ck;
        for (int pass = 0; pass < 2; pass++) {
            const bool k256 = pass == 0;
            if (k256 ? !(k256A || k256V) : (k256A && k256V)) continue;
            __syncthreads();
            ab_quant_pad(sx, dim, k256, xq, xd, xs);
            __syncthreads();
            for (int ch = warp; ch < nchunk && staged; ch += AB_WARPS) {
                const int m = ch < cq ? 0 : ch < cq + ck ? 1 : 2;
                const int lc = m == 0 ? ch : m == 1 ? ch - cq : ch - cq - ck;
                const AbStage &st = m == 0 ? sq : m == 1 ? sk : sv;
                if ((m <= 1 ? k256A : k256V) != k256) continue;
                const int r0 = lc * SA, nS = min(SA, st.rb - st.ra - r0);
                const int pq = ab_pad_qs(k256), ps = ab_pad_ss(k256);
                const float a = m <= 1 ? ab_rows<TA>(st, r0, nS, xv, tsm, lane, pq, ps)
                                       : ab_rows<TV>(st, r0, nS, xv, tsm, lane, pq, ps);
                float *dst = (m == 0 ? A.q : m == 1 ? A.k : A.v) + st.ra + r0;
                if (lane < nS) dst[lane] = a;
            }
        }
    }
    mark(10);
    if (!ab_barrier(ctr, base + (unsigned long long)G * ++nbar, err)) goto out;
    mark(1);

    mark(2);

    // ---- P3: attention chunks ------------------------------------------------------------
    if (pos_ok) {
        const int grp = warp / AB_GRP_WARPS, gl = tid % (AB_GRP_WARPS * 32), gwarp = warp % AB_GRP_WARPS;
        const int ngrp = A.groups;  // groups per CTA that fit in shared memory
        const int KS = hd + 4;
        const size_t per = ab_att_per(hd, GQ);
        const int live = (pos + 1 + ATT_CH - 1) / ATT_CH, items = nkv * live;
        if (grp < ngrp) {
            float *sK = att_sm + grp * per, *sV = sK + ATT_CH * KS, *qs = sV + ATT_CH * hd, *sc = qs + GQ * hd;
            float *gqs = sc + GQ * ATT_CH, *gks = gqs + hd, *css = gks + hd;  // head-norm weights, (cos, sin) pairs
            uint32_t hph = 0;  // phase of this group's head-row and cache-row barriers
            const bool kv_bulk = hd % 4 == 0;  // 16-byte rows: one bulk copy per cache row
            for (int it = c * ngrp + grp; it < items; it += G * ngrp) {
                const int g = it / live, sp = it % live;
                const int t0 = sp * ATT_CH, n = min(ATT_CH, pos + 1 - t0);
                const bool fresh = t0 + n - 1 == pos;  // the chunk of the new position: its k, v made here
                const int nold = fresh ? n - 1 : n;
                const float *kb = A.kc + (size_t)t0 * kvd + (size_t)g * hd;
                const float *vb = A.vc + (size_t)t0 * kvd + (size_t)g * hd;
                const int q4 = hd / 4;
                // headNorm + RoPE of this group's query heads (llama.zig:938-950, :830-858), and in
                // the fresh chunk of the new key (then appended to the cache) and value rows. Their
                // rows, weights and (cos, sin) pairs are loaded first, ahead of the cache rows' copies
                // (requests queued behind those wait for them); the heads are then prepared, one
                // warp per head in shared memory, while the cache rows stream in.
                const int nhp = GQ + (fresh ? 2 : 0);
                // the rows (written by other CTAs before the last grid barrier) by bulk copies: one
                // request per row instead of a load per element (many SMs read the same lines)
                if (gl == 0) {
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    const uint32_t hb = (uint32_t)hd * 4;
                    const bool rope_bulk = (A.rope_dim * 4) % 16 == 0;
                    const uint32_t bytes = (uint32_t)GQ * hb + (fresh ? 2 * hb : 0) + (A.q_norm ? hb : 0) +
                                           (A.k_norm ? hb : 0) + (rope_bulk ? (uint32_t)A.rope_dim * 4 : 0);
                    mbar_expect_tx(&mbh[grp], bytes);
                    bulk_g2s(qs, A.q + (size_t)g * GQ * hd, (uint32_t)GQ * hb, &mbh[grp]);
                    if (fresh) {
                        bulk_g2s(sK + (n - 1) * KS, A.k + (size_t)g * hd, hb, &mbh[grp]);
                        bulk_g2s(sV + (n - 1) * hd, A.v + (size_t)g * hd, hb, &mbh[grp]);
                    }
                    if (A.q_norm) bulk_g2s(gqs, A.q_norm, hb, &mbh[grp]);
                    if (A.k_norm) bulk_g2s(gks, A.k_norm, hb, &mbh[grp]);
                    if (rope_bulk) bulk_g2s(css, A.rope + (size_t)pos * A.rope_dim, (uint32_t)A.rope_dim * 4, &mbh[grp]);
                }
                if ((A.rope_dim * 4) % 16 != 0)
                    for (int i = gl; i < A.rope_dim; i += AB_GRP_WARPS * 32) css[i] = __ldg(A.rope + (size_t)pos * A.rope_dim + i);
                if (!mbar_wait(&mbh[grp], hph & 1, STAGE_POLLS_AB) && lane == 0) atomicOr(err, 2u);
                if (grp == 0) mark(28);
                asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                if (kv_bulk) {
                    // the cache rows by the copy engine (two requests per position): the head
                    // preparation's shared-memory traffic does not queue behind them
                    // (spread over the group's lanes: each issues at most a few, so no warp's own
                    // head preparation waits long behind the issue)
                    if (gl == 0) mbar_expect_tx(&mbkv[grp], (uint32_t)nold * 2 * hd * 4);
                    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                    for (int i = gl; i < 2 * nold; i += AB_GRP_WARPS * 32) {
                        const int j = i >> 1;
                        if (i & 1) bulk_g2s(sV + j * hd, vb + (size_t)j * kvd, (uint32_t)hd * 4, &mbkv[grp]);
                        else bulk_g2s(sK + j * KS, kb + (size_t)j * kvd, (uint32_t)hd * 4, &mbkv[grp]);
                    }
                } else {
                    for (int i = gl; i < nold * q4; i += AB_GRP_WARPS * 32) {
                        const int j = i / q4, c4 = (i % q4) * 4;
                        ab_cp16(sK + j * KS + c4, kb + (size_t)j * kvd + c4);
                        ab_cp16(sV + j * hd + c4, vb + (size_t)j * kvd + c4);
                    }
                    asm volatile("cp.async.commit_group;\n" ::: "memory");
                }
                if (grp == 0) mark(12);
                if (A.serial || AB_HEAD_COMPACT) {
                    for (int hh = gwarp; hh < nhp; hh += AB_GRP_WARPS) {
                        const bool isq = hh < GQ, isk = hh == GQ;
                        float *v = isq ? qs + hh * hd : isk ? sK + (n - 1) * KS : sV + (n - 1) * hd;
                        const bool norm = isq ? A.q_norm != nullptr : isk && A.k_norm != nullptr;
                        float *cache = isq ? nullptr : (isk ? A.kc : A.vc) + (size_t)pos * kvd + (size_t)g * hd;
                        ab_head_smem(v, norm ? (isq ? gqs : gks) : nullptr, hh <= GQ, css, A.rope_dim / 2, A.neox, hd,
                                     A.eps, A.serial, cache, lane);
                    }
                } else {  // this warp's heads side by side (independent chains interleaved)
                    constexpr int HW = (16 + 2 + AB_GRP_WARPS - 1) / AB_GRP_WARPS;
                    float *vr[HW];
                    float ss[HW];
#pragma unroll
                    for (int t = 0; t < HW; t++) {
                        const int hh = gwarp + AB_GRP_WARPS * t;
                        vr[t] = hh < GQ ? qs + hh * hd : hh == GQ ? sK + (n - 1) * KS : sV + (n - 1) * hd;
                        const bool norm = hh < nhp && (hh < GQ ? A.q_norm != nullptr : hh == GQ && A.k_norm != nullptr);
                        ss[t] = 0.0f;
                        if (norm)
                            for (int i = lane; i < hd; i += 32) ss[t] = fadd(ss[t], fmul(vr[t][i], vr[t][i]));
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                        for (int t = 0; t < HW; t++) ss[t] = fadd(ss[t], __shfl_xor_sync(0xffffffffu, ss[t], o));
                    __syncwarp();
                    const int half = A.rope_dim / 2;
#pragma unroll
                    for (int t = 0; t < HW; t++) {
                        const int hh = gwarp + AB_GRP_WARPS * t;
                        if (hh >= nhp) continue;
                        const bool norm = hh < GQ ? A.q_norm != nullptr : hh == GQ && A.k_norm != nullptr;
                        float *v = vr[t];
                        if (norm) {
                            const float inv = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss[t], (float)hd), A.eps)));
                            const float *gm = hh < GQ ? gqs : gks;
                            for (int i = lane; i < hd; i += 32) v[i] = fmul(fmul(v[i], inv), gm[i]);
                        }
                    }
                    __syncwarp();
#pragma unroll
                    for (int t = 0; t < HW; t++) {
                        const int hh = gwarp + AB_GRP_WARPS * t;
                        if (hh >= nhp || hh > GQ) continue;  // RoPE on queries and the key
                        float *v = vr[t];
                        for (int j = lane; j < half; j += 32) {
                            const int ia = A.neox ? j : 2 * j, ib = A.neox ? j + half : 2 * j + 1;
                            const float a = v[ia], b = v[ib], co = css[2 * j], si = css[2 * j + 1];
                            v[ia] = fsub(fmul(a, co), fmul(b, si));
                            v[ib] = fadd(fmul(a, si), fmul(b, co));
                        }
                    }
                    __syncwarp();
#pragma unroll
                    for (int t = 0; t < HW; t++) {
                        const int hh = gwarp + AB_GRP_WARPS * t;
                        if (hh < GQ || hh >= nhp) continue;  // the new key and value rows -> the cache
                        float *cache = (hh == GQ ? A.kc : A.vc) + (size_t)pos * kvd + (size_t)g * hd;
                        for (int i = lane; i < hd; i += 32) cache[i] = vr[t][i];
                    }
                }
                if (grp == 0) mark(13);
                if (kv_bulk) {
                    if (!mbar_wait(&mbkv[grp], hph & 1, STAGE_POLLS_AB) && lane == 0) atomicOr(err, 2u);
                } else {
                    asm volatile("cp.async.wait_all;\n" ::: "memory");
                }
                hph++;
                asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                if (grp == 0) mark(14);
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
                if (grp == 0) mark(15);
                // records head-major: [query head][split][RS] (a head's records are one contiguous run)
                float *rec = A.part + ((size_t)g * GQ * A.nsplit + sp) * RS;
                for (int hh = gwarp; hh < GQ; hh += AB_GRP_WARPS) {
                    const float v = lane < n ? sc[hh * ATT_CH + lane] : -INFINITY;
                    const float m = warp_max(v);
                    const float e = lane < n ? exp_f(v - m) : 0.0f;
                    if (lane < n) sc[hh * ATT_CH + lane] = e;
                    const float l = ab_warp_sum(e);
                    if (lane == 0) {
                        rec[(size_t)hh * A.nsplit * RS + hd] = m;
                        rec[(size_t)hh * A.nsplit * RS + hd + 1] = l;
                    }
                }
                asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                if (grp == 0) mark(16);
                for (int d = gl; d < hd; d += AB_GRP_WARPS * 32) {
                    float acc[16];
#pragma unroll
                    for (int hh = 0; hh < 16; hh++) acc[hh] = 0.0f;
                    int j = 0;
                    for (; j + 4 <= n; j += 4) {  // four positions per score load (broadcast float4)
                        const float v0 = sV[j * hd + d], v1 = sV[(j + 1) * hd + d];
                        const float v2 = sV[(j + 2) * hd + d], v3 = sV[(j + 3) * hd + d];
#pragma unroll
                        for (int hh = 0; hh < 16; hh++)
                            if (hh < GQ) {
                                const float4 s4 = *reinterpret_cast<const float4 *>(sc + hh * ATT_CH + j);
                                acc[hh] = fmaf(s4.w, v3, fmaf(s4.z, v2, fmaf(s4.y, v1, fmaf(s4.x, v0, acc[hh]))));
                            }
                    }
                    for (; j < n; j++) {
                        const float vv = sV[j * hd + d];
#pragma unroll
                        for (int hh = 0; hh < 16; hh++)
                            if (hh < GQ) acc[hh] = fmaf(sc[hh * ATT_CH + j], vv, acc[hh]);
                    }
#pragma unroll
                    for (int hh = 0; hh < 16; hh++)
                        if (hh < GQ) rec[(size_t)hh * A.nsplit * RS + d] = acc[hh];
                }
                asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(AB_GRP_WARPS * 32) : "memory");
                if (grp == 0) mark(17);
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
            const size_t stride = (size_t)RS;  // consecutive splits of one head
            const int e0 = c * 256, h0 = e0 / hd, h1 = min((e0 + 255) / hd, nh - 1), nlh = h1 - h0 + 1;
            float *wsm = att_sm;                                   // [heads][live]
            float *val = att_sm + ((nlh * live + 3) & ~3);         // [256] (16-byte aligned)
            // every record of this CTA's heads by bulk copies (written by other CTAs: one request per
            // record instead of a load per float), when they fit in shared memory
            float *recs = val + 256;                     // [heads][live][RS]
            const bool bulk = A.merge_bulk;
            if (bulk) {
                if (tid == 0) {  // one copy per head: its live records are contiguous
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    mbar_expect_tx(&mbm[0], (uint32_t)(nlh * live * RS * 4));
                    for (int lh = 0; lh < nlh; lh++)
                        bulk_g2s(recs + (size_t)lh * live * RS, A.part + (size_t)(h0 + lh) * A.nsplit * RS,
                                 (uint32_t)(live * RS * 4), &mbm[0]);
                }
                if (!mbar_wait(&mbm[0], 0, STAGE_POLLS_AB) && lane == 0) atomicOr(err, 2u);
            }
            for (int lh = warp; lh < nlh; lh += AB_WARPS) {
                const int h = h0 + lh;
                const float *rec = bulk ? recs + (size_t)lh * live * RS : A.part + (size_t)h * A.nsplit * RS;
                const size_t rst = bulk ? (size_t)RS : stride;
                float *w = wsm + lh * live;
                float M = -INFINITY;
                for (int s2 = lane; s2 < live; s2 += 32) M = fmaxf(M, rec[s2 * rst + hd]);
                M = warp_max(M);
                float L = 0.0f;
                for (int s2 = lane; s2 < live; s2 += 32) {
                    const float ws = exp_f(rec[s2 * rst + hd] - M);
                    w[s2] = ws;
                    L = fmaf(rec[s2 * rst + hd + 1], ws, L);
                }
                L = ab_warp_sum(L);
                if (lane == 0) Ls[lh] = L;
            }
            __syncthreads();
            mark(18);
            if (tid < 256) {
                const int e = e0 + tid;
                float o = 0.0f;
                if (e < qd) {
                    const int h = e / hd, d = e % hd, lh = h - h0;
                    const float *rec = bulk ? recs + (size_t)lh * live * RS + d : A.part + (size_t)h * A.nsplit * RS + d;
                    const size_t rst = bulk ? (size_t)RS : stride;
                    const float *w = wsm + lh * live;
#pragma unroll 32
                    for (int s2 = 0; s2 < live; s2++) o = fmaf(rec[s2 * rst], w[s2], o);
                    o = o / Ls[lh];
                }
                val[tid] = o;
            }
            __syncthreads();
            mark(19);
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
        // the quantized attention output (written by the merge CTAs) into shared memory, padded
        int8_t *pq8 = reinterpret_cast<int8_t *>(att_sm);
        float *pd = reinterpret_cast<float *>(pq8 + ab_al16(ab_pad_qbytes(qd)));
        int32_t *ps32 = reinterpret_cast<int32_t *>(pd + ab_al16((size_t)qd / 32 * 4) / 4);
        if (k256O && (qd / 256) % 4 == 0) {  // per block: its quants and sums by bulk copies, padded
            const int nbo = qd / 256;
            if (warp == 0) {
                if (lane == 0) {
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    mbar_expect_tx(&mbm[1], (uint32_t)nbo * (256 + 64) + (uint32_t)nbo * 4);
                    bulk_g2s(pd, A.ad, (uint32_t)nbo * 4, &mbm[1]);
                }
                __syncwarp();
                for (int b = lane; b < nbo; b += 32) {
                    bulk_g2s(pq8 + (size_t)b * ab_pad_qs(true), A.aq + (size_t)b * 256, 256, &mbm[1]);
                    bulk_g2s(ps32 + (size_t)b * ab_pad_ss(true), A.as + (size_t)b * 16, 64, &mbm[1]);
                }
            }
            if (!mbar_wait(&mbm[1], 0, STAGE_POLLS_AB) && lane == 0) atomicOr(err, 2u);
        } else {
            const int BEo = QT<TO>::BE, nbo = qd / BEo, qso = ab_pad_qs(k256O), sso = ab_pad_ss(k256O);
            const int c16 = BEo / 16;  // 16-byte chunks per block
            for (int i = tid; i < nbo * c16; i += AB_THREADS) {
                const int b = i / c16, cc = i - b * c16;
                *reinterpret_cast<int4 *>(pq8 + (size_t)b * qso + 16 * cc) =
                    __ldcg(reinterpret_cast<const int4 *>(A.aq + (size_t)b * BEo) + cc);
            }
            const int spb = QT<TO>::SPB;
            for (int i = tid; i < nbo * spb; i += AB_THREADS) ps32[(i / spb) * sso + i % spb] = __ldcg(A.as + i);
            for (int i = tid; i < nbo; i += AB_THREADS) pd[i] = __ldcg(A.ad + i);
        }
        __syncthreads();
        const XV av{pq8, pd, ps32};
        const int nco = (ob - oa + SO - 1) / SO;
        for (int ch = warp; ch < nco && staged; ch += AB_WARPS) {
            const int r0 = ch * SO, nS = min(SO, ob - oa - r0);
            const float a = ab_rows<TO>(so, r0, nS, av, tsm, lane, ab_pad_qs(k256O), ab_pad_ss(k256O));
            if (lane < nS)  // llama.zig:1195 add
                A.x[oa + r0 + lane] = fadd(xres_ok ? xres[r0 + lane] : A.x[oa + r0 + lane], a);
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!A.normed) goto out;  // the MoE layer's router kernel applies the FFN norm itself
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
    return ab_al16((size_t)dim * 4) + ab_al16(ab_pad_qbytes(dim)) + ab_al16((size_t)dim / 32 * 4) +
           ab_al16(ab_pad_sbytes(dim));
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
    const size_t per = ab_att_per(A.hd, GQ) * 4;
    const size_t nsplit = (ctx + ATT_CH - 1) / ATT_CH;
    const size_t merge_nb = ((size_t)(256 / A.hd + 2) * nsplit + 256) * 4;
    const size_t merge_b = merge_nb + 16 + (size_t)(256 / A.hd + 1) * nsplit * (A.hd + 4) * 4;
    const size_t fixed = ab_al128(ab_fixed_smem(A.dim));
    const size_t limit = 225 * 1024;
    if (fixed + ost + std::max(qkv, merge_nb) > limit) return 0;
    if (fixed + ost + ab_al16(ab_pad_qbytes(qd)) + ab_al16((size_t)qd / 32 * 4) + ab_al16(ab_pad_sbytes(qd)) > limit) return 0;
    const size_t room = limit - fixed - ost;
    // the merge reads its records by bulk copies when they fit beside the staging
    A.merge_bulk = std::max(qkv, merge_b) <= room;
    const size_t merge = A.merge_bulk ? merge_b : merge_nb;
    const int groups = (int)std::min<size_t>(AB_WARPS / AB_GRP_WARPS, room / per);
    if (groups < 1) return 0;
    A.groups = groups;
    A.off_o = fixed;
    A.off_u = fixed + ost;
    const size_t p5 = ab_al16(ab_pad_qbytes(qd)) + ab_al16((size_t)qd / 32 * 4) + ab_al16(ab_pad_sbytes(qd));
    A.smem = A.off_u + std::max(std::max(std::max(qkv, (size_t)groups * per), std::max(merge, (size_t)AB_WARPS * MAX_AB_HD * 4)),
                                p5);
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
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    // with programmatic dependent launch the q/k/v weight copies overlap the previous kernel's
    // tail; if the runtime refuses the combination, the launch is cooperative only
    static int pdl_ok = getenv("LOOM_CUDA_NO_AB_PDL") ? 0 : 1;
    count_launch();
    if (pdl_ok) {
        cfg.numAttrs = 2;
        e = cudaLaunchKernelEx(&cfg, fn, A);
        if (e == cudaSuccess) return e;
        cudaGetLastError();
        pdl_ok = 0;
    }
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, A);
}

}  // namespace loom
