// moe_tc.cu -- the expert FFN of batched prefill on the 5th-generation tensor
// cores, as warp-specialized persistent kernels.
//
// Arithmetic (unchanged from the reference, ggml.zig kBlockDot :1002): each
// MMA carries integer sub-block products that fp16 holds exactly,
//   A = the weight's folded sub-block values   Q4_K  sc * q        (<= 945)
//                                              Q6_K  sc * (q - 32) (|.| <= 1024 when |sc| <= 32;
//                                                    any int8 sc: split in two tiles, FMT 2)
//   B = the int8 activations of quantizeX256 (ggml.zig:776),
// accumulated in f32 in TMEM over half a super-block (128 products, every
// partial sum an integer below 2^24, so exact). The epilogue adds the two
// halves as integers, forms the reference's float tail per super-block and
// accumulates the blocks in block order from +0: results equal the CPU's bit
// for bit.
//
// Work unit ("tile"): one expert x 128 weight rows x up to TC_N of the
// expert's tokens, all super-blocks of the row. Tiles are numbered expert by
// expert, row tile by row tile, token chunk by token chunk (consecutive tiles
// share weights, which stay in L2), and CTA c takes tiles c, c + grid, ...
//
// Roles of one CTA (576 threads, one CTA per SM):
//   warp 8       producer: per super-block, one 2D tensor copy (TMA, into
//                this CTA only) of the tile's 128 raw weight rows per matrix and
//                one bulk copy per token row into a 2-stage ring, completion by
//                mbarrier transaction count
//   warps 10-17  converters: raw stage -> fp16 operand tiles (K = 64 per
//                stage, K-major core-matrix layout) in a 2-stage ring; per
//                super-block also the rows' float scales and the tokens' scales
//                for the epilogue (4-slot ring)
//   warp 9       one thread issues the MMAs (M 128, N = tokens rounded up to
//                16, K 16) into TMEM, two super-block accumulators in flight
//   warps 0-7    epilogue: TMEM -> integer dots -> float tail per super-block;
//                at the end of the tile SwiGLU (gate/up) or the down output
// Every wait is bounded: on a timeout the kernel raises bit 64 of the error
// word, stops taking tiles, lets its copies and MMAs drain and frees TMEM.
#include <cuda.h>  // CUtensorMap (the encoder is reached through the runtime's driver entry point)
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "decode.cuh"
#include "umma.cuh"
#include "warpdot.cuh"

namespace loom {

constexpr int TC_N = MOE_TC_N;      // tokens per tile (the MMA's N after rounding up to 16)
constexpr int TC_EPI_WARPS = 8;     // warps 0-7: TMEM lane quarter = warp % 4, token half = warp / 4
constexpr int TC_PRO_WARP = 8;
constexpr int TC_MMA_WARP = 9;
constexpr int TC_CVT_WARP0 = 10, TC_CVT_WARPS = 8;
constexpr int TC_THREADS = (TC_CVT_WARP0 + TC_CVT_WARPS) * 32;

constexpr int TC_RS = 2, TC_OS = 2, TC_HS = 4;
constexpr uint32_t TC_POLLS = 1u << 21;   // suspending polls (drains)
constexpr int TC_XPITCH = 272;      // token row pitch in a raw stage: 16-byte reads by consecutive rows are conflict-free

// FMT 0: gate and up, Q4_K (two matrices); FMT 1: down, Q6_K (one matrix).
// FMT 2: down, Q6_K with any int8 sub-block scale: q - 32 = 8 (qh - 4) + ql
// (qh = q >> 3, ql = q & 7) splits the folded value into two operand tiles,
//   hi = sc * (qh - 4) (|.| <= 512) and lo = sc * ql (|.| <= 896),
// each exact in fp16 with 128-product partial sums below 2^24; the epilogue
// forms the integer 8 I_hi + I_lo. One raw matrix, two operand matrices.
template <int FMT> struct TcFmt;
template <> struct TcFmt<0> {
    static constexpr int MATS = 2, RMATS = 2, WPITCH = 144;  // raw Q4_K block
};
template <> struct TcFmt<1> {
    static constexpr int MATS = 1, RMATS = 1, WPITCH = 208;  // Q6_K quants [128][192], then int8 scales [128][16]
};
template <> struct TcFmt<2> {
    static constexpr int MATS = 2, RMATS = 1, WPITCH = 208;
};

// 2D tensor maps of the weights, rows x bytes: FMT 0 gate, up, shared gate,
// shared up (box 144 x 128); FMT 1 down quants (box 192 x 128), down scales
// (box 16 x 128), the shared expert's quants and scales.
struct TcMaps {
    CUtensorMap m[4];
};

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

template <int FMT> struct TcLayout {
    static constexpr int MATS = TcFmt<FMT>::MATS, WPITCH = TcFmt<FMT>::WPITCH;
    static constexpr size_t RAW_W = (size_t)TcFmt<FMT>::RMATS * 128 * WPITCH, RAW_X = (size_t)TC_N * TC_XPITCH;
    static constexpr size_t RAW = RAW_W + RAW_X;
    static constexpr size_t OP_A = (size_t)8 * 128 * 16, OP = MATS * OP_A + (size_t)8 * TC_N * 16;
    static constexpr size_t HDR = (size_t)MATS * 128 * 16;      // per row: d, dmin, mins (2 words)
    static constexpr size_t TOK = (size_t)TC_N * 4 + (size_t)TC_N * 16;  // per token: xd, packed per-32 sums
    static constexpr size_t SMEM = TC_RS * RAW + TC_OS * OP + TC_HS * (HDR + TOK);
    static constexpr uint32_t TMEM_COLS = MATS == 2 ? 512 : 256;  // 2 buffers x MATS x 2 halves x TC_N
};

struct TcTile {
    int e, rt, c0, nc;
    bool shared;
};

// Tile t of this launch (RT row tiles per expert, CH slots per token chunk);
// false past the last tile.
__device__ __forceinline__ bool tc_tile(const DecodeArgs &A, int RT, int t, TcTile &o, int CH = TC_N) {
    const int nexp = A.n_local + (A.has_shared ? 1 : 0);
    const int *pre = A.tc_pre;
    if (t >= pre[nexp] * RT) return false;
    int lo = 0, hi = nexp;  // the last expert whose first tile is <= t
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] * RT <= t) lo = mid;
        else hi = mid;
    }
    const int nch = pre[lo + 1] - pre[lo], loc = t - pre[lo] * RT;
    o.e = lo;
    o.shared = lo == A.n_local;
    o.rt = loc / nch;
    o.c0 = (loc % nch) * CH;
    const int n = o.shared ? A.T : A.grp_cnt[lo];
    o.nc = n - o.c0 < CH ? n - o.c0 : CH;
    return true;
}

__device__ __forceinline__ int tc_slot(const DecodeArgs &A, const TcTile &tl, int i) {
    return tl.shared ? A.T * A.n_used + tl.c0 + i : A.grp_list[A.grp_off[tl.e] + tl.c0 + i];
}

// The tile tables (tc_pre, grp_cnt, grp_off) copied into shared memory at
// kernel start: the per-tile lookups (a binary search over tc_pre, then the
// group offset) would otherwise be chains of dependent global loads that stall
// the warps at every tile boundary.
struct TileTab {
    const int *pre, *cnt, *off;
};
__host__ __device__ constexpr size_t tc_tab_bytes(int n_local) { return ((size_t)3 * (n_local + 3) * 4 + 15) & ~(size_t)15; }
// every thread of the CTA; a __syncthreads() must follow before the first use
__device__ __forceinline__ TileTab tc_tab_load(const DecodeArgs &A, int *buf) {
    const int nexp = A.n_local + (A.has_shared ? 1 : 0), n = A.n_local + 3;
    for (int i = threadIdx.x; i <= nexp; i += blockDim.x) buf[i] = A.tc_pre[i];
    for (int i = threadIdx.x; i < A.n_local; i += blockDim.x) {
        buf[n + i] = A.grp_cnt[i];
        buf[2 * n + i] = A.grp_off[i];
    }
    return TileTab{buf, buf + n, buf + 2 * n};
}
__device__ __forceinline__ bool tc_tile(const DecodeArgs &A, const TileTab &tt, int RT, int t, TcTile &o,
                                        int CH = TC_N) {
    const int nexp = A.n_local + (A.has_shared ? 1 : 0);
    const int *pre = tt.pre;
    if (t >= pre[nexp] * RT) return false;
    int lo = 0, hi = nexp;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] * RT <= t) lo = mid;
        else hi = mid;
    }
    const int nch = pre[lo + 1] - pre[lo], loc = t - pre[lo] * RT;
    o.e = lo;
    o.shared = lo == A.n_local;
    o.rt = loc / nch;
    o.c0 = (loc % nch) * CH;
    const int n = o.shared ? A.T : tt.cnt[lo];
    o.nc = n - o.c0 < CH ? n - o.c0 : CH;
    return true;
}
__device__ __forceinline__ int tc_slot(const DecodeArgs &A, const TileTab &tt, const TcTile &tl, int i) {
    return tl.shared ? A.T * A.n_used + tl.c0 + i : A.grp_list[tt.off[tl.e] + tl.c0 + i];
}

__device__ __forceinline__ void tc_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// 8 consecutive f32 accumulator columns of TMEM lane quarter q (exact integers)
__device__ __forceinline__ void tmem_f8(uint32_t tmem, int q, uint32_t col, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(tmem + ((uint32_t)(32 * q) << 16) + col));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t tc_h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 tc_u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// scaleMinK4 (ggml.zig:1332-1340) with the 12 scale bytes in three words
__device__ __forceinline__ void tc_scale_min(int j, uint32_t y, uint32_t z, uint32_t w, int &sc, int &mn) {
    auto byte = [&](int i) -> int { return (int)(((i < 4 ? y : i < 8 ? z : w) >> (8 * (i & 3))) & 0xFF); };
    if (j < 4) {
        sc = byte(j) & 63;
        mn = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
        mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

// Exact small-integer -> fp16 through the fp16 "magic" 1024: 0x6400 | v is
// 1024 + v for 0 <= v < 1024; one HFMA2 / HSUB2 of exactly representable
// operands with an exactly representable result is exact.
// Q4_K: one word of nibble bytes -> sc_lo * (low nibbles) and sc_hi * (high
// nibbles) as fp16 pairs (bytes 0,1 and 2,3).
__device__ __forceinline__ void tc_q4_word(uint32_t w, __half2 sl2, __half2 offl, __half2 sh16, __half2 offh,
                                           uint32_t &lo01, uint32_t &lo23, uint32_t &hi01, uint32_t &hi23) {
    const uint32_t p01 = __byte_perm(w, 0, 0x4140), p23 = __byte_perm(w, 0, 0x4342);
    lo01 = tc_h2u(__hfma2(tc_u2h((p01 & 0x000F000Fu) | 0x64006400u), sl2, offl));  // (1024 + q) sc - 1024 sc
    lo23 = tc_h2u(__hfma2(tc_u2h((p23 & 0x000F000Fu) | 0x64006400u), sl2, offl));
    hi01 = tc_h2u(__hfma2(tc_u2h((p01 & 0x00F000F0u) | 0x64006400u), sh16, offh));  // (1024 + 16q) sc/16 - 64 sc
    hi23 = tc_h2u(__hfma2(tc_u2h((p23 & 0x00F000F0u) | 0x64006400u), sh16, offh));
}
// 8 int8 -> 8 fp16, exact: (1024 + (v + 128)) - 1152
__device__ __forceinline__ uint4 tc_h8(uint32_t lo, uint32_t hi) {
    const __half2 k = tc_u2h(0x64806480u);
    lo ^= 0x80808080u;
    hi ^= 0x80808080u;
    return make_uint4(tc_h2u(__hsub2(tc_u2h(__byte_perm(lo, 0x64646464u, 0x7170)), k)),
                      tc_h2u(__hsub2(tc_u2h(__byte_perm(lo, 0x64646464u, 0x7372)), k)),
                      tc_h2u(__hsub2(tc_u2h(__byte_perm(hi, 0x64646464u, 0x7170)), k)),
                      tc_h2u(__hsub2(tc_u2h(__byte_perm(hi, 0x64646464u, 0x7372)), k)));
}

// Operand tiles use the K-major 128-byte-swizzle layout: one row per 128
// bytes (64 fp16 of K, the K extent of a stage), 8-row atoms of 1 KB, the
// 16-byte chunk c of row r stored at chunk position c ^ (r % 8). Stores by
// consecutive rows and the tensor core's reads are free of bank conflicts.
__device__ __forceinline__ size_t tc_sw(int r, int c) { return (size_t)r * 128 + (size_t)((c ^ (r & 7)) << 4); }

// Shared-memory matrix descriptor of such a tile (1 KB aligned): start >> 4,
// leading offset 1 (unused for swizzled K-major), stride offset 1024 B (next
// 8-row atom), version 1 (bit 46), layout SWIZZLE_128B (2 in bits [61,64)).
// A K step of 16 fp16 (32 bytes) inside the atom advances the start by 2.
__device__ __forceinline__ uint64_t tc_desc_sw128(const void *tile) {
    return (uint64_t)((smem_u32(tile) >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__host__ __device__ constexpr uint32_t tc_idesc(int M, int N) {  // kind::f16, fp16 A and B, f32 D, K-major
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct TcBars {
    uint64_t raw_full[TC_RS], raw_empty[TC_RS], op_full[TC_OS], op_empty[TC_OS];
    uint64_t acc_full[2], acc_empty[2], hdr_full[TC_HS], hdr_empty[TC_HS], drain;
    uint32_t tmem;
    int err;
    int prof;  // cycle profile on for this CTA
};

// Diagnostic cycle profile of CTA 0 (loom_cuda_tc_profile): per wait site
// the clock64 cycles spent waiting, plus per role the cycles from its first
// tile to its end.
constexpr int TC_PROF_SLOTS = 24;
__device__ int g_tc_prof_on = 0;
__device__ unsigned long long g_tc_prof[2][TC_PROF_SLOTS];  // by FMT
// `on`: the CTA's copy of (g_tc_prof_on && blockIdx.x == 0), read once at kernel start
__device__ __forceinline__ void tc_prof_add(int on, int fmt, int slot, long long cyc) {
    if (on) atomicAdd(&g_tc_prof[fmt != 0][slot], (unsigned long long)cyc);
}

// bounded wait by one thread; a timeout raises the CTA's error flag
__device__ __forceinline__ bool tc_wait(TcBars &B, uint64_t *bar, uint32_t parity, int *gerr, int fmt = 0,
                                        int slot = -1) {
    if (*reinterpret_cast<volatile int *>(&B.err)) return false;
    const long long c0 = B.prof ? clock64() : 0;
    const bool ok = mbar_wait(bar, parity, TC_POLLS);
    if (slot >= 0) tc_prof_add(B.prof, fmt, slot, clock64() - c0);
    if (ok) return true;
    *reinterpret_cast<volatile int *>(&B.err) = 1;
    if (gerr) atomicOr(gerr, 64);
    return false;
}
__device__ __forceinline__ bool tc_ok(TcBars &B) { return *reinterpret_cast<volatile int *>(&B.err) == 0; }

// The epilogue's per-block scalars that live in global memory (the token's
// xd and per-16 sums, the Q6_K row's d), loaded a super-block ahead into
// registers so their latency overlaps a block's conversion.
template <int FMT, int NB>
__device__ __forceinline__ void tc_pf_load(const DecodeArgs &A, const TcTile &t, int blk, int slot, int ct, int R,
                                           int stride, float &xd, float &d, int4 (&s)[4]) {
    if (ct < t.nc) {
        if (FMT == 0) {
            const size_t tk = t.shared ? (size_t)(t.c0 + ct) : (size_t)(slot / A.n_used);
            xd = A.x256.d[tk * NB + blk];
            const int4 *ss = reinterpret_cast<const int4 *>(A.x256.s + (tk * NB + blk) * 16);
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++) s[k4] = ss[k4];
        } else {
            xd = A.ad[(size_t)slot * (stride / 32) + blk];
        }
    }
    if (FMT != 0) {
        const int r0 = t.rt * 128;
        if (ct < 128 && r0 + ct < R) {
            const WDev w = t.shared ? A.sdn : A.dn;
            const uint64_t pl = t.shared ? 0 : (uint64_t)t.e * R * NB;
            d = f16_to_f32(w.d[pl + (uint64_t)(r0 + ct) * NB + blk]);
        }
    }
}

template <int FMT, int NB>
__global__ void __launch_bounds__(TC_THREADS, 1) k_moe_tc(DecodeArgs A, const __grid_constant__ TcMaps M) {
    using Ly = TcLayout<FMT>;
    constexpr int MATS = Ly::MATS;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ TcBars B;
    uint8_t *raw = sm, *ops = sm + TC_RS * Ly::RAW, *hdr = ops + TC_OS * Ly::OP, *tok = hdr + TC_HS * Ly::HDR;
    const TileTab TT = tc_tab_load(A, reinterpret_cast<int *>(sm + Ly::SMEM));
    const int R = FMT == 0 ? A.ffn : A.dim;  // weight rows
    const int RT = (R + 127) / 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    {
        TcTile t0;
        if (!tc_tile(A, RT, blockIdx.x, t0)) return;  // no work for this CTA
    }
    if (warp == 0) tmem_alloc(&B.tmem, Ly::TMEM_COLS);
    if (tid == 0) {
        for (int i = 0; i < TC_RS; i++) {
            mbar_init(&B.raw_full[i], 1);
            mbar_init(&B.raw_empty[i], TC_CVT_WARPS);
        }
        for (int i = 0; i < TC_OS; i++) {
            mbar_init(&B.op_full[i], TC_CVT_WARPS);
            mbar_init(&B.op_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&B.acc_full[i], 1);
            mbar_init(&B.acc_empty[i], TC_EPI_WARPS);
        }
        for (int i = 0; i < TC_HS; i++) {
            mbar_init(&B.hdr_full[i], TC_CVT_WARPS);
            mbar_init(&B.hdr_empty[i], TC_EPI_WARPS);
        }
        mbar_init(&B.drain, 1);
        B.err = 0;
        B.prof = g_tc_prof_on && blockIdx.x == 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem;
    const int dim = A.dim, stride = A.act_stride;

    const long long t_start = clock64();
    if (warp == TC_PRO_WARP) {
        // ---- producer ----------------------------------------------------------------------
        uint32_t gb = 0;
        TcTile tl;
        bool run = true;
        for (int ti = blockIdx.x; run && tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) {
            const int row0 = tl.rt * 128;
            const int8_t *src[2] = {nullptr, nullptr};  // this lane's token rows (i = lane, lane + 32), block 0
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int i = lane + 32 * u;
                if (i < tl.nc) {
                    const int slot = tc_slot(A, TT, tl, i);
                    src[u] = FMT == 0 ? A.x256.q + (size_t)(tl.shared ? tl.c0 + i : slot / A.n_used) * dim
                                      : A.aq + (size_t)slot * stride;
                }
            }
            for (int blk = 0; blk < NB; blk++, gb++) {
                const int s = gb % TC_RS;
                int ok = 1;
                if (lane == 0) ok = gb >= TC_RS ? tc_wait(B, &B.raw_empty[s], ((gb / TC_RS) - 1) & 1, A.err, FMT, 0) : tc_ok(B);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    run = false;
                    break;
                }
                uint8_t *W = raw + (size_t)s * Ly::RAW, *X = W + Ly::RAW_W;
                // full boxes always land (rows past the tensor read as zero, rows of the next expert are ignored)
                const uint32_t bytes = (uint32_t)Ly::RAW_W + (uint32_t)tl.nc * 256;
                if (lane == 0) {
                    mbar_expect_tx(&B.raw_full[s], bytes);
                    const int y = (tl.shared ? 0 : tl.e * R) + row0, m0 = tl.shared ? 2 : 0;
                    if (FMT == 0) {
                        tma_load_2d(W, &M.m[m0], blk * 144, y, &B.raw_full[s]);
                        tma_load_2d(W + 128 * 144, &M.m[m0 + 1], blk * 144, y, &B.raw_full[s]);
                    } else {
                        tma_load_2d(W, &M.m[m0], blk * 192, y, &B.raw_full[s]);
                        tma_load_2d(W + 128 * 192, &M.m[m0 + 1], blk * 16, y, &B.raw_full[s]);
                    }
                }
                __syncwarp();
#pragma unroll
                for (int u = 0; u < 2; u++)
                    if (src[u]) bulk_g2s(X + (size_t)(lane + 32 * u) * TC_XPITCH, src[u] + blk * 256, 256, &B.raw_full[s]);
            }
        }
        // drain: the last stages' copies must land before the CTA can exit
        if (lane == 0 && !run)
            for (uint32_t g = gb > TC_RS ? gb - TC_RS : 0; g < gb; g++)
                mbar_wait(&B.raw_full[g % TC_RS], (g / TC_RS) & 1, TC_POLLS);
    } else if (warp >= TC_CVT_WARP0) {
        // ---- converters ----------------------------------------------------------------------
        const int ct = tid - TC_CVT_WARP0 * 32;
        uint32_t gb = 0, gq = 0;
        // the epilogue's per-block scalars that live in global memory (token scales, Q6_K row
        // scales) are loaded one super-block ahead, so their latency overlaps a block's work
        float pf_xd = 0.0f, pf_d = 0.0f;
        int4 pf_s[4];
        // this thread's token slot (ct < nc) of the current and of the next tile, read a tile ahead
        int slot_cur = 0, slot_nxt = 0;
#define TC_PF_LOAD(t, blk, slot) tc_pf_load<FMT, NB>(A, (t), (blk), (slot), ct, R, stride, pf_xd, pf_d, pf_s)
        TcTile tl, tn;
        if (tc_tile(A, TT, RT, blockIdx.x, tl)) {
            if (ct < tl.nc) slot_cur = tc_slot(A, TT, tl, ct);
            TC_PF_LOAD(tl, 0, slot_cur);
        }
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) {
            const bool has_next = tc_tile(A, TT, RT, ti + gridDim.x, tn);
            if (has_next && ct < tn.nc) slot_nxt = tc_slot(A, TT, tn, ct);
            const int row0 = tl.rt * 128, rows = R - row0 < 128 ? R - row0 : 128;
            const int N = (tl.nc + 15) & ~15;
            bool run = true;
            for (int blk = 0; blk < NB && run; blk++, gb++) {
                const int s = gb % TC_RS, hs = gb % TC_HS;
                // each converter warp waits on its own (no CTA-level barrier: warps drift within the rings)
                int ok = 1;
                if (lane == 0) {
                    ok = tc_wait(B, &B.raw_full[s], (gb / TC_RS) & 1, A.err, FMT, ct == 0 ? 1 : -1);
                    if (ok && gb >= TC_HS)
                        ok = tc_wait(B, &B.hdr_empty[hs], ((gb / TC_HS) - 1) & 1, A.err, FMT, ct == 0 ? 2 : -1);
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    run = false;
                    break;
                }
                const uint8_t *W = raw + (size_t)s * Ly::RAW, *X = W + Ly::RAW_W;
                const long long c_h = clock64();
                // the epilogue's per-block scalars: rows' scales, tokens' scales
                {
                    uint4 *H = reinterpret_cast<uint4 *>(hdr + (size_t)hs * Ly::HDR);
                    if (FMT == 0) {
                        const int mat = ct >> 7, r = ct & 127;
                        if (r < rows) {
                            const uint4 hd = *reinterpret_cast<const uint4 *>(W + (size_t)ct * 144);
                            const uint32_t m0 = hd.z & 0x3F3F3F3Fu;
                            const uint32_t m1 = ((hd.w >> 4) & 0x0F0F0F0Fu) | (((hd.z >> 6) & 0x03030303u) << 4);
                            H[mat * 128 + r] = make_uint4(__float_as_uint(f16_to_f32((uint16_t)(hd.x & 0xFFFF))),
                                                          __float_as_uint(f16_to_f32((uint16_t)(hd.x >> 16))), m0, m1);
                        }
                    } else if (ct < rows) {
                        H[ct].x = __float_as_uint(pf_d);
                    }
                    float *txd = reinterpret_cast<float *>(tok + (size_t)hs * Ly::TOK);
                    uint4 *tbs = reinterpret_cast<uint4 *>(txd + TC_N);
                    if (ct < tl.nc) {
                        txd[ct] = pf_xd;
                        if (FMT == 0) {
                            uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
                            for (int k4 = 0; k4 < 4; k4++) {  // per-32 sum bs = 256 hi + lo (lo unsigned, hi signed)
                                const int4 v = pf_s[k4];
                                const int b0 = v.x + v.y, b1 = v.z + v.w, k = 2 * k4;
                                lo[k >> 2] |= (uint32_t)(b0 & 0xFF) << (8 * (k & 3));
                                hi[k >> 2] |= (uint32_t)((b0 >> 8) & 0xFF) << (8 * (k & 3));
                                lo[(k + 1) >> 2] |= (uint32_t)(b1 & 0xFF) << (8 * ((k + 1) & 3));
                                hi[(k + 1) >> 2] |= (uint32_t)((b1 >> 8) & 0xFF) << (8 * ((k + 1) & 3));
                            }
                            tbs[ct] = make_uint4(lo[0], lo[1], hi[0], hi[1]);
                        }
                    }
                    if (blk + 1 < NB) {
                        TC_PF_LOAD(tl, blk + 1, slot_cur);
                    } else if (has_next) {
                        TC_PF_LOAD(tn, 0, slot_nxt);
                    }
                    __syncwarp();  // one arrival per converter warp (256 arrivals on one word serialise)
                    if (lane == 0) tc_arrive(&B.hdr_full[hs]);
                }
                if (ct == 0) tc_prof_add(B.prof, FMT, 16, clock64() - c_h);
                for (int q = 0; q < 4; q++, gq++) {
                    const long long c_q = clock64();
                    const int os = gq % TC_OS;
                    int ok2 = 1;
                    if (lane == 0)
                        ok2 = gq >= TC_OS ? tc_wait(B, &B.op_empty[os], ((gq / TC_OS) - 1) & 1, A.err, FMT, ct == 0 ? 3 : -1)
                                          : tc_ok(B);
                    if (!__shfl_sync(0xffffffffu, ok2, 0)) {
                        run = false;
                        break;
                    }
                    uint8_t *O = ops + (size_t)os * Ly::OP;
                    const long long c_a = clock64();
                    if (ct == 0) tc_prof_add(B.prof, FMT, 17, c_a - c_q);
                    if (FMT == 0) {  // thread = (matrix, row): two 16-byte reads of this quarter's 32 nibble bytes
                        const int mat = ct >> 7, r = ct & 127;
                        uint8_t *tA = O + (size_t)mat * Ly::OP_A;
                        if (r < rows) {
                            const uint8_t *wr = W + (size_t)ct * 144;
                            const uint4 hd = *reinterpret_cast<const uint4 *>(wr);
                            int sl, ml, sh, mh;
                            tc_scale_min(2 * q, hd.y, hd.z, hd.w, sl, ml);
                            tc_scale_min(2 * q + 1, hd.y, hd.z, hd.w, sh, mh);
                            const __half2 sl2 = __half2half2(__int2half_rn(sl)), offl = __half2half2(__int2half_rn(-1024 * sl));
                            const __half2 sh16 = __half2half2(__float2half_rn((float)sh * 0.0625f)),
                                          offh = __half2half2(__int2half_rn(-64 * sh));
#pragma unroll
                            for (int cc = 0; cc < 2; cc++) {
                                const uint4 v = *reinterpret_cast<const uint4 *>(wr + 16 + 32 * q + 16 * cc);
                                uint32_t a0, a1, b0, b1, c0, c1, d0, d1;
                                tc_q4_word(v.x, sl2, offl, sh16, offh, a0, a1, b0, b1);
                                tc_q4_word(v.y, sl2, offl, sh16, offh, c0, c1, d0, d1);
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, 2 * cc)) = make_uint4(a0, a1, c0, c1);
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, 4 + 2 * cc)) = make_uint4(b0, b1, d0, d1);
                                tc_q4_word(v.z, sl2, offl, sh16, offh, a0, a1, b0, b1);
                                tc_q4_word(v.w, sl2, offl, sh16, offh, c0, c1, d0, d1);
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, 2 * cc + 1)) = make_uint4(a0, a1, c0, c1);
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, 5 + 2 * cc)) = make_uint4(b0, b1, d0, d1);
                            }
                        } else {
#pragma unroll
                            for (int c = 0; c < 8; c++)
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, c)) = make_uint4(0, 0, 0, 0);
                        }
                    } else {  // thread = (row, 16-byte quarter j of the half's 64 ql bytes), two rows:
                              // 8 consecutive lanes read 2 rows x 4 chunks (row pitch 192 B): conflict-free
                        const int h = q >> 1, p = q & 1, j = ct & 3;
                        const int gp = j >> 1, hl = j & 1, gg = 2 * p + gp;  // values l = 16 hl .. 16 hl + 15 of group gg
                        uint8_t *tA = O;
                        const __half2 k1056 = tc_u2h(0x64206420u);  // 1024 + 32
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            const int r = (ct >> 2) + 64 * u;
                            const int c0 = 4 * gp + 2 * hl;  // output chunks c0, c0 + 1
                            if (r < rows) {
                                const uint8_t *wr = W + (size_t)r * 192;
                                const uint4 l4 = *reinterpret_cast<const uint4 *>(wr + 64 * h + 16 * j);
                                const uint4 h4 = *reinterpret_cast<const uint4 *>(wr + 128 + 32 * h + 16 * hl);
                                const int sc = (int)*reinterpret_cast<const int8_t *>(W + 128 * 192 + (size_t)r * 16 + 8 * h +
                                                                                      2 * gg + hl);
                                const __half2 sc2 = __half2half2(__int2half_rn(sc));
                                const uint32_t lw[4] = {l4.x, l4.y, l4.z, l4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
                                uint32_t o[8];
                                uint32_t o2[8];  // FMT 2: the lo tile (o holds hi)
#pragma unroll
                                for (int w = 0; w < 4; w++) {
                                    const uint32_t lo4 = (p ? lw[w] >> 4 : lw[w]) & 0x0F0F0F0Fu;
                                    const uint32_t qb = lo4 | (((hw[w] >> (2 * gg)) & 0x03030303u) << 4);
                                    if (FMT == 1) {
                                        o[2 * w] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(qb, 0x64646464u, 0x7170)), k1056), sc2));
                                        o[2 * w + 1] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(qb, 0x64646464u, 0x7372)), k1056), sc2));
                                    } else {
                                        const __half2 k1028 = tc_u2h(0x64046404u), k1024 = tc_u2h(0x64006400u);
                                        const uint32_t qh = (qb >> 3) & 0x07070707u, ql = qb & 0x07070707u;
                                        o[2 * w] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(qh, 0x64646464u, 0x7170)), k1028), sc2));
                                        o[2 * w + 1] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(qh, 0x64646464u, 0x7372)), k1028), sc2));
                                        o2[2 * w] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(ql, 0x64646464u, 0x7170)), k1024), sc2));
                                        o2[2 * w + 1] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(ql, 0x64646464u, 0x7372)), k1024), sc2));
                                    }
                                }
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, c0)) = make_uint4(o[0], o[1], o[2], o[3]);
                                *reinterpret_cast<uint4 *>(tA + tc_sw(r, c0 + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                                if (FMT == 2) {
                                    uint8_t *tL = tA + Ly::OP_A;
                                    *reinterpret_cast<uint4 *>(tL + tc_sw(r, c0)) = make_uint4(o2[0], o2[1], o2[2], o2[3]);
                                    *reinterpret_cast<uint4 *>(tL + tc_sw(r, c0 + 1)) = make_uint4(o2[4], o2[5], o2[6], o2[7]);
                                }
                            } else {
#pragma unroll
                                for (int m = 0; m < MATS; m++) {
                                    *reinterpret_cast<uint4 *>(tA + m * Ly::OP_A + tc_sw(r, c0)) = make_uint4(0, 0, 0, 0);
                                    *reinterpret_cast<uint4 *>(tA + m * Ly::OP_A + tc_sw(r, c0 + 1)) = make_uint4(0, 0, 0, 0);
                                }
                            }
                        }
                    }
                    const long long c_b = clock64();
                    {   // tokens: thread = (token i, chunk pair cp) -> chunks 2cp, 2cp + 1
                        uint8_t *tB = O + MATS * Ly::OP_A;
                        const int i = ct & 63, cp = ct >> 6;
                        if (i < N) {
                            uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
                            if (i < tl.nc) {
                                const uint4 v = *reinterpret_cast<const uint4 *>(X + (size_t)i * TC_XPITCH + 64 * q + 16 * cp);
                                o0 = tc_h8(v.x, v.y);
                                o1 = tc_h8(v.z, v.w);
                            }
                            *reinterpret_cast<uint4 *>(tB + tc_sw(i, 2 * cp)) = o0;
                            *reinterpret_cast<uint4 *>(tB + tc_sw(i, 2 * cp + 1)) = o1;
                        }
                    }
                    fence_async_smem();  // this thread's operand stores -> the tensor core's proxy
                    __syncwarp();
                    if (lane == 0) tc_arrive(&B.op_full[os]);
                    if (ct == 0) {
                        const long long c_e = clock64();
                        tc_prof_add(B.prof, FMT, 14, c_b - c_a);
                        tc_prof_add(B.prof, FMT, 15, c_e - c_b);
                        tc_prof_add(B.prof, FMT, 18, clock64() - c_e);
                    }
                }
                if (run) {
                    __syncwarp();
                    if (lane == 0) tc_arrive(&B.raw_empty[s]);
                }
            }
            if (!run) break;
            slot_cur = slot_nxt;
        }
    } else if (warp == TC_MMA_WARP) {
        // ---- MMA issuer ----------------------------------------------------------------------
        if (lane == 0) {
            uint32_t gb = 0, gq = 0;
            TcTile tl;
            for (int ti = blockIdx.x; tc_ok(B) && tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) {
                const int N = (tl.nc + 15) & ~15;
                const uint32_t idesc = tc_idesc(128, N);
                bool run = true;
                for (int blk = 0; blk < NB && run; blk++, gb++) {
                    const int b = gb & 1;
                    if (gb >= 2 && !tc_wait(B, &B.acc_empty[b], ((gb >> 1) - 1) & 1, A.err, FMT, 4)) {
                        run = false;
                        break;
                    }
                    for (int q = 0; q < 4; q++, gq++) {
                        const int os = gq % TC_OS;
                        if (!tc_wait(B, &B.op_full[os], (gq / TC_OS) & 1, A.err, FMT, 5)) {
                            run = false;
                            break;
                        }
                        tc_fence_after();
                        const uint8_t *O = ops + (size_t)os * Ly::OP;
                        const uint64_t bd = tc_desc_sw128(O + MATS * Ly::OP_A);
#pragma unroll
                        for (int mat = 0; mat < MATS; mat++) {
                            const uint64_t ad = tc_desc_sw128(O + mat * Ly::OP_A);
                            const uint32_t dcol = (uint32_t)b * (MATS * 2 * TC_N) + (uint32_t)(mat * 2 + (q >> 1)) * TC_N;
#pragma unroll
                            for (int k = 0; k < 4; k++)
                                umma_bf16(tmem + dcol, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                                          (q & 1) || k > 0);
                        }
                        umma_commit(&B.op_empty[os]);
                        if (q == 3) umma_commit(&B.acc_full[b]);
                    }
                }
                if (!run) break;
            }
            // drain: every MMA issued must complete before TMEM and shared memory are released
            umma_commit(&B.drain);
            mbar_wait(&B.drain, 0, TC_POLLS);
        }
        __syncwarp();
    } else if (warp < TC_EPI_WARPS) {
        // ---- epilogue (warps 0-7) ------------------------------------------------------------
        const int qq = warp & 3, th = warp >> 2, r = 32 * qq + lane;
        uint32_t gb = 0;
        TcTile tl;
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) {
            const int row0 = tl.rt * 128, rows = R - row0 < 128 ? R - row0 : 128;
            // lane l: the slot of this warp's l-th token, for the stores at the end of the tile
            const int my_ti = 8 * (2 * (lane >> 3) + th) + (lane & 7);
            const int my_slot = my_ti < tl.nc ? tc_slot(A, TT, tl, my_ti) : 0;
            float acc[MATS][32];
#pragma unroll
            for (int m = 0; m < MATS; m++)
#pragma unroll
                for (int i = 0; i < 32; i++) acc[m][i] = 0.0f;
            bool run = true;
            for (int blk = 0; blk < NB; blk++, gb++) {
                const int b = gb & 1, hs = gb % TC_HS;
                int ok = 1;  // each epilogue warp waits on its own
                if (lane == 0) {
                    ok = tc_wait(B, &B.acc_full[b], (gb >> 1) & 1, A.err, FMT, tid == 0 ? 6 : -1);
                    if (ok) ok = tc_wait(B, &B.hdr_full[hs], (gb / TC_HS) & 1, A.err, FMT, tid == 0 ? 7 : -1);
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    run = false;
                    break;
                }
                tc_fence_after();
                const uint4 *H = reinterpret_cast<const uint4 *>(hdr + (size_t)hs * Ly::HDR);
                const float *txd = reinterpret_cast<const float *>(tok + (size_t)hs * Ly::TOK);
                const uint4 *tbs = reinterpret_cast<const uint4 *>(txd + TC_N);
                uint4 hr[MATS];
#pragma unroll
                for (int m = 0; m < MATS; m++) hr[m] = H[m * 128 + r];
#pragma unroll
                for (int j = 0; j < 4; j++) {  // token groups of 8, alternating between the two warp halves
                    const int t0 = 8 * (2 * j + th);
                    if (t0 >= tl.nc) break;  // warp-uniform
                    if (FMT == 2) {  // one output: I = 8 I_hi + I_lo, every part an exact integer
                        float h0[8], h1[8], l0[8], l1[8];
                        const uint32_t col = (uint32_t)b * (MATS * 2 * TC_N) + (uint32_t)t0;
                        tmem_f8(tmem, qq, col, h0);
                        tmem_f8(tmem, qq, col + TC_N, h1);
                        tmem_f8(tmem, qq, col + 2 * TC_N, l0);
                        tmem_f8(tmem, qq, col + 3 * TC_N, l1);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const int ti2 = t0 + i;
                            if (ti2 < tl.nc) {
                                const int I = 8 * (__float2int_rn(h0[i]) + __float2int_rn(h1[i])) + __float2int_rn(l0[i]) +
                                              __float2int_rn(l1[i]);
                                acc[0][8 * j + i] = fadd(acc[0][8 * j + i],
                                                         fmul(fmul(txd[ti2], __uint_as_float(hr[0].x)), __int2float_rn(I)));
                            }
                        }
                        continue;
                    }
#pragma unroll
                    for (int m = 0; m < MATS; m++) {
                        float v0[8], v1[8];
                        const uint32_t col = (uint32_t)b * (MATS * 2 * TC_N) + (uint32_t)(m * 2) * TC_N + (uint32_t)t0;
                        tmem_f8(tmem, qq, col, v0);
                        tmem_f8(tmem, qq, col + TC_N, v1);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const int ti2 = t0 + i;
                            if (ti2 < tl.nc) {
                                // the halves hold exact integers: their f32 sum rounds like (float) of the integer sum
                                const float fI = fadd(v0[i], v1[i]);
                                const float xd = txd[ti2];
                                if (FMT == 0) {
                                    // mins term M = sum_sub mn * bs through dp4a on bs = 256 hi + lo (exact)
                                    const uint4 bp = tbs[ti2];
                                    const int M = (int)__dp4a(hr[m].z, bp.x, __dp4a(hr[m].w, bp.y, 0u)) +
                                                  256 * dp4a_us(hr[m].z, (int)bp.z, dp4a_us(hr[m].w, (int)bp.w, 0));
                                    const float d = __uint_as_float(hr[m].x), dmin = __uint_as_float(hr[m].y);
                                    acc[m][8 * j + i] =
                                        fadd(acc[m][8 * j + i], fmul(xd, fsub(fmul(d, fI), fmul(dmin, (float)M))));
                                } else {
                                    acc[m][8 * j + i] = fadd(acc[m][8 * j + i], fmul(fmul(xd, __uint_as_float(hr[m].x)), fI));
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    tc_arrive(&B.acc_empty[b]);
                    tc_arrive(&B.hdr_empty[hs]);
                }
            }
            if (!run) break;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const int ti2 = 8 * (2 * (i >> 3) + th) + (i & 7);
                if (ti2 >= tl.nc) break;  // warp-uniform
                const int slot = __shfl_sync(0xffffffffu, my_slot, i);
                if (r < rows) {
                    if (FMT == 0) {
                        const float g = acc[0][i], u = acc[MATS - 1][i];
                        A.act[(size_t)slot * stride + row0 + r] = fmul(fdiv(g, fadd(1.0f, exp_f(-g))), u);
                    } else {
                        A.y[(size_t)slot * dim + row0 + r] = acc[0][i];
                    }
                }
            }
        }
    }
    {   // role spans: producer 8, converters 9, MMA 10, epilogue 11; whole CTA 12; tiles 13
        const long long span = clock64() - t_start;
        if (tid == TC_PRO_WARP * 32) tc_prof_add(B.prof, FMT, 8, span);
        if (tid == TC_CVT_WARP0 * 32) tc_prof_add(B.prof, FMT, 9, span);
        if (tid == TC_MMA_WARP * 32) tc_prof_add(B.prof, FMT, 10, span);
        if (tid == 0) tc_prof_add(B.prof, FMT, 11, span);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
        tc_prof_add(B.prof, FMT, 12, clock64() - t_start);
        int nt = 0;
        TcTile tl;
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) nt++;
        tc_prof_add(B.prof, FMT, 13, nt);
    }
    if (warp == 0) tmem_free(tmem, Ly::TMEM_COLS);
}

// ==== down projection on dequantized fp16 tiles (the default) ============================
// The north star's form of the batched expert FFN, for the down projection:
// the Q6_K weights dequantized to fp16 values (d sc)(q - 32) (the f32 product
// of dequantBlockQ6K, ggml.zig:1420, rounded once), the activations the
// reference's int8 quantization of quantizeX256 (ggml.zig:776) dequantized to
// fp16 (xd * q), one f32 TMEM accumulator per (row, token) over the whole row,
// and no per-block epilogue: the epilogue runs once per tile. The result stays
// within ~3e-4 relative L2 of the reference's integer arithmetic (fp16 keeps
// 11 significant bits of every operand; the int8 activations are reproduced
// exactly before the rounding). Gate/up keep the integer-exact kernel: their
// output is re-quantized to int8 for down, where operand rounding would move
// int8 roundings. loom_cuda_tc_exact(1) runs down integer-exact too.
//
// Same tiles, producer and bounded waits as k_moe_tc, with more converter
// warps (the conversion is the kernel's critical path) and a deeper operand
// ring:
//   warps 0-3    epilogue: TMEM lane quarter = warp, every token of the tile
//   warp 4       producer
//   warp 5       MMA issuer (one accumulator per tile, two tile buffers)
//   warps 6-21   converters: thread = (row, 16-value quarter) of the weight
//                tile, (token, 8-value chunk) of the activation tile
// Operand values are limited to the fp16 range (|x| < 65504).
constexpr int TCF_EPI_WARPS = 4, TCF_PRO_WARP = 4, TCF_MMA_WARP = 5, TCF_CVT_WARP0 = 6, TCF_CVT_WARPS = 16;
constexpr int TCF_THREADS = (TCF_CVT_WARP0 + TCF_CVT_WARPS) * 32;
constexpr int TCF_OS = 4;
constexpr uint32_t TCF_POLLS = 1u << 20;  // suspending polls of up to 4 us each
constexpr int TCF_ACC = 4;  // accumulators per tile (one per K step of a sub-stage), summed by the epilogue
struct TcfLayout {
    static constexpr size_t RAW_W = (size_t)128 * 208, RAW_X = (size_t)TC_N * TC_XPITCH;
    static constexpr size_t RAW = RAW_W + RAW_X;
    static constexpr size_t OP_A = (size_t)8 * 128 * 16, OP = OP_A + (size_t)8 * TC_N * 16;
    static constexpr size_t SMEM = TC_RS * RAW + TCF_OS * OP;
    static constexpr uint32_t TMEM_COLS = 2 * TCF_ACC * TC_N;  // 2 tile buffers x TCF_ACC x TC_N
};
struct TcfBars {
    uint64_t raw_full[TC_RS], raw_empty[TC_RS], op_full[TCF_OS], op_empty[TCF_OS];
    uint64_t acc_full[2], acc_empty[2], drain;
    uint32_t tmem;
    int err;
    int prof;
};

__device__ __forceinline__ uint32_t tcf_h2(float a) {  // f32 -> fp16 pair (a, a)
    const __half h = __float2half_rn(a);
    return tc_h2u(__halves2half2(h, h));
}

// bounded wait by one thread; a timeout raises the CTA's error flag (as tc_wait)
__device__ __forceinline__ bool tcf_wait(TcfBars &B, uint64_t *bar, uint32_t parity, int *gerr, int slot = -1) {
    if (*reinterpret_cast<volatile int *>(&B.err)) return false;
    const long long c0 = B.prof ? clock64() : 0;
    const bool ok = mbar_wait_hint(bar, parity, TCF_POLLS, 4000);
    if (slot >= 0) tc_prof_add(B.prof, 1, slot, clock64() - c0);
    if (ok) return true;
    *reinterpret_cast<volatile int *>(&B.err) = 1;
    if (gerr) atomicOr(gerr, 64);
    return false;
}

// Power-of-two exponent E of a down-projection token: its largest block scale
// xd times 127 lies in [2^(E-1), 2^E), so its operand values xd q 2^-E lie
// below 1 in magnitude (far inside fp16's range); the epilogue multiplies by
// 2^E, which is exact.
template <int NB>
__device__ __forceinline__ int tcf_exp_of(const float (&xd)[NB]) {
    float m = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; b++) m = fmaxf(m, fabsf(xd[b]));
    int e = 0;
    if (m > 0.0f && m < 1e30f) frexpf(m * 127.0f, &e);
    return max(-100, min(100, e));
}
template <int NB>
__device__ __forceinline__ int tcf_tok_exp(const DecodeArgs &A, int slot) {
    float xd[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) xd[b] = A.ad[(size_t)slot * (A.act_stride / 32) + b];
    return tcf_exp_of<NB>(xd);
}
__device__ __forceinline__ float tcf_pow2(int e) { return __int_as_float((127 + e) << 23); }

template <int NB>
__global__ void __launch_bounds__(TCF_THREADS, 1) k_moe_tcf(DecodeArgs A, const __grid_constant__ TcMaps M) {
    using Ly = TcfLayout;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ TcfBars B;
    uint8_t *raw = sm, *ops = sm + TC_RS * Ly::RAW;
    const TileTab TT = tc_tab_load(A, reinterpret_cast<int *>(sm + Ly::SMEM));
    const int R = A.dim;  // weight rows
    const int RT = (R + 127) / 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    {
        TcTile t0;
        if (!tc_tile(A, RT, blockIdx.x, t0)) return;  // no work for this CTA
    }
    if (warp == 0) tmem_alloc(&B.tmem, Ly::TMEM_COLS);
    if (tid == 0) {
        for (int i = 0; i < TC_RS; i++) {
            mbar_init(&B.raw_full[i], 1);
            mbar_init(&B.raw_empty[i], TCF_CVT_WARPS);
        }
        for (int i = 0; i < TCF_OS; i++) {
            mbar_init(&B.op_full[i], TCF_CVT_WARPS);
            mbar_init(&B.op_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&B.acc_full[i], 1);
            mbar_init(&B.acc_empty[i], TCF_EPI_WARPS);
        }
        mbar_init(&B.drain, 1);
        B.err = 0;
        B.prof = g_tc_prof_on && blockIdx.x == 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem;
    const int dim = A.dim, stride = A.act_stride;
    const long long t_start = clock64();

    if (warp == TCF_PRO_WARP) {
        // ---- producer (as k_moe_tc) ------------------------------------------------------------
        uint32_t gb = 0;
        TcTile tl;
        bool run = true;
        for (int ti = blockIdx.x; run && tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) {
            const int row0 = tl.rt * 128;
            const int8_t *src[2] = {nullptr, nullptr};
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int i = lane + 32 * u;
                if (i < tl.nc) src[u] = A.aq + (size_t)tc_slot(A, TT, tl, i) * stride;
            }
            for (int blk = 0; blk < NB; blk++, gb++) {
                const int s = gb % TC_RS;
                int ok = 1;
                if (lane == 0) ok = gb >= TC_RS ? tcf_wait(B, &B.raw_empty[s], ((gb / TC_RS) - 1) & 1, A.err, 0) : 1;
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    run = false;
                    break;
                }
                uint8_t *W = raw + (size_t)s * Ly::RAW, *X = W + Ly::RAW_W;
                if (lane == 0) {
                    mbar_expect_tx(&B.raw_full[s], (uint32_t)Ly::RAW_W + (uint32_t)tl.nc * 256);
                    const int y = (tl.shared ? 0 : tl.e * R) + row0, m0 = tl.shared ? 2 : 0;
                    tma_load_2d(W, &M.m[m0], blk * 192, y, &B.raw_full[s]);
                    tma_load_2d(W + 128 * 192, &M.m[m0 + 1], blk * 16, y, &B.raw_full[s]);
                }
                __syncwarp();
#pragma unroll
                for (int u = 0; u < 2; u++)
                    if (src[u]) bulk_g2s(X + (size_t)(lane + 32 * u) * TC_XPITCH, src[u] + blk * 256, 256, &B.raw_full[s]);
            }
        }
        if (lane == 0 && !run)
            for (uint32_t g = gb > TC_RS ? gb - TC_RS : 0; g < gb; g++)
                mbar_wait(&B.raw_full[g % TC_RS], (g / TC_RS) & 1, TC_POLLS);
    } else if (warp >= TCF_CVT_WARP0) {
        // ---- converters: raw stage -> dequantized fp16 operand tiles ---------------------------
        const int ct = tid - TCF_CVT_WARP0 * 32;
        const int r = ct >> 2, j = ct & 3;          // weight row, 16-value quarter of the 64-value sub-stage
        const int ti_tok = ct & 63, ch = ct >> 6;   // activation token, 8-value chunk
        const int gp = j >> 1, hl = j & 1, c0 = 4 * gp + 2 * hl;
        uint32_t gb = 0, gq = 0;
        // read a block ahead: the converted token's scale xd and the row's f16 d
        float pf_xd = 0.0f, pf_d = 0.0f;
        int slot_cur = 0, slot_nxt = 0;  // the slot of token ti_tok in this / the next tile
        float inv_cur = 1.0f;            // 2^-E of that token (tcf_tok_exp)
        float nxd[NB];                   // the next tile's token: its block scales, loaded a tile ahead
#pragma unroll
        for (int b = 0; b < NB; b++) nxd[b] = 0.0f;
        auto pf = [&](const TcTile &t, int blk, int slot) {
            if (ti_tok < t.nc) pf_xd = A.ad[(size_t)slot * (stride / 32) + blk];
            const WDev &w = t.shared ? A.sdn : A.dn;
            const uint64_t pl = t.shared ? 0 : (uint64_t)t.e * R * NB;
            const int rr = t.rt * 128 + r;
            pf_d = rr < R ? f16_to_f32(w.d[pl + (uint64_t)rr * NB + blk]) : 0.0f;
        };
        TcTile tl, tn;
        if (tc_tile(A, TT, RT, blockIdx.x, tl)) {
            if (ti_tok < tl.nc) {
                slot_cur = tc_slot(A, TT, tl, ti_tok);
                inv_cur = tcf_pow2(-tcf_tok_exp<NB>(A, slot_cur));
            }
            pf(tl, 0, slot_cur);
        }
        const __half2 k1056 = tc_u2h(0x64206420u);  // 1024 + 32
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) {
            const bool has_next = tc_tile(A, TT, RT, ti + gridDim.x, tn);
            if (has_next && ti_tok < tn.nc) {
                slot_nxt = tc_slot(A, TT, tn, ti_tok);
#pragma unroll
                for (int b = 0; b < NB; b++) nxd[b] = A.ad[(size_t)slot_nxt * (stride / 32) + b];
            }
            const int row0 = tl.rt * 128, rows = R - row0 < 128 ? R - row0 : 128;
            const int N = (tl.nc + 15) & ~15;
            bool run = true;
            for (int blk = 0; blk < NB && run; blk++, gb++) {
                const int s = gb % TC_RS;
                int ok = 1;
                if (lane == 0) ok = tcf_wait(B, &B.raw_full[s], (gb / TC_RS) & 1, A.err, ct == 0 ? 1 : -1);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    run = false;
                    break;
                }
                const uint8_t *W = raw + (size_t)s * Ly::RAW, *X = W + Ly::RAW_W;
                const float xd = pf_xd, dr = pf_d;
                if (blk + 1 < NB) pf(tl, blk + 1, slot_cur);
                else if (has_next) pf(tn, 0, slot_nxt);
                const __half2 xd2 = tc_u2h(tcf_h2(fmul(xd, inv_cur)));
                const uint8_t *wr = W + (size_t)r * 192;
                const int8_t *scr = reinterpret_cast<const int8_t *>(W + 128 * 192 + (size_t)r * 16);
                for (int q = 0; q < 4; q++, gq++) {
                    const long long c_0 = clock64();
                    const int os = gq % TCF_OS;
                    const int h = q >> 1, p = q & 1, gg = 2 * p + gp;
                    int ok2 = 1;
                    if (lane == 0) ok2 = gq >= TCF_OS ? tcf_wait(B, &B.op_empty[os], ((gq / TCF_OS) - 1) & 1, A.err, ct == 0 ? 3 : -1) : 1;
                    if (!__shfl_sync(0xffffffffu, ok2, 0)) {
                        run = false;
                        break;
                    }
                    uint4 l4 = make_uint4(0, 0, 0, 0), h4 = l4;
                    int sc = 0;
                    if (r < rows) {
                        l4 = *reinterpret_cast<const uint4 *>(wr + 64 * h + 16 * j);
                        h4 = *reinterpret_cast<const uint4 *>(wr + 128 + 32 * h + 16 * hl);
                        sc = scr[8 * h + 2 * gg + hl];
                    }
                    uint2 xv = make_uint2(0, 0);
                    if (ti_tok < tl.nc) xv = *reinterpret_cast<const uint2 *>(X + (size_t)ti_tok * TC_XPITCH + 64 * q + 8 * ch);
                    uint8_t *O = ops + (size_t)os * Ly::OP;
                    const long long c_1 = clock64();
                    {   // weights: (d sc)(q - 32), the f32 product of dequantBlockQ6K rounded to fp16
                        const __half2 S = tc_u2h(tcf_h2(fmul(dr, (float)sc)));
                        const uint32_t lw[4] = {l4.x, l4.y, l4.z, l4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
                        uint32_t o[8];
#pragma unroll
                        for (int w = 0; w < 4; w++) {
                            const uint32_t lo4 = (p ? lw[w] >> 4 : lw[w]) & 0x0F0F0F0Fu;
                            const uint32_t qb = lo4 | (((hw[w] >> (2 * gg)) & 0x03030303u) << 4);
                            o[2 * w] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(qb, 0x64646464u, 0x7170)), k1056), S));
                            o[2 * w + 1] = tc_h2u(__hmul2(__hsub2(tc_u2h(__byte_perm(qb, 0x64646464u, 0x7372)), k1056), S));
                        }
                        *reinterpret_cast<uint4 *>(O + tc_sw(r, c0)) = make_uint4(o[0], o[1], o[2], o[3]);
                        *reinterpret_cast<uint4 *>(O + tc_sw(r, c0 + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                    }
                    const long long c_2 = clock64();
                    if (ti_tok < N) {  // activations: xd * q of the int8 values, in fp16
                        uint4 o = tc_h8(xv.x, xv.y);
                        o = make_uint4(tc_h2u(__hmul2(tc_u2h(o.x), xd2)), tc_h2u(__hmul2(tc_u2h(o.y), xd2)),
                                       tc_h2u(__hmul2(tc_u2h(o.z), xd2)), tc_h2u(__hmul2(tc_u2h(o.w), xd2)));
                        *reinterpret_cast<uint4 *>(O + Ly::OP_A + tc_sw(ti_tok, ch)) = o;  // zero past nc
                    }
                    const long long c_3 = clock64();
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) tc_arrive(&B.op_full[os]);
                    if (ct == 0) {
                        tc_prof_add(B.prof, 1, 17, c_1 - c_0);
                        tc_prof_add(B.prof, 1, 14, c_2 - c_1);
                        tc_prof_add(B.prof, 1, 15, c_3 - c_2);
                        tc_prof_add(B.prof, 1, 18, clock64() - c_3);
                    }
                }
                if (run) {
                    __syncwarp();
                    if (lane == 0) tc_arrive(&B.raw_empty[s]);
                }
            }
            if (!run) break;
            slot_cur = slot_nxt;
            inv_cur = tcf_pow2(-tcf_exp_of<NB>(nxd));
        }
    } else if (warp == TCF_MMA_WARP) {
        // ---- MMA issuer: one accumulator over the whole row, two tile buffers -------------------
        if (lane == 0) {
            uint32_t gt = 0, gq = 0;
            TcTile tl;
            bool run = true;
            for (int ti = blockIdx.x; run && tc_tile(A, TT, RT, ti, tl); ti += gridDim.x, gt++) {
                const int N = (tl.nc + 15) & ~15;
                const uint32_t idesc = tc_idesc(128, N);
                const int b = gt & 1;
                if (gt >= 2 && !tcf_wait(B, &B.acc_empty[b], ((gt >> 1) - 1) & 1, A.err, 4)) break;
                for (int blk = 0; blk < NB && run; blk++) {
                    for (int q = 0; q < 4; q++, gq++) {
                        const int os = gq % TCF_OS;
                        if (!tcf_wait(B, &B.op_full[os], (gq / TCF_OS) & 1, A.err, 5)) {
                            run = false;
                            break;
                        }
                        tc_fence_after();
                        const uint8_t *O = ops + (size_t)os * Ly::OP;
                        const uint64_t ad = tc_desc_sw128(O), bd = tc_desc_sw128(O + Ly::OP_A);
#pragma unroll
                        for (int k = 0; k < 4; k++)  // four independent accumulators: no MMA waits on the previous
                            umma_bf16(tmem + (uint32_t)(b * TCF_ACC + k) * TC_N, ad + (uint64_t)(2 * k),
                                      bd + (uint64_t)(2 * k), idesc, (blk | q) != 0);
                        umma_commit(&B.op_empty[os]);
                    }
                }
                if (run) umma_commit(&B.acc_full[b]);
            }
            umma_commit(&B.drain);
            mbar_wait(&B.drain, 0, TC_POLLS);
        }
        __syncwarp();
    } else {
        // ---- epilogue (warps 0-3): once per tile, every token -----------------------------------
        const int r = 32 * warp + lane;
        uint32_t gt = 0;
        TcTile tl;
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl); ti += gridDim.x, gt++) {
            const int row0 = tl.rt * 128, rows = R - row0 < 128 ? R - row0 : 128;
            const int slot_a = lane < tl.nc ? tc_slot(A, TT, tl, lane) : 0;        // token lane
            const int slot_b = lane + 32 < tl.nc ? tc_slot(A, TT, tl, lane + 32) : 0;  // token lane + 32
            const float sc_a = lane < tl.nc ? tcf_pow2(tcf_tok_exp<NB>(A, slot_a)) : 1.0f;
            const float sc_b = lane + 32 < tl.nc ? tcf_pow2(tcf_tok_exp<NB>(A, slot_b)) : 1.0f;
            const int b = gt & 1;
            int ok = 1;
            if (lane == 0) ok = tcf_wait(B, &B.acc_full[b], (gt >> 1) & 1, A.err, tid == 0 ? 6 : -1);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();
            for (int t0 = 0; t0 < tl.nc; t0 += 8) {  // warp-uniform
                float v[8], w[8];
                tmem_f8(tmem, warp, (uint32_t)(b * TCF_ACC) * TC_N + (uint32_t)t0, v);
#pragma unroll
                for (int c = 1; c < TCF_ACC; c++) {
                    tmem_f8(tmem, warp, (uint32_t)(b * TCF_ACC + c) * TC_N + (uint32_t)t0, w);
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = fadd(v[i], w[i]);
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int t = t0 + i;
                    const int slot = __shfl_sync(0xffffffffu, t < 32 ? slot_a : slot_b, t & 31);
                    const float sc = __shfl_sync(0xffffffffu, t < 32 ? sc_a : sc_b, t & 31);
                    if (t < tl.nc && r < rows) A.y[(size_t)slot * dim + row0 + r] = fmul(v[i], sc);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tc_arrive(&B.acc_empty[b]);
        }
    }
    {   // role spans: producer 8, converters 9, MMA 10, epilogue 11; whole CTA 12; tiles 13
        const long long span = clock64() - t_start;
        if (tid == TCF_PRO_WARP * 32) tc_prof_add(B.prof, 1, 8, span);
        if (tid == TCF_CVT_WARP0 * 32) tc_prof_add(B.prof, 1, 9, span);
        if (tid == TCF_MMA_WARP * 32) tc_prof_add(B.prof, 1, 10, span);
        if (tid == 0) tc_prof_add(B.prof, 1, 11, span);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
        tc_prof_add(B.prof, 1, 12, clock64() - t_start);
        int nt = 0;
        TcTile tl;
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl); ti += gridDim.x) nt++;
        tc_prof_add(B.prof, 1, 13, nt);
    }
    if (warp == 0) tmem_free(tmem, Ly::TMEM_COLS);
}

using TcFn = void (*)(DecodeArgs, TcMaps);

typedef CUresult (*TcEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                               const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static TcEncodeFn tc_encoder() {
    static TcEncodeFn f = nullptr;
    if (!f) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f = reinterpret_cast<TcEncodeFn>(p);
    }
    return f;
}

// rows x row_bytes bytes, box of 128 rows x box_bytes (false without an encoder or a base)
static bool tc_map(CUtensorMap &m, const void *base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes) {
    TcEncodeFn enc = tc_encoder();
    if (!enc || !base || rows == 0) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_bytes, 128};
    const cuuint32_t es[2] = {1, 1};
    return enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static TcFn tc_gu_fn(int nb) {
    switch (nb) {
        case 4: return k_moe_tc<0, 4>;
        case 8: return k_moe_tc<0, 8>;
        case 16: return k_moe_tc<0, 16>;
        case 28: return k_moe_tc<0, 28>;
    }
    return nullptr;
}
static TcFn tcf_dn_fn(int nb) {
    switch (nb) {
        case 2: return k_moe_tcf<2>;
        case 3: return k_moe_tcf<3>;
        case 4: return k_moe_tcf<4>;
        case 8: return k_moe_tcf<8>;
    }
    return nullptr;
}
static TcFn tc_dn_fn(int nb, bool split) {
    switch (nb) {
        case 2: return split ? k_moe_tc<2, 2> : k_moe_tc<1, 2>;
        case 3: return split ? k_moe_tc<2, 3> : k_moe_tc<1, 3>;
        case 4: return split ? k_moe_tc<2, 4> : k_moe_tc<1, 4>;
        case 8: return split ? k_moe_tc<2, 8> : k_moe_tc<1, 8>;
    }
    return nullptr;
}
// Small Q6_K scales (every |sc| <= 32) take the one-tile fold; others the split.
static bool tc_dn_split(const DecodeArgs &A) {
    return !(A.dn.pad_ & WDEV_Q6K_SMALL_SCALES) || (A.has_shared && !(A.sdn.pad_ & WDEV_Q6K_SMALL_SCALES));
}

// 1: the bit-exact integer kernels (k_moe_tc); 0: the dequantized fp16 kernels (k_moe_tcf)
int g_tc_exact = 0;

bool moe_mma_supported(const DecodeArgs &A) {
    if (A.g.type != T_Q4_K || A.u.type != T_Q4_K || A.dn.type != T_Q6_K) return false;
    if (A.dim % 256 || A.ffn % 256 || A.n_local + 1 > 1024) return false;
    if (!tc_gu_fn(A.dim / 256) || !tc_dn_fn(A.ffn / 256, false)) return false;
    if (!tc_encoder()) return false;
    if (A.has_shared && (A.sg.type != T_Q4_K || A.su.type != T_Q4_K || A.sdn.type != T_Q6_K || A.shexp_ffn != A.ffn))
        return false;
    return true;
}

// gate/up on the tensor cores, the activations' quantization, down on the
// tensor cores: after the grouping kernel (which wrote A.tc_pre), before the
// combine. One CTA per SM; CTAs without a tile return at once.
cudaError_t launch_moe_mma(const DecodeArgs &A, cudaStream_t st, cudaError_t (*quant)(const DecodeArgs &, cudaStream_t)) {
    static int n_sm = 0;
    if (!n_sm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (n_sm <= 0) n_sm = 148;
    }
    // gate/up stay integer-exact in every mode: their output is re-quantized to int8 for down, and
    // fp16 operand rounding there moves int8 roundings (one moved step is ~1e-3 of the layer output)
    const bool split = tc_dn_split(A), exact = g_tc_exact != 0;
    TcFn gf = tc_gu_fn(A.dim / 256);
    TcFn df = exact ? tc_dn_fn(A.ffn / 256, split) : tcf_dn_fn(A.ffn / 256);
    const int nbg = A.dim / 256, nbd = A.ffn / 256;
    TcMaps mg, md;
    memset(&mg, 0, sizeof mg);
    memset(&md, 0, sizeof md);
    const uint64_t gr = (uint64_t)A.n_local * A.ffn, dr = (uint64_t)A.n_local * A.dim;
    bool ok = tc_map(mg.m[0], A.g.q, nbg * 144ull, gr, 144) && tc_map(mg.m[1], A.u.q, nbg * 144ull, gr, 144) &&
              tc_map(md.m[0], A.dn.q, nbd * 192ull, dr, 192) && tc_map(md.m[1], A.dn.sc, nbd * 16ull, dr, 16);
    if (ok && A.has_shared)
        ok = tc_map(mg.m[2], A.sg.q, nbg * 144ull, (uint64_t)A.shexp_ffn, 144) &&
             tc_map(mg.m[3], A.su.q, nbg * 144ull, (uint64_t)A.shexp_ffn, 144) &&
             tc_map(md.m[2], A.sdn.q, nbd * 192ull, (uint64_t)A.dim, 192) &&
             tc_map(md.m[3], A.sdn.sc, nbd * 16ull, (uint64_t)A.dim, 16);
    if (!ok) return cudaErrorInvalidValue;
    const size_t gs = TcLayout<0>::SMEM + tc_tab_bytes(A.n_local);
    const size_t ds = (!exact ? TcfLayout::SMEM : split ? TcLayout<2>::SMEM : TcLayout<1>::SMEM) + tc_tab_bytes(A.n_local);
    cudaError_t e = cudaFuncSetAttribute(gf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gs);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(df, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ds);
    if (e != cudaSuccess) return e;
    count_launch();
    gf<<<n_sm, TC_THREADS, gs, st>>>(A, mg);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = quant(A, st)) != cudaSuccess) return e;
    count_launch();
    df<<<n_sm, exact ? TC_THREADS : TCF_THREADS, ds, st>>>(A, md);
    return cudaGetLastError();
}

// ---- Q6_K scale range of a tensor ---------------------------------------------------------
__global__ void k_q6k_scale_max(const int8_t *sc, uint64_t n, int *out) {
    int m = 0;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const int v = sc[i];
        m = max(m, v < 0 ? -v : v);
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

int q6k_max_scale(const uint8_t *sc, uint64_t nblk, int *d_tmp, cudaStream_t st) {
    if (cudaMemsetAsync(d_tmp, 0, 4, st) != cudaSuccess) return -1;
    const uint64_t n = nblk * 16;
    const unsigned grid = (unsigned)std::min<uint64_t>(1024, (n + 255) / 256 + 1);
    k_q6k_scale_max<<<grid, 256, 0, st>>>(reinterpret_cast<const int8_t *>(sc), n, d_tmp);
    count_launch();
    int h = -1;
    if (cudaMemcpyAsync(&h, d_tmp, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    return h;
}

}  // namespace loom

using namespace loom;

extern "C" int loom_cuda_tc_profile(int enable, unsigned long long *out, size_t n);
extern "C" int loom_cuda_tc_exact(int on);

int loom_cuda_tc_exact(int on) {
    const int prev = g_tc_exact;
    g_tc_exact = on ? 1 : 0;
    return prev;
}

// Diagnostic entry (no counterpart in the reference): enable (1) / disable (0)
// the tensor-core kernels' cycle profile of CTA 0, zeroing it; then (any
// enable value < 0) copy min(n, 32) counters (gate/up then down, 16 each).
int loom_cuda_tc_profile(int enable, unsigned long long *out, size_t n) {
    if (enable >= 0) {
        static const unsigned long long zero[2][TC_PROF_SLOTS] = {};
        if (cudaMemcpyToSymbol(g_tc_prof, zero, sizeof zero) != cudaSuccess) return 2;
        if (cudaMemcpyToSymbol(g_tc_prof_on, &enable, sizeof enable) != cudaSuccess) return 2;
        return 0;
    }
    unsigned long long h[2][TC_PROF_SLOTS];
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyFromSymbol(h, g_tc_prof, sizeof h) != cudaSuccess) return 2;
    memcpy(out, h, std::min(n, (size_t)(2 * TC_PROF_SLOTS)) * 8);
    return 0;
}

namespace loom {

// ==== expert FFN of small batches with dp4a (a few tokens per expert) ======================
// The same tiles and staging as the tensor-core kernels (TMA 2D weight boxes
// of 128 rows per super-block, bulk copies of the tile's token rows, a
// 2-stage ring), but the dots run on the integer pipes: each compute thread
// owns one weight row, unpacks each super-block once into int8 words and
// dots it with every token of the tile by dp4a, exactly the reference's
// integer arithmetic (ggml.zig kBlockDot :1002; Q4_K I = sum_j sc_j (q . x)_j
// and M = sum_j mn_j bs_j, Q6_K I = sum_j sc_j ((q . x)_j - 32 s_j)), then its
// float tail per block, accumulated in block order. Two CTAs per SM.
//
// Roles (288 threads): warps 0-7 compute (gate/up: thread = (matrix, row),
// all tokens; down: thread = (token half, row)), warp 8 the producer.
// Tiles hold up to DP_CH tokens of one expert.
constexpr int DP_CH = MOE_DP_CH;        // tokens per tile
constexpr int DP_CWARPS = 8, DP_THREADS = (DP_CWARPS + 1) * 32;
constexpr int DP_RS = 2;

template <int FMT> struct DpLayout {
    static constexpr int MATS = FMT == 0 ? 2 : 1;
    static constexpr size_t RAW_W = FMT == 0 ? (size_t)2 * 128 * 144 : (size_t)128 * 192 + 128 * 16;
    static constexpr size_t RAW = RAW_W + (size_t)DP_CH * 256;        // + the tokens' int8 rows of the block
    static constexpr size_t TOKW = FMT == 0 ? 12 : 20;               // words per token per block: xd, sums
    static constexpr size_t TOK = (size_t)DP_CH * TOKW * 4;
    static constexpr size_t XCHG = FMT == 0 ? (size_t)256 * DP_CH * 4 : 0;  // gate/up: the accumulators [token][thread]
    static constexpr size_t SMEM = DP_RS * (RAW + TOK) + XCHG;
};

struct DpBars {
    uint64_t full[DP_RS], empty[DP_RS];
    int err;
};

template <int FMT, int NB>
__global__ void __launch_bounds__(DP_THREADS, 2) k_moe_dp4a(DecodeArgs A, const __grid_constant__ TcMaps M) {
    using Ly = DpLayout<FMT>;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ DpBars B;
    uint8_t *raw = sm, *tokb = sm + DP_RS * Ly::RAW;
    float *xchg = reinterpret_cast<float *>(tokb + DP_RS * Ly::TOK);
    const TileTab TT = tc_tab_load(A, reinterpret_cast<int *>(sm + Ly::SMEM));
    const int R = FMT == 0 ? A.ffn : A.dim, RT = (R + 127) / 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int dim = A.dim, stride = A.act_stride;
    {
        TcTile t0;
        if (!tc_tile(A, RT, blockIdx.x, t0, DP_CH)) return;
    }
    if (tid == 0) {
        for (int i = 0; i < DP_RS; i++) {
            mbar_init(&B.full[i], 1);
            mbar_init(&B.empty[i], DP_CWARPS);
        }
        B.err = 0;
    }
    __syncthreads();
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {  // one lane waits; the verdict is the warp's
        int ok = 1;
        if (lane == 0) {
            ok = !*reinterpret_cast<volatile int *>(&B.err) && mbar_wait(bar, parity, TC_POLLS);
            if (!ok) {
                *reinterpret_cast<volatile int *>(&B.err) = 1;
                if (A.err) atomicOr(A.err, 64);
            }
        }
        return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };

    if (warp == DP_CWARPS) {
        // ---- producer ----------------------------------------------------------------------
        uint32_t gb = 0;
        bool run = true;
        TcTile tl;
        for (int ti = blockIdx.x; run && tc_tile(A, TT, RT, ti, tl, DP_CH); ti += gridDim.x) {
            const int row0 = tl.rt * 128;
            const int8_t *src = nullptr;  // this lane's token row (i = lane)
            if (lane < tl.nc) {
                const int slot = tc_slot(A, TT, tl, lane);
                src = FMT == 0 ? A.x256.q + (size_t)(tl.shared ? tl.c0 + lane : slot / A.n_used) * dim
                               : A.aq + (size_t)slot * stride;
            }
            for (int blk = 0; blk < NB; blk++, gb++) {
                const int s = gb % DP_RS;
                if (gb >= DP_RS && !wait(&B.empty[s], ((gb / DP_RS) - 1) & 1)) {
                    run = false;
                    break;
                }
                uint8_t *W = raw + (size_t)s * Ly::RAW, *X = W + Ly::RAW_W;
                if (lane == 0) {
                    mbar_expect_tx(&B.full[s], (uint32_t)Ly::RAW_W + (uint32_t)tl.nc * 256);
                    const int y = (tl.shared ? 0 : tl.e * R) + row0, m0 = tl.shared ? 2 : 0;
                    if (FMT == 0) {
                        tma_load_2d(W, &M.m[m0], blk * 144, y, &B.full[s]);
                        tma_load_2d(W + 128 * 144, &M.m[m0 + 1], blk * 144, y, &B.full[s]);
                    } else {
                        tma_load_2d(W, &M.m[m0], blk * 192, y, &B.full[s]);
                        tma_load_2d(W + 128 * 192, &M.m[m0 + 1], blk * 16, y, &B.full[s]);
                    }
                }
                __syncwarp();
                if (src) bulk_g2s(X + (size_t)lane * 256, src + blk * 256, 256, &B.full[s]);
            }
        }
        if (lane == 0 && !run)  // the last stages' copies must land before the CTA can exit
            for (uint32_t g = gb > DP_RS ? gb - DP_RS : 0; g < gb; g++)
                mbar_wait(&B.full[g % DP_RS], (g / DP_RS) & 1, TC_POLLS);
    } else {
        // ---- compute ----------------------------------------------------------------------
        const int r = tid & 127, hi = tid >> 7;  // FMT 0: hi = matrix; FMT 1: hi = token half
        uint32_t gb = 0;
        TcTile tl;
        for (int ti = blockIdx.x; tc_tile(A, TT, RT, ti, tl, DP_CH); ti += gridDim.x) {
            const int row0 = tl.rt * 128, rows = R - row0 < 128 ? R - row0 : 128;
            // this thread's token (tid < nc): its slot, for the per-block scalars and the stores
            const int my_slot = tid < tl.nc ? tc_slot(A, TT, tl, tid) : 0;
            const size_t my_tok = tl.shared ? (size_t)(tl.c0 + tid) : (size_t)(my_slot / A.n_used);
            float acc[FMT == 0 ? 1 : DP_CH / 2];  // down: in registers; gate/up: in shared memory (xchg)
#pragma unroll
            for (int i = 0; i < (FMT == 0 ? 1 : DP_CH / 2); i++) acc[i] = 0.0f;
            if (FMT == 0)
#pragma unroll
                for (int i = 0; i < DP_CH; i++) xchg[i * 256 + tid] = 0.0f;
            bool run = true;
            for (int blk = 0; blk < NB; blk++, gb++) {
                const int s = gb % DP_RS;
                if (!wait(&B.full[s], (gb / DP_RS) & 1)) {
                    run = false;
                    break;
                }
                // the tokens' per-block scalars into the stage's token words
                uint32_t *TK = reinterpret_cast<uint32_t *>(tokb + (size_t)s * Ly::TOK);
                if (tid < tl.nc) {
                    uint32_t *tw = TK + (size_t)tid * Ly::TOKW;
                    if (FMT == 0) {
                        tw[0] = __float_as_uint(A.x256.d[my_tok * NB + blk]);
                        const int4 *ss = reinterpret_cast<const int4 *>(A.x256.s + (my_tok * NB + blk) * 16);
                        uint32_t lo[2] = {0, 0}, hb[2] = {0, 0};
#pragma unroll
                        for (int k4 = 0; k4 < 4; k4++) {  // per-32 sums bs = 256 hi + lo (lo unsigned, hi signed bytes)
                            const int4 v = ss[k4];
                            const int b0 = v.x + v.y, b1 = v.z + v.w, k = 2 * k4;
                            lo[k >> 2] |= (uint32_t)(b0 & 0xFF) << (8 * (k & 3));
                            hb[k >> 2] |= (uint32_t)((b0 >> 8) & 0xFF) << (8 * (k & 3));
                            lo[(k + 1) >> 2] |= (uint32_t)(b1 & 0xFF) << (8 * ((k + 1) & 3));
                            hb[(k + 1) >> 2] |= (uint32_t)((b1 >> 8) & 0xFF) << (8 * ((k + 1) & 3));
                        }
                        tw[4] = lo[0];
                        tw[5] = lo[1];
                        tw[6] = hb[0];
                        tw[7] = hb[1];
                    } else {
                        tw[0] = __float_as_uint(A.ad[(size_t)my_slot * (stride / 32) + blk]);
                        const int4 *ss = reinterpret_cast<const int4 *>(A.as + (size_t)my_slot * (stride / 16) + blk * 16);
#pragma unroll
                        for (int k4 = 0; k4 < 4; k4++) *reinterpret_cast<int4 *>(tw + 4 + 4 * k4) = ss[k4];
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"r"(DP_CWARPS * 32) : "memory");
                const uint8_t *W = raw + (size_t)s * Ly::RAW;
                const int8_t *X = reinterpret_cast<const int8_t *>(W + Ly::RAW_W);
                if (FMT == 0) {
                    const uint8_t *wr = W + (size_t)(hi * 128 + r) * 144;
                    const uint4 hd = *reinterpret_cast<const uint4 *>(wr);
                    const float d = f16_to_f32((uint16_t)(hd.x & 0xFFFF)), dmin = f16_to_f32((uint16_t)(hd.x >> 16));
                    // scaleMinK4 for all 8 sub-blocks at once, as bytes: scales s0 (0-3), s1 (4-7); mins m0, m1
                    const uint32_t s0 = hd.y & 0x3F3F3F3Fu;
                    const uint32_t s1 = (hd.w & 0x0F0F0F0Fu) | (((hd.y >> 6) & 0x03030303u) << 4);
                    const uint32_t m0 = hd.z & 0x3F3F3F3Fu;
                    const uint32_t m1 = ((hd.w >> 4) & 0x0F0F0F0Fu) | (((hd.z >> 6) & 0x03030303u) << 4);
#pragma unroll
                    for (int g = 0; g < DP_CH / 8; g++) {
                        if (8 * g >= tl.nc) break;  // uniform
                        int isum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
                        for (int j = 0; j < 4; j++) {  // sub-blocks 2j (low nibbles), 2j + 1 (high)
                            const uint4 q0 = *reinterpret_cast<const uint4 *>(wr + 16 + 32 * j);
                            const uint4 q1 = *reinterpret_cast<const uint4 *>(wr + 32 + 32 * j);
                            const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                            const uint32_t sw = j < 2 ? s0 : s1;
                            const int sca = (int)((sw >> (16 * (j & 1))) & 0xFF), scb = (int)((sw >> (16 * (j & 1) + 8)) & 0xFF);
                            int lo[8], hv[8];
#pragma unroll
                            for (int w = 0; w < 8; w++) {
                                lo[w] = (int)(qw[w] & 0x0F0F0F0Fu);
                                hv[w] = (int)((qw[w] >> 4) & 0x0F0F0F0Fu);
                            }
#pragma unroll
                            for (int t = 0; t < 8; t++) {
                                const int i = 8 * g + t;
                                if (i < tl.nc) {
                                    const int4 *xp = reinterpret_cast<const int4 *>(X + (size_t)i * 256 + 64 * j);
                                    const int4 x0 = xp[0], x1 = xp[1], x2 = xp[2], x3 = xp[3];
                                    int a = 0, b = 0;
                                    a = __dp4a(lo[0], x0.x, a); a = __dp4a(lo[1], x0.y, a);
                                    a = __dp4a(lo[2], x0.z, a); a = __dp4a(lo[3], x0.w, a);
                                    a = __dp4a(lo[4], x1.x, a); a = __dp4a(lo[5], x1.y, a);
                                    a = __dp4a(lo[6], x1.z, a); a = __dp4a(lo[7], x1.w, a);
                                    b = __dp4a(hv[0], x2.x, b); b = __dp4a(hv[1], x2.y, b);
                                    b = __dp4a(hv[2], x2.z, b); b = __dp4a(hv[3], x2.w, b);
                                    b = __dp4a(hv[4], x3.x, b); b = __dp4a(hv[5], x3.y, b);
                                    b = __dp4a(hv[6], x3.z, b); b = __dp4a(hv[7], x3.w, b);
                                    isum[t] += sca * a + scb * b;
                                }
                            }
                        }
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            const int i = 8 * g + t;
                            if (i < tl.nc) {
                                const uint32_t *tw = TK + (size_t)i * Ly::TOKW;
                                // mins term M = sum_j mn_j bs_j through dp4a on bs = 256 hi + lo (exact)
                                const int Mi = (int)__dp4a(m0, tw[4], __dp4a(m1, tw[5], 0u)) +
                                               256 * dp4a_us(m0, (int)tw[6], dp4a_us(m1, (int)tw[7], 0));
                                const float xd = __uint_as_float(tw[0]);
                                float &a = xchg[i * 256 + tid];
                                a = fadd(a, fmul(xd, fsub(fmul(d, (float)isum[t]), fmul(dmin, (float)Mi))));
                            }
                        }
                    }
                } else {
                    const uint8_t *wr = W + (size_t)r * 192;
                    const int8_t *scb = reinterpret_cast<const int8_t *>(W + 128 * 192 + (size_t)r * 16);
                    float d = 0.0f;
                    if (r < rows) {
                        const WDev w = tl.shared ? A.sdn : A.dn;
                        const uint64_t pl = tl.shared ? 0 : (uint64_t)tl.e * R * NB;
                        d = f16_to_f32(w.d[pl + (uint64_t)(row0 + r) * NB + blk]);
                    }
#pragma unroll
                    for (int g = 0; g < DP_CH / 16; g++) {  // this thread's tokens: DP_CH / 2 * hi + 8 g + t
                        const int i0 = DP_CH / 2 * hi + 8 * g;
                        if (i0 >= tl.nc) break;  // uniform per warp
                        int isum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
                        for (int n = 0; n < 2; n++) {  // halves of 128 values
                            const uint4 h0 = *reinterpret_cast<const uint4 *>(wr + 128 + 32 * n);
                            const uint4 h1 = *reinterpret_cast<const uint4 *>(wr + 128 + 32 * n + 16);
                            const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
                            for (int gg = 0; gg < 4; gg++) {  // 32 values 128 n + 32 gg + l
                                const uint4 l0 = *reinterpret_cast<const uint4 *>(wr + 64 * n + 32 * (gg & 1));
                                const uint4 l1 = *reinterpret_cast<const uint4 *>(wr + 64 * n + 32 * (gg & 1) + 16);
                                const uint32_t ql[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                                int qv[8];
#pragma unroll
                                for (int w = 0; w < 8; w++)
                                    qv[w] = (int)((((gg >> 1) ? ql[w] >> 4 : ql[w]) & 0x0F0F0F0Fu) |
                                                  (((qh[w] >> (2 * gg)) & 0x03030303u) << 4));
                                const int s0 = scb[8 * n + 2 * gg], s1 = scb[8 * n + 2 * gg + 1];
#pragma unroll
                                for (int t = 0; t < 8; t++) {
                                    const int i = i0 + t;
                                    if (i < tl.nc) {
                                        const int4 *xp = reinterpret_cast<const int4 *>(X + (size_t)i * 256 + 128 * n + 32 * gg);
                                        const int4 x0 = xp[0], x1 = xp[1];
                                        int a = 0, b = 0;
                                        a = __dp4a(qv[0], x0.x, a); a = __dp4a(qv[1], x0.y, a);
                                        a = __dp4a(qv[2], x0.z, a); a = __dp4a(qv[3], x0.w, a);
                                        b = __dp4a(qv[4], x1.x, b); b = __dp4a(qv[5], x1.y, b);
                                        b = __dp4a(qv[6], x1.z, b); b = __dp4a(qv[7], x1.w, b);
                                        const uint32_t *tw = TK + (size_t)i * Ly::TOKW + 4;  // per-16 sums
                                        const int k = 8 * n + 2 * gg;
                                        isum[t] += s0 * (a - 32 * (int)tw[k]) + s1 * (b - 32 * (int)tw[k + 1]);
                                    }
                                }
                            }
                        }
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            const int i = i0 + t;
                            if (i < tl.nc) {
                                const float xd = __uint_as_float(TK[(size_t)i * Ly::TOKW]);
                                acc[8 * g + t] = fadd(acc[8 * g + t], fmul(fmul(xd, d), (float)isum[t]));
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) tc_arrive(&B.empty[s]);
            }
            if (!run) break;
            if (FMT == 0) {  // act = silu(gate) * up, the up row's sums from thread 128 + r
                asm volatile("bar.sync 1, %0;" ::"r"(DP_CWARPS * 32) : "memory");
                if (hi == 0 && r < rows)
#pragma unroll
                    for (int i = 0; i < DP_CH; i++) {
                        if (i >= tl.nc) break;
                        const int slot = tc_slot(A, TT, tl, i);
                        const float g = xchg[i * 256 + r], u = xchg[i * 256 + 128 + r];
                        A.act[(size_t)slot * stride + row0 + r] = fmul(fdiv(g, fadd(1.0f, exp_f(-g))), u);
                    }
                asm volatile("bar.sync 1, %0;" ::"r"(DP_CWARPS * 32) : "memory");  // xchg zeroed by the next tile
            } else if (r < rows) {
#pragma unroll
                for (int k = 0; k < DP_CH / 2; k++) {
                    const int i = DP_CH / 2 * hi + k;
                    if (i >= tl.nc) break;
                    A.y[(size_t)tc_slot(A, TT, tl, i) * dim + row0 + r] = acc[k];
                }
            }
        }
    }
    __syncthreads();
}

using DpFn = void (*)(DecodeArgs, TcMaps);

static DpFn dp_gu_fn(int nb) {
    switch (nb) {
        case 4: return k_moe_dp4a<0, 4>;
        case 8: return k_moe_dp4a<0, 8>;
        case 16: return k_moe_dp4a<0, 16>;
        case 28: return k_moe_dp4a<0, 28>;
    }
    return nullptr;
}
static DpFn dp_dn_fn(int nb) {
    switch (nb) {
        case 2: return k_moe_dp4a<1, 2>;
        case 3: return k_moe_dp4a<1, 3>;
        case 4: return k_moe_dp4a<1, 4>;
        case 8: return k_moe_dp4a<1, 8>;
    }
    return nullptr;
}

bool moe_dp4a_supported(const DecodeArgs &A) {
    if (A.g.type != T_Q4_K || A.u.type != T_Q4_K || A.dn.type != T_Q6_K) return false;
    if (A.dim % 256 || A.ffn % 256 || A.n_local + 1 > 1024) return false;
    if (!dp_gu_fn(A.dim / 256) || !dp_dn_fn(A.ffn / 256) || !tc_encoder()) return false;
    if (A.has_shared && (A.sg.type != T_Q4_K || A.su.type != T_Q4_K || A.sdn.type != T_Q6_K || A.shexp_ffn != A.ffn))
        return false;
    return true;
}

cudaError_t launch_moe_dp4a(const DecodeArgs &A, cudaStream_t st, cudaError_t (*quant)(const DecodeArgs &, cudaStream_t)) {
    static int n_sm = 0;
    if (!n_sm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (n_sm <= 0) n_sm = 148;
    }
    DpFn gf = dp_gu_fn(A.dim / 256), df = dp_dn_fn(A.ffn / 256);
    const int nbg = A.dim / 256, nbd = A.ffn / 256;
    TcMaps mg, md;
    memset(&mg, 0, sizeof mg);
    memset(&md, 0, sizeof md);
    const uint64_t gr = (uint64_t)A.n_local * A.ffn, dr = (uint64_t)A.n_local * A.dim;
    bool ok = tc_map(mg.m[0], A.g.q, nbg * 144ull, gr, 144) && tc_map(mg.m[1], A.u.q, nbg * 144ull, gr, 144) &&
              tc_map(md.m[0], A.dn.q, nbd * 192ull, dr, 192) && tc_map(md.m[1], A.dn.sc, nbd * 16ull, dr, 16);
    if (ok && A.has_shared)
        ok = tc_map(mg.m[2], A.sg.q, nbg * 144ull, (uint64_t)A.shexp_ffn, 144) &&
             tc_map(mg.m[3], A.su.q, nbg * 144ull, (uint64_t)A.shexp_ffn, 144) &&
             tc_map(md.m[2], A.sdn.q, nbd * 192ull, (uint64_t)A.dim, 192) &&
             tc_map(md.m[3], A.sdn.sc, nbd * 16ull, (uint64_t)A.dim, 16);
    if (!ok) return cudaErrorInvalidValue;
    const size_t gs = DpLayout<0>::SMEM + tc_tab_bytes(A.n_local), ds = DpLayout<1>::SMEM + tc_tab_bytes(A.n_local);
    cudaError_t e = cudaFuncSetAttribute(gf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gs);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(df, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ds);
    if (e != cudaSuccess) return e;
    count_launch();
    gf<<<2 * n_sm, DP_THREADS, gs, st>>>(A, mg);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = quant(A, st)) != cudaSuccess) return e;
    count_launch();
    df<<<2 * n_sm, DP_THREADS, ds, st>>>(A, md);
    return cudaGetLastError();
}

}  // namespace loom
