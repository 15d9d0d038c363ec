// loom_oracle.cpp -- TEST INFRASTRUCTURE ONLY: CPU restatement of the
// reference's CPU kernels for the quantized MoE forward path. It checks the
// CUDA backend and is the timed CPU baseline; the product never links it.
//
// Source followed (ch4r10t33r/loom):
//   src/gguf/ggml.zig   block formats, quantizers, int8-activation matvecs,
//                       batched matmul, dequantRow, the row-parallel pool
//   src/gguf/moe.zig    route()
//   src/core/tensor.zig softmax / silu / sigmoid / swiglu / rmsnorm
//   src/gguf/llama.zig  denseFFN + moeRun's weighted accumulation
//   src/gguf/deepseek.zig  moeFfnBlockRouted / moeFfnBlock call sites
// Build with -ffp-contract=off (no FMA contraction, as Zig) and no fast-math.
#include "loom_oracle.h"

#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace {

constexpr size_t QK_0 = 32;
constexpr size_t QK_K = 256;
constexpr size_t Q4_0_BLOCK = 18;
constexpr size_t Q8_0_BLOCK = 34;
constexpr size_t Q4_K_BLOCK = 144;
constexpr size_t Q4_1_BLOCK = 20;   // ggml.zig:89: d, m, qs[16]
constexpr size_t Q5_1_BLOCK = 24;   // ggml.zig:91: d, m, qh (u32), qs[16]
constexpr size_t Q5_0_BLOCK = 22;   // ggml.zig:90: d, qh (u32), qs[16]
constexpr size_t Q5_K_BLOCK = 176;  // ggml.zig:87-159: d, dmin, scales[12], qh[32], qs[128]
constexpr size_t Q2_K_BLOCK = 84;   // scales[16], qs[64], d, dmin
constexpr size_t Q3_K_BLOCK = 110;  // hmask[32], qs[64], scales[12], d
constexpr size_t Q6_K_BLOCK = 210;

// ggml.zig:260 f16FromBytes: exact widening of an IEEE half.
inline float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal half -> normal float
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
inline float f16at(const uint8_t *p) { return f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

inline bool finitef(float v) { return std::isfinite(v); }

// ggml.zig:1067-1074 toI8Saturating: non-finite -> 0, round half away from
// zero, saturate at +-127.
inline int8_t to_i8_sat(float v) {
    if (!finitef(v)) return 0;
    float r = std::round(v);
    if (r >= 127.0f) return 127;
    if (r <= -127.0f) return -127;
    return (int8_t)(int)r;
}

// ggml.zig:1332-1340 scaleMinK4
inline void scale_min_k4(int j, const uint8_t *s, int &sc, int &mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// ---- quantizers ---------------------------------------------------------------

// ggml.zig:776-801 quantizeX256 (one 256-wide block)
void quant256(const float *src, int8_t *q, float *d_out, int32_t *bsum) {
    float amax = 0.0f;
    for (size_t i = 0; i < QK_K; i++)
        if (finitef(src[i])) amax = std::fmax(amax, std::fabs(src[i]));
    const float d = amax / 127.0f;
    const float inv = (d != 0.0f && finitef(d)) ? 1.0f / d : 0.0f;
    for (size_t s = 0; s < QK_K / 16; s++) {
        int32_t sum = 0;
        for (size_t i = 0; i < 16; i++) {
            int8_t v = to_i8_sat(src[s * 16 + i] * inv);
            q[s * 16 + i] = v;
            sum += v;
        }
        bsum[s] = sum;
    }
    *d_out = finitef(d) ? d : 0.0f;
}

// ggml.zig:1077-1100 quantizeX (one 32-wide block)
void quant32(const float *src, int8_t *q, float *d_out, int32_t *sum_out) {
    float amax = 0.0f;
    for (size_t i = 0; i < QK_0; i++)
        if (finitef(src[i])) amax = std::fmax(amax, std::fabs(src[i]));
    const float d = amax / 127.0f;
    const float inv = (d != 0.0f && finitef(d)) ? 1.0f / d : 0.0f;
    int32_t sum = 0;
    for (size_t i = 0; i < QK_0; i++) {
        int8_t v = to_i8_sat(src[i] * inv);
        q[i] = v;
        sum += v;
    }
    *d_out = finitef(d) ? d : 0.0f;
    *sum_out = sum;
}

struct XQ {  // quantized activation vector
    std::vector<int8_t> q;
    std::vector<float> d;
    std::vector<int32_t> s;  // bsum16 (K) or sum32 (Q4_0/Q8_0)
};

bool uses_q8k(int t) { return t == OR_Q4_K || t == OR_Q6_K || t == OR_Q2_K || t == OR_Q3_K || t == OR_Q5_K; }

void quantize(int t, const float *x, size_t cols, XQ &xq) {
    xq.q.resize(cols);
    if (uses_q8k(t)) {
        xq.d.resize(cols / QK_K);
        xq.s.resize(cols / 16);
        for (size_t b = 0; b < cols / QK_K; b++)
            quant256(x + b * QK_K, &xq.q[b * QK_K], &xq.d[b], &xq.s[b * 16]);
    } else {
        xq.d.resize(cols / QK_0);
        xq.s.resize(cols / QK_0);
        for (size_t b = 0; b < cols / QK_0; b++)
            quant32(x + b * QK_0, &xq.q[b * QK_0], &xq.d[b], &xq.s[b]);
    }
}

// ---- per-block dots ------------------------------------------------------------

inline int32_t dot32(const int8_t *w, const int8_t *x) {
    int32_t s = 0;
    for (int i = 0; i < 32; i++) s += (int32_t)w[i] * (int32_t)x[i];
    return s;
}

// ggml.zig:882-997 kDecode (q4_k) + :1002-1021 kBlockDot
inline float q4k_block_dot(const uint8_t *blk, const int8_t *xq, float xd, const int32_t *bsum) {
    const float d = f16at(blk);
    const float dmin = f16at(blk + 2);
    const uint8_t *scales = blk + 4;
    const uint8_t *qs = blk + 16;
    int32_t isum = 0, msum = 0;
    int8_t w[32];
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        scale_min_k4(j, scales, sc, mn);
        const uint8_t *src = qs + (j / 2) * 32;
        if (j & 1)
            for (int i = 0; i < 32; i++) w[i] = (int8_t)(src[i] >> 4);
        else
            for (int i = 0; i < 32; i++) w[i] = (int8_t)(src[i] & 0x0F);
        isum += sc * dot32(w, xq + j * 32);
        msum += mn * (bsum[2 * j] + bsum[2 * j + 1]);
    }
    return xd * (d * (float)isum - dmin * (float)msum);
}

// ggml.zig:882-997 kDecode (q6_k) + kBlockDot (no min)
inline float q6k_block_dot(const uint8_t *blk, const int8_t *xq, float xd) {
    const uint8_t *ql_all = blk;
    const uint8_t *qh_all = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    const float d = f16at(blk + 208);
    int32_t isum = 0;
    int8_t w[32];
    for (int half = 0; half < 2; half++) {
        const uint8_t *ql = ql_all + half * 64;
        const uint8_t *qh = qh_all + half * 32;
        for (int gg = 0; gg < 4; gg++) {
            for (int i = 0; i < 32; i++) {
                uint8_t a = ql[i], bb = ql[32 + i], h = qh[i];
                uint8_t q;
                switch (gg) {
                    case 0: q = (a & 0x0F) | ((h & 3) << 4); break;
                    case 1: q = (bb & 0x0F) | (((h >> 2) & 3) << 4); break;
                    case 2: q = (a >> 4) | (((h >> 4) & 3) << 4); break;
                    default: q = (bb >> 4) | (((h >> 6) & 3) << 4); break;
                }
                w[i] = (int8_t)((int)q - 32);
            }
            const int g = half * 4 + gg;
            int32_t lo = 0, hi = 0;
            for (int i = 0; i < 16; i++) lo += (int32_t)w[i] * xq[g * 32 + i];
            for (int i = 16; i < 32; i++) hi += (int32_t)w[i] * xq[g * 32 + i];
            isum += lo * (int32_t)sc[2 * g] + hi * (int32_t)sc[2 * g + 1];
        }
    }
    return xd * d * (float)isum;
}

// ggml.zig:1196-1223 matvecQ40Int, one block
inline float q40_block_dot(const uint8_t *blk, const int8_t *xq, float xd) {
    const float d = f16at(blk);
    const uint8_t *qs = blk + 2;
    int32_t dot = 0, sum = 0;
    for (int i = 0; i < 16; i++) {
        int32_t lo = qs[i] & 0x0F, hi = qs[i] >> 4;
        dot += lo * (int32_t)xq[i] + hi * (int32_t)xq[i + 16];
        sum += (int32_t)xq[i] + (int32_t)xq[i + 16];
    }
    return d * xd * (float)(dot - 8 * sum);
}

// ggml.zig:1242-1275 matvecQ41Int (q4_1 / q5_1), one block: the min folds
// out as m * sum(xq): xd * (d * dot + m * sum)
inline float q41_block_dot(int t, const uint8_t *blk, const int8_t *xq, float xd) {
    const float d = f16at(blk), m = f16at(blk + 2);
    uint32_t qh = 0;
    if (t == OR_Q5_1) std::memcpy(&qh, blk + 4, 4);
    const uint8_t *qs = blk + (t == OR_Q5_1 ? 8 : 4);
    int32_t dot = 0, sum = 0;
    for (int i = 0; i < 16; i++) {
        const int32_t lo = (qs[i] & 0x0F) | (t == OR_Q5_1 ? (int32_t)(((qh >> i) << 4) & 0x10) : 0);
        const int32_t hi = (qs[i] >> 4) | (t == OR_Q5_1 ? (int32_t)((qh >> (i + 12)) & 0x10) : 0);
        dot += lo * (int32_t)xq[i] + hi * (int32_t)xq[i + 16];
        sum += (int32_t)xq[i] + (int32_t)xq[i + 16];
    }
    return xd * (d * (float)dot + m * (float)sum);
}

// ggml.zig:1277-1294 matvecQ80Int, one block
inline float q80_block_dot(const uint8_t *blk, const int8_t *xq, float xd) {
    const float d = f16at(blk);
    return d * xd * (float)dot32((const int8_t *)(blk + 2), xq);
}

// ggml.zig:1173-1191 q3kScales: 12 packed bytes -> 16 six-bit scales
inline void q3k_scales(const uint8_t *p, uint8_t out[16]) {
    uint32_t aux[4];
    std::memcpy(&aux[0], p, 4);
    std::memcpy(&aux[1], p + 4, 4);
    std::memcpy(&aux[2], p + 8, 4);
    const uint32_t kmask1 = 0x03030303u, kmask2 = 0x0f0f0f0fu, tmp = aux[2];
    aux[2] = ((aux[0] >> 4) & kmask2) | (((tmp >> 4) & kmask1) << 4);
    aux[3] = ((aux[1] >> 4) & kmask2) | (((tmp >> 6) & kmask1) << 4);
    aux[0] = (aux[0] & kmask2) | (((tmp >> 0) & kmask1) << 4);
    aux[1] = (aux[1] & kmask2) | (((tmp >> 2) & kmask1) << 4);
    std::memcpy(out, aux, 16);
}

// ggml.zig:844-997 kDecode for q2_k / q3_k / q5_k into the uniform shape:
// eight 32-wide int8 weight groups (group g = values 32g..32g+31, per-16
// sub-blocks 2g and 2g+1), sixteen per-16 scales and mins, d and dmin.
struct KDec {
    int8_t w[256];
    int32_t sc[16], mn[16];
    float d, dmin;
    bool has_min;
};

inline void k_decode(int t, const uint8_t *blk, KDec &k) {
    switch (t) {
        case OR_Q5_K: {
            k.d = f16at(blk);
            k.dmin = f16at(blk + 2);
            k.has_min = true;
            const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
            for (int j = 0; j < 8; j++) {
                int sc, mn;
                scale_min_k4(j, scales, sc, mn);
                k.sc[2 * j] = k.sc[2 * j + 1] = sc;
                k.mn[2 * j] = k.mn[2 * j + 1] = mn;
                for (int l = 0; l < 32; l++) {
                    const uint8_t b = qs[(j / 2) * 32 + l];
                    const int nib = (j % 2) ? (b >> 4) : (b & 0x0F);
                    const int hb = (qh[l] >> (j % 2 + 2 * (j / 2))) & 1;  // the fifth bit of sub-block j
                    k.w[32 * j + l] = (int8_t)(nib | (hb << 4));
                }
            }
            break;
        }
        case OR_Q2_K: {
            const uint8_t *scales = blk, *qs = blk + 16;
            k.d = f16at(blk + 80);
            k.dmin = f16at(blk + 82);
            k.has_min = true;
            for (int j = 0; j < 16; j++) {
                k.sc[j] = scales[j] & 0xF;
                k.mn[j] = scales[j] >> 4;
            }
            for (int half = 0; half < 2; half++)
                for (int shift = 0; shift < 4; shift++)
                    for (int l = 0; l < 32; l++)
                        k.w[32 * (half * 4 + shift) + l] = (int8_t)((qs[half * 32 + l] >> (2 * shift)) & 3);
            break;
        }
        case OR_Q3_K: {
            const uint8_t *hmask = blk, *qs = blk + 32;
            uint8_t sc16[16];
            q3k_scales(blk + 96, sc16);
            k.d = f16at(blk + 108);
            k.dmin = 0.0f;
            k.has_min = false;
            for (int j = 0; j < 16; j++) {
                k.sc[j] = (int32_t)sc16[j] - 32;
                k.mn[j] = 0;
            }
            for (int half = 0; half < 2; half++)
                for (int shift = 0; shift < 4; shift++) {
                    const int idx = half * 4 + shift;
                    for (int l = 0; l < 32; l++) {
                        const int q2 = (qs[half * 32 + l] >> (2 * shift)) & 3;
                        const int off = (hmask[l] & (1 << idx)) ? 0 : 4;  // subtract 4 where the high bit is clear
                        k.w[32 * idx + l] = (int8_t)(q2 - off);
                    }
                }
            break;
        }
    }
}

// ggml.zig:1002-1021 kBlockDot on a uniform decode
inline float k_block_dot(const KDec &k, const int8_t *xq, float xd, const int32_t *bsum) {
    int32_t isum = 0;
    for (int j = 0; j < 16; j++) {
        int32_t s = 0;
        for (int l = 0; l < 16; l++) s += (int32_t)k.w[16 * j + l] * (int32_t)xq[16 * j + l];
        isum += s * k.sc[j];
    }
    if (k.has_min) {
        int32_t msum = 0;
        for (int j = 0; j < 16; j++) msum += k.mn[j] * bsum[j];
        return xd * (k.d * (float)isum - k.dmin * (float)msum);
    }
    return xd * k.d * (float)isum;
}

// One row against a quantized activation.
float row_dot(int t, const uint8_t *row, const XQ &xq, size_t cols) {
    float acc = 0.0f;
    switch (t) {
        case OR_Q4_K:
            for (size_t b = 0; b < cols / QK_K; b++)
                acc += q4k_block_dot(row + b * Q4_K_BLOCK, &xq.q[b * QK_K], xq.d[b], &xq.s[b * 16]);
            break;
        case OR_Q6_K:
            for (size_t b = 0; b < cols / QK_K; b++)
                acc += q6k_block_dot(row + b * Q6_K_BLOCK, &xq.q[b * QK_K], xq.d[b]);
            break;
        case OR_Q4_0:
            for (size_t b = 0; b < cols / QK_0; b++)
                acc += q40_block_dot(row + b * Q4_0_BLOCK, &xq.q[b * QK_0], xq.d[b]);
            break;
        case OR_Q4_1:
        case OR_Q5_1: {
            const size_t bb = or_block_bytes(t);
            for (size_t b = 0; b < cols / QK_0; b++) acc += q41_block_dot(t, row + b * bb, &xq.q[b * QK_0], xq.d[b]);
            break;
        }
        case OR_Q2_K:
        case OR_Q3_K:
        case OR_Q5_K: {  // matvecK256 :1024 over the uniform decode
            const size_t bb = or_block_bytes(t);
            KDec k;
            for (size_t b = 0; b < cols / QK_K; b++) {
                k_decode(t, row + b * bb, k);
                acc += k_block_dot(k, &xq.q[b * QK_K], xq.d[b], &xq.s[b * 16]);
            }
            break;
        }
        case OR_Q8_0:
            for (size_t b = 0; b < cols / QK_0; b++)
                acc += q80_block_dot(row + b * Q8_0_BLOCK, &xq.q[b * QK_0], xq.d[b]);
            break;
    }
    return acc;
}

// ---- pool (ggml.zig:279-398): spin workers, row chunks, submitter works ------

struct Pool {
    int n = 0;  // live workers (excluding the submitting thread)
    std::vector<std::thread> threads;
    std::atomic<bool> quit{false};
    std::atomic<uint64_t> seq{0};
    std::atomic<size_t> active{0};
    std::atomic<size_t> cursor{0};
    size_t rows = 0, chunk = 0;
    const std::function<void(size_t, size_t)> *job = nullptr;
};
Pool pool;
constexpr size_t MIN_ROWS_PER_THREAD = 64;  // ggml.zig:263
constexpr uint32_t SPIN_BEFORE_YIELD = 40000;  // ggml.zig:268

void run_chunks() {
    for (;;) {
        size_t start = pool.cursor.fetch_add(pool.chunk, std::memory_order_acq_rel);
        if (start >= pool.rows) return;
        size_t end = std::min(start + pool.chunk, pool.rows);
        (*pool.job)(start, end);
    }
}

void worker_main() {
    uint64_t seen = 0;
    uint32_t idle = 0;
    for (;;) {
        uint64_t s = pool.seq.load(std::memory_order_acquire);
        if (s == seen) {
            if (pool.quit.load(std::memory_order_acquire)) return;
            if (++idle < SPIN_BEFORE_YIELD) {
#if defined(__x86_64__)
                __builtin_ia32_pause();
#endif
            } else {
                std::this_thread::yield();
            }
            continue;
        }
        idle = 0;
        seen = s;
        if (pool.quit.load(std::memory_order_acquire)) return;
        run_chunks();
        pool.active.fetch_sub(1, std::memory_order_release);
    }
}

// Row-parallel execution with the reference's chunking rule (ggml.zig:212-213):
// chunk = max(64, ceil(rows / (2*(workers+1)))).  Row splitting is exact, so the
// result is independent of the worker count.
void parallel_rows(size_t rows, const std::function<void(size_t, size_t)> &fn) {
    const int workers = pool.n;
    if (workers == 0 || rows < 2 * MIN_ROWS_PER_THREAD) {
        fn(0, rows);
        return;
    }
    size_t per = (rows + (workers + 1) * 2 - 1) / ((workers + 1) * 2);
    if (per < MIN_ROWS_PER_THREAD) per = MIN_ROWS_PER_THREAD;
    pool.job = &fn;
    pool.rows = rows;
    pool.chunk = per;
    pool.cursor.store(0, std::memory_order_relaxed);
    pool.active.store(workers, std::memory_order_relaxed);
    pool.seq.fetch_add(1, std::memory_order_release);
    run_chunks();
    uint32_t spins = 0;
    while (pool.active.load(std::memory_order_acquire) != 0) {
        if (++spins < SPIN_BEFORE_YIELD) {
#if defined(__x86_64__)
            __builtin_ia32_pause();
#endif
        } else {
            std::this_thread::yield();
        }
    }
}

}  // namespace

extern "C" {

size_t or_block_elems(int t) {
    switch (t) {
        case OR_F32: case OR_F16: return 1;
        case OR_Q4_0: case OR_Q4_1: case OR_Q5_0: case OR_Q5_1: case OR_Q8_0: return QK_0;
        case OR_Q2_K: case OR_Q3_K: case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return QK_K;
    }
    return 0;
}

size_t or_block_bytes(int t) {
    switch (t) {
        case OR_F32: return 4;
        case OR_F16: return 2;
        case OR_Q4_0: return Q4_0_BLOCK;
        case OR_Q8_0: return Q8_0_BLOCK;
        case OR_Q4_K: return Q4_K_BLOCK;
        case OR_Q6_K: return Q6_K_BLOCK;
        case OR_Q2_K: return Q2_K_BLOCK;
        case OR_Q3_K: return Q3_K_BLOCK;
        case OR_Q5_K: return Q5_K_BLOCK;
        case OR_Q4_1: return Q4_1_BLOCK;
        case OR_Q5_1: return Q5_1_BLOCK;
        case OR_Q5_0: return Q5_0_BLOCK;
    }
    return 0;
}

size_t or_row_bytes(int t, size_t n) {
    size_t be = or_block_elems(t);
    if (be == 0) return 0;
    return (n / be) * or_block_bytes(t);
}

void or_parallel_begin(int n) {
    if (pool.n != 0) return;
    int want = n > 32 ? 32 : n;  // MAX_WORKERS, ggml.zig:259
    if (want <= 1) return;
    pool.quit.store(false);
    pool.seq.store(0);
    pool.active.store(0);
    for (int i = 0; i + 1 < want; i++) pool.threads.emplace_back(worker_main);
    pool.n = (int)pool.threads.size();
}

void or_parallel_end(void) {
    if (pool.n == 0) return;
    pool.quit.store(true, std::memory_order_release);
    pool.seq.fetch_add(1, std::memory_order_release);
    for (auto &t : pool.threads) t.join();
    pool.threads.clear();
    pool.n = 0;
}

int or_pool_workers(void) { return pool.n; }

// ggml.zig:198-217 dotF32: four 8-lane accumulators, 32 per step, an 8-wide
// tail into acc0, then (acc0+acc1+acc2+acc3) reduced lane 0..7 in order
// (@reduce(.Add) lowered as an ordered reduction), then a scalar tail.
float or_dot_f32(const float *a, const float *b, size_t n) {
    float acc[4][8] = {};
    size_t i = 0;
    for (; i + 32 <= n; i += 32)
        for (int k = 0; k < 4; k++)
            for (int j = 0; j < 8; j++) acc[k][j] += a[i + 8 * k + j] * b[i + 8 * k + j];
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; j++) acc[0][j] += a[i + j] * b[i + j];
    float v[8];
    for (int j = 0; j < 8; j++) v[j] = ((acc[0][j] + acc[1][j]) + acc[2][j]) + acc[3][j];
    float r = v[0];
    for (int j = 1; j < 8; j++) r += v[j];
    for (; i < n; i++) r += a[i] * b[i];
    return r;
}

void or_quantize_x256(const float *x, size_t cols, int8_t *q, float *d, int32_t *bsum) {
    for (size_t b = 0; b < cols / QK_K; b++) quant256(x + b * QK_K, q + b * QK_K, d + b, bsum + b * 16);
}

void or_quantize_x32(const float *x, size_t cols, int8_t *q, float *d, int32_t *sum) {
    for (size_t b = 0; b < cols / QK_0; b++) quant32(x + b * QK_0, q + b * QK_0, d + b, sum + b);
}

// ggml.zig:1739-1857 dequantRow (f32, q4_0, q8_0, q4_k, q6_k)
int or_dequant_row(int t, float *out, const uint8_t *data, size_t r, size_t cols) {
    const size_t rb = or_row_bytes(t, cols);
    const uint8_t *row = data + r * rb;
    switch (t) {
        case OR_F32:
            std::memcpy(out, row, cols * 4);
            return 0;
        case OR_Q4_K:  // dequantBlockQ4K, ggml.zig:1342-1374
            for (size_t b = 0; b < cols / QK_K; b++) {
                const uint8_t *blk = row + b * Q4_K_BLOCK;
                const float d = f16at(blk), dmin = f16at(blk + 2);
                const uint8_t *scales = blk + 4, *qs = blk + 16;
                float *v = out + b * QK_K;
                for (int j = 0; j < 4; j++) {
                    int sc, mn;
                    scale_min_k4(2 * j, scales, sc, mn);
                    const float d1 = d * (float)sc, m1 = dmin * (float)mn;
                    scale_min_k4(2 * j + 1, scales, sc, mn);
                    const float d2 = d * (float)sc, m2 = dmin * (float)mn;
                    for (int l = 0; l < 32; l++) {
                        v[64 * j + l] = d1 * (float)(qs[32 * j + l] & 0x0F) - m1;
                        v[64 * j + 32 + l] = d2 * (float)(qs[32 * j + l] >> 4) - m2;
                    }
                }
            }
            return 0;
        case OR_Q6_K:  // dequantBlockQ6K, ggml.zig:1420-1474
            for (size_t b = 0; b < cols / QK_K; b++) {
                const uint8_t *blk = row + b * Q6_K_BLOCK;
                const float d = f16at(blk + 208);
                float *v = out + b * QK_K;
                for (int n = 0; n < 2; n++) {
                    const uint8_t *ql = blk + 64 * n, *qh = blk + 128 + 32 * n;
                    const int8_t *sc = (const int8_t *)(blk + 192 + 8 * n);
                    for (int l = 0; l < 32; l++) {
                        const int is = l / 16;
                        const float s1 = d * (float)sc[is], s2 = d * (float)sc[is + 2];
                        const float s3 = d * (float)sc[is + 4], s4 = d * (float)sc[is + 6];
                        const uint8_t a = ql[l], bb = ql[l + 32], h = qh[l];
                        const float q1 = (float)((a & 0x0F) | ((h & 3) << 4));
                        const float q2 = (float)((bb & 0x0F) | (((h >> 2) & 3) << 4));
                        const float q3 = (float)((a >> 4) | (((h >> 4) & 3) << 4));
                        const float q4 = (float)((bb >> 4) | (((h >> 6) & 3) << 4));
                        v[128 * n + l] = s1 * (q1 - 32.0f);
                        v[128 * n + l + 32] = s2 * (q2 - 32.0f);
                        v[128 * n + l + 64] = s3 * (q3 - 32.0f);
                        v[128 * n + l + 96] = s4 * (q4 - 32.0f);
                    }
                }
            }
            return 0;
        case OR_Q5_K:  // dequantBlockQ5K, ggml.zig:1376-1418
            for (size_t b = 0; b < cols / QK_K; b++) {
                const uint8_t *blk = row + b * Q5_K_BLOCK;
                const float d = f16at(blk), dmin = f16at(blk + 2);
                const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
                float *v = out + b * QK_K;
                for (int j = 0; j < 4; j++) {
                    int sc, mn;
                    scale_min_k4(2 * j, scales, sc, mn);
                    const float d1 = d * (float)sc, m1 = dmin * (float)mn;
                    scale_min_k4(2 * j + 1, scales, sc, mn);
                    const float d2 = d * (float)sc, m2 = dmin * (float)mn;
                    const uint8_t hb1 = (uint8_t)(1u << (2 * j)), hb2 = (uint8_t)(2u << (2 * j));
                    for (int l = 0; l < 32; l++) {
                        const uint8_t q = qs[32 * j + l];
                        v[64 * j + l] = d1 * ((float)(q & 0x0F) + ((qh[l] & hb1) ? 16.0f : 0.0f)) - m1;
                        v[64 * j + 32 + l] = d2 * ((float)(q >> 4) + ((qh[l] & hb2) ? 16.0f : 0.0f)) - m2;
                    }
                }
            }
            return 0;
        case OR_Q2_K:  // dequantBlockQ2K, ggml.zig:1476-1505
            for (size_t b = 0; b < cols / QK_K; b++) {
                const uint8_t *blk = row + b * Q2_K_BLOCK;
                const uint8_t *scales = blk, *qs = blk + 16;
                const float d = f16at(blk + 80), dmin = f16at(blk + 82);
                float *v = out + b * QK_K;
                int y = 0, is = 0;
                for (int n = 0; n < 2; n++)
                    for (int j = 0; j < 4; j++)
                        for (int half = 0; half < 2; half++) {
                            const uint8_t sc = scales[is++];
                            const float dl = d * (float)(sc & 0xF), ml = dmin * (float)(sc >> 4);
                            for (int l = 0; l < 16; l++)
                                v[y++] = dl * (float)((qs[32 * n + half * 16 + l] >> (2 * j)) & 3) - ml;
                        }
            }
            return 0;
        case OR_Q3_K:  // dequantBlockQ3K, ggml.zig:1508-1540
            for (size_t b = 0; b < cols / QK_K; b++) {
                const uint8_t *blk = row + b * Q3_K_BLOCK;
                const uint8_t *hmask = blk, *qs = blk + 32;
                uint8_t sc16[16];
                q3k_scales(blk + 96, sc16);
                const float d = f16at(blk + 108);
                float *v = out + b * QK_K;
                int y = 0, is = 0;
                for (int n = 0; n < 2; n++)
                    for (int j = 0; j < 4; j++) {
                        const uint8_t m = (uint8_t)(1u << (4 * n + j));
                        for (int half = 0; half < 2; half++) {
                            const float dl = d * (float)((int)sc16[is++] - 32);
                            for (int l = 0; l < 16; l++) {
                                const int idx = half * 16 + l;
                                const int q2 = (qs[32 * n + idx] >> (2 * j)) & 3;
                                v[y++] = dl * (float)(q2 - ((hmask[idx] & m) ? 0 : 4));
                            }
                        }
                    }
            }
            return 0;
        case OR_Q5_0:  // dequantRow :1772-1793: (q - 16) * d
            for (size_t b = 0; b < cols / QK_0; b++) {
                const uint8_t *blk = row + b * Q5_0_BLOCK;
                const float s = f16at(blk);
                uint32_t qh;
                std::memcpy(&qh, blk + 2, 4);
                for (int j = 0; j < 16; j++) {
                    const int xh0 = (int)(((qh >> j) << 4) & 0x10), xh1 = (int)((qh >> (j + 12)) & 0x10);
                    out[b * 32 + j] = (float)(((blk[6 + j] & 0x0F) | xh0) - 16) * s;
                    out[b * 32 + j + 16] = (float)(((blk[6 + j] >> 4) | xh1) - 16) * s;
                }
            }
            return 0;
        case OR_Q4_1:
        case OR_Q5_1:  // dequantRow :1795-1819: q * d + m
            for (size_t b = 0; b < cols / QK_0; b++) {
                const uint8_t *blk = row + b * or_block_bytes(t);
                const float d = f16at(blk), m = f16at(blk + 2);
                uint32_t qh = 0;
                if (t == OR_Q5_1) std::memcpy(&qh, blk + 4, 4);
                const uint8_t *qs = blk + (t == OR_Q5_1 ? 8 : 4);
                for (int j = 0; j < 16; j++) {
                    const int lo = (qs[j] & 0x0F) | (t == OR_Q5_1 ? (int)(((qh >> j) << 4) & 0x10) : 0);
                    const int hi = (qs[j] >> 4) | (t == OR_Q5_1 ? (int)((qh >> (j + 12)) & 0x10) : 0);
                    out[b * 32 + j] = (float)lo * d + m;
                    out[b * 32 + j + 16] = (float)hi * d + m;
                }
            }
            return 0;
        case OR_Q4_0:
            for (size_t b = 0; b < cols / QK_0; b++) {
                const uint8_t *blk = row + b * Q4_0_BLOCK;
                const float s = f16at(blk);
                for (int j = 0; j < 16; j++) {
                    out[b * 32 + j] = (float)((int)(blk[2 + j] & 0x0F) - 8) * s;
                    out[b * 32 + j + 16] = (float)((int)(blk[2 + j] >> 4) - 8) * s;
                }
            }
            return 0;
        case OR_Q8_0:
            for (size_t b = 0; b < cols / QK_0; b++) {
                const uint8_t *blk = row + b * Q8_0_BLOCK;
                const float s = f16at(blk);
                for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * s;
            }
            return 0;
    }
    return -1;
}

// ggml.zig:602-659 matvec/dispatch: the activation is quantized once per call
// (matvecK256 :1024, matvecQ40Int :1196, matvecQ80Int :1277); rows are
// independent dots, split over the pool.
// ggml.zig:1673-1704 matvecQ50: q5_0 stays on f32 activations. Per block the
// partial runs j = 0..15 as partial += w0*x[j] + w1*x[j+16]; blocks whose
// scale is 0 are skipped; acc += partial * scale in block order.
static float q50_row(const uint8_t *row, const float *x, size_t cols) {
    float acc = 0.0f;
    for (size_t b = 0; b < cols / QK_0; b++) {
        const uint8_t *blk = row + b * Q5_0_BLOCK;
        const float scale = f16at(blk);
        if (scale == 0.0f) continue;
        uint32_t qh;
        std::memcpy(&qh, blk + 2, 4);
        const float *xb = x + b * QK_0;
        float partial = 0.0f;
        for (int j = 0; j < 16; j++) {
            const int xh0 = (int)(((qh >> j) << 4) & 0x10), xh1 = (int)((qh >> (j + 12)) & 0x10);
            const float w0 = (float)(((blk[6 + j] & 0xF) | xh0) - 16);
            const float w1 = (float)(((blk[6 + j] >> 4) | xh1) - 16);
            partial += w0 * xb[j] + w1 * xb[j + 16];
        }
        acc += partial * scale;
    }
    return acc;
}

int or_matvec(int t, float *out, const uint8_t *data, const float *x, size_t rows, size_t cols) {
    if (t == OR_Q5_0) {
        if (cols % QK_0) return -1;
        const size_t rb = or_row_bytes(t, cols);
        parallel_rows(rows, [&](size_t r0, size_t r1) {
            for (size_t r = r0; r < r1; r++) out[r] = q50_row(data + r * rb, x, cols);
        });
        return 0;
    }
    if (t == OR_F32) {
        const float *w = (const float *)data;
        parallel_rows(rows, [&](size_t r0, size_t r1) {
            for (size_t r = r0; r < r1; r++) out[r] = or_dot_f32(w + r * cols, x, cols);
        });
        return 0;
    }
    if (or_block_elems(t) == 0 || t == OR_F16) return -1;
    if (cols % or_block_elems(t) != 0) return -1;
    XQ xq;
    quantize(t, x, cols, xq);
    const size_t rb = or_row_bytes(t, cols);
    parallel_rows(rows, [&](size_t r0, size_t r1) {
        for (size_t r = r0; r < r1; r++) out[r] = row_dot(t, data + r * rb, xq, cols);
    });
    return 0;
}

// ggml.zig:504-563 matmul: out[k*rows + r]; bit-identical to n matvecs
// (the reference's own invariant, test ggml.zig:2132). Each token's activation
// is quantized once; every row is decoded against all n tokens.
int or_matmul(int t, float *out, const uint8_t *data, const float *xs, size_t n, size_t rows, size_t cols) {
    if (t == OR_F32 || t == OR_Q5_0) {  // q5_0 has no batched kernel: n matvecs (ggml.zig:516-526)
        for (size_t k = 0; k < n; k++) or_matvec(t, out + k * rows, data, xs + k * cols, rows, cols);
        return 0;
    }
    if (or_block_elems(t) == 0 || t == OR_F16) return -1;
    std::vector<XQ> xq(n);
    for (size_t k = 0; k < n; k++) quantize(t, xs + k * cols, cols, xq[k]);
    const size_t rb = or_row_bytes(t, cols);
    parallel_rows(rows, [&](size_t r0, size_t r1) {
        for (size_t r = r0; r < r1; r++)
            for (size_t k = 0; k < n; k++) out[k * rows + r] = row_dot(t, data + r * rb, xq[k], cols);
    });
    return 0;
}

// f32 e^x, correctly rounded (a double-precision exp rounded once; exact to
// f32 except within ~2^-29 of a rounding boundary). Zig's f32 @exp and glibc's
// expf are both within ~0.5 ulp of this and differ from it, and from each
// other, in rare last-bit cases; the correctly rounded value is the common
// definition the oracle and the device kernels share.
static inline float exp_f(float x) { return (float)std::exp((double)x); }

// tensor.zig:18-28
void or_softmax(float *x, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; i++) m = std::fmax(m, x[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        x[i] = exp_f(x[i] - m);
        sum += x[i];
    }
    const float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) x[i] *= inv;
}

float or_silu(float x) { return x / (1.0f + exp_f(-x)); }      // tensor.zig:30
float or_sigmoid(float x) { return 1.0f / (1.0f + exp_f(-x)); }  // tensor.zig:34

// tensor.zig:9-15
void or_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    const float scale = 1.0f / std::sqrt(ss / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

// moe.zig:106-158 route
// sampler.zig:7-15
size_t or_argmax(const float *logits, size_t n) {
    size_t best = 0;
    float best_v = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (logits[i] > best_v) {
            best_v = logits[i];
            best = i;
        }
    return best;
}

int or_route(const float *logits, const float *bias, size_t n_expert, size_t n_used, int gating,
             int weights_norm, float weights_scale, uint32_t *ids, float *gates) {
    return or_route_grouped(logits, bias, n_expert, n_used, gating, weights_norm, weights_scale, 1, 1, ids, gates);
}

// Group-limited selection (DeepSeek-V3's published routing; the reference has
// no implementation): the n_expert experts form n_group equal groups of
// consecutive ids; a group's score is the sum of its two largest biased
// choices (its one choice when a group holds one expert); the topk_group
// groups with the highest scores are kept (serial first-max scan, lowest
// group index on ties) and every expert outside them is masked to -inf before
// moe.zig's k-round top-k. n_group = 1 (or topk_group = n_group) masks
// nothing, which is exactly moe.zig:106-158 route.
static int or_group_mask(float *choice, size_t n_expert, size_t n_group, size_t topk_group) {
    if (n_group <= 1 || topk_group >= n_group) return 0;
    const size_t gs = n_expert / n_group;
    float gsc[32];
    for (size_t g = 0; g < n_group; g++) {
        float top1 = -INFINITY, top2 = -INFINITY;
        for (size_t e = g * gs; e < (g + 1) * gs; e++) {
            const float c = choice[e];
            if (c > top1) {
                top2 = top1;
                top1 = c;
            } else if (c > top2) {
                top2 = c;
            }
        }
        gsc[g] = gs == 1 ? top1 : top1 + top2;
    }
    uint32_t keep = 0;
    for (size_t k = 0; k < topk_group; k++) {
        int best = -1;
        float bv = -INFINITY;
        for (size_t g = 0; g < n_group; g++) {
            if (keep >> g & 1u) continue;
            if (best < 0 || gsc[g] > bv) {
                best = (int)g;
                bv = gsc[g];
            }
        }
        keep |= 1u << best;
    }
    for (size_t e = 0; e < n_expert; e++)
        if (!(keep >> (e / gs) & 1u)) choice[e] = -INFINITY;
    return 0;
}

int or_route_grouped(const float *logits, const float *bias, size_t n_expert, size_t n_used, int gating,
                     int weights_norm, float weights_scale, size_t n_group, size_t topk_group, uint32_t *ids,
                     float *gates) {
    if (n_expert > 1024 || n_used > 64 || n_used > n_expert) return -1;  // MAX_EXPERTS/MAX_SELECTED, moe.zig:48-49
    if (n_group == 0 || n_group > 32 || n_expert % n_group || topk_group == 0 || topk_group > n_group ||
        n_used > topk_group * (n_expert / n_group))
        return -1;
    float scores[1024], choice[1024];
    bool used[1024] = {};
    if (gating == 2) {
        for (size_t i = 0; i < n_expert; i++) scores[i] = or_sigmoid(logits[i]);
    } else {
        std::memcpy(scores, logits, n_expert * 4);
        if (gating == 1) or_softmax(scores, n_expert);
    }
    std::memcpy(choice, scores, n_expert * 4);
    if (bias)
        for (size_t i = 0; i < n_expert; i++) choice[i] += bias[i];
    or_group_mask(choice, n_expert, n_group, topk_group);
    for (size_t k = 0; k < n_used; k++) {
        size_t best = 0;
        float best_v = -INFINITY;
        for (size_t e = 0; e < n_expert; e++) {
            if (!used[e] && choice[e] > best_v) {
                best_v = choice[e];
                best = e;
            }
        }
        used[best] = true;
        ids[k] = (uint32_t)best;
        gates[k] = scores[best];
    }
    if (gating == 3) or_softmax(gates, n_used);
    if (weights_norm) {
        float sum = 0.0f;
        for (size_t k = 0; k < n_used; k++) sum += gates[k];
        const float denom = std::fmax(sum, 6.103515625e-5f);
        for (size_t k = 0; k < n_used; k++) gates[k] /= denom;
    }
    if (weights_scale != 1.0f)
        for (size_t k = 0; k < n_used; k++) gates[k] *= weights_scale;
    return 0;
}

// llama.zig:952-958 denseFFN then moeRun's `acc += gate * out` (:1397).
static int dense_ffn(const or_expert &e, const float *normed, size_t dim, float *ffn_out,
                     std::vector<float> &g, std::vector<float> &u) {
    g.resize(e.ffn);
    u.resize(e.ffn);
    if (or_matvec(e.gate_type, g.data(), e.gate, normed, e.ffn, dim)) return -1;
    if (or_matvec(e.up_type, u.data(), e.up, normed, e.ffn, dim)) return -1;
    for (size_t i = 0; i < e.ffn; i++) g[i] = or_silu(g[i]) * u[i];  // tensor.zig:53 swiglu
    if (or_matvec(e.down_type, ffn_out, e.down, g.data(), dim, e.ffn)) return -1;
    return 0;
}

int or_moe_ffn_block(const float *normed, size_t dim, const or_expert *experts, size_t n, float *out) {
    std::vector<float> g, u, v(dim);
    for (size_t i = 0; i < dim; i++) out[i] = 0.0f;
    for (size_t k = 0; k < n; k++) {
        if (dense_ffn(experts[k], normed, dim, v.data(), g, u)) return -1;
        for (size_t i = 0; i < dim; i++) out[i] += experts[k].weight * v[i];
    }
    return 0;
}

int or_moe_ffn_routed(const float *normed, size_t dim, const float *logits, const float *bias,
                      int gate_type, const uint8_t *gate3d, int up_type, const uint8_t *up3d,
                      int down_type, const uint8_t *down3d, size_t ffn,
                      const int *shexp_types, const uint8_t *const *shexp, size_t shexp_ffn,
                      size_t n_expert, size_t n_used, int gating_sigmoid, int weights_norm,
                      float weights_scale, float *out) {
    uint32_t ids[64];
    float gates[64];
    if (or_route(logits, bias, n_expert, n_used, gating_sigmoid ? 2 : 1, weights_norm, weights_scale, ids, gates))
        return -1;
    const size_t gp = ffn * or_row_bytes(gate_type, dim);
    const size_t up_ = ffn * or_row_bytes(up_type, dim);
    const size_t dp = dim * or_row_bytes(down_type, ffn);
    std::vector<or_expert> ex(n_used);
    for (size_t k = 0; k < n_used; k++) {
        ex[k] = or_expert{gate_type, up_type, down_type, gate3d + ids[k] * gp, up3d + ids[k] * up_,
                          down3d + ids[k] * dp, gates[k], ffn};
    }
    if (or_moe_ffn_block(normed, dim, ex.data(), n_used, out)) return -1;
    if (shexp) {  // deepseek.zig:1498-1508: shared expert, added plainly
        or_expert se{shexp_types[0], shexp_types[1], shexp_types[2], shexp[0], shexp[1], shexp[2], 1.0f, shexp_ffn};
        std::vector<float> g, u, v(dim);
        if (dense_ffn(se, normed, dim, v.data(), g, u)) return -1;
        for (size_t i = 0; i < dim; i++) out[i] += v[i];
    }
    return 0;
}

int or_moe_layer(const float *x, size_t T, size_t dim, const float *router_w, int gate_type,
                 const uint8_t *gate3d, int up_type, const uint8_t *up3d, int down_type,
                 const uint8_t *down3d, size_t ffn, size_t n_expert, size_t n_used, int gating,
                 int weights_norm, float weights_scale, float *out, uint32_t *ids_out) {
    std::vector<float> logits(n_expert);
    uint32_t ids[64];
    float gates[64];
    const size_t gp = ffn * or_row_bytes(gate_type, dim);
    const size_t up_ = ffn * or_row_bytes(up_type, dim);
    const size_t dp = dim * or_row_bytes(down_type, ffn);
    std::vector<or_expert> ex(n_used);
    for (size_t t = 0; t < T; t++) {
        const float *xt = x + t * dim;
        or_matvec(OR_F32, logits.data(), (const uint8_t *)router_w, xt, n_expert, dim);
        if (or_route(logits.data(), nullptr, n_expert, n_used, gating, weights_norm, weights_scale, ids, gates))
            return -1;
        for (size_t k = 0; k < n_used; k++) {
            if (ids_out) ids_out[t * n_used + k] = ids[k];
            ex[k] = or_expert{gate_type, up_type, down_type, gate3d + ids[k] * gp, up3d + ids[k] * up_,
                              down3d + ids[k] * dp, gates[k], ffn};
        }
        if (or_moe_ffn_block(xt, dim, ex.data(), n_used, out + t * dim)) return -1;
    }
    return 0;
}

// ---- seeded synthetic tensors -------------------------------------------------
// Counter-based: word(seed, i) = splitmix64(seed * K + i). A block b of a
// quantized tensor draws words [b*16, b*16+16)... (see synth_block).

static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline uint64_t word(uint64_t seed, uint64_t i) { return splitmix64(seed * 0xD1B54A32D192ED03ull + i); }
static inline float unit24(uint64_t w) { return (float)(w >> 40) * (1.0f / 16777216.0f); }

uint16_t or_f32_to_f16_rne(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    uint32_t sign = (b >> 16) & 0x8000u;
    int32_t e = (int32_t)((b >> 23) & 0xFF) - 127 + 15;
    uint32_t m = b & 0x7FFFFFu;
    if (e <= 0 || e >= 31) return (uint16_t)sign;  // generator only emits normal halves
    uint32_t h = ((uint32_t)e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}
float or_f16_to_f32(uint16_t h) { return f16_bits_to_f32(h); }

// words per block: enough for the largest block (210 B) plus two scale words
static constexpr uint64_t WPB = 32;

static inline void put_bytes(uint8_t *dst, size_t n, uint64_t seed, uint64_t w0) {
    for (size_t i = 0; i < n; i += 8) {
        uint64_t w = word(seed, w0 + i / 8);
        for (size_t j = 0; j < 8 && i + j < n; j++) dst[i + j] = (uint8_t)(w >> (8 * j));
    }
}
static inline uint16_t rand_scale(uint64_t w, float lo, float span) {
    float u = unit24(w);
    float a = span * u;
    float d = lo + a;
    return or_f32_to_f16_rne(d);
}

void or_synth(int type, void *out, uint64_t blk0, uint64_t nblk, uint64_t seed, float sigma) {
    uint8_t *o = (uint8_t *)out;
    for (uint64_t i = 0; i < nblk; i++) {
        const uint64_t b = blk0 + i;
        const uint64_t w0 = b * WPB;
        switch (type) {
            case OR_F32: {
                uint64_t w[3] = {word(seed, w0), word(seed, w0 + 1), word(seed, w0 + 2)};
                float s = 0.0f;
                for (int k = 0; k < 12; k++) s += (float)((w[k / 4] >> (16 * (k % 4))) & 0xFFFF) * (1.0f / 65536.0f);
                float v = (s - 6.0f) * sigma;
                std::memcpy(o + i * 4, &v, 4);
                break;
            }
            case OR_Q4_K: {
                uint8_t *blk = o + i * Q4_K_BLOCK;
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                uint16_t dm = rand_scale(word(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = dm & 0xFF; blk[3] = dm >> 8;
                put_bytes(blk + 4, 140, seed, w0 + 2);
                break;
            }
            case OR_Q6_K: {
                uint8_t *blk = o + i * Q6_K_BLOCK;
                put_bytes(blk, 192, seed, w0 + 2);
                uint8_t sc[16];
                put_bytes(sc, 16, seed, w0 + 26);
                for (int k = 0; k < 16; k++) blk[192 + k] = (uint8_t)(int8_t)((int)(sc[k] % 64) - 32);
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                blk[208] = d & 0xFF; blk[209] = d >> 8;
                break;
            }
            case OR_Q5_0: {  // f16 d ~U(1e-3, 1e-2), random high bits and nibbles
                uint8_t *blk = o + i * Q5_0_BLOCK;
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8;
                put_bytes(blk + 2, 20, seed, w0 + 2);
                break;
            }
            case OR_Q4_1:
            case OR_Q5_1: {  // f16 d, m ~U(1e-3, 1e-2), random (high bits and) nibbles
                uint8_t *blk = o + i * (type == OR_Q4_1 ? Q4_1_BLOCK : Q5_1_BLOCK);
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                uint16_t m = rand_scale(word(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = m & 0xFF; blk[3] = m >> 8;
                put_bytes(blk + 4, type == OR_Q4_1 ? 16 : 20, seed, w0 + 2);
                break;
            }
            case OR_Q5_K: {  // as Q4_K: f16 d, dmin ~U(1e-3, 1e-2), random scales, high bits and nibbles
                uint8_t *blk = o + i * Q5_K_BLOCK;
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                uint16_t dm = rand_scale(word(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = dm & 0xFF; blk[3] = dm >> 8;
                put_bytes(blk + 4, 172, seed, w0 + 2);
                break;
            }
            case OR_Q2_K: {  // random scale/min nibbles and quants, f16 d, dmin ~U(1e-3, 1e-2)
                uint8_t *blk = o + i * Q2_K_BLOCK;
                put_bytes(blk, 80, seed, w0 + 2);
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                uint16_t dm = rand_scale(word(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[80] = d & 0xFF; blk[81] = d >> 8; blk[82] = dm & 0xFF; blk[83] = dm >> 8;
                break;
            }
            case OR_Q3_K: {  // random high-bit mask, quants and packed 6-bit scales, f16 d ~U(1e-3, 1e-2)
                uint8_t *blk = o + i * Q3_K_BLOCK;
                put_bytes(blk, 108, seed, w0 + 2);
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                blk[108] = d & 0xFF; blk[109] = d >> 8;
                break;
            }
            case OR_Q4_0: {
                uint8_t *blk = o + i * Q4_0_BLOCK;
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 1.9e-2f);
                blk[0] = d & 0xFF; blk[1] = d >> 8;
                put_bytes(blk + 2, 16, seed, w0 + 2);
                break;
            }
            case OR_Q8_0: {
                uint8_t *blk = o + i * Q8_0_BLOCK;
                uint16_t d = rand_scale(word(seed, w0), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8;
                put_bytes(blk + 2, 32, seed, w0 + 2);
                break;
            }
        }
    }
}

}  // extern "C"

// ---- llama.zig:1111-1228 step ---------------------------------------------------

// llama.zig:821-826 ropeTheta
static void rope_theta(size_t i, size_t rope_dim, size_t pos, float base, float &c, float &s) {
    const float exponent = (float)i / (float)rope_dim;
    const float freq = std::pow(base, -exponent);
    const float angle = (float)pos * freq;
    c = std::cos(angle);
    s = std::sin(angle);
}

// llama.zig:830-839 ropeNorm (adjacent pairs) and :845-856 ropeNeox (split halves)
static void rope_apply(int neox, float *vec, size_t rope_dim, size_t pos, float base) {
    if (neox) {
        const size_t half = rope_dim / 2;
        for (size_t i = 0; i < half; i++) {
            float c, s;
            rope_theta(2 * i, rope_dim, pos, base, c, s);
            const float a = vec[i], b = vec[i + half];
            vec[i] = a * c - b * s;
            vec[i + half] = a * s + b * c;
        }
    } else {
        for (size_t i = 0; i + 1 < rope_dim; i += 2) {
            float c, s;
            rope_theta(i, rope_dim, pos, base, c, s);
            const float a = vec[i], b = vec[i + 1];
            vec[i] = a * c - b * s;
            vec[i + 1] = a * s + b * c;
        }
    }
}

// llama.zig:938-950 headNorm
static void head_norm(float *vec, const float *g, size_t n_heads, size_t hd, float eps) {
    if (!g) return;
    for (size_t h = 0; h < n_heads; h++) {
        float *head = vec + h * hd;
        float ss = 0.0f;
        for (size_t i = 0; i < hd; i++) ss += head[i] * head[i];
        const float inv = 1.0f / std::sqrt(ss / (float)hd + eps);
        for (size_t i = 0; i < hd; i++) head[i] = head[i] * inv * g[i];
    }
}

// ggml.zig:222-231 axpy (elementwise, no contraction)
static void axpy(float *out, const float *v, float w, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = out[i] + w * v[i];
}

int or_llama_step(const or_llama_model *m, float *k_cache, float *v_cache, uint32_t token, size_t pos,
                  float *logits) {
    const size_t dim = m->dim, hd = m->head_dim, nh = m->n_heads, nkv = m->n_kv_heads;
    if (token >= m->vocab || pos >= m->ctx_len || nkv == 0 || nh % nkv) return -1;
    const size_t kvd = nkv * hd, qd = nh * hd, q_per_kv = nh / nkv;
    const float scale = m->attn_logit_mul / std::sqrt((float)hd);
    std::vector<float> x(dim), normed(dim), q(qd), k(kvd), v(kvd), att(qd), proj(dim), scores(pos + 1), acc(dim);
    if (or_dequant_row(m->embd_type, x.data(), m->token_embd, token, dim)) return -1;  // :1122
    for (size_t li = 0; li < m->n_layers; li++) {
        const or_llama_layer &l = m->layers[li];
        or_rmsnorm(normed.data(), x.data(), l.attn_norm, dim, m->eps);               // :1139
        if (or_matvec(l.wq_type, q.data(), l.wq, normed.data(), qd, dim)) return -1;  // :1140-1142
        if (or_matvec(l.wk_type, k.data(), l.wk, normed.data(), kvd, dim)) return -1;
        if (or_matvec(l.wv_type, v.data(), l.wv, normed.data(), kvd, dim)) return -1;
        head_norm(q.data(), l.q_norm, nh, hd, m->eps);                               // :1148-1149
        head_norm(k.data(), l.k_norm, nkv, hd, m->eps);
        for (size_t h = 0; h < nh; h++) rope_apply(m->rope_neox, q.data() + h * hd, m->rope_dim, pos, m->rope_base);
        for (size_t h = 0; h < nkv; h++) rope_apply(m->rope_neox, k.data() + h * hd, m->rope_dim, pos, m->rope_base);
        const size_t base = (li * m->ctx_len + pos) * kvd;                            // :1157
        std::memcpy(k_cache + base, k.data(), kvd * 4);
        std::memcpy(v_cache + base, v.data(), kvd * 4);
        const size_t seq = pos + 1;
        for (size_t h = 0; h < nh; h++) {                                             // :1171-1191
            const size_t kvh = h / q_per_kv;
            const float *qh = q.data() + h * hd;
            for (size_t t = 0; t < seq; t++)
                scores[t] = or_dot_f32(qh, k_cache + (li * m->ctx_len + t) * kvd + kvh * hd, hd) * scale;
            or_softmax(scores.data(), seq);
            float *oh = att.data() + h * hd;
            for (size_t i = 0; i < hd; i++) oh[i] = 0.0f;
            for (size_t t = 0; t < seq; t++) axpy(oh, v_cache + (li * m->ctx_len + t) * kvd + kvh * hd, scores[t], hd);
        }
        if (or_matvec(l.wo_type, proj.data(), l.wo, att.data(), dim, qd)) return -1;  // :1193
        for (size_t i = 0; i < dim; i++) x[i] += proj[i];                             // :1195
        or_rmsnorm(normed.data(), x.data(), l.ffn_norm, dim, m->eps);                 // :1216/:1222
        if (!l.router) {  // :1212-1218 denseFFN then add
            or_expert e{l.gate_type, l.up_type, l.down_type, l.gate, l.up, l.down, 1.0f, l.ffn};
            std::vector<float> g, u;
            if (dense_ffn(e, normed.data(), dim, acc.data(), g, u)) return -1;
        } else {  // :1224 moeLayer, then add(x, moe_acc)
            if (or_moe_layer(normed.data(), 1, dim, l.router, l.gate_type, l.gate, l.up_type, l.up, l.down_type,
                             l.down, l.ffn, m->n_expert, m->n_used, m->gating, m->weights_norm, m->weights_scale,
                             acc.data(), nullptr))
                return -1;
        }
        for (size_t i = 0; i < dim; i++) x[i] += acc[i];
    }
    or_rmsnorm(normed.data(), x.data(), m->output_norm, dim, m->eps);                 // :1226-1227
    return or_matvec(m->output_type, logits, m->output, normed.data(), m->vocab, dim);
}

// ---- deepseek.zig:1275-1537 step, attnLayer :851-1049 -----------------------------

// deepseek.zig:615-629 ropeNormPlain (adjacent pairs over the whole vector)
static void rope_norm_plain(float *vec, size_t n, size_t pos, float base) {
    for (size_t i = 0; 2 * i + 1 < n; i++) {
        float c, s;
        rope_theta(2 * i, n, pos, base, c, s);
        const float a = vec[2 * i], b = vec[2 * i + 1];
        vec[2 * i] = a * c - b * s;
        vec[2 * i + 1] = a * s + b * c;
    }
}

int or_deepseek_step(const or_ds_model *m, float *c_cache, float *r_cache, uint32_t token, size_t pos,
                     float *logits) {
    const size_t dim = m->dim, nh = m->n_heads, nope = m->nope, rope = m->rope, kvr = m->kv_lora, vd = m->v_head;
    const size_t kd = nope + rope;
    if (token >= m->vocab || pos >= m->ctx_len) return -1;
    std::vector<float> x(dim), normed(dim), q(nh * kd), qa_lat(m->q_lora ? m->q_lora : 1), kv_a(kvr + rope),
        qabs(nh * kvr), row(kvr), scores(pos + 1), c_acc(kvr), head_out(nh * vd), proj(dim), acc(dim), v(dim);
    if (or_dequant_row(m->embd_type, x.data(), m->token_embd, token, dim)) return -1;  // :1292
    for (size_t li = 0; li < m->n_layers; li++) {
        const or_ds_layer &l = m->layers[li];
        or_rmsnorm(normed.data(), x.data(), l.attn_norm, dim, m->eps);  // :860
        if (m->q_lora) {                                                // :862-865
            if (or_matvec(l.q_a_type, qa_lat.data(), l.q_a, normed.data(), m->q_lora, dim)) return -1;
            or_rmsnorm(qa_lat.data(), qa_lat.data(), l.q_a_norm, m->q_lora, m->eps);
            if (or_matvec(l.q_b_type, q.data(), l.q_b, qa_lat.data(), nh * kd, m->q_lora)) return -1;
        } else if (or_matvec(l.wq_type, q.data(), l.wq, normed.data(), nh * kd, dim)) {
            return -1;
        }
        if (or_matvec(l.kv_a_type, kv_a.data(), l.kv_a, normed.data(), kvr + rope, dim)) return -1;  // :870
        float *c_kv = c_cache + (li * m->ctx_len + pos) * kvr;
        or_rmsnorm(c_kv, kv_a.data(), l.kv_a_norm, kvr, m->eps);                                    // :872
        float *k_rope = r_cache + (li * m->ctx_len + pos) * rope;
        std::memcpy(k_rope, kv_a.data() + kvr, rope * 4);
        rope_norm_plain(k_rope, rope, pos, m->rope_base);                                           // :875
        for (size_t h = 0; h < nh; h++) rope_norm_plain(q.data() + h * kd + nope, rope, pos, m->rope_base);
        const size_t seq = pos + 1;
        const size_t kb_rb = or_row_bytes(l.kv_b_type, kvr);
        for (size_t h = 0; h < nh; h++) {  // :944-958 absorb: qa = sum_r q_nope[r] * W_k row r
            float *qa = qabs.data() + h * kvr;
            for (size_t j = 0; j < kvr; j++) qa[j] = 0.0f;
            const uint8_t *k_rows = l.kv_b + h * (nope + vd) * kb_rb;
            for (size_t r = 0; r < nope; r++) {
                if (or_dequant_row(l.kv_b_type, row.data(), k_rows, r, kvr)) return -1;
                axpy(qa, row.data(), q[h * kd + r], kvr);
            }
        }
        for (size_t h = 0; h < nh; h++) {  // :966-986 scores, softmax, weighted sum in compressed space
            const float *qa = qabs.data() + h * kvr, *qr = q.data() + h * kd + nope;
            for (size_t t = 0; t < seq; t++) {
                const float *c_t = c_cache + (li * m->ctx_len + t) * kvr;
                const float *kr_t = r_cache + (li * m->ctx_len + t) * rope;
                scores[t] = (or_dot_f32(qa, c_t, kvr) + or_dot_f32(qr, kr_t, rope)) * m->attn_scale;
            }
            or_softmax(scores.data(), seq);
            for (size_t j = 0; j < kvr; j++) c_acc[j] = 0.0f;
            for (size_t t = 0; t < seq; t++) axpy(c_acc.data(), c_cache + (li * m->ctx_len + t) * kvr, scores[t], kvr);
            // :988 W_v applied once per head
            if (or_matvec(l.kv_b_type, head_out.data() + h * vd, l.kv_b + (h * (nope + vd) + nope) * kb_rb,
                          c_acc.data(), vd, kvr))
                return -1;
        }
        if (or_matvec(l.wo_type, proj.data(), l.wo, head_out.data(), dim, nh * vd)) return -1;  // :991
        for (size_t i = 0; i < dim; i++) x[i] += proj[i];
        or_rmsnorm(normed.data(), x.data(), l.ffn_norm, dim, m->eps);  // :1326
        if (!l.router) {                                               // :1328-1330 dense
            or_expert e{l.gate_type, l.up_type, l.down_type, l.gate, l.up, l.down, 1.0f, l.ffn};
            std::vector<float> g, u;
            if (dense_ffn(e, normed.data(), dim, acc.data(), g, u)) return -1;
        } else {  // :1332-1507 router, route, experts in selection order, shared expert added
            std::vector<float> lg(m->n_expert);
            if (or_matvec(OR_F32, lg.data(), (const uint8_t *)l.router, normed.data(), m->n_expert, dim)) return -1;
            uint32_t ids[64];
            float gates[64];
            if (or_route_grouped(lg.data(), l.router_bias, m->n_expert, m->n_used, m->gating_sigmoid ? 2 : 1,
                                 m->weights_norm, m->weights_scale, m->n_group ? m->n_group : 1,
                                 m->topk_group ? m->topk_group : 1, ids, gates))
                return -1;
            const size_t gp = l.ffn * or_row_bytes(l.gate_type, dim), upb = l.ffn * or_row_bytes(l.up_type, dim);
            const size_t dp = dim * or_row_bytes(l.down_type, l.ffn);
            std::vector<or_expert> ex(m->n_used);
            for (size_t k = 0; k < m->n_used; k++)
                ex[k] = or_expert{l.gate_type, l.up_type, l.down_type, l.gate + ids[k] * gp, l.up + ids[k] * upb,
                                  l.down + ids[k] * dp, gates[k], l.ffn};
            if (or_moe_ffn_block(normed.data(), dim, ex.data(), m->n_used, acc.data())) return -1;
            if (l.sh_gate) {  // deepseek.zig:1498-1508: shared expert added plainly
                or_expert se{l.sh_gate_type, l.sh_up_type, l.sh_down_type, l.sh_gate, l.sh_up, l.sh_down, 1.0f,
                             l.sh_ffn};
                std::vector<float> g, u;
                if (dense_ffn(se, normed.data(), dim, v.data(), g, u)) return -1;
                for (size_t i = 0; i < dim; i++) acc[i] += v[i];
            }
        }
        for (size_t i = 0; i < dim; i++) x[i] += acc[i];
    }
    or_rmsnorm(normed.data(), x.data(), m->output_norm, dim, m->eps);
    return or_matvec(m->output_type, logits, m->output, normed.data(), m->vocab, dim);
}
