// kernels.cu -- dequant, activation quantization, matvec/matmul, router and
// the MoE expert kernels of the CUDA backend (sm_100a).
#include <atomic>

#include "kernels.cuh"
#include "rowdot.cuh"
#include "devutil.cuh"

namespace loom {

static std::atomic<uint64_t> g_launches{0};
uint64_t launches() { return g_launches.load(); }
void count_launch() { g_launches.fetch_add(1); }
void count_launches(uint64_t n) { g_launches.fetch_add(n); }

static inline unsigned cdiv(uint64_t a, uint64_t b) { return (unsigned)((a + b - 1) / b); }

// ---- seeded synthetic tensors ---------------------------------------------------
// Counter-based generator: word(seed, i) = splitmix64(seed*K + i); block b draws
// words [32b, 32b+32). The host-side test oracle implements the same function,
// so any sampled block can be regenerated on the CPU bit for bit.

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t rword(uint64_t seed, uint64_t i) {
    return splitmix64(seed * 0xD1B54A32D192ED03ull + i);
}
__device__ __forceinline__ float unit24(uint64_t w) { return (float)(w >> 40) * (1.0f / 16777216.0f); }

// f32 -> f16 round-to-nearest-even for positive normal-range values (the
// generator's scale ranges); integer arithmetic, identical on host and device.
__device__ __forceinline__ uint16_t f32_to_f16_rne(float f) {
    uint32_t b = __float_as_uint(f);
    uint32_t sign = (b >> 16) & 0x8000u;
    int32_t e = (int32_t)((b >> 23) & 0xFF) - 127 + 15;
    uint32_t m = b & 0x7FFFFFu;
    if (e <= 0 || e >= 31) return (uint16_t)sign;
    uint32_t h = ((uint32_t)e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}
__device__ __forceinline__ uint16_t rand_scale(uint64_t w, float lo, float span) {
    return f32_to_f16_rne(fadd(lo, fmul(span, unit24(w))));
}
__device__ __forceinline__ void put_bytes(uint8_t *dst, int n, uint64_t seed, uint64_t w0) {
    for (int i = 0; i < n; i += 8) {
        uint64_t w = rword(seed, w0 + i / 8);
        for (int j = 0; j < 8 && i + j < n; j++) dst[i + j] = (uint8_t)(w >> (8 * j));
    }
}

__global__ void k_synth(int type, uint8_t *raw, uint64_t blk0, uint64_t nblk, uint64_t seed, float sigma) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nblk; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = blk0 + i;
        const uint64_t w0 = b * 32;
        switch (type) {
            case T_F32: {
                uint64_t w[3] = {rword(seed, w0), rword(seed, w0 + 1), rword(seed, w0 + 2)};
                float s = 0.0f;
                for (int k = 0; k < 12; k++) s = fadd(s, (float)((w[k / 4] >> (16 * (k % 4))) & 0xFFFF) * (1.0f / 65536.0f));
                reinterpret_cast<float *>(raw)[i] = fmul(fsub(s, 6.0f), sigma);
                break;
            }
            case T_Q4_K: {
                uint8_t *blk = raw + i * 144;
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                uint16_t dm = rand_scale(rword(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = dm & 0xFF; blk[3] = dm >> 8;
                put_bytes(blk + 4, 140, seed, w0 + 2);
                break;
            }
            case T_Q6_K: {
                uint8_t *blk = raw + i * 210;
                put_bytes(blk, 192, seed, w0 + 2);
                uint8_t sc[16];
                put_bytes(sc, 16, seed, w0 + 26);
                for (int k = 0; k < 16; k++) blk[192 + k] = (uint8_t)(int8_t)((int)(sc[k] % 64) - 32);
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                blk[208] = d & 0xFF; blk[209] = d >> 8;
                break;
            }
            case T_Q5_0: {
                uint8_t *blk = raw + i * 22;
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8;
                put_bytes(blk + 2, 20, seed, w0 + 2);
                break;
            }
            case T_Q4_1:
            case T_Q5_1: {
                uint8_t *blk = raw + i * (type == T_Q4_1 ? 20 : 24);
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                uint16_t m = rand_scale(rword(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = m & 0xFF; blk[3] = m >> 8;
                put_bytes(blk + 4, type == T_Q4_1 ? 16 : 20, seed, w0 + 2);
                break;
            }
            case T_Q5_K: {
                uint8_t *blk = raw + i * 176;
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                uint16_t dm = rand_scale(rword(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = dm & 0xFF; blk[3] = dm >> 8;
                put_bytes(blk + 4, 172, seed, w0 + 2);
                break;
            }
            case T_Q2_K: {
                uint8_t *blk = raw + i * 84;
                put_bytes(blk, 80, seed, w0 + 2);
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                uint16_t dm = rand_scale(rword(seed, w0 + 1), 1e-3f, 9e-3f);
                blk[80] = d & 0xFF; blk[81] = d >> 8; blk[82] = dm & 0xFF; blk[83] = dm >> 8;
                break;
            }
            case T_Q3_K: {
                uint8_t *blk = raw + i * 110;
                put_bytes(blk, 108, seed, w0 + 2);
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                blk[108] = d & 0xFF; blk[109] = d >> 8;
                break;
            }
            case T_Q4_0: {
                uint8_t *blk = raw + i * 18;
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 1.9e-2f);
                blk[0] = d & 0xFF; blk[1] = d >> 8;
                put_bytes(blk + 2, 16, seed, w0 + 2);
                break;
            }
            case T_Q8_0: {
                uint8_t *blk = raw + i * 34;
                uint16_t d = rand_scale(rword(seed, w0), 1e-3f, 9e-3f);
                blk[0] = d & 0xFF; blk[1] = d >> 8;
                put_bytes(blk + 2, 32, seed, w0 + 2);
                break;
            }
        }
    }
}

void launch_synth(int type, uint8_t *raw, uint64_t blk0, uint64_t nblk, uint64_t seed, float sigma, cudaStream_t st) {
    if (nblk == 0) return;
    unsigned g = cdiv(nblk, 256);
    if (g > 148 * 64) g = 148 * 64;
    k_synth<<<g, 256, 0, st>>>(type, raw, blk0, nblk, seed, sigma);
    count_launch();
}

// ---- GGUF bytes <-> device layout ------------------------------------------------

__global__ void k_repack(int type, const uint8_t *raw, uint8_t *q, uint8_t *sc, uint16_t *d, uint64_t nblk) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblk; b += (uint64_t)gridDim.x * blockDim.x) {
        switch (type) {
            case T_Q6_K: {
                const uint8_t *src = raw + b * 210;
                for (int i = 0; i < 192; i++) q[b * 192 + i] = src[i];
                for (int i = 0; i < 16; i++) sc[b * 16 + i] = src[192 + i];
                d[b] = (uint16_t)(src[208] | (src[209] << 8));
                break;
            }
            case T_Q8_0: {
                const uint8_t *src = raw + b * 34;
                d[b] = (uint16_t)(src[0] | (src[1] << 8));
                for (int i = 0; i < 32; i++) q[b * 32 + i] = src[2 + i];
                break;
            }
            case T_Q5_0: {  // quants | d | the 32 high bits
                const uint8_t *src = raw + b * 22;
                d[b] = (uint16_t)(src[0] | (src[1] << 8));
                for (int i = 0; i < 4; i++) sc[b * 4 + i] = src[2 + i];
                for (int i = 0; i < 16; i++) q[b * 16 + i] = src[6 + i];
                break;
            }
            case T_Q4_1:
            case T_Q5_1: {  // quants | d, m | (Q5_1) the 32 high bits
                const uint8_t *src = raw + b * (type == T_Q4_1 ? 20 : 24);
                const int qo = type == T_Q4_1 ? 4 : 8;
                for (int i = 0; i < 16; i++) q[b * 16 + i] = src[qo + i];
                d[2 * b] = (uint16_t)(src[0] | (src[1] << 8));
                d[2 * b + 1] = (uint16_t)(src[2] | (src[3] << 8));
                if (type == T_Q5_1)
                    for (int i = 0; i < 4; i++) sc[b * 4 + i] = src[4 + i];
                break;
            }
            case T_Q2_K: {  // scales + quants | d, dmin
                const uint8_t *src = raw + b * 84;
                for (int i = 0; i < 80; i++) q[b * 80 + i] = src[i];
                d[2 * b] = (uint16_t)(src[80] | (src[81] << 8));
                d[2 * b + 1] = (uint16_t)(src[82] | (src[83] << 8));
                break;
            }
            case T_Q3_K: {  // high-bit mask + quants | packed scales (12 of 16 bytes) | d
                const uint8_t *src = raw + b * 110;
                for (int i = 0; i < 96; i++) q[b * 96 + i] = src[i];
                for (int i = 0; i < 16; i++) sc[b * 16 + i] = i < 12 ? src[96 + i] : 0;
                d[b] = (uint16_t)(src[108] | (src[109] << 8));
                break;
            }
            case T_Q4_0: {
                const uint8_t *src = raw + b * 18;
                d[b] = (uint16_t)(src[0] | (src[1] << 8));
                for (int i = 0; i < 16; i++) q[b * 16 + i] = src[2 + i];
                break;
            }
        }
    }
}

void launch_repack(int type, const uint8_t *raw, uint8_t *q, uint8_t *sc, uint16_t *d, uint64_t nblk, cudaStream_t st) {
    if (nblk == 0) return;
    unsigned g = cdiv(nblk, 256);
    if (g > 148 * 64) g = 148 * 64;
    k_repack<<<g, 256, 0, st>>>(type, raw, q, sc, d, nblk);
    count_launch();
}

__global__ void k_unpack(WDev w, uint8_t *raw, uint64_t nblk) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblk; b += (uint64_t)gridDim.x * blockDim.x) {
        switch (w.type) {
            case T_Q4_K:
                for (int i = 0; i < 144; i++) raw[b * 144 + i] = w.q[b * 144 + i];
                break;
            case T_Q5_K:
                for (int i = 0; i < 176; i++) raw[b * 176 + i] = w.q[b * 176 + i];
                break;
            case T_Q5_0: {
                uint8_t *dst = raw + b * 22;
                dst[0] = w.d[b] & 0xFF;
                dst[1] = w.d[b] >> 8;
                for (int i = 0; i < 4; i++) dst[2 + i] = w.sc[b * 4 + i];
                for (int i = 0; i < 16; i++) dst[6 + i] = w.q[b * 16 + i];
                break;
            }
            case T_Q4_1:
            case T_Q5_1: {
                const bool q5 = w.type == T_Q5_1;
                uint8_t *dst = raw + b * (q5 ? 24 : 20);
                dst[0] = w.d[2 * b] & 0xFF;
                dst[1] = w.d[2 * b] >> 8;
                dst[2] = w.d[2 * b + 1] & 0xFF;
                dst[3] = w.d[2 * b + 1] >> 8;
                if (q5)
                    for (int i = 0; i < 4; i++) dst[4 + i] = w.sc[b * 4 + i];
                for (int i = 0; i < 16; i++) dst[(q5 ? 8 : 4) + i] = w.q[b * 16 + i];
                break;
            }
            case T_Q2_K: {
                uint8_t *dst = raw + b * 84;
                for (int i = 0; i < 80; i++) dst[i] = w.q[b * 80 + i];
                dst[80] = w.d[2 * b] & 0xFF;
                dst[81] = w.d[2 * b] >> 8;
                dst[82] = w.d[2 * b + 1] & 0xFF;
                dst[83] = w.d[2 * b + 1] >> 8;
                break;
            }
            case T_Q3_K: {
                uint8_t *dst = raw + b * 110;
                for (int i = 0; i < 96; i++) dst[i] = w.q[b * 96 + i];
                for (int i = 0; i < 12; i++) dst[96 + i] = w.sc[b * 16 + i];
                dst[108] = w.d[b] & 0xFF;
                dst[109] = w.d[b] >> 8;
                break;
            }
            case T_Q6_K: {
                uint8_t *dst = raw + b * 210;
                for (int i = 0; i < 192; i++) dst[i] = w.q[b * 192 + i];
                for (int i = 0; i < 16; i++) dst[192 + i] = w.sc[b * 16 + i];
                dst[208] = w.d[b] & 0xFF;
                dst[209] = w.d[b] >> 8;
                break;
            }
            case T_Q8_0: {
                uint8_t *dst = raw + b * 34;
                dst[0] = w.d[b] & 0xFF;
                dst[1] = w.d[b] >> 8;
                for (int i = 0; i < 32; i++) dst[2 + i] = w.q[b * 32 + i];
                break;
            }
            case T_Q4_0: {
                uint8_t *dst = raw + b * 18;
                dst[0] = w.d[b] & 0xFF;
                dst[1] = w.d[b] >> 8;
                for (int i = 0; i < 16; i++) dst[2 + i] = w.q[b * 16 + i];
                break;
            }
        }
    }
}

void launch_unpack(int type, const WDev &w, uint8_t *raw, uint64_t nblk, cudaStream_t st) {
    (void)type;
    if (nblk == 0) return;
    unsigned g = cdiv(nblk, 256);
    if (g > 148 * 64) g = 148 * 64;
    k_unpack<<<g, 256, 0, st>>>(w, raw, nblk);
    count_launch();
}

// ---- dequant (bit-exact with dequantRow, ggml.zig:1739-1857) -----------------------

// element i of global block gb (bit-exact with dequantRow)
__device__ __forceinline__ float dequant_at(const WDev &w, uint64_t gb, int i) {
    float v = 0.0f;
    switch (w.type) {
        case T_F32:
            v = reinterpret_cast<const float *>(w.q)[gb];
            break;
        case T_Q4_K: {  // dequantBlockQ4K :1342: (d*sc)*q - (dmin*m)
            const uint8_t *blk = w.q + gb * 144;
            const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const float dmin = f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const int j = i / 64, l = i % 64;
            const int sb = 2 * j + (l >= 32);
            const uint8_t byte = blk[16 + 32 * j + (l & 31)];
            const int q = l < 32 ? (byte & 0x0F) : (byte >> 4);
            int sc, mn;
            scale_min_k4(sb, blk + 4, sc, mn);
            v = fsub(fmul(fmul(d, (float)sc), (float)q), fmul(dmin, (float)mn));
            break;
        }
        case T_Q6_K: {  // dequantBlockQ6K :1420: (d*sc)*(q-32)
            const uint8_t *qb = w.q + gb * 192;
            const int8_t *scs = reinterpret_cast<const int8_t *>(w.sc + gb * 16);
            const float d = f16_to_f32(w.d[gb]);
            const int n = i / 128, r = i % 128, g = r / 32, l = r % 32;
            const uint8_t a = qb[64 * n + l], bb = qb[64 * n + 32 + l], h = qb[128 + 32 * n + l];
            int q;
            switch (g) {
                case 0: q = (a & 0x0F) | ((h & 3) << 4); break;
                case 1: q = (bb & 0x0F) | (((h >> 2) & 3) << 4); break;
                case 2: q = (a >> 4) | (((h >> 4) & 3) << 4); break;
                default: q = (bb >> 4) | (((h >> 6) & 3) << 4); break;
            }
            const float s = fmul(d, (float)scs[8 * n + l / 16 + 2 * g]);
            v = fmul(s, fsub((float)q, 32.0f));
            break;
        }
        case T_Q5_0: {  // dequantRow :1772: (q - 16) * d
            const uint8_t byte = w.q[gb * 16 + (i & 15)];
            const uint32_t qh = (uint32_t)w.sc[gb * 4] | ((uint32_t)w.sc[gb * 4 + 1] << 8) |
                                ((uint32_t)w.sc[gb * 4 + 2] << 16) | ((uint32_t)w.sc[gb * 4 + 3] << 24);
            const int q = (i < 16 ? (byte & 0x0F) : (byte >> 4)) | (int)((qh >> i) & 1) << 4;
            v = fmul((float)(q - 16), f16_to_f32(w.d[gb]));
            break;
        }
        case T_Q4_1:
        case T_Q5_1: {  // dequantRow :1795: q*d + m
            const uint8_t byte = w.q[gb * 16 + (i & 15)];
            int q = i < 16 ? (byte & 0x0F) : (byte >> 4);
            if (w.type == T_Q5_1) {
                const uint32_t qh = (uint32_t)w.sc[gb * 4] | ((uint32_t)w.sc[gb * 4 + 1] << 8) |
                                    ((uint32_t)w.sc[gb * 4 + 2] << 16) | ((uint32_t)w.sc[gb * 4 + 3] << 24);
                q |= (int)((qh >> i) & 1) << 4;  // value i < 16: bit i; value 16 + j: bit 16 + j
            }
            v = fadd(fmul((float)q, f16_to_f32(w.d[2 * gb])), f16_to_f32(w.d[2 * gb + 1]));
            break;
        }
        case T_Q5_K: {  // dequantBlockQ5K :1376: (d*sc)*(q + 16 h) - (dmin*m)
            const uint8_t *blk = w.q + gb * 176;
            const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const float dmin = f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const int j = i / 64, l = i % 64, sb = 2 * j + (l >= 32);
            const uint8_t byte = blk[48 + 32 * j + (l & 31)];
            const int q = l < 32 ? (byte & 0x0F) : (byte >> 4);
            const bool hb = (blk[16 + (l & 31)] >> sb) & 1;
            int sc, mn;
            scale_min_k4(sb, blk + 4, sc, mn);
            v = fsub(fmul(fmul(d, (float)sc), fadd((float)q, hb ? 16.0f : 0.0f)), fmul(dmin, (float)mn));
            break;
        }
        case T_Q2_K: {  // dequantBlockQ2K :1476: (d*sc)*q - (dmin*m), sub-block j = i / 16
            const uint8_t *qb = w.q + gb * 80;
            const float d = f16_to_f32(w.d[2 * gb]), dmin = f16_to_f32(w.d[2 * gb + 1]);
            const int g = i / 32, l = i % 32, j = i / 16;
            const uint8_t sc = qb[j];
            const int q = (qb[16 + 32 * (g / 4) + l] >> (2 * (g % 4))) & 3;
            v = fsub(fmul(fmul(d, (float)(sc & 0xF)), (float)q), fmul(dmin, (float)(sc >> 4)));
            break;
        }
        case T_Q3_K: {  // dequantBlockQ3K :1508: (d*(sc-32))*(q - 4 [high bit clear])
            const uint8_t *qb = w.q + gb * 96;
            const int g = i / 32, l = i % 32, j = i / 16;
            const int q2 = (qb[32 + 32 * (g / 4) + l] >> (2 * (g % 4))) & 3;
            const int off = (qb[l] >> g) & 1 ? 0 : 4;
            v = fmul(fmul(f16_to_f32(w.d[gb]), (float)(q3k_scale(w.sc + gb * 16, j) - 32)), (float)(q2 - off));
            break;
        }
        case T_Q4_0: {
            const uint8_t byte = w.q[gb * 16 + (i & 15)];
            const int q = i < 16 ? (byte & 0x0F) : (byte >> 4);
            v = fmul((float)(q - 8), f16_to_f32(w.d[gb]));
            break;
        }
        case T_Q8_0:
            v = fmul((float)(int8_t)w.q[gb * 32 + i], f16_to_f32(w.d[gb]));
            break;
    }
    return v;
}

__global__ void k_dequant(WDev w, uint64_t gb0, uint64_t nelem, float *out) {
    const int be = block_elems(w.type);
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < nelem; e += (uint64_t)gridDim.x * blockDim.x)
        out[e] = dequant_at(w, gb0 + e / be, (int)(e % be));
}

// Embedding lookup (llama.zig:1122 dequantRow of token_embd) of the token held
// in device memory; an id >= vocab reads row vocab - 1 (the caller's contract
// is id < vocab; this only keeps the read inside the tensor).
// row blockIdx.y: token tok[y] into x + y * dim (one row per token of a batch)
__global__ void k_embed(WDev w, int dim, const uint32_t *tok, int vocab, float *x) {
    x += (size_t)blockIdx.y * dim;
    const uint32_t t = min(tok[blockIdx.y], (uint32_t)(vocab - 1));
    const int be = block_elems(w.type);
    const uint64_t gb0 = (uint64_t)t * (dim / be);
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x)
        x[e] = dequant_at(w, gb0 + e / be, e % be);
}

void launch_embed(const WDev &w, int dim, const uint32_t *tok, int vocab, float *x, cudaStream_t st, int ntok) {
    k_embed<<<dim3(cdiv(dim, 256), ntok), 256, 0, st>>>(w, dim, tok, vocab, x);
    count_launch();
}

// MLA absorption (deepseek.zig:944-958): for head h and latent column j,
// qa[h][j] = sum over r < nope, in order from +0, of q[h*kd + r] * W[h*(nope+vd) + r][j]
// (axpy of each dequantized W_k row, exact dequantRow values), W = attn_kv_b [nh*(nope+vd)][kvr].
constexpr int MLA_AB_COLS = 64;  // latent columns per CTA of k_mla_absorb
__global__ void __launch_bounds__(512) k_mla_absorb(WDev w, int kvr, int nope, int vd, int kd, const float *q, float *qa) {
    // this CTA: head h, latent columns [j0, j0 + 64); every W_k value it needs dequantized into
    // shared memory by all threads at once, then each column's sum over the rows in order
    extern __shared__ float wk_s[];  // [nope][64], then the head's q rows [nope]
    const int h = blockIdx.y, j0 = blockIdx.x * MLA_AB_COLS, tid = threadIdx.x;
    const int be = block_elems(w.type), nb = kvr / be, nc = min(MLA_AB_COLS, kvr - j0);
    float *qs = wk_s + nope * MLA_AB_COLS;
    for (int i = tid; i < nope * MLA_AB_COLS; i += blockDim.x) {
        const int r = i / MLA_AB_COLS, jj = i % MLA_AB_COLS, j = j0 + jj;
        const uint64_t row = (uint64_t)h * (nope + vd) + r;
        wk_s[i] = jj < nc ? dequant_at(w, row * nb + j / be, j % be) : 0.0f;
    }
    for (int r = tid; r < nope; r += blockDim.x) qs[r] = __ldg(q + (size_t)h * kd + r);
    __syncthreads();
    if (tid < nc) {
        float a = 0.0f;
#pragma unroll 8
        for (int r = 0; r < nope; r++) a = fadd(a, fmul(qs[r], wk_s[r * MLA_AB_COLS + tid]));
        qa[(size_t)h * kvr + j0 + tid] = a;
    }
}

// W_v per head (deepseek.zig:988): out[h*vd + r] = W[h*(nope+vd) + nope + r] . c_h, the
// bit-exact quantized row dot of the tensor's type against head h's activation
// (token h of x).
__global__ void __launch_bounds__(256) k_mla_wv(WDev w, int nope, int vd, int nb, int n_heads, XQ x, float *out) {
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (i >= n_heads * vd) return;
    const int h = i / vd, r = i % vd;
    float acc[1] = {0.0f};
    rowdot<1>(w, ((uint64_t)h * (nope + vd) + nope + r) * nb, nb, x, h, 1, acc, lane);
    if (lane == 0) out[i] = acc[0];
}

void launch_mla_absorb(const WDev &w, int kvr, int nope, int vd, int kd, int n_heads, const float *q, float *qa,
                       cudaStream_t st) {
    const size_t smem = (size_t)nope * (MLA_AB_COLS + 1) * 4;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k_mla_absorb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_mla_absorb<<<dim3(cdiv(kvr, MLA_AB_COLS), n_heads), 512, smem, st>>>(w, kvr, nope, vd, kd, q, qa);
    count_launch();
}

void launch_mla_wv(const WDev &w, int kvr, int nope, int vd, int n_heads, const XQ &x, float *out, cudaStream_t st) {
    const int nb = kvr / block_elems(w.type);
    k_mla_wv<<<cdiv((uint64_t)n_heads * vd, 8), 256, 0, st>>>(w, nope, vd, nb, n_heads, x, out);
    count_launch();
}

void launch_dequant(const WDev &w, uint64_t gb0, uint64_t nblk, float *out, cudaStream_t st) {
    const uint64_t n = nblk * (uint64_t)block_elems(w.type);
    if (n == 0) return;
    unsigned g = cdiv(n, 256);
    if (g > 148 * 64) g = 148 * 64;
    k_dequant<<<g, 256, 0, st>>>(w, gb0, n, out);
    count_launch();
}

// ---- activation quantization (quantizeX256 :776 / quantizeX :1077) ---------------
// Each lane holds 8 consecutive values. 256-wide blocks: one warp per block,
// per-16 sums from lane pairs. 32-wide blocks: four lanes per block, eight
// blocks per warp.

__global__ void k_quant_act(const float *x, int ntok, int cols, int xstride, int kind256, int8_t *q, float *d,
                            int32_t *s, int dstride, int sstride) {
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    if (kind256) {
        const int nb = cols / 256;
        for (int item = warp; item < ntok * nb; item += nwarps) {
            const int t = item / nb, b = item % nb;
            const int off = b * 256 + lane * 8;
            quant_lane8(x + (size_t)t * xstride + off, true, 32, q + (size_t)t * cols + off, d + (size_t)t * dstride + b,
                        s + (size_t)t * sstride + b * 16 + lane / 2, nullptr, lane);
        }
    } else {
        const int nb = cols / 32;
        const int ng = (nb + 7) / 8;
        for (int item = warp; item < ntok * ng; item += nwarps) {
            const int t = item / ng, g = item % ng;
            const int b = g * 8 + lane / 4;
            const bool live = b < nb;
            const int off = b * 32 + (lane & 3) * 8;
            quant_lane8(x + (size_t)t * xstride + off, live, 4, q + (size_t)t * cols + off, d + (size_t)t * dstride + b,
                        nullptr, s + (size_t)t * sstride + b, lane);
        }
    }
}

// act = silu(g) * u (tensor.zig:30,53; the fused kernels' order: g / (1 + e^-g), then * u)
__global__ void k_swiglu(const float *g, const float *u, int n, float *act) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        act[i] = fmul(fdiv(g[i], fadd(1.0f, exp_f(-g[i]))), u[i]);
}

void launch_swiglu(const float *g, const float *u, int n, float *act, cudaStream_t st) {
    k_swiglu<<<cdiv(n, 256), 256, 0, st>>>(g, u, n, act);
    count_launch();
}

void launch_quant_act(const float *x, int ntok, int cols, int xstride, int kind256, int8_t *q, float *d, int32_t *s,
                      int dstride, int sstride, cudaStream_t st) {
    const int items = kind256 ? ntok * (cols / 256) : ntok * ((cols / 32 + 7) / 8);
    if (items == 0) return;
    const int threads = 128;
    unsigned g = cdiv((uint64_t)items * 32, threads);
    if (g > 148 * 16) g = 148 * 16;
    k_quant_act<<<g, threads, 0, st>>>(x, ntok, cols, xstride, kind256, q, d, s, dstride, sstride);
    count_launch();
}

// ---- matvec / matmul (ggml.zig:602 matvec, :504 matmul) ---------------------------
// One warp per row; the row's blocks are decoded once per group of NT tokens.

constexpr int MM_NT = 4;

__global__ void __launch_bounds__(256) k_mm(WDev w, uint64_t gb_base, int rows, int nb, XQ x, int ntok, float *out) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    for (int t0 = 0; t0 < ntok; t0 += MM_NT) {
        float acc[MM_NT] = {};
        const int nt = min(MM_NT, ntok - t0);
        rowdot<MM_NT>(w, gb_base + (uint64_t)r * nb, nb, x, t0, nt, acc, lane);
        if (lane == 0)
            for (int k = 0; k < nt; k++) out[(size_t)(t0 + k) * rows + r] = acc[k];
    }
}

void launch_mm(const WDev &w, uint64_t gb_base, int rows, int cols, const XQ &x, int ntok, float *out, cudaStream_t st) {
    if (rows == 0 || ntok == 0) return;
    const int nb = cols / block_elems(w.type);
    k_mm<<<cdiv(rows, 8), 256, 0, st>>>(w, gb_base, rows, nb, x, ntok, out);
    count_launch();
}

// matvecQ50 (ggml.zig:1673-1704): one warp per (row, token); lane b takes
// block b's partial (j = 0..15: partial += w0*x[j] + w1*x[j+16], in order),
// a zero-scale block contributes nothing (the reference skips it, so its
// non-finite activations never reach the sum), and the block terms
// partial*scale are added in block order from +0.
__global__ void __launch_bounds__(256) k_mm_q50(WDev w, uint64_t gb_base, int rows, int nb, const float *xs, int ntok,
                                                float *out) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int cols = nb * 32;
    for (int t = 0; t < ntok; t++) {
        const float *x = xs + (size_t)t * cols;
        float acc = 0.0f;
        for (int b0 = 0; b0 < nb; b0 += 32) {
            const int b = b0 + lane;
            float term = 0.0f;
            if (b < nb) {
                const uint64_t gb = gb_base + (uint64_t)r * nb + b;
                const float scale = f16_to_f32(__ldg(w.d + gb));
                if (scale != 0.0f) {
                    const uint4 qv = ld_stream_v4(w.q + gb * 16);
                    const uint32_t qh = __ldg(reinterpret_cast<const uint32_t *>(w.sc) + gb);
                    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
                    const float *xb = x + (size_t)b * 32;
                    float partial = 0.0f;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const uint32_t byte = (qw[j >> 2] >> (8 * (j & 3))) & 0xFF;
                        const int q0 = (int)((byte & 0x0F) | (((qh >> j) << 4) & 0x10)) - 16;
                        const int q1 = (int)((byte >> 4) | ((qh >> (j + 12)) & 0x10)) - 16;
                        partial = fadd(partial, fadd(fmul((float)q0, __ldg(xb + j)), fmul((float)q1, __ldg(xb + j + 16))));
                    }
                    term = fmul(partial, scale);
                }
            }
            const int lim = min(32, nb - b0);
            for (int g = 0; g < lim; g++) acc = fadd(acc, __shfl_sync(0xffffffffu, term, g));
        }
        if (lane == 0) out[(size_t)t * rows + r] = acc;
    }
}

void launch_mm_q50(const WDev &w, uint64_t gb_base, int rows, int cols, const float *xs, int ntok, float *out,
                   cudaStream_t st) {
    if (rows == 0 || ntok == 0) return;
    k_mm_q50<<<cdiv(rows, 8), 256, 0, st>>>(w, gb_base, rows, cols / 32, xs, ntok, out);
    count_launch();
}

__global__ void __launch_bounds__(256) k_mm_f32(const float *W, int rows, int cols, const float *xs, int ntok, float *out) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    for (int t = 0; t < ntok; t++) {
        const float v = rowdot_f32(W + (size_t)r * cols, xs + (size_t)t * cols, cols, lane);
        if (lane == 0) out[(size_t)t * rows + r] = v;
    }
}

void launch_mm_f32(const float *W, int rows, int cols, const float *xs, int ntok, float *out, cudaStream_t st) {
    if (rows == 0 || ntok == 0) return;
    k_mm_f32<<<cdiv(rows, 8), 256, 0, st>>>(W, rows, cols, xs, ntok, out);
    count_launch();
}

// ---- router (moe.zig:106-158 route) ------------------------------------------------
// One warp per token. Scores and the biased choice live in shared memory;
// top-k is k rounds of a warp arg-max that keeps the lowest index on ties and
// never selects a value that is not > -inf (the serial scan's strict '>').

__global__ void __launch_bounds__(ROUTE_THREADS) k_route(const float *logits, const float *bias, int ne, int nk,
                                                         int gating, int weights_norm, float weights_scale, int *ids,
                                                         float *gates, int n_group, int topk_group) {
    extern __shared__ float sm[];  // scores[ne] | choice[ne] | ids[64] | gates[64] | red[8]
    const int t = blockIdx.x;
    float *choice = sm + ne;
    for (int e = threadIdx.x; e < ne; e += blockDim.x) choice[e] = logits[(size_t)t * ne + e];
    __syncthreads();
    route_block(choice, bias, ne, nk, gating, weights_norm, weights_scale, sm, choice,
                reinterpret_cast<int *>(sm + 2 * ne), sm + 2 * ne + 64, sm + 2 * ne + 128, ids + (size_t)t * nk,
                gates + (size_t)t * nk, n_group, topk_group);
}

void launch_route(const float *logits, const float *bias, int T, int n_expert, int n_used, int gating, int weights_norm,
                  float weights_scale, int *ids, float *gates, cudaStream_t st, int n_group, int topk_group) {
    if (T == 0) return;
    k_route<<<T, ROUTE_THREADS, (2 * n_expert + 136) * sizeof(float), st>>>(
        logits, bias, n_expert, n_used, gating, weights_norm, weights_scale, ids, gates, n_group, topk_group);
    count_launch();
}

// ---- slot sources -----------------------------------------------------------------
// A slot is one (token, expert) pair. Host-listed experts (moeFfnBlock) come as
// an array built on the host; routed layers derive each slot in registers from
// the layer description and the router's ids/gates: slot t*n_used + k is token
// t's k-th selected expert, slot T*n_used + t its shared expert. Experts outside
// this rank's range get ffn = 0 (skipped).

struct HostSlots {
    const Slot *p;
    __device__ __forceinline__ Slot get(int i) const { return p[i]; }
};

struct RoutedSlots {
    RoutedLayerDev L;
    const int *ids;
    const float *gates;
    int T;
    int act_stride;
    __device__ __forceinline__ Slot get(int i) const {
        Slot s;
        const int nr = T * L.n_used;
        if (i < nr) {
            const int t = i / L.n_used;
            const int le = __ldg(ids + i) - L.expert0;
            const bool local = le >= 0 && le < L.n_local;
            s.g = L.g;
            s.u = L.u;
            s.dn = L.dn;
            s.gb_g = local ? (uint64_t)le * L.plane_blk_g : 0;
            s.gb_u = local ? (uint64_t)le * L.plane_blk_u : 0;
            s.gb_dn = local ? (uint64_t)le * L.plane_blk_dn : 0;
            s.ffn = local ? L.ffn : 0;
            s.token = t;
            s.weight = __ldg(gates + i);
        } else {
            s.g = L.sg;
            s.u = L.su;
            s.dn = L.sdn;
            s.gb_g = s.gb_u = s.gb_dn = 0;
            s.ffn = L.shexp_ffn;
            s.token = i - nr;
            s.weight = 1.0f;
        }
        s.act_off = i * act_stride;
        return s;
    }
};

// ---- expert FFN ------------------------------------------------------------------
// gate/up (+SwiGLU): warp per (slot, row). act = silu(g) * u, silu(g) = g/(1+e^-g)
// (tensor.zig:30, :53).

template <class Src>
__global__ void __launch_bounds__(256) k_gateup(Src src, int dim, XQ x256, XQ x32, float *act) {
    const Slot s = src.get(blockIdx.y);
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= s.ffn) return;
    const int nbg = dim / block_elems(s.g.type), nbu = dim / block_elems(s.u.type);
    float g[1] = {0.0f}, u[1] = {0.0f};
    rowdot<1>(s.g, s.gb_g + (uint64_t)r * nbg, nbg, act256(s.g.type) ? x256 : x32, s.token, 1, g, lane);
    rowdot<1>(s.u, s.gb_u + (uint64_t)r * nbu, nbu, act256(s.u.type) ? x256 : x32, s.token, 1, u, lane);
    if (lane == 0) {
        const float sl = fdiv(g[0], fadd(1.0f, exp_f(-g[0])));
        act[s.act_off + r] = fmul(sl, u[0]);
    }
}

// Quantize each slot's activation in the format its down projection reads.
template <class Src>
__global__ void k_quant_slots(Src src, const float *act, int8_t *aq, float *ad, int32_t *as) {
    const Slot s = src.get(blockIdx.y);
    if (s.ffn == 0) return;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float *x = act + s.act_off;
    int8_t *q = aq + s.act_off;
    float *d = ad + s.act_off / 32;
    int32_t *sm = as + s.act_off / 16;
    if (act256(s.dn.type)) {
        for (int b = warp; b < s.ffn / 256; b += nw)
            quant_lane8(x + b * 256 + lane * 8, true, 32, q + b * 256 + lane * 8, d + b, sm + b * 16 + lane / 2, nullptr,
                        lane);
    } else {
        const int nb = s.ffn / 32, ng = (nb + 7) / 8;
        for (int gi = warp; gi < ng; gi += nw) {
            const int b = gi * 8 + lane / 4;
            const bool live = b < nb;
            const int off = b * 32 + (lane & 3) * 8;
            quant_lane8(x + off, live, 4, q + off, d + b, nullptr, sm + b, lane);
        }
    }
}

// down + weighted combine: warp per (token, output row); the token's slots are
// summed in selection order, then the shared expert is added (llama.zig:1397,
// deepseek.zig:1498-1508).
template <class Src>
__global__ void __launch_bounds__(256) k_down(Src src, int T, int nk, int has_shared, int dim, const int8_t *aq,
                                              const float *ad, const int32_t *as, float *out, const float *residual) {
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= dim) return;
    float acc = 0.0f;
    const int n = nk + (has_shared ? 1 : 0);
    for (int k = 0; k < n; k++) {
        const Slot s = src.get(k < nk ? t * nk + k : T * nk + t);
        if (s.ffn == 0) continue;
        XQ xa;
        xa.q = aq + s.act_off;
        xa.d = ad + s.act_off / 32;
        xa.s = as + s.act_off / 16;
        xa.cols = s.ffn;
        xa.dstride = 0;
        xa.sstride = 0;
        xa.kind256 = act256(s.dn.type);
        const int nb = s.ffn / block_elems(s.dn.type);
        float y[1] = {0.0f};
        rowdot<1>(s.dn, s.gb_dn + (uint64_t)r * nb, nb, xa, 0, 1, y, lane);
        acc = k < nk ? fadd(acc, fmul(s.weight, y[0])) : fadd(acc, y[0]);
    }
    if (lane == 0) out[(size_t)t * dim + r] = residual ? fadd(residual[(size_t)t * dim + r], acc) : acc;
}

template <class Src>
static void run_expert_kernels(const Src &src, int T, int nk, int has_shared, int n_slots, int max_ffn, int dim,
                               const XQ &x256, const XQ &x32, float *act, int8_t *aq, float *ad, int32_t *as,
                               float *out, const float *residual, cudaStream_t st) {
    if (n_slots == 0) return;
    k_gateup<Src><<<dim3(cdiv(max_ffn, 8), n_slots), 256, 0, st>>>(src, dim, x256, x32, act);
    count_launch();
    k_quant_slots<Src><<<dim3(1, n_slots), 256, 0, st>>>(src, act, aq, ad, as);
    count_launch();
    k_down<Src><<<dim3(cdiv(dim, 8), T), 256, 0, st>>>(src, T, nk, has_shared, dim, aq, ad, as, out, residual);
    count_launch();
}

void launch_experts_host(const Slot *slots, int n, int max_ffn, int dim, const XQ &x256, const XQ &x32, float *act,
                         int8_t *aq, float *ad, int32_t *as, float *out, cudaStream_t st) {
    run_expert_kernels(HostSlots{slots}, 1, n, 0, n, max_ffn, dim, x256, x32, act, aq, ad, as, out, nullptr, st);
}

void launch_experts_routed(const RoutedLayerDev &L, const int *ids, const float *gates, int T, int act_stride,
                           const XQ &x256, const XQ &x32, float *act, int8_t *aq, float *ad, int32_t *as, float *out,
                           const float *residual, cudaStream_t st) {
    const int n_slots = T * L.n_used + (L.has_shared ? T : 0);
    const int max_ffn = L.has_shared ? max(L.ffn, L.shexp_ffn) : L.ffn;
    run_expert_kernels(RoutedSlots{L, ids, gates, T, act_stride}, T, L.n_used, L.has_shared, n_slots, max_ffn, L.dim,
                       x256, x32, act, aq, ad, as, out, residual, st);
}

}  // namespace loom

namespace loom {

// ---- greedy sampling (sampler.zig:7-15 argmax) --------------------------------------
// The reference scans with a strict '>' from -inf: the first maximum wins, NaN
// is never taken, and nothing above -inf gives index 0. Here every value above
// -inf becomes the 64-bit key (order key of the value, ~index): the largest
// key is the largest value at its lowest index. Blocks fold their best key
// into *slot with atomicMax; the last block to finish (counter) writes the
// index and re-arms slot and counter for the next call.
__global__ void __launch_bounds__(256) k_argmax(const float *v, int n, unsigned long long *slot, unsigned *count,
                                                uint32_t *out) {
    unsigned long long best = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = __ldg(v + i);
        if (x > -INFINITY) {  // false for NaN and -inf
            const unsigned long long k = ((unsigned long long)f32_order_key(x) << 32) | (0xFFFFFFFFu - (uint32_t)i);
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
        best = ob > best ? ob : best;
    }
    __shared__ unsigned long long wb[8];
    __shared__ bool last;
    if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = wb[w] > best ? wb[w] : best;
        best = wb[0] > best ? wb[0] : best;
        if (best) atomicMax(slot, best);
        __threadfence();
        last = atomicAdd(count, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const unsigned long long k = atomicExch(slot, 0ull);
        *out = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
        *count = 0;
    }
}

void launch_argmax(const float *v, int n, unsigned long long *slot, unsigned *count, uint32_t *out, cudaStream_t st) {
    const int grid = n <= 256 ? 1 : (n + 2047) / 2048 < 148 ? (n + 2047) / 2048 : 148;
    k_argmax<<<grid, 256, 0, st>>>(v, n, slot, count, out);
    count_launch();
}

}  // namespace loom
