// digest.cu -- SHA-256 of device-resident weight bytes, and the verified
// upload: every content-addressed shard (an expert's gate, up and down
// extents) is hashed on the device over the GGUF bytes its kernels will
// read, and compared with the shard's digest before use.
//
// The digest is SHA-256 (FIPS 180-4), the reference's content address for
// weight ranges (src/core/hash.zig:12-23); a shard's digest covers its
// extents in order, as src/p2p/weights.zig:862-872 feeds them to one hasher.
// One thread hashes one shard (SHA-256 is serial within a message); a model's
// thousands of expert shards fill the GPU.
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <set>
#include <vector>

#include "../../include/loom_cuda.h"
#include "common.cuh"
#include "kernels.cuh"

namespace loom {
bool rt_tensor(uint64_t h, WDev *w, int *type, uint64_t *nblk);
cudaStream_t rt_stream(void *s);
int rt_need_init();
int rt_decline(const char *why);
int rt_fail(const char *what, cudaError_t e);
int rt_place(int type, const void *data, size_t bytes, uint64_t *handle, uint64_t *blk0, uint64_t *nblk);
void rt_evict(uint64_t handle);
}  // namespace loom

namespace {

using namespace loom;

// FIPS 180-4 section 4.2.2: the first 32 bits of the fractional parts of the
// cube roots of the first 64 primes.
__constant__ uint32_t K256[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }
__device__ __forceinline__ uint32_t bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

__device__ __forceinline__ void compress(uint32_t h[8], uint32_t w[16]) {
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
#pragma unroll
    for (int i = 0; i < 64; i++) {
        if (i >= 16) {
            const uint32_t x = w[(i + 1) & 15], y = w[(i + 14) & 15];
            const uint32_t s0 = rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3);
            const uint32_t s1 = rotr(y, 17) ^ rotr(y, 19) ^ (y >> 10);
            w[i & 15] += s0 + s1 + w[(i + 9) & 15];
        }
        const uint32_t t1 = k + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K256[i] + w[i & 15];
        const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
        k = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += k;
}

struct Seg {
    const uint8_t *p;
    uint64_t len;
};

// Sequential reader over a shard's segments, padded as SHA-256 pads: the
// message, 0x80, zeros, the 64-bit big-endian bit length.
struct Reader {
    const Seg *seg;
    int nseg, si;
    uint64_t off, pos, total;
    __device__ uint32_t byte() {
        const uint64_t p = pos++;
        if (p < total) {
            while (off >= seg[si].len) {
                si++;
                off = 0;
            }
            return seg[si].p[off++];
        }
        if (p == total) return 0x80;
        const uint64_t padded = (total + 9 + 63) & ~63ull;
        if (p >= padded - 8) return (uint32_t)(((total * 8) >> (8 * (padded - 1 - p))) & 0xff);
        return 0;
    }
};

// out[i] = SHA-256 of the concatenated segments seg[first[i] .. first[i+1]).
__global__ void __launch_bounds__(64) k_sha256(const Seg *seg, const int *first, int n, uint8_t *out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    Reader r{seg + first[i], first[i + 1] - first[i], 0, 0, 0, 0};
    for (int s = 0; s < r.nseg; s++) r.total += r.seg[s].len;
    uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    const uint64_t nblocks = (r.total + 9 + 63) / 64;
    for (uint64_t bk = 0; bk < nblocks; bk++) {
        uint32_t w[16];
        // skip exhausted segments so the fast path sees the current one
        while (r.pos < r.total && r.off >= r.seg[r.si].len) {
            r.si++;
            r.off = 0;
        }
        const uint8_t *p = r.pos < r.total ? r.seg[r.si].p + r.off : nullptr;
        const bool whole = r.pos + 64 <= r.total && r.seg[r.si].len - r.off >= 64;
        if (whole && ((uintptr_t)p & 15) == 0) {
            const uint4 *v = reinterpret_cast<const uint4 *>(p);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint4 x = __ldg(v + j);
                w[4 * j] = bswap(x.x);
                w[4 * j + 1] = bswap(x.y);
                w[4 * j + 2] = bswap(x.z);
                w[4 * j + 3] = bswap(x.w);
            }
            r.off += 64;
            r.pos += 64;
        } else if (whole && ((uintptr_t)p & 3) == 0) {
            const uint32_t *v = reinterpret_cast<const uint32_t *>(p);
#pragma unroll
            for (int j = 0; j < 16; j++) w[j] = bswap(__ldg(v + j));
            r.off += 64;
            r.pos += 64;
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                uint32_t x = 0;
                for (int b = 0; b < 4; b++) x = (x << 8) | r.byte();
                w[j] = x;
            }
        }
        compress(h, w);
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        out[32 * i + 4 * j] = h[j] >> 24;
        out[32 * i + 4 * j + 1] = (h[j] >> 16) & 0xff;
        out[32 * i + 4 * j + 2] = (h[j] >> 8) & 0xff;
        out[32 * i + 4 * j + 3] = h[j] & 0xff;
    }
}

// The device layout's regions advanced by `blk` blocks.
WDev advance(WDev w, uint64_t blk) {
    const int t = w.type;
    w.q += blk * (uint64_t)layout_qbytes(t);
    if (w.sc) w.sc += blk * (uint64_t)((t == T_Q6_K || t == T_Q3_K) ? 16 : 4);
    if (w.d) w.d += blk * (uint64_t)((t == T_Q2_K || t == T_Q4_1 || t == T_Q5_1) ? 2 : 1);
    return w;
}

bool raw_layout(int t) { return t == T_F32 || t == T_Q4_K || t == T_Q5_K; }

struct Extent {
    WDev w;
    uint64_t blk0, nblk;
};

constexpr size_t SCRATCH_CAP = 1ull << 30;  // unpacked bytes held at once
size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

// Digests of `groups` of extents (group g = ext[first[g] .. first[g+1])).
int digest_groups(const std::vector<Extent> &ext, const std::vector<int> &first, std::vector<uint8_t> &out) {
    cudaStream_t st = rt_stream(nullptr);
    const int n = (int)first.size() - 1;
    out.assign((size_t)n * 32, 0);
    uint8_t *scratch = nullptr, *d_out = nullptr;
    Seg *d_seg = nullptr;
    int *d_first = nullptr;
    size_t scratch_cap = 0;
    int rc = 0;
    auto ck = [&](cudaError_t e, const char *what) {
        if (e != cudaSuccess && !rc) rc = rt_fail(what, e);
        return e == cudaSuccess;
    };
    int g0 = 0;
    while (g0 < n && !rc) {
        // a batch of groups whose unpacked bytes fit the scratch (at least one group)
        int g1 = g0;
        size_t need = 0;
        while (g1 < n) {
            size_t gneed = 0;
            for (int e = first[g1]; e < first[g1 + 1]; e++)
                if (!raw_layout(ext[e].w.type)) gneed += al256(ext[e].nblk * (size_t)block_bytes(ext[e].w.type));
            if (g1 > g0 && need + gneed > SCRATCH_CAP) break;
            need += gneed;
            g1++;
        }
        if (need > scratch_cap) {
            if (scratch) cudaFree(scratch);
            scratch = nullptr;
            scratch_cap = 0;
            if (!ck(cudaMalloc(&scratch, need), "cudaMalloc(digest scratch)")) break;
            scratch_cap = need;
        }
        std::vector<Seg> seg;
        std::vector<int> f{0};
        size_t so = 0;
        for (int g = g0; g < g1; g++) {
            for (int e = first[g]; e < first[g + 1]; e++) {
                const Extent &x = ext[e];
                const int t = x.w.type;
                const size_t bytes = x.nblk * (size_t)block_bytes(t);
                if (raw_layout(t)) {
                    seg.push_back({x.w.q + x.blk0 * (size_t)block_bytes(t), bytes});
                } else {
                    launch_unpack(t, advance(x.w, x.blk0), scratch + so, x.nblk, st);
                    seg.push_back({scratch + so, bytes});
                    so += al256(bytes);
                }
            }
            f.push_back((int)seg.size());
        }
        const int m = g1 - g0;
        if (!ck(cudaGetLastError(), "unpack")) break;
        if (!ck(cudaMalloc(&d_seg, std::max<size_t>(seg.size(), 1) * sizeof(Seg)), "cudaMalloc(digest)")) break;
        if (!ck(cudaMalloc(&d_first, f.size() * sizeof(int)), "cudaMalloc(digest)")) break;
        if (!ck(cudaMalloc(&d_out, (size_t)m * 32), "cudaMalloc(digest)")) break;
        ck(cudaMemcpyAsync(d_seg, seg.data(), seg.size() * sizeof(Seg), cudaMemcpyHostToDevice, st), "digest copy");
        ck(cudaMemcpyAsync(d_first, f.data(), f.size() * sizeof(int), cudaMemcpyHostToDevice, st), "digest copy");
        if (!rc) {
            k_sha256<<<(m + 63) / 64, 64, 0, st>>>(d_seg, d_first, m, d_out);
            count_launch();
            ck(cudaGetLastError(), "k_sha256");
        }
        ck(cudaMemcpyAsync(out.data() + (size_t)g0 * 32, d_out, (size_t)m * 32, cudaMemcpyDeviceToHost, st),
           "digest copy");
        ck(cudaStreamSynchronize(st), "digest sync");
        cudaFree(d_seg);
        cudaFree(d_first);
        cudaFree(d_out);
        d_seg = nullptr;
        d_first = nullptr;
        d_out = nullptr;
        g0 = g1;
    }
    if (d_seg) cudaFree(d_seg);
    if (d_first) cudaFree(d_first);
    if (d_out) cudaFree(d_out);
    if (scratch) cudaFree(scratch);
    return rc;
}

}  // namespace

extern "C" {

int loom_cuda_sha256_device(const void *d_bytes, size_t bytes, uint8_t digest[32]) {
    if (int rc = rt_need_init()) return rc;
    cudaStream_t st = rt_stream(nullptr);
    const Seg s{static_cast<const uint8_t *>(d_bytes), bytes};
    const int f[2] = {0, 1};
    Seg *d_seg = nullptr;
    int *d_first = nullptr;
    uint8_t *d_out = nullptr;
    int rc = 0;
    cudaError_t e = cudaMalloc(&d_seg, sizeof s);
    if (e == cudaSuccess) e = cudaMalloc(&d_first, sizeof f);
    if (e == cudaSuccess) e = cudaMalloc(&d_out, 32);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_seg, &s, sizeof s, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_first, f, sizeof f, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        k_sha256<<<1, 64, 0, st>>>(d_seg, d_first, 1, d_out);
        count_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(digest, d_out, 32, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = rt_fail("sha256_device", e);
    cudaFree(d_seg);
    cudaFree(d_first);
    cudaFree(d_out);
    return rc;
}

int loom_cuda_tensor_sha256(loom_tensor t, uint64_t blk0, uint64_t nblk, uint8_t digest[32]) {
    if (int rc = rt_need_init()) return rc;
    WDev w;
    int type;
    uint64_t tn;
    if (!rt_tensor(t, &w, &type, &tn)) return rt_decline("unknown tensor");
    if (blk0 > tn || nblk > tn - blk0) return rt_decline("block range outside the tensor");
    std::vector<Extent> ext;
    if (nblk) ext.push_back({w, blk0, nblk});
    std::vector<int> first{0, (int)ext.size()};
    std::vector<uint8_t> out;
    if (int rc = digest_groups(ext, first, out)) return rc;
    std::memcpy(digest, out.data(), 32);
    return LOOM_CUDA_OK;
}

int loom_cuda_verify_shards(const loom_shard *shards, size_t n, uint8_t *bad, size_t *n_bad) {
    if (int rc = rt_need_init()) return rc;
    std::vector<Extent> ext;
    std::vector<uint64_t> owner;  // tensor handle of each extent
    std::vector<int> first{0};
    for (size_t i = 0; i < n; i++) {
        const loom_shard &s = shards[i];
        if (s.n_ext < 0 || s.n_ext > 4) return rt_decline("a shard has 0..4 extents");
        for (int e = 0; e < s.n_ext; e++) {
            const loom_weight &x = s.ext[e];
            uint64_t h = 0, b0 = 0, nb = 0;
            if (int rc = rt_place(x.ggml_type, x.data, x.bytes, &h, &b0, &nb)) return rc;
            WDev w;
            int type;
            uint64_t tn;
            if (!rt_tensor(h, &w, &type, &tn)) return rt_decline("unknown tensor");
            ext.push_back({w, b0, nb});
            owner.push_back(h);
        }
        first.push_back((int)ext.size());
    }
    std::vector<uint8_t> out;
    if (int rc = digest_groups(ext, first, out)) return rc;
    size_t nb = 0;
    std::set<uint64_t> evict;
    for (size_t i = 0; i < n; i++) {
        const bool mismatch = std::memcmp(out.data() + 32 * i, shards[i].digest, 32) != 0;
        if (bad) bad[i] = mismatch;
        if (!mismatch) continue;
        nb++;
        for (int e = first[i]; e < first[i + 1]; e++) evict.insert(owner[e]);
    }
    for (uint64_t h : evict) rt_evict(h);
    if (n_bad) *n_bad = nb;
    return LOOM_CUDA_OK;
}

}  // extern "C"
