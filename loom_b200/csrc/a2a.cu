// a2a.cu -- the all-to-all form of expert parallelism: tokens stay on the rank
// that owns them (token-sharded attention), routed activation rows travel to
// the rank holding the selected expert and the expert outputs travel back.
//
// Per layer, on every rank:
//   pack     slot i = (token i / n_used, its (i % n_used)-th expert) goes to
//            the expert's owner; slots are ordered by destination rank and,
//            within one destination, by slot index (a stable partition), so
//            the layout is deterministic
//   gather   send_x[p] = x[token of the slot at position p]
//   (exchange of counts, rows and expert ids over NCCL: ep.cu)
//   experts  the receiver runs each received row through its one expert with
//            weight 1.0, so the row that comes back is that expert's output
//            exactly (0 + 1*y == y)
//   combine  out[t] = residual + ((sum over k in selection order of
//            gate_k * y_k) + shared expert), the order of the single-GPU
//            combine (llama.zig:1397, deepseek.zig:1498-1508), so the result is
//            bit-identical to the unsharded layer.
#include "devutil.cuh"
#include "ep.cuh"
#include "kernels.cuh"

namespace loom {

// Owner of expert e when ranks hold [r*ne/world, (r+1)*ne/world).
__device__ __forceinline__ int a2a_owner(int e, int ne, int world) {
    int r = (int)(((long long)e * world) / ne);
    while (r + 1 < world && (long long)(r + 1) * ne / world <= e) r++;
    while (r > 0 && (long long)r * ne / world > e) r--;
    return r;
}

constexpr int PACK_THREADS = 1024;

// One CTA. cnt[world]: slots per destination; send_eid/send_tok/slot_pos as
// described above. cap > 0 (fixed-capacity form): destination r's run starts
// at r*cap instead of after the runs before it, and its cap - cnt[r] unused
// entries get expert -1 and token -1 (no row: the receiver's grouping skips
// ids outside its shard, and nothing is gathered for them).
__global__ void __launch_bounds__(PACK_THREADS) k_a2a_pack(const int *ids, int n_slots, int n_used, int n_expert,
                                                           int world, int cap, int *send_eid, int *send_tok,
                                                           int *slot_pos, int *cnt) {
    __shared__ int s_cnt[A2A_MAX_RANKS], s_base[A2A_MAX_RANKS], s_wsum[PACK_THREADS / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < world) s_cnt[tid] = 0;
    __syncthreads();
    for (int i = tid; i < n_slots; i += PACK_THREADS) atomicAdd(&s_cnt[a2a_owner(ids[i], n_expert, world)], 1);
    __syncthreads();
    if (tid == 0) {
        int b = 0;
        for (int r = 0; r < world; r++) {
            s_base[r] = cap > 0 ? r * cap : b;
            b += s_cnt[r];
            cnt[r] = s_cnt[r];
        }
    }
    __syncthreads();
    if (cap > 0)
        for (int i = tid; i < world * cap; i += PACK_THREADS)
            if (i % cap >= s_cnt[i / cap]) {
                send_eid[i] = -1;
                send_tok[i] = -1;
            }
    for (int c = 0; c < n_slots; c += PACK_THREADS) {
        const int i = c + tid;
        const int e = i < n_slots ? ids[i] : 0;
        const int d = i < n_slots ? a2a_owner(e, n_expert, world) : -1;
        for (int r = 0; r < world; r++) {
            const unsigned m = __ballot_sync(0xffffffffu, d == r);
            if (lane == 0) s_wsum[warp] = __popc(m);
            __syncthreads();
            int woff = 0, tot = 0;
            for (int w = 0; w < PACK_THREADS / 32; w++) {
                const int v = s_wsum[w];
                woff += w < warp ? v : 0;
                tot += v;
            }
            if (d == r) {
                const int p = s_base[r] + woff + __popc(m & ((1u << lane) - 1u));
                send_eid[p] = e;
                send_tok[p] = i / n_used;
                slot_pos[i] = p;
            }
            __syncthreads();
            if (tid == 0) s_base[r] += tot;
            __syncthreads();
        }
    }
}

__global__ void k_a2a_gather(const float *x, const int *send_tok, int dim, float *send_x) {
    const int p = blockIdx.x;
    if (send_tok[p] < 0) return;  // an unused entry of a fixed-capacity run
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)send_tok[p] * dim);
    float4 *dst = reinterpret_cast<float4 *>(send_x + (size_t)p * dim);
    for (int c = threadIdx.x; c < dim / 4; c += blockDim.x) dst[c] = src[c];
}

__global__ void k_a2a_fill(float *v, int n, float val) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = val;
}

__global__ void k_a2a_combine(const float *y_back, const int *slot_pos, const float *gates, const float *y_sh,
                              const float *residual, float *out, int n_used, int dim) {
    const int t = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= dim) return;
    float acc = 0.0f;
    for (int k = 0; k < n_used; k++) {
        const int i = t * n_used + k;
        acc = fadd(acc, fmul(gates[i], y_back[(size_t)slot_pos[i] * dim + c]));
    }
    if (y_sh) acc = fadd(acc, y_sh[(size_t)t * dim + c]);
    out[(size_t)t * dim + c] = residual ? fadd(residual[(size_t)t * dim + c], acc) : acc;
}

static inline unsigned cdiv_u(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

void launch_a2a_pack(const int *ids, int T, int n_used, int n_expert, int world, int cap, const float *x, int dim,
                     int *send_eid, int *send_tok, int *slot_pos, int *cnt, float *send_x, cudaStream_t st) {
    const int n = T * n_used;
    k_a2a_pack<<<1, PACK_THREADS, 0, st>>>(ids, n, n_used, n_expert, world, cap, send_eid, send_tok, slot_pos, cnt);
    count_launch();
    const int np = cap > 0 ? world * cap : n;
    if (n == 0) return;
    k_a2a_gather<<<np, 128, 0, st>>>(x, send_tok, dim, send_x);
    count_launch();
}

void launch_a2a_fill(float *v, int n, float val, cudaStream_t st) {
    if (n == 0) return;
    k_a2a_fill<<<cdiv_u(n, 256), 256, 0, st>>>(v, n, val);
    count_launch();
}

void launch_a2a_combine(const float *y_back, const int *slot_pos, const float *gates, const float *y_sh,
                        const float *residual, float *out, int T, int n_used, int dim, cudaStream_t st) {
    if (T == 0) return;
    k_a2a_combine<<<dim3(cdiv_u(dim, 256), T), 256, 0, st>>>(y_back, slot_pos, gates, y_sh, residual, out, n_used,
                                                             dim);
    count_launch();
}

}  // namespace loom
