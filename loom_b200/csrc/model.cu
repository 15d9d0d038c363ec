// model.cu -- whole-model decode on the device (include/loom_cuda.h,
// loom_cuda_model_*): the reference's token step (src/gguf/llama.zig:1111-1228)
// with the residual stream, the KV cache and every layer resident in HBM.
//
// Per layer (llama.zig:1138-1225):
//   k_rmsnorm_q        attention RMSNorm + quantization of the normed vector
//   k_mm x3            q, k, v matvecs (bit-exact with ggml.matvec)
//   k_qk_rope          headNorm + RoPE, k/v appended to the cache at pos
//   k_attn_*           softmax attention over rows 0..pos
//   k_quant_act, k_mm  output projection
//   k_rmsnorm_q        residual add + FFN RMSNorm
//   MoE layer          loom_cuda_moe_forward (routed, or a dense FFN run as one
//                      expert of weight 1.0, which adds exactly y: 0 + 1*y = y),
//                      residual included
// then the final RMSNorm, the output head and the argmax.
// The step reads token and position from device memory, so one CUDA graph
// replays every step; loom_cuda_model_decode wraps it with one host->device
// and one device->host copy.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_map>
#include <vector>

#include "../../include/loom_cuda.h"
#include "attn.cuh"
#include "attn_block.cuh"
#include "gemv.cuh"
#include "model_kernel.cuh"
#include "kernels.cuh"

namespace loom {
bool rt_tensor(uint64_t h, WDev *w, int *type, uint64_t *nblk);
cudaStream_t rt_stream(void *s);
int rt_need_init();
int rt_decline(const char *why);
int rt_fail(const char *what, cudaError_t e);
uint64_t rt_buf_gen();
cudaError_t rt_wait();
void rt_moe_prenorm(const float *w, float eps);
}  // namespace loom

using namespace loom;

namespace {

#define MCK(call)                                         \
    do {                                                  \
        cudaError_t e_ = (call);                          \
        if (e_ != cudaSuccess) return rt_fail(#call, e_); \
    } while (0)

struct Mat {
    WDev w{};
    int type = 0;
    int rows = 0, cols = 0;
};

struct LayerRt {
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *qn = nullptr, *kn = nullptr;
    Mat wq, wk, wv, wo;
    loom_moe_desc moe{};
    bool dense = false;
    bool fused = false;       // the attention half runs as one cooperative launch (attn_block.cu)
    Mat q_a, q_b, kv_a, kv_b;  // multi-head latent attention
    Mat fg, fu, fd;            // dense FFN on the streamed matvec (dense_stream)
    bool dense_stream = false;
    const float *q_a_norm = nullptr, *kv_a_norm = nullptr;
    AttnBlockArgs blk{};
};

struct Model {
    size_t dim = 0, n_layers = 0, nh = 0, nkv = 0, hd = 0, rope_dim = 0, vocab = 0, ctx = 0;
    float eps = 0, scale = 0;
    int neox = 0;
    bool serial_norm = false, ordered_attn = false, exact = false;
    bool fold_ffn_norm = false;  // fused layers: the MoE router kernel applies the FFN RMSNorm
    bool mla = false;  // DeepSeek multi-head latent attention
    size_t kvr = 0, qlora = 0, nope = 0, vd = 0, kd = 0;
    float *qa_lat = nullptr, *qa_n = nullptr, *kva = nullptr, *qabs = nullptr, *cacc = nullptr;
    float *mla_part = nullptr;  // split-position MLA attention records
    float *dg = nullptr, *du = nullptr, *dact_f = nullptr;  // dense FFN: gate, up, SwiGLU rows
    XQW dact{};                                              // ... and the quantized activation
    XQW l256{}, l32{}, c256{}, c32{};  // q_a output quantized for q_b; per-head compressed results for W_v
    Mat embd, out;
    const float *out_norm = nullptr;
    std::vector<LayerRt> L;
    bool need256 = false, need32 = false;  // kinds the normed vector is quantized to
    bool att256 = false, att32 = false;    // kinds of the attention output
    std::vector<void *> allocs;
    float *kc = nullptr, *vc = nullptr, *rope = nullptr;
    float *x[2] = {nullptr, nullptr}, *normed = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
          *proj = nullptr, *part = nullptr, *logits = nullptr, *zero_logit = nullptr;
    XQW n256{}, n32{}, a256{}, a32{};
    unsigned long long *ab_bar = nullptr;  // grid-barrier state of the fused attention kernel
    unsigned long long *ab_trace = nullptr;  // diagnostic: phase timestamps of one layer's fused attention
    bool persistent = false;  // every layer in one persistent launch (model_kernel.cu)
    MkArgs mk{};
    MkLayer *mk_layers = nullptr;
    float *mk_logits = nullptr, *mk_act = nullptr;
    uint32_t *io_dev = nullptr;   // token, pos, next (graph path)
    uint32_t *io_host = nullptr;  // pinned mirror
    float *h_logits = nullptr;    // pinned
    cudaGraphExec_t exec = nullptr;
    uint64_t exec_gen = 0;
    int calls = 0;
    size_t max_ffn = 0, max_ne = 1, max_nu = 1;  // the MoE layers' largest shape (scratch sizing)
    // batched prefill (loom_cuda_model_prefill): row buffers for up to pf_cap tokens
    size_t pf_cap = 0;
    float *pf_x[2] = {nullptr, nullptr}, *pf_normed = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr,
          *pf_att = nullptr, *pf_proj = nullptr, *pf_zero = nullptr;
    XQW pf_n256{}, pf_n32{}, pf_a256{}, pf_a32{};
    uint32_t *pf_tok = nullptr, *pf_pos = nullptr;
    // batched decode of many sequences (loom_cuda_model_decode_batch): their own caches
    size_t bd_cap = 0;
    float *bkc = nullptr, *bvc = nullptr, *bd_logits = nullptr, *bd_part = nullptr;
    uint32_t *bd_pos = nullptr, *bd_next = nullptr;
};

std::unordered_map<uint64_t, Model *> g_models;
uint64_t g_next_model = 1;

template <class T> int dalloc(Model &m, T *&p, size_t n, bool zero = false) {
    void *v = nullptr;
    const size_t bytes = std::max<size_t>(n * sizeof(T), 256);
    MCK(cudaMalloc(&v, bytes));
    m.allocs.push_back(v);
    if (zero) MCK(cudaMemset(v, 0, bytes));
    p = static_cast<T *>(v);
    return 0;
}

void free_model(Model *m) {
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->ab_trace) cudaFree(m->ab_trace);
    for (void *p : m->allocs) cudaFree(p);
    if (m->io_host) cudaFreeHost(m->io_host);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    delete m;
}

bool mm_type_ok(int t) {
    return t == T_F32 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0 || is_kquant(t);
}

// A [rows][cols] matrix view of a tensor; false when the tensor is unknown, of
// an unsupported type or too small.
bool mat(loom_tensor h, size_t rows, size_t cols, Mat &m) {
    uint64_t nblk = 0;
    if (!rt_tensor(h, &m.w, &m.type, &nblk)) return false;
    if (!mm_type_ok(m.type)) return false;
    const size_t be = block_elems(m.type);
    if (cols % be || nblk < rows * (cols / be)) return false;
    m.rows = (int)rows;
    m.cols = (int)cols;
    return true;
}

const float *f32_vec(loom_tensor h, size_t n, bool &ok) {
    WDev w;
    int type = 0;
    uint64_t nblk = 0;
    if (!rt_tensor(h, &w, &type, &nblk) || type != T_F32 || nblk < n) {
        ok = false;
        return nullptr;
    }
    return reinterpret_cast<const float *>(w.q);
}

// the activation kinds a matvec of type t reads
void need_kind(int t, bool &k256, bool &k32) {
    if (t == T_F32 || t == T_Q5_0) return;  // f32 activations
    if (act256(t))
        k256 = true;
    else
        k32 = true;
}

bool getenv_stream_off() {  // LOOM_CUDA_NO_GEMV_STREAM=1: the warp-engine matvec for every size (comparisons)
    static const int off = getenv("LOOM_CUDA_NO_GEMV_STREAM") ? 1 : 0;
    return off != 0;
}

void matvec(const Mat &m, const float *xf, const XQW &x256, const XQW &x32, float *out, cudaStream_t st) {
    if (m.type == T_F32) {
        launch_mm_f32(reinterpret_cast<const float *>(m.w.q), m.rows, m.cols, xf, 1, out, st);
    } else if (m.type == T_Q5_0) {
        launch_mm_q50(m.w, 0, m.rows, m.cols, xf, 1, out, st);
    } else {
        const XQ x = act256(m.type) ? XQ{x256.q, x256.d, x256.s, m.cols, m.cols / 256, m.cols / 16, 1}
                                    : XQ{x32.q, x32.d, x32.s, m.cols, m.cols / 32, m.cols / 32, 0};
        if (gemv_stream_supported(m.type, (int)m.rows, (int)m.cols) && !getenv_stream_off())
            launch_gemv_stream(m.w, (int)m.rows, (int)m.cols, x, out, st);  // large: tiles streamed through smem
        else if (gemv_supported(m.type, m.cols))
            launch_gemv(m.w, m.rows, m.cols, x, out, st);  // warp engine, weights loaded ahead of the wait
        else
            launch_mm(m.w, 0, m.rows, m.cols, x, 1, out, st);
    }
}

int alloc_xq(Model &m, XQW &q, size_t cols, bool k256) {
    if (int rc = dalloc(m, q.q, cols)) return rc;
    if (int rc = dalloc(m, q.d, cols / (k256 ? 256 : 32) + 1)) return rc;
    return dalloc(m, q.s, cols / (k256 ? 16 : 32) + 1);
}

// A dense FFN on the streamed matvec: normed x already quantized in m.n256;
// xn = x + W_down . (silu(W_gate . x) * (W_up . x)).
void dense_ffn_stream(Model &m, const LayerRt &l, const float *x, float *xn, cudaStream_t st) {
    const int dim = (int)m.dim, f = (int)l.moe.ffn;
    const XQ xq{m.n256.q, m.n256.d, m.n256.s, dim, dim / 256, dim / 16, 1};
    launch_gemv_stream(l.fg.w, f, dim, xq, m.dg, st);
    launch_gemv_stream(l.fu.w, f, dim, xq, m.du, st);
    launch_swiglu(m.dg, m.du, f, m.dact_f, st);
    launch_quant_act(m.dact_f, 1, f, f, 1, m.dact.q, m.dact.d, m.dact.s, f / 256, f / 16, st);
    launch_gemv_stream(l.fd.w, dim, f, XQ{m.dact.q, m.dact.d, m.dact.s, f, f / 256, f / 16, 1}, xn, st, x);
}

// The step on device memory: token id at tok[0], position at pos[0].
int run_step(Model &m, const uint32_t *tok, const uint32_t *pos, float *logits, uint32_t *next, cudaStream_t st) {
    const int dim = (int)m.dim, nh = (int)m.nh, nkv = (int)m.nkv, hd = (int)m.hd, qd = nh * hd;
    const size_t layer_stride = m.ctx * m.nkv * m.hd;
    const XQW none{};
    launch_embed(m.embd.w, dim, tok, (int)m.vocab, m.x[0], st);
    int cur = 0;
    if (m.persistent) {  // every layer in one launch; then the head below
        MkArgs a = m.mk;
        a.x = m.x[0];
        a.pos = pos;
        MCK(launch_model_kernel(a, st));
    }
    for (size_t li = 0; li < m.n_layers && !m.persistent; li++) {
        const LayerRt &l = m.L[li];
        float *x = m.x[cur];
        if (m.mla) {  // deepseek.zig:851-1049 attnLayer, then the FFN
            launch_rmsnorm_q(x, nullptr, l.attn_norm, dim, m.eps, m.normed, m.need256 ? m.n256 : none,
                             m.need32 ? m.n32 : none, m.serial_norm, st);
            if (m.qlora) {
                matvec(l.q_a, m.normed, m.n256, m.n32, m.qa_lat, st);
                const bool k256 = act256(l.q_b.type), kq = l.q_b.type != T_F32 && l.q_b.type != T_Q5_0;
                launch_rmsnorm_q(m.qa_lat, nullptr, l.q_a_norm, (int)m.qlora, m.eps, m.qa_n, kq && k256 ? m.l256 : none,
                                 kq && !k256 ? m.l32 : none, m.exact || m.qlora <= (size_t)RN_SERIAL_MAX, st);
                matvec(l.q_b, m.qa_n, m.l256, m.l32, m.q, st);
            } else {
                matvec(l.wq, m.normed, m.n256, m.n32, m.q, st);
            }
            matvec(l.kv_a, m.normed, m.n256, m.n32, m.kva, st);
            const int kvr = (int)m.kvr, rope = (int)m.rope_dim;
            float *cc = m.kc + li * m.ctx * m.kvr, *rc = m.vc + li * m.ctx * m.rope_dim;
            launch_mla_front(m.kva, l.kv_a_norm, kvr, rope, m.eps, m.q, nh, (int)m.kd, (int)m.nope, m.rope, pos,
                             (int)m.ctx, cc, rc, st);
            launch_mla_absorb(l.kv_b.w, kvr, (int)m.nope, (int)m.vd, (int)m.kd, nh, m.q, m.qabs, st);
            if (m.ordered_attn)
                launch_mla_attn(m.qabs, m.q, kvr, rope, (int)m.kd, (int)m.nope, nh, m.scale, pos, (int)m.ctx, cc, rc,
                                m.cacc, st);
            else
                launch_mla_split(m.qabs, m.q, kvr, rope, (int)m.kd, (int)m.nope, nh, m.scale, pos, (int)m.ctx, cc, rc,
                                 m.mla_part, m.cacc, reinterpret_cast<int *>(m.ab_bar + 2), st);
            const bool ck = act256(l.kv_b.type);
            const XQW &cq = ck ? m.c256 : m.c32;
            launch_quant_act(m.cacc, nh, kvr, kvr, ck, cq.q, cq.d, cq.s, ck ? kvr / 256 : kvr / 32, ck ? kvr / 16 : kvr / 32,
                             st);
            launch_mla_wv(l.kv_b.w, kvr, (int)m.nope, (int)m.vd, nh,
                          XQ{cq.q, cq.d, cq.s, kvr, ck ? kvr / 256 : kvr / 32, ck ? kvr / 16 : kvr / 32, ck ? 1 : 0},
                          m.att, st);
            const int hv = nh * (int)m.vd;
            if (l.wo.type != T_F32 && l.wo.type != T_Q5_0) {
                const bool k256 = act256(l.wo.type);
                const XQW &a = k256 ? m.a256 : m.a32;
                launch_quant_act(m.att, 1, hv, hv, k256, a.q, a.d, a.s, k256 ? hv / 256 : hv / 32, k256 ? hv / 16 : hv / 32,
                                 st);
            }
            matvec(l.wo, m.att, m.a256, m.a32, m.proj, st);
            launch_rmsnorm_q(x, m.proj, l.ffn_norm, dim, m.eps, m.normed, l.dense_stream ? m.n256 : none, none,
                             m.serial_norm, st);
            float *xn = m.x[cur ^ 1];
            if (l.dense_stream)
                dense_ffn_stream(m, l, x, xn, st);
            else if (int rc2 = loom_cuda_moe_forward(&l.moe, m.normed, 1, xn, x, l.dense ? m.zero_logit : nullptr,
                                                     nullptr, st))
                return rc2;
            cur ^= 1;
            continue;
        }
        if (l.fused) {  // one cooperative launch: norm, q/k/v, RoPE, attention, output projection, FFN norm
            AttnBlockArgs a = l.blk;
            a.x = x;
            a.pos = pos;
            MCK(launch_attn_block(a, st));
            float *xn = m.x[cur ^ 1];
            if (l.dense_stream) {
                launch_rmsnorm_q(x, nullptr, l.ffn_norm, dim, m.eps, m.normed, m.n256, none, m.serial_norm, st);
                dense_ffn_stream(m, l, x, xn, st);
                cur ^= 1;
                continue;
            }
            if (m.fold_ffn_norm) rt_moe_prenorm(l.ffn_norm, m.eps);  // the router kernel normalizes x itself
            if (int rc = loom_cuda_moe_forward(&l.moe, m.fold_ffn_norm ? x : m.normed, 1, xn, x,
                                               l.dense ? m.zero_logit : nullptr, nullptr, st))
                return rc;
            cur ^= 1;
            continue;
        }
        launch_rmsnorm_q(x, nullptr, l.attn_norm, dim, m.eps, m.normed, m.need256 ? m.n256 : none,
                         m.need32 ? m.n32 : none, m.serial_norm, st);
        matvec(l.wq, m.normed, m.n256, m.n32, m.q, st);
        matvec(l.wk, m.normed, m.n256, m.n32, m.k, st);
        matvec(l.wv, m.normed, m.n256, m.n32, m.v, st);
        float *kc = m.kc + li * layer_stride, *vc = m.vc + li * layer_stride;
        launch_qk_rope(m.q, m.k, m.v, l.qn, l.kn, nh, nkv, hd, (int)m.rope_dim, m.neox, m.rope, m.eps, pos,
                       (int)m.ctx, kc, vc, st);
        const bool wq_kind = l.wo.type != T_F32 && l.wo.type != T_Q5_0;
        const bool k256 = wq_kind && act256(l.wo.type);
        const bool fused_q = wq_kind && !m.ordered_attn && attn_merge_quantizes(nh, hd, (int)m.ctx);
        launch_attention(m.q, kc, vc, nh, nkv, hd, m.scale, pos, (int)m.ctx, m.part, m.att, m.ordered_attn,
                         fused_q && k256 ? m.a256 : none, fused_q && !k256 ? m.a32 : none, st);
        if (wq_kind && !fused_q) {
            const XQW &a = k256 ? m.a256 : m.a32;
            launch_quant_act(m.att, 1, qd, qd, k256, a.q, a.d, a.s, k256 ? qd / 256 : qd / 32,
                             k256 ? qd / 16 : qd / 32, st);
        }
        matvec(l.wo, m.att, m.a256, m.a32, m.proj, st);
        // x += proj (llama.zig:1195), then the FFN norm; the MoE layer quantizes normed itself
        launch_rmsnorm_q(x, m.proj, l.ffn_norm, dim, m.eps, m.normed, l.dense_stream ? m.n256 : none, none,
                         m.serial_norm, st);
        float *xn = m.x[cur ^ 1];
        if (l.dense_stream)
            dense_ffn_stream(m, l, x, xn, st);
        else if (int rc = loom_cuda_moe_forward(&l.moe, m.normed, 1, xn, x, l.dense ? m.zero_logit : nullptr, nullptr, st))
            return rc;
        cur ^= 1;
    }
    XQW o256 = none, o32 = none;
    if (m.out.type != T_F32 && m.out.type != T_Q5_0) {
        if (act256(m.out.type))
            o256 = m.n256;
        else
            o32 = m.n32;
    }
    launch_rmsnorm_q(m.x[cur], nullptr, m.out_norm, dim, m.eps, m.normed, o256, o32, m.serial_norm, st);
    float *lg = logits ? logits : m.logits;
    matvec(m.out, m.normed, m.n256, m.n32, lg, st);
    if (next) {
        if (int rc = loom_cuda_argmax(lg, m.vocab, next, st)) return rc;
    }
    MCK(cudaGetLastError());
    return LOOM_CUDA_OK;
}

// A matrix times ntok token rows: out[k * rows + r] (ggml.matmul, ggml.zig:504: bit-identical to
// ntok matvecs); xf are the f32 rows, x256 / x32 their quantized forms (token stride = one row).
void matmul_rows(const Mat &m, const float *xf, const XQW &x256, const XQW &x32, int ntok, float *out,
                 cudaStream_t st) {
    if (m.type == T_F32) {
        launch_mm_f32(reinterpret_cast<const float *>(m.w.q), m.rows, m.cols, xf, ntok, out, st);
    } else if (m.type == T_Q5_0) {
        launch_mm_q50(m.w, 0, m.rows, m.cols, xf, ntok, out, st);
    } else {
        const XQ x = act256(m.type) ? XQ{x256.q, x256.d, x256.s, m.cols, m.cols / 256, m.cols / 16, 1}
                                    : XQ{x32.q, x32.d, x32.s, m.cols, m.cols / 32, m.cols / 32, 0};
        if (ntok < 8 || !launch_mm_tiled(m.w, m.rows, m.cols, x, ntok, out, st))
            launch_mm(m.w, 0, m.rows, m.cols, x, ntok, out, st);
    }
}

int alloc_prefill(Model &m, size_t n) {
    if (n <= m.pf_cap) return 0;
    const size_t dim = m.dim, qd = m.nh * m.hd, kvd = m.nkv * m.hd;
    int rc = 0;
    if ((rc = dalloc(m, m.pf_x[0], n * dim)) || (rc = dalloc(m, m.pf_x[1], n * dim)) ||
        (rc = dalloc(m, m.pf_normed, n * dim)) || (rc = dalloc(m, m.pf_q, n * qd)) || (rc = dalloc(m, m.pf_k, n * kvd)) ||
        (rc = dalloc(m, m.pf_v, n * kvd)) || (rc = dalloc(m, m.pf_att, n * qd)) || (rc = dalloc(m, m.pf_proj, n * dim)) ||
        (rc = dalloc(m, m.pf_zero, n, true)) || (rc = dalloc(m, m.pf_tok, n)) || (rc = dalloc(m, m.pf_pos, 1)) ||
        (rc = alloc_xq(m, m.pf_n256, n * dim, true)) || (rc = alloc_xq(m, m.pf_n32, n * dim, false)) ||
        (rc = alloc_xq(m, m.pf_a256, n * qd, true)) || (rc = alloc_xq(m, m.pf_a32, n * qd, false)))
        return rc;
    m.pf_cap = n;
    return 0;
}

// llama.zig:1698-1825 stepBatch: n tokens at positions pos_base .. pos_base + n - 1 through the
// model layer by layer (every token's row through a layer before the next layer), the KV cache
// rows appended, each token attending causally to rows 0..its position; the last token's logits.
// Per layer: RMSNorm of every row (+ quantization), q/k/v as matmuls over the rows (bit-identical
// to per-row matvecs), headNorm + RoPE + cache append per token, the ordered attention per
// (head, token), the output projection as a matmul, the residual add and the FFN RMSNorm, then
// the MoE (or dense) FFN on all rows through the expert-major batch path (the reference runs it
// token by token through the single-token path: the same integer arithmetic, except the
// tensor cores' fp16 down projection when the experts average >= 16 tokens).
int run_prefill(Model &m, int n, int pos_base, cudaStream_t st) {
    const int dim = (int)m.dim, nh = (int)m.nh, nkv = (int)m.nkv, hd = (int)m.hd, qd = nh * hd;
    const size_t layer_stride = m.ctx * m.nkv * m.hd;
    const XQW none{};
    launch_embed(m.embd.w, dim, m.pf_tok, (int)m.vocab, m.pf_x[0], st, n);
    int cur = 0;
    for (size_t li = 0; li < m.n_layers; li++) {
        const LayerRt &l = m.L[li];
        float *x = m.pf_x[cur];
        launch_rmsnorm_q(x, nullptr, l.attn_norm, dim, m.eps, m.pf_normed, m.need256 ? m.pf_n256 : none,
                         m.need32 ? m.pf_n32 : none, m.serial_norm, st, n);
        matmul_rows(l.wq, m.pf_normed, m.pf_n256, m.pf_n32, n, m.pf_q, st);
        matmul_rows(l.wk, m.pf_normed, m.pf_n256, m.pf_n32, n, m.pf_k, st);
        matmul_rows(l.wv, m.pf_normed, m.pf_n256, m.pf_n32, n, m.pf_v, st);
        float *kc = m.kc + li * layer_stride, *vc = m.vc + li * layer_stride;
        launch_qk_rope(m.pf_q, m.pf_k, m.pf_v, l.qn, l.kn, nh, nkv, hd, (int)m.rope_dim, m.neox, m.rope, m.eps,
                       m.pf_pos, (int)m.ctx, kc, vc, st, n);
        // the reference's order where the model keeps it (exact_order, short contexts); else the batched form
        if (m.ordered_attn || !launch_attention_prefill_rows(m.pf_q, kc, vc, nh, nkv, hd, m.scale, m.pf_pos, (int)m.ctx,
                                                             m.pf_att, n, pos_base + n - 1, st))
            launch_attention_ordered_rows(m.pf_q, kc, vc, nh, nkv, hd, m.scale, m.pf_pos, (int)m.ctx, m.pf_att, n, st);
        if (l.wo.type != T_F32 && l.wo.type != T_Q5_0) {
            const bool k256 = act256(l.wo.type);
            const XQW &a = k256 ? m.pf_a256 : m.pf_a32;
            launch_quant_act(m.pf_att, n, qd, qd, k256, a.q, a.d, a.s, k256 ? qd / 256 : qd / 32, k256 ? qd / 16 : qd / 32,
                             st);
        }
        matmul_rows(l.wo, m.pf_att, m.pf_a256, m.pf_a32, n, m.pf_proj, st);
        // x += proj (llama.zig:1781), then the FFN norm of every row
        launch_rmsnorm_q(x, m.pf_proj, l.ffn_norm, dim, m.eps, m.pf_normed, none, none, m.serial_norm, st, n);
        float *xn = m.pf_x[cur ^ 1];
        if (int rc = loom_cuda_moe_forward(&l.moe, m.pf_normed, (size_t)n, xn, x, l.dense ? m.pf_zero : nullptr, nullptr,
                                           st))
            return rc;
        cur ^= 1;
    }
    MCK(cudaGetLastError());
    return cur;  // the buffer holding the final rows
}

// llama.zig:1939 decodeBatch: B sequences one token each, sequence b at position pos[b] with its
// own KV cache (m.bkc / m.bvc: [B][layers][ctx][kv dim]); the prefill's row-batched kernels with
// per-row positions and cache bases, the attention per (head or KV head, sequence), the FFN of
// all B rows on the expert-major batch path, then every row's final norm, head and argmax.
int run_decode_batch(Model &m, int B, cudaStream_t st) {
    const int dim = (int)m.dim, nh = (int)m.nh, nkv = (int)m.nkv, hd = (int)m.hd, qd = nh * hd;
    const size_t layer_stride = m.ctx * m.nkv * m.hd, seq_stride = m.n_layers * layer_stride;
    const XQW none{};
    launch_embed(m.embd.w, dim, m.pf_tok, (int)m.vocab, m.pf_x[0], st, B);
    int cur = 0;
    for (size_t li = 0; li < m.n_layers; li++) {
        const LayerRt &l = m.L[li];
        float *x = m.pf_x[cur];
        launch_rmsnorm_q(x, nullptr, l.attn_norm, dim, m.eps, m.pf_normed, m.need256 ? m.pf_n256 : none,
                         m.need32 ? m.pf_n32 : none, m.serial_norm, st, B);
        matmul_rows(l.wq, m.pf_normed, m.pf_n256, m.pf_n32, B, m.pf_q, st);
        matmul_rows(l.wk, m.pf_normed, m.pf_n256, m.pf_n32, B, m.pf_k, st);
        matmul_rows(l.wv, m.pf_normed, m.pf_n256, m.pf_n32, B, m.pf_v, st);
        float *kc = m.bkc + li * layer_stride, *vc = m.bvc + li * layer_stride;
        launch_qk_rope(m.pf_q, m.pf_k, m.pf_v, l.qn, l.kn, nh, nkv, hd, (int)m.rope_dim, m.neox, m.rope, m.eps,
                       m.bd_pos, (int)m.ctx, kc, vc, st, B, 1, seq_stride);
        if (m.ordered_attn)
            launch_attention_ordered_rows(m.pf_q, kc, vc, nh, nkv, hd, m.scale, m.bd_pos, (int)m.ctx, m.pf_att, B, st, 1,
                                          seq_stride);
        else  // the single-sequence step's split form, one grid over every sequence's chunks
            launch_attention_split_rows(m.pf_q, kc, vc, nh, nkv, hd, m.scale, m.bd_pos, (int)m.ctx, m.bd_part, m.pf_att, B,
                                        seq_stride, st);
        if (l.wo.type != T_F32 && l.wo.type != T_Q5_0) {
            const bool k256 = act256(l.wo.type);
            const XQW &a = k256 ? m.pf_a256 : m.pf_a32;
            launch_quant_act(m.pf_att, B, qd, qd, k256, a.q, a.d, a.s, k256 ? qd / 256 : qd / 32, k256 ? qd / 16 : qd / 32,
                             st);
        }
        matmul_rows(l.wo, m.pf_att, m.pf_a256, m.pf_a32, B, m.pf_proj, st);
        launch_rmsnorm_q(x, m.pf_proj, l.ffn_norm, dim, m.eps, m.pf_normed, none, none, m.serial_norm, st, B);
        float *xn = m.pf_x[cur ^ 1];
        if (int rc = loom_cuda_moe_forward(&l.moe, m.pf_normed, (size_t)B, xn, x, l.dense ? m.pf_zero : nullptr, nullptr,
                                           st))
            return rc;
        cur ^= 1;
    }
    XQW o256 = none, o32 = none;
    if (m.out.type != T_F32 && m.out.type != T_Q5_0) {
        if (act256(m.out.type))
            o256 = m.pf_n256;
        else
            o32 = m.pf_n32;
    }
    launch_rmsnorm_q(m.pf_x[cur], nullptr, m.out_norm, dim, m.eps, m.pf_normed, o256, o32, m.serial_norm, st, B);
    matmul_rows(m.out, m.pf_normed, m.pf_n256, m.pf_n32, B, m.bd_logits, st);
    for (int b = 0; b < B; b++)
        if (int rc = loom_cuda_argmax(m.bd_logits + (size_t)b * m.vocab, m.vocab, m.bd_next + b, st)) return rc;
    MCK(cudaGetLastError());
    return LOOM_CUDA_OK;
}

Model *find(uint64_t h) {
    auto it = g_models.find(h);
    return it == g_models.end() ? nullptr : it->second;
}

// (cos, sin) of every rotation pair j at every position, in the reference's
// theta progression (llama.zig:821-826 ropeTheta with index 2j: exponent =
// 2j / rope_dim, freq = base^-exponent, angle = pos * freq), in f32.
std::vector<float> rope_table(size_t ctx, size_t rope_dim, float base) {
    const size_t half = rope_dim / 2;
    std::vector<float> t(ctx * half * 2);
    for (size_t j = 0; j < half; j++) {
        const float exponent = (float)(2 * j) / (float)rope_dim;
        const float freq = std::pow(base, -exponent);
        for (size_t p = 0; p < ctx; p++) {
            const float angle = (float)p * freq;
            t[(p * half + j) * 2] = std::cos(angle);
            t[(p * half + j) * 2 + 1] = std::sin(angle);
        }
    }
    return t;
}

}  // namespace

extern "C" {

int loom_cuda_model_create(const loom_model_desc *d, uint64_t *handle) {
    if (int rc = rt_need_init()) return rc;
    if (!d || !handle || !d->layers) return rt_decline("no model description");
    if (d->dim == 0 || d->n_layers == 0 || d->n_heads == 0 || d->n_kv_heads == 0 || d->vocab == 0 || d->ctx_len == 0)
        return rt_decline("empty model shape");
    if (d->n_heads % d->n_kv_heads || d->n_heads / d->n_kv_heads > 16)
        return rt_decline("n_heads must be a multiple of n_kv_heads, at most 16 query heads per KV head");
    if (d->head_dim < 8 || d->head_dim % 2 || d->head_dim > 256)
        return rt_decline("head_dim must be even, >= 8 and <= 256");
    if (d->rope_dim > d->head_dim || d->rope_dim % 2) return rt_decline("rope_dim must be even and <= head_dim");
    if (d->dim > 16384 || d->ctx_len > (1u << 18) || d->vocab > 0x7FFFFFFFu) return rt_decline("model shape too large");
    if (d->mla && (!d->kv_lora || !d->nope || !d->v_head || d->nope + d->rope_dim != d->head_dim ||
                   d->ctx_len > (size_t)ATT_ORDERED_LIMIT))
        return rt_decline("MLA: head_dim must be nope + rope_dim, kv_lora/v_head nonzero, ctx_len <= 32768");
    if (!d->mla) {  // the split attention's merge keeps (256 / hd + 1) x chunks weights in shared memory
        const size_t hpc = std::min<size_t>(256 / d->head_dim + 1, d->n_heads);
        const size_t nsplit = (d->ctx_len + ATT_CH - 1) / ATT_CH;
        if (!d->exact_order && d->ctx_len > (size_t)ATT_ORDERED_MAX && hpc * nsplit * 4 > 200 * 1024)
            return rt_decline("context too long for this head_dim");
    }
    Model *m = new Model();
    auto bail = [&](int rc) {
        free_model(m);
        return rc;
    };
    m->dim = d->dim;
    m->n_layers = d->n_layers;
    m->nh = d->n_heads;
    m->nkv = d->n_kv_heads;
    m->hd = d->head_dim;
    m->rope_dim = d->rope_dim;
    m->vocab = d->vocab;
    m->ctx = d->ctx_len;
    m->eps = d->eps;
    m->neox = d->rope_neox;
    m->serial_norm = d->exact_order || d->dim <= (size_t)RN_SERIAL_MAX;
    m->ordered_attn = d->exact_order || d->ctx_len <= (size_t)ATT_ORDERED_MAX;
    if (m->ordered_attn && d->ctx_len > (size_t)ATT_ORDERED_LIMIT) {
        delete m;
        return rt_decline("exact_order takes contexts up to 32768 positions");
    }
    m->scale = d->attn_logit_mul / std::sqrt((float)d->head_dim);  // llama.zig:1116
    m->exact = d->exact_order != 0;
    if (d->mla) {
        m->mla = true;
        m->kvr = d->kv_lora;
        m->qlora = d->q_lora;
        m->nope = d->nope;
        m->vd = d->v_head;
        m->kd = d->nope + d->rope_dim;
        m->scale = d->mla_scale;
        // the reference's order up to the ordered limit (and with exact_order); past it the
        // split-position form
        m->ordered_attn = d->exact_order || d->ctx_len <= (size_t)ATT_ORDERED_MAX ||
                          !mla_split_supported((int)d->kv_lora, (int)d->rope_dim);
    }
    const size_t dim = d->dim, qd = d->n_heads * d->head_dim, kvd = d->n_kv_heads * d->head_dim;
    const size_t hv = m->mla ? d->n_heads * d->v_head : qd;  // attention output width (the output projection's input)
    if (!mat(d->token_embd, d->vocab, dim, m->embd)) return bail(rt_decline("token_embd: unknown tensor or wrong size"));
    if (!mat(d->output, d->vocab, dim, m->out)) return bail(rt_decline("output: unknown tensor or wrong size"));
    bool ok = true;
    m->out_norm = f32_vec(d->output_norm, dim, ok);
    if (!ok) return bail(rt_decline("output_norm must be f32 [dim]"));
    size_t max_ffn = 0, max_ne = 1, max_nu = 1, max_dense = 0;
    for (size_t li = 0; li < d->n_layers; li++) {
        const loom_model_layer &s = d->layers[li];
        LayerRt l;
        l.attn_norm = f32_vec(s.attn_norm, dim, ok);
        l.ffn_norm = f32_vec(s.ffn_norm, dim, ok);
        if (s.q_norm) l.qn = f32_vec(s.q_norm, d->head_dim, ok);
        if (s.k_norm) l.kn = f32_vec(s.k_norm, d->head_dim, ok);
        if (!ok) return bail(rt_decline("layer norms must be f32 [dim] / [head_dim]"));
        if (m->mla) {  // deepseek.zig:860-875 tensors
            const bool qok = m->qlora ? mat(s.q_a, m->qlora, dim, l.q_a) && mat(s.q_b, qd, m->qlora, l.q_b) &&
                                            (l.q_a_norm = f32_vec(s.q_a_norm, m->qlora, ok)) != nullptr
                                      : mat(s.wq, qd, dim, l.wq);
            l.kv_a_norm = f32_vec(s.kv_a_norm, m->kvr, ok);
            if (!qok || !ok || !mat(s.kv_a, m->kvr + d->rope_dim, dim, l.kv_a) ||
                !mat(s.kv_b, d->n_heads * (m->nope + m->vd), m->kvr, l.kv_b) || !mat(s.wo, dim, hv, l.wo))
                return bail(rt_decline("MLA weights: unknown tensor, unsupported type or wrong size"));
            if (l.kv_b.type == T_F32 || l.kv_b.type == T_Q5_0)
                return bail(rt_decline("MLA: kv_b must be a quantized type with int8 activations"));
            if (m->qlora) {
                need_kind(l.q_a.type, m->need256, m->need32);
                if ((act256(l.q_b.type) && m->qlora % 256) || m->qlora % 32)
                    return bail(rt_decline("MLA: q_lora width does not fit q_b's blocks"));
            } else {
                need_kind(l.wq.type, m->need256, m->need32);
            }
            need_kind(l.kv_a.type, m->need256, m->need32);
        } else if (!mat(s.wq, qd, dim, l.wq) || !mat(s.wk, kvd, dim, l.wk) || !mat(s.wv, kvd, dim, l.wv) ||
                   !mat(s.wo, dim, qd, l.wo)) {
            return bail(rt_decline("attention weights: unknown tensor, unsupported type or wrong size"));
        }
        if (s.moe.n_expert) {
            l.moe = s.moe;
            if (l.moe.dim != dim) return bail(rt_decline("MoE layer dim differs from the model's"));
            max_ffn = std::max(max_ffn, std::max(l.moe.ffn, l.moe.shexp_ffn));
            max_ne = std::max(max_ne, l.moe.n_expert);
            max_nu = std::max(max_nu, l.moe.n_used);
        } else {
            if (!s.ffn_gate || !s.ffn_up || !s.ffn_down || !s.ffn) return bail(rt_decline("dense FFN tensors missing"));
            l.dense = true;
            loom_moe_desc &e = l.moe;
            e.dim = dim;
            e.ffn = s.ffn;
            e.n_expert = 1;
            e.n_used = 1;
            e.gating = 1;
            e.weights_norm = 1;
            e.weights_scale = 1.0f;
            e.gate = s.ffn_gate;
            e.up = s.ffn_up;
            e.down = s.ffn_down;
            max_ffn = std::max(max_ffn, s.ffn);
            // large dense FFNs (DeepSeek's first layers) on the streamed matvec: gate, up, SwiGLU, down + residual
            if (!getenv("LOOM_CUDA_NO_GEMV_STREAM") && mat(s.ffn_gate, s.ffn, dim, l.fg) && mat(s.ffn_up, s.ffn, dim, l.fu) &&
                mat(s.ffn_down, dim, s.ffn, l.fd) && act256(l.fg.type) && l.fg.type == l.fu.type &&
                act256(l.fd.type) && gemv_stream_shape_ok(l.fg.type, (int)dim) &&
                gemv_stream_shape_ok(l.fd.type, (int)s.ffn)) {
                l.dense_stream = true;
                max_dense = std::max(max_dense, s.ffn);
            }
        }
        if (!m->mla) {
            need_kind(l.wq.type, m->need256, m->need32);
            need_kind(l.wk.type, m->need256, m->need32);
            need_kind(l.wv.type, m->need256, m->need32);
        }
        need_kind(l.wo.type, m->att256, m->att32);
        m->L.push_back(l);
    }
    m->max_ffn = max_ffn;
    m->max_ne = max_ne;
    m->max_nu = max_nu;
    need_kind(m->out.type, m->need256, m->need32);
    if ((m->need256 && dim % 256) || (m->att256 && hv % 256))
        return bail(rt_decline("a K-quant projection needs a width that is a multiple of 256"));
    if ((m->need32 && dim % 32) || (m->att32 && hv % 32)) return bail(rt_decline("width not a multiple of 32"));
    // the MoE scratch, sized now so the step never allocates (graph capture)
    if (int rc = loom_cuda_reserve(1, dim, max_ffn, max_ne, max_nu)) return bail(rc);
    int rc = 0;
    // caches: k/v rows [layers][ctx][n_kv*hd]; MLA: compressed rows [..][kv_lora] and rope rows [..][rope]
    const size_t cache_k = d->n_layers * d->ctx_len * (m->mla ? m->kvr : kvd);
    const size_t cache_v = d->n_layers * d->ctx_len * (m->mla ? d->rope_dim : kvd);
    if (m->mla) {
        const size_t ql = m->qlora ? m->qlora : 1, lat = d->n_heads * m->kvr;
        if ((rc = dalloc(*m, m->qa_lat, ql)) || (rc = dalloc(*m, m->qa_n, ql)) || (rc = alloc_xq(*m, m->l256, ql, true)) ||
            (rc = alloc_xq(*m, m->l32, ql, false)) || (rc = dalloc(*m, m->kva, m->kvr + d->rope_dim)) ||
            (rc = dalloc(*m, m->qabs, lat)) || (rc = dalloc(*m, m->cacc, lat)) || (rc = alloc_xq(*m, m->c256, lat, true)) ||
            (rc = alloc_xq(*m, m->c32, lat, false)))
            return bail(rc);
    }
    if ((rc = dalloc(*m, m->kc, cache_k, true)) || (rc = dalloc(*m, m->vc, cache_v, true)) ||
        (rc = dalloc(*m, m->rope, d->ctx_len * d->rope_dim)) || (rc = dalloc(*m, m->x[0], dim)) ||
        (rc = dalloc(*m, m->x[1], dim)) || (rc = dalloc(*m, m->normed, dim)) || (rc = dalloc(*m, m->q, qd)) ||
        (rc = dalloc(*m, m->k, kvd)) || (rc = dalloc(*m, m->v, kvd)) || (rc = dalloc(*m, m->att, qd)) ||
        (rc = dalloc(*m, m->proj, dim)) ||
        (rc = dalloc(*m, m->part, attn_part_floats((int)m->nh, (int)m->nkv, (int)m->hd, (int)m->ctx))) ||
        (rc = dalloc(*m, m->logits, d->vocab)) || (rc = dalloc(*m, m->zero_logit, 1, true)) ||
        (rc = dalloc(*m, m->io_dev, 4, true)) || (rc = alloc_xq(*m, m->n256, dim, true)) ||
        (rc = alloc_xq(*m, m->n32, dim, false)) || (rc = alloc_xq(*m, m->a256, std::max(qd, hv), true)) ||
        (rc = alloc_xq(*m, m->a32, std::max(qd, hv), false)))
        return bail(rc);
    if ((rc = dalloc(*m, m->ab_bar, 64, true))) return bail(rc);
    if (max_dense && ((rc = dalloc(*m, m->dg, max_dense)) || (rc = dalloc(*m, m->du, max_dense)) ||
                      (rc = dalloc(*m, m->dact_f, max_dense)) || (rc = alloc_xq(*m, m->dact, max_dense, true))))
        return bail(rc);
    if (m->mla && !m->ordered_attn && (rc = dalloc(*m, m->mla_part, mla_part_floats((int)m->nh, (int)m->kvr, (int)m->ctx))))
        return bail(rc);
    // The FFN RMSNorm moves into the MoE layer's router kernel (one grid barrier
    // and one single-CTA phase less per layer) where the tree-order norm is used.
    m->fold_ffn_norm = !m->serial_norm && !getenv("LOOM_CUDA_NO_NORM_FOLD");
    if (!m->ordered_attn && !m->mla && !getenv("LOOM_CUDA_NO_ATTN_BLOCK")) {
        for (size_t li = 0; li < d->n_layers; li++) {
            LayerRt &l = m->L[li];
            AttnBlockArgs &a = l.blk;
            a.normed = m->fold_ffn_norm ? nullptr : m->normed;
            a.attn_norm = l.attn_norm;
            a.ffn_norm = l.ffn_norm;
            a.q_norm = l.qn;
            a.k_norm = l.kn;
            a.eps = m->eps;
            a.serial = m->serial_norm;
            a.wq = l.wq.w;
            a.wk = l.wk.w;
            a.wv = l.wv.w;
            a.wo = l.wo.w;
            a.dim = (int)dim;
            a.n_heads = (int)m->nh;
            a.n_kv = (int)m->nkv;
            a.hd = (int)m->hd;
            a.rope_dim = (int)m->rope_dim;
            a.neox = m->neox;
            a.rope = m->rope;
            a.scale = m->scale;
            a.ctx = (int)m->ctx;
            a.kc = m->kc + li * d->ctx_len * kvd;
            a.vc = m->vc + li * d->ctx_len * kvd;
            a.q = m->q;
            a.k = m->k;
            a.v = m->v;
            a.part = m->part;
            a.nsplit = (int)((m->ctx + ATT_CH - 1) / ATT_CH);
            const bool o256 = act256(l.wo.type);
            a.aq = o256 ? m->a256.q : m->a32.q;
            a.ad = o256 ? m->a256.d : m->a32.d;
            a.as = o256 ? m->a256.s : m->a32.s;
            a.bar = m->ab_bar;
            l.fused = attn_block_plan(a, l.wq.type, l.wk.type, l.wv.type, l.wo.type, m->ctx) != 0;
        }
    }
    // every layer in one persistent launch when each is a fused-attention, plain routed layer
    // of one shape (no shared expert, bias-free or biased, unsharded, plain top-k)
    // Opt-in (LOOM_CUDA_PERSISTENT=1): correct and tested, but measured slower than the per-layer
    // launches (B200: 0.92 vs 0.74 ms for 8 Qwen3 layers + head at ctx 2048): with 12 warps per SM its
    // dot and staging phases are latency-bound.
    bool all = getenv("LOOM_CUDA_PERSISTENT") != nullptr;
    for (size_t li = 0; li < d->n_layers && all; li++) {
        const LayerRt &l = m->L[li];
        const loom_moe_desc &e = l.moe, &e0 = m->L[0].moe;
        all = l.fused && !l.dense && !e.shexp_gate && (e.n_local == 0 || e.n_local == e.n_expert) && e.expert0 == 0 &&
              e.n_group <= 1 && e.n_expert == e0.n_expert && e.n_used == e0.n_used && e.ffn == e0.ffn &&
              e.gating == e0.gating && e.weights_norm == e0.weights_norm && e.weights_scale == e0.weights_scale;
    }
    if (all) {
        std::vector<MkLayer> hl(d->n_layers);
        int tg = -1, tu = -1, td = -1;
        for (size_t li = 0; li < d->n_layers && all; li++) {
            const LayerRt &l = m->L[li];
            MkLayer &o = hl[li];
            o.attn_norm = l.attn_norm;
            o.ffn_norm = l.ffn_norm;
            o.q_norm = l.qn;
            o.k_norm = l.kn;
            o.wq = l.wq.w;
            o.wk = l.wk.w;
            o.wv = l.wv.w;
            o.wo = l.wo.w;
            o.kc = l.blk.kc;
            o.vc = l.blk.vc;
            WDev rw{};
            int rty = 0, gty = 0, uty = 0, dty = 0;
            uint64_t nb = 0, ng = 0, nu = 0, nd = 0;
            all = rt_tensor(l.moe.router, &rw, &rty, &nb) && rty == T_F32 && nb >= l.moe.n_expert * dim &&
                  rt_tensor(l.moe.gate, &o.g, &gty, &ng) && rt_tensor(l.moe.up, &o.u, &uty, &nu) &&
                  rt_tensor(l.moe.down, &o.dn, &dty, &nd);
            if (!all) break;
            const size_t be_g = block_elems(gty), be_d = block_elems(dty);
            all = be_g && be_d && ng >= l.moe.n_expert * l.moe.ffn * (dim / be_g) &&
                  nu >= l.moe.n_expert * l.moe.ffn * (dim / be_g) && nd >= l.moe.n_expert * dim * (l.moe.ffn / be_d) &&
                  (tg < 0 || (tg == gty && tu == uty && td == dty));
            tg = gty;
            tu = uty;
            td = dty;
            o.router = reinterpret_cast<const float *>(rw.q);
            o.bias = nullptr;
            if (l.moe.router_bias) {
                WDev bw{};
                int bty = 0;
                uint64_t bn = 0;
                all = all && rt_tensor(l.moe.router_bias, &bw, &bty, &bn) && bty == T_F32 && bn >= l.moe.n_expert;
                o.bias = reinterpret_cast<const float *>(bw.q);
            }
        }
        if (all) {
            const loom_moe_desc &e0 = m->L[0].moe;
            MkArgs &a = m->mk;
            a.n_layers = (int)d->n_layers;
            a.dim = (int)dim;
            a.n_heads = (int)m->nh;
            a.n_kv = (int)m->nkv;
            a.hd = (int)m->hd;
            a.rope_dim = (int)m->rope_dim;
            a.neox = m->neox;
            a.rope = m->rope;
            a.scale = m->scale;
            a.eps = m->eps;
            a.serial = m->serial_norm;
            a.ctx = (int)m->ctx;
            a.n_expert = (int)e0.n_expert;
            a.n_used = (int)e0.n_used;
            a.ffn = (int)e0.ffn;
            a.gating = e0.gating ? e0.gating : 1;
            a.weights_norm = e0.weights_norm;
            a.weights_scale = e0.weights_scale;
            a.q = m->q;
            a.k = m->k;
            a.v = m->v;
            a.part = m->part;
            a.nsplit = (int)((m->ctx + ATT_CH - 1) / ATT_CH);
            a.aq = m->a256.q;
            a.ad = m->a256.d;
            a.as = m->a256.s;
            a.bar = m->ab_bar;
            const LayerRt &l0 = m->L[0];
            if (model_kernel_plan(a, l0.wq.type, l0.wk.type, l0.wv.type, l0.wo.type, tg, tu, td)) {
                if ((rc = dalloc(*m, m->mk_layers, d->n_layers)) || (rc = dalloc(*m, m->mk_logits, e0.n_expert)) ||
                    (rc = dalloc(*m, m->mk_act, e0.n_used * e0.ffn)))
                    return bail(rc);
                cudaError_t ce = cudaMemcpy(m->mk_layers, hl.data(), hl.size() * sizeof(MkLayer), cudaMemcpyHostToDevice);
                if (ce != cudaSuccess) return bail(rt_fail("model layer table upload", ce));
                a.layers = m->mk_layers;
                a.logits = m->mk_logits;
                a.act = m->mk_act;
                m->persistent = true;
            }
        }
    }
    if (d->rope_dim) {
        const std::vector<float> tab = rope_table(d->ctx_len, d->rope_dim, d->rope_base);
        cudaError_t e = cudaMemcpy(m->rope, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(rt_fail("rope table upload", e));
    }
    cudaError_t e = cudaHostAlloc(&m->io_host, 16, cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaHostAlloc(&m->h_logits, d->vocab * 4, cudaHostAllocDefault);
    if (e != cudaSuccess) return bail(rt_fail("cudaHostAlloc(model staging)", e));
    const uint64_t h = g_next_model++;
    g_models[h] = m;
    *handle = h;
    return LOOM_CUDA_OK;
}

int loom_cuda_model_step(uint64_t handle, const uint32_t *d_token, const uint32_t *d_pos, float *d_logits,
                         uint32_t *d_next, void *stream) {
    if (int rc = rt_need_init()) return rc;
    Model *m = find(handle);
    if (!m) return rt_decline("unknown model handle");
    if (!d_token || !d_pos) return rt_decline("token and position pointers are required");
    return run_step(*m, d_token, d_pos, d_logits, d_next, rt_stream(stream));
}

int loom_cuda_model_decode(uint64_t handle, uint32_t token, size_t pos, float *logits, uint32_t *next) {
    if (int rc = rt_need_init()) return rc;
    Model *m = find(handle);
    if (!m) return rt_decline("unknown model handle");
    if (token >= m->vocab) return rt_decline("token id out of range (llama.zig:1121)");
    if (pos >= m->ctx) return rt_decline("position beyond the context length");
    cudaStream_t st = rt_stream(nullptr);
    m->io_host[0] = token;
    m->io_host[1] = (uint32_t)pos;
    // one H2D copy of (token, pos), the step, one D2H copy of the token
    auto record = [&]() -> int {
        MCK(cudaMemcpyAsync(m->io_dev, m->io_host, 8, cudaMemcpyHostToDevice, st));
        if (int rc = run_step(*m, m->io_dev, m->io_dev + 1, m->logits, m->io_dev + 2, st)) return rc;
        MCK(cudaMemcpyAsync(m->io_host + 2, m->io_dev + 2, 4, cudaMemcpyDeviceToHost, st));
        return 0;
    };
    if (m->exec && m->exec_gen != rt_buf_gen()) {  // a scratch buffer the graph points at has moved
        cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    if (!m->exec && m->calls++ > 0) {  // the first call runs eagerly (sizes every buffer); then capture
        const uint64_t gen = rt_buf_gen();
        MCK(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
        const int rc = record();
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(st, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return rt_fail("cudaStreamEndCapture(model)", e);
        e = cudaGraphInstantiate(&m->exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) {
            m->exec = nullptr;
            return rt_fail("cudaGraphInstantiate(model)", e);
        }
        m->exec_gen = gen;
    }
    if (m->exec) {
        MCK(cudaGraphLaunch(m->exec, st));
    } else if (int rc = record()) {
        return rc;
    }
    if (logits) MCK(cudaMemcpyAsync(m->h_logits, m->logits, m->vocab * 4, cudaMemcpyDeviceToHost, st));
    MCK(rt_wait());
    if (next) *next = m->io_host[2];
    if (logits) std::memcpy(logits, m->h_logits, m->vocab * 4);
    return LOOM_CUDA_OK;
}

int loom_cuda_model_prefill(uint64_t handle, const uint32_t *tokens, size_t n, size_t pos_base, float *logits,
                            uint32_t *next) {
    if (int rc = rt_need_init()) return rc;
    Model *mp = find(handle);
    if (!mp) return rt_decline("unknown model handle");
    Model &m = *mp;
    if (m.mla) return rt_decline("prefill: multi-head latent attention models decode token by token");
    if (m.persistent) return rt_decline("prefill: not with the persistent whole-token kernel");
    if (!tokens || n == 0) return rt_decline("prefill: no tokens");
    if (pos_base + n > m.ctx) return rt_decline("prefill: positions beyond the context");
    for (size_t i = 0; i < n; i++)
        if (tokens[i] >= m.vocab) return rt_decline("prefill: token id out of range");
    if ((size_t)ATT_ORDERED_LIMIT < m.ctx) return rt_decline("prefill: context beyond the ordered attention's limit");
    if (int rc = alloc_prefill(m, n)) return rc;
    if (int rc = loom_cuda_reserve(n, m.dim, std::max<size_t>(m.max_ffn, 1), m.max_ne, m.max_nu)) return rc;
    cudaStream_t st = rt_stream(nullptr);
    const uint32_t pb = (uint32_t)pos_base;
    MCK(cudaMemcpyAsync(m.pf_tok, tokens, n * 4, cudaMemcpyHostToDevice, st));
    MCK(cudaMemcpyAsync(m.pf_pos, &pb, 4, cudaMemcpyHostToDevice, st));
    const int cur = run_prefill(m, (int)n, (int)pos_base, st);
    if (cur < 0 || cur > 1) return cur;
    // the last token: final RMSNorm, the head, the argmax (llama.zig:1820-1824)
    const XQW none{};
    XQW o256 = none, o32 = none;
    if (m.out.type != T_F32 && m.out.type != T_Q5_0) {
        if (act256(m.out.type))
            o256 = m.n256;
        else
            o32 = m.n32;
    }
    launch_rmsnorm_q(m.pf_x[cur] + (n - 1) * m.dim, nullptr, m.out_norm, (int)m.dim, m.eps, m.normed, o256, o32,
                     m.serial_norm, st);
    matvec(m.out, m.normed, m.n256, m.n32, m.logits, st);
    if (int rc = loom_cuda_argmax(m.logits, m.vocab, m.io_dev + 2, st)) return rc;
    if (logits) MCK(cudaMemcpyAsync(logits, m.logits, m.vocab * 4, cudaMemcpyDeviceToHost, st));
    uint32_t nx = 0;
    MCK(cudaMemcpyAsync(&nx, m.io_dev + 2, 4, cudaMemcpyDeviceToHost, st));
    MCK(cudaStreamSynchronize(st));
    if (next) *next = nx;
    return LOOM_CUDA_OK;
}

int loom_cuda_model_decode_batch(uint64_t handle, const uint32_t *tokens, const uint32_t *positions, size_t B,
                                 float *logits, uint32_t *next) {
    if (int rc = rt_need_init()) return rc;
    Model *mp = find(handle);
    if (!mp) return rt_decline("unknown model handle");
    Model &m = *mp;
    if (m.mla) return rt_decline("decode_batch: multi-head latent attention models decode one sequence");
    if (m.persistent) return rt_decline("decode_batch: not with the persistent whole-token kernel");
    if (!tokens || !positions || B == 0) return rt_decline("decode_batch: no sequences");
    if (m.bd_cap && B > m.bd_cap) return rt_decline("decode_batch: more sequences than the first call's batch");
    for (size_t i = 0; i < B; i++)
        if (tokens[i] >= m.vocab || positions[i] >= m.ctx) return rt_decline("decode_batch: token or position out of range");
    if ((size_t)ATT_ORDERED_LIMIT < m.ctx) return rt_decline("decode_batch: context beyond the ordered attention's limit");
    if (int rc = alloc_prefill(m, B)) return rc;
    if (!m.bd_cap) {  // the sequences' caches (zeroed), logits and next tokens, sized by the first call
        const size_t cache = B * m.n_layers * m.ctx * m.nkv * m.hd;
        int rc = 0;
        if ((rc = dalloc(m, m.bkc, cache, true)) || (rc = dalloc(m, m.bvc, cache, true)) ||
            (rc = dalloc(m, m.bd_logits, B * m.vocab)) || (rc = dalloc(m, m.bd_pos, B)) || (rc = dalloc(m, m.bd_next, B)) ||
            (rc = dalloc(m, m.bd_part, B * attn_part_floats((int)m.nh, (int)m.nkv, (int)m.hd, (int)m.ctx))))
            return rc;
        m.bd_cap = B;
    }
    if (int rc = loom_cuda_reserve(B, m.dim, std::max<size_t>(m.max_ffn, 1), m.max_ne, m.max_nu)) return rc;
    cudaStream_t st = rt_stream(nullptr);
    MCK(cudaMemcpyAsync(m.pf_tok, tokens, B * 4, cudaMemcpyHostToDevice, st));
    MCK(cudaMemcpyAsync(m.bd_pos, positions, B * 4, cudaMemcpyHostToDevice, st));
    if (int rc = run_decode_batch(m, (int)B, st)) return rc;
    if (logits) MCK(cudaMemcpyAsync(logits, m.bd_logits, B * m.vocab * 4, cudaMemcpyDeviceToHost, st));
    if (next) MCK(cudaMemcpyAsync(next, m.bd_next, B * 4, cudaMemcpyDeviceToHost, st));
    MCK(cudaStreamSynchronize(st));
    return LOOM_CUDA_OK;
}

int loom_cuda_model_read_kv(uint64_t handle, size_t layer, size_t pos, float *k, float *v) {
    if (int rc = rt_need_init()) return rc;
    Model *m = find(handle);
    if (!m) return rt_decline("unknown model handle");
    if (layer >= m->n_layers || pos >= m->ctx) return rt_decline("cache row out of range");
    // GQA: key and value rows (n_kv*hd each); MLA: compressed row (kv_lora) and rope row (rope_dim)
    const size_t kw = m->mla ? m->kvr : m->nkv * m->hd, vw = m->mla ? m->rope_dim : m->nkv * m->hd;
    MCK(cudaStreamSynchronize(rt_stream(nullptr)));
    if (k) MCK(cudaMemcpy(k, m->kc + (layer * m->ctx + pos) * kw, kw * 4, cudaMemcpyDeviceToHost));
    if (v) MCK(cudaMemcpy(v, m->vc + (layer * m->ctx + pos) * vw, vw * 4, cudaMemcpyDeviceToHost));
    return LOOM_CUDA_OK;
}

int loom_cuda_model_error(uint64_t handle) {
    Model *m = find(handle);
    if (!m) return -1;
    if (cudaStreamSynchronize(rt_stream(nullptr)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return -1;
    unsigned long long h[4] = {};
    if (cudaMemcpy(h, m->ab_bar, sizeof h, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    const int e = (int)(unsigned)h[2];
    if (e && cudaMemset(m->ab_bar, 0, 32 * sizeof(unsigned long long)) != cudaSuccess) return -1;  // re-arm (counter, flag)
    return e;
}

int loom_cuda_model_trace(uint64_t handle, int layer, unsigned long long *out, size_t n) {
    if (int rc = rt_need_init()) return rc;
    Model *m = find(handle);
    if (!m) return rt_decline("unknown model handle");
    if (layer >= 0) {
        if ((size_t)layer >= m->n_layers) return rt_decline("layer out of range");
        if (!m->ab_trace) MCK(cudaMalloc(&m->ab_trace, 32 * sizeof(unsigned long long)));
        MCK(cudaMemset(m->ab_trace, 0, 32 * sizeof(unsigned long long)));
        for (auto &l : m->L) l.blk.trace = nullptr;
        m->L[layer].blk.trace = m->ab_trace;
        if (m->exec) {  // a captured graph holds the old arguments
            cudaGraphExecDestroy(m->exec);
            m->exec = nullptr;
        }
        return LOOM_CUDA_OK;
    }
    if (!m->ab_trace) return rt_decline("tracing was not enabled");
    MCK(cudaDeviceSynchronize());
    MCK(cudaMemcpy(out, m->ab_trace, std::min<size_t>(n, 32) * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    return LOOM_CUDA_OK;
}

int loom_cuda_model_free(uint64_t handle) {
    Model *m = find(handle);
    if (!m) return LOOM_CUDA_DECLINED;
    cudaDeviceSynchronize();
    g_models.erase(handle);
    free_model(m);
    return LOOM_CUDA_OK;
}

}  // extern "C"
