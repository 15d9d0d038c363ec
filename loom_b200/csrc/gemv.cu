// gemv.cu -- one-token matvec on the warp engine (warpdot.cuh): each warp
// takes S consecutive rows, issues every 16-byte weight load of those rows
// before touching the activations (so the loads are in flight while the
// producer of x is still finishing: programmatic dependent launch), then
// forms the reference's integer block dots and adds each row's block terms in
// block order (ggml.zig:1002-1042 kBlockDot / matvecK256; :1196 / :1277 for
// Q4_0 / Q8_0). Bit-identical to k_mm and to the CPU reference.
#include "gemv.cuh"
#include "pdl.cuh"
#include "warpdot.cuh"

namespace loom {

namespace {

constexpr int GV_WARPS = 8;

struct GvRows {
    WDev w;
    int r0, nb;
    XQ x;
    __device__ __forceinline__ void at(int s, WDev &ww, uint64_t &gb, XV &xv) const {
        ww = w;
        gb = (uint64_t)(r0 + s) * nb;
        xv = XV{x.q, x.d, x.s};
    }
};

template <int TY, int S, int MAXU>
__global__ void __launch_bounds__(GV_WARPS * 32) k_gemv(WDev w, int rows, int nb, XQ x, float *out) {
    const int lane = threadIdx.x & 31;
    const int r0 = (blockIdx.x * GV_WARPS + (threadIdx.x >> 5)) * S;
    if (r0 >= rows) {
        pdl_wait_();
        return;
    }
    const int nS = min(S, rows - r0);
    const GvRows st{w, r0, nb, x};
    WFrags<TY, MAXU> fr;
    wd_load<TY, S, MAXU>(st, nb, nS, fr, lane);
    pdl_wait_();
    pdl_trigger_();
    float acc[S];
    wd_finish<TY, S, MAXU>(st, nb, nS, fr, acc, lane);
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < S; s++)
            if (s < nS) out[r0 + s] = acc[s];
    }
}

// units a warp holds: MAXU fragments x (32 / lanes per block)
template <int TY> constexpr int gv_maxu() { return TY == T_Q4_K ? 8 : TY == T_Q6_K ? 4 : TY == T_Q8_0 ? 4 : 2; }
template <int TY> constexpr int gv_units() { return gv_maxu<TY>() * (32 / QT<TY>::LPB); }

template <int TY> cudaError_t gv_launch(const WDev &w, int rows, int nb, const XQ &x, float *out, cudaStream_t st) {
    constexpr int MAXU = gv_maxu<TY>();
    const int cap = gv_units<TY>() / nb;  // rows a warp can hold
    if (cap >= 4)
        return launch_pdl_(k_gemv<TY, 4, MAXU>, dim3((rows + GV_WARPS * 4 - 1) / (GV_WARPS * 4)), dim3(GV_WARPS * 32),
                           0, st, w, rows, nb, x, out);
    if (cap >= 2)
        return launch_pdl_(k_gemv<TY, 2, MAXU>, dim3((rows + GV_WARPS * 2 - 1) / (GV_WARPS * 2)), dim3(GV_WARPS * 32),
                           0, st, w, rows, nb, x, out);
    return launch_pdl_(k_gemv<TY, 1, MAXU>, dim3((rows + GV_WARPS - 1) / GV_WARPS), dim3(GV_WARPS * 32), 0, st, w,
                       rows, nb, x, out);
}

}  // namespace

bool gemv_supported(int type, int cols) {
    const int be = block_elems(type);
    if (be == 0 || cols % be) return false;
    const int nb = cols / be;
    switch (type) {
        case T_Q4_K: return nb <= gv_units<T_Q4_K>();
        case T_Q6_K: return nb <= gv_units<T_Q6_K>();
        case T_Q8_0: return nb <= gv_units<T_Q8_0>();
        case T_Q4_0: return nb <= gv_units<T_Q4_0>();
        default: return false;
    }
}

cudaError_t launch_gemv(const WDev &w, int rows, int cols, const XQ &x, float *out, cudaStream_t st) {
    const int nb = cols / block_elems(w.type);
    switch (w.type) {
        case T_Q4_K: return gv_launch<T_Q4_K>(w, rows, nb, x, out, st);
        case T_Q6_K: return gv_launch<T_Q6_K>(w, rows, nb, x, out, st);
        case T_Q8_0: return gv_launch<T_Q8_0>(w, rows, nb, x, out, st);
        case T_Q4_0: return gv_launch<T_Q4_0>(w, rows, nb, x, out, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace loom
