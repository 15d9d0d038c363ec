"""ctypes view of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle (loom_oracle.cpp) restates the reference's CPU kernels
(ch4r10t33r/loom src/gguf/ggml.zig, src/gguf/moe.zig, src/core/tensor.zig).
Only the test suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg use it, and only as the checker / the timed CPU reference. The
product library never loads it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libloom_oracle.so")

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 6, 7, 8, 10, 11, 12, 13, 14
BLOCK_ELEMS = {F32: 1, Q4_0: 32, Q4_1: 32, Q5_0: 32, Q5_1: 32, Q8_0: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256,
               Q6_K: 256}
BLOCK_BYTES = {F32: 4, Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q8_0: 34, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176,
               Q6_K: 210}


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, sz, fp = C.c_void_p, C.c_size_t, C.c_float
        L.or_row_bytes.restype = sz
        L.or_row_bytes.argtypes = [C.c_int, sz]
        L.or_dequant_row.argtypes = [C.c_int, vp, vp, sz, sz]
        L.or_matvec.argtypes = [C.c_int, vp, vp, vp, sz, sz]
        L.or_matmul.argtypes = [C.c_int, vp, vp, vp, sz, sz, sz]
        L.or_dot_f32.restype = fp
        L.or_dot_f32.argtypes = [vp, vp, sz]
        L.or_quantize_x256.argtypes = [vp, sz, vp, vp, vp]
        L.or_quantize_x32.argtypes = [vp, sz, vp, vp, vp]
        L.or_softmax.argtypes = [vp, sz]
        L.or_silu.restype = fp
        L.or_silu.argtypes = [fp]
        L.or_sigmoid.restype = fp
        L.or_sigmoid.argtypes = [fp]
        L.or_route.argtypes = [vp, vp, sz, sz, C.c_int, C.c_int, fp, vp, vp]
        L.or_argmax.restype = sz
        L.or_argmax.argtypes = [vp, sz]
        L.or_route_grouped.argtypes = [vp, vp, sz, sz, C.c_int, C.c_int, fp, sz, sz, vp, vp]
        L.or_moe_ffn_block.argtypes = [vp, sz, vp, sz, vp]
        L.or_moe_ffn_routed.argtypes = [vp, sz, vp, vp, C.c_int, vp, C.c_int, vp, C.c_int, vp, sz,
                                        vp, vp, sz, sz, sz, C.c_int, C.c_int, fp, vp]
        L.or_moe_layer.argtypes = [vp, sz, sz, vp, C.c_int, vp, C.c_int, vp, C.c_int, vp, sz, sz,
                                   sz, C.c_int, C.c_int, fp, vp, vp]
        L.or_llama_step.argtypes = [vp, vp, vp, C.c_uint32, sz, vp]
        L.or_deepseek_step.argtypes = [vp, vp, vp, C.c_uint32, sz, vp]
        L.or_synth.argtypes = [C.c_int, vp, C.c_uint64, C.c_uint64, C.c_uint64, fp]
        L.or_f32_to_f16_rne.restype = C.c_uint16
        L.or_f32_to_f16_rne.argtypes = [fp]
        L.or_parallel_begin.argtypes = [C.c_int]
        L.or_pool_workers.restype = C.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


class Expert(C.Structure):
    _fields_ = [("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("weight", C.c_float), ("ffn", C.c_size_t)]


def row_bytes(t: int, n: int) -> int:
    return int(lib().or_row_bytes(t, n))


def parallel_begin(n: int) -> None:
    lib().or_parallel_begin(n)


def parallel_end() -> None:
    lib().or_parallel_end()


def dequant_row(t, data, r, cols):
    out = np.empty(cols, np.float32)
    assert lib().or_dequant_row(t, _p(out), _p(data), r, cols) == 0
    return out


def dequant(t, data, rows, cols):
    return np.stack([dequant_row(t, data, r, cols) for r in range(rows)])


def matvec(t, data, x, rows, cols):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(rows, np.float32)
    assert lib().or_matvec(t, _p(out), _p(data), _p(x), rows, cols) == 0
    return out


def matmul(t, data, xs, rows, cols):
    xs = np.ascontiguousarray(xs, np.float32)
    n = xs.shape[0]
    out = np.empty((n, rows), np.float32)
    assert lib().or_matmul(t, _p(out), _p(data), _p(xs), n, rows, cols) == 0
    return out


def dot_f32(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().or_dot_f32(_p(a), _p(b), a.size))


def quantize_x256(x):
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    q = np.empty(n, np.int8)
    d = np.empty(n // 256, np.float32)
    s = np.empty(n // 16, np.int32)
    lib().or_quantize_x256(_p(x), n, _p(q), _p(d), _p(s))
    return q, d, s


def quantize_x32(x):
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    q = np.empty(n, np.int8)
    d = np.empty(n // 32, np.float32)
    s = np.empty(n // 32, np.int32)
    lib().or_quantize_x32(_p(x), n, _p(q), _p(d), _p(s))
    return q, d, s


def softmax(x):
    x = np.array(x, np.float32)
    lib().or_softmax(_p(x), x.size)
    return x


def silu(v):
    return float(lib().or_silu(v))


def sigmoid(v):
    return float(lib().or_sigmoid(v))


def argmax(logits):
    """sampler.zig:7-15 argmax."""
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().or_argmax(_p(logits), logits.size))


def route(logits, n_used, gating=1, weights_norm=True, weights_scale=1.0, bias=None, n_group=1,
          topk_group=1):
    """moe.zig:106-158 route; n_group > 1 adds DeepSeek-V3's group-limited
    selection (or_route_grouped)."""
    logits = np.ascontiguousarray(logits, np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ids = np.empty(n_used, np.uint32)
    gates = np.empty(n_used, np.float32)
    if n_group > 1:
        rc = lib().or_route_grouped(_p(logits), _p(bias), logits.size, n_used, gating, int(weights_norm),
                                    weights_scale, n_group, topk_group, _p(ids), _p(gates))
        assert rc == 0
        return ids, gates
    rc = lib().or_route(_p(logits), _p(bias), logits.size, n_used, gating, int(weights_norm),
                        weights_scale, _p(ids), _p(gates))
    assert rc == 0
    return ids, gates


def moe_ffn_block(normed, experts, dim):
    """experts: list of dicts {gate_type, up_type, down_type, gate, up, down, weight, ffn}."""
    normed = np.ascontiguousarray(normed, np.float32)
    arr = (Expert * len(experts))()
    keep = []
    for i, e in enumerate(experts):
        keep += [e["gate"], e["up"], e["down"]]
        arr[i] = Expert(e["gate_type"], e["up_type"], e["down_type"], _p(e["gate"]).value,
                        _p(e["up"]).value, _p(e["down"]).value, e["weight"], e["ffn"])
    out = np.empty(dim, np.float32)
    assert lib().or_moe_ffn_block(_p(normed), dim, C.cast(arr, C.c_void_p), len(experts), _p(out)) == 0
    return out


def moe_ffn_routed(normed, logits, gate, up, down, ffn, n_used, gating_sigmoid=False,
                   weights_norm=True, weights_scale=1.0, bias=None, shexp=None, shexp_ffn=0):
    """gate/up/down: (type, bytes) of the full 3D tensors; shexp: 3 x (type, bytes) or None."""
    normed = np.ascontiguousarray(normed, np.float32)
    logits = np.ascontiguousarray(logits, np.float32)
    dim = normed.size
    out = np.empty(dim, np.float32)
    st = sp = None
    if shexp is not None:
        st = (C.c_int * 3)(*[t for t, _ in shexp])
        sp = (C.c_void_p * 3)(*[_p(b).value for _, b in shexp])
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().or_moe_ffn_routed(_p(normed), dim, _p(logits), _p(b), gate[0], _p(gate[1]), up[0],
                                 _p(up[1]), down[0], _p(down[1]), ffn,
                                 C.cast(st, C.c_void_p) if st else None,
                                 C.cast(sp, C.c_void_p) if sp else None, shexp_ffn, logits.size,
                                 n_used, int(gating_sigmoid), int(weights_norm), weights_scale, _p(out))
    assert rc == 0
    return out


def moe_layer(x, router_w, gate, up, down, ffn, n_expert, n_used, gating=1, weights_norm=True,
              weights_scale=1.0):
    x = np.ascontiguousarray(x, np.float32)
    T, dim = x.shape
    out = np.empty((T, dim), np.float32)
    ids = np.empty((T, n_used), np.uint32)
    rc = lib().or_moe_layer(_p(x), T, dim, _p(router_w), gate[0], _p(gate[1]), up[0], _p(up[1]),
                            down[0], _p(down[1]), ffn, n_expert, n_used, gating, int(weights_norm),
                            weights_scale, _p(out), _p(ids))
    assert rc == 0
    return out, ids


def synth(t, nblk, seed, blk0=0, sigma=1.0):
    """Seeded synthetic blocks (same generator as the CUDA backend's device synth)."""
    nbytes = nblk * BLOCK_BYTES[t]
    out = np.empty(nbytes, np.uint8)
    lib().or_synth(t, _p(out), blk0, nblk, seed, sigma)
    return out.view(np.float32) if t == F32 else out


def f32_to_f16_rne(v):
    return int(lib().or_f32_to_f16_rne(v))


class LlamaLayer(C.Structure):
    """or_llama_layer: one decoder layer (llama.zig:136-200)."""
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p),
                ("wq_type", C.c_int), ("wk_type", C.c_int), ("wv_type", C.c_int), ("wo_type", C.c_int),
                ("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("ffn", C.c_size_t), ("router", C.c_void_p)]


class LlamaModel(C.Structure):
    """or_llama_model."""
    _fields_ = [("dim", C.c_size_t), ("n_layers", C.c_size_t), ("n_heads", C.c_size_t), ("n_kv_heads", C.c_size_t),
                ("head_dim", C.c_size_t), ("rope_dim", C.c_size_t), ("vocab", C.c_size_t), ("ctx_len", C.c_size_t),
                ("eps", C.c_float), ("rope_base", C.c_float), ("attn_logit_mul", C.c_float),
                ("rope_neox", C.c_int), ("n_expert", C.c_size_t), ("n_used", C.c_size_t),
                ("gating", C.c_int), ("weights_norm", C.c_int), ("weights_scale", C.c_float),
                ("embd_type", C.c_int), ("token_embd", C.c_void_p), ("output_norm", C.c_void_p),
                ("output_type", C.c_int), ("output", C.c_void_p), ("layers", C.POINTER(LlamaLayer))]


class LlamaRunner:
    """llama.zig:1111-1228 step on host tensors, with its own f32 KV cache.

    `tensors` maps the GGUF tensor names of a model spec (loom_b200.model.ModelSpec)
    to (type, numpy bytes or floats)."""

    def __init__(self, spec, tensors):
        self.spec, self.t = spec, tensors  # keep the arrays alive
        c = spec
        self._layers = (LlamaLayer * c.n_layers)()
        for i in range(c.n_layers):
            L = self._layers[i]
            g = lambda n: tensors.get(f"blk.{i}.{n}")  # noqa: E731
            L.attn_norm, L.ffn_norm = _p(g("attn_norm")[1]), _p(g("ffn_norm")[1])
            for nm, tn in (("q", "attn_q"), ("k", "attn_k"), ("v", "attn_v"), ("o", "attn_output")):
                ty, data = g(tn)
                setattr(L, f"w{nm}_type", ty)
                setattr(L, f"w{nm}", _p(data))
            L.q_norm = _p(g("attn_q_norm")[1]) if g("attn_q_norm") else None
            L.k_norm = _p(g("attn_k_norm")[1]) if g("attn_k_norm") else None
            moe = g("ffn_gate_inp") is not None
            sfx = "_exps" if moe else ""
            for nm in ("gate", "up", "down"):
                ty, data = g(f"ffn_{nm}{sfx}")
                setattr(L, f"{nm}_type", ty)
                setattr(L, nm, _p(data))
            L.ffn = c.moe_ffn if moe else c.ffn
            L.router = _p(g("ffn_gate_inp")[1]) if moe else None
        M = LlamaModel()
        M.dim, M.n_layers, M.n_heads, M.n_kv_heads = c.dim, c.n_layers, c.n_heads, c.n_kv_heads
        M.head_dim, M.rope_dim, M.vocab, M.ctx_len = c.head_dim, c.rope_dim, c.vocab, c.ctx_len
        M.eps, M.rope_base, M.attn_logit_mul, M.rope_neox = c.eps, c.rope_base, 1.0, int(c.rope_neox)
        M.n_expert, M.n_used, M.gating, M.weights_norm, M.weights_scale = c.n_expert, c.n_used, 1, 1, 1.0
        M.embd_type, M.token_embd = tensors["token_embd"][0], _p(tensors["token_embd"][1])
        M.output_norm = _p(tensors["output_norm"][1])
        M.output_type, M.output = tensors["output"][0], _p(tensors["output"][1])
        M.layers = self._layers
        self.m = M
        kvd = c.n_kv_heads * c.head_dim
        self.kc = np.zeros(c.n_layers * c.ctx_len * kvd, np.float32)
        self.vc = np.zeros_like(self.kc)

    def step(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self.spec.vocab, np.float32)
        rc = lib().or_llama_step(C.byref(self.m), _p(self.kc), _p(self.vc), token, pos, _p(logits))
        assert rc == 0
        return logits


class DsLayer(C.Structure):
    """or_ds_layer: one DeepSeek-V2/V3 decoder layer."""
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p),
                ("wq_type", C.c_int), ("wq", C.c_void_p),
                ("q_a_type", C.c_int), ("q_a", C.c_void_p), ("q_a_norm", C.c_void_p),
                ("q_b_type", C.c_int), ("q_b", C.c_void_p),
                ("kv_a_type", C.c_int), ("kv_a", C.c_void_p), ("kv_a_norm", C.c_void_p),
                ("kv_b_type", C.c_int), ("kv_b", C.c_void_p), ("wo_type", C.c_int), ("wo", C.c_void_p),
                ("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p), ("ffn", C.c_size_t),
                ("router", C.c_void_p), ("router_bias", C.c_void_p),
                ("sh_gate_type", C.c_int), ("sh_up_type", C.c_int), ("sh_down_type", C.c_int),
                ("sh_gate", C.c_void_p), ("sh_up", C.c_void_p), ("sh_down", C.c_void_p), ("sh_ffn", C.c_size_t)]


class DsModel(C.Structure):
    """or_ds_model."""
    _fields_ = [("dim", C.c_size_t), ("n_layers", C.c_size_t), ("n_heads", C.c_size_t), ("nope", C.c_size_t),
                ("rope", C.c_size_t), ("kv_lora", C.c_size_t), ("q_lora", C.c_size_t), ("v_head", C.c_size_t),
                ("vocab", C.c_size_t), ("ctx_len", C.c_size_t), ("eps", C.c_float), ("rope_base", C.c_float),
                ("attn_scale", C.c_float), ("n_expert", C.c_size_t), ("n_used", C.c_size_t),
                ("gating_sigmoid", C.c_int), ("weights_norm", C.c_int), ("weights_scale", C.c_float),
                ("embd_type", C.c_int), ("token_embd", C.c_void_p), ("output_norm", C.c_void_p),
                ("output_type", C.c_int), ("output", C.c_void_p), ("layers", C.POINTER(DsLayer)),
                ("n_group", C.c_size_t), ("topk_group", C.c_size_t)]


class DeepseekRunner:
    """deepseek.zig:1275-1537 step (attnLayer :851-1049) on host tensors, with
    its own compressed caches (c: [layers][ctx][kv_lora], r: [layers][ctx][rope])."""

    def __init__(self, spec, tensors):
        self.spec, self.t = spec, tensors
        c = spec
        self._layers = (DsLayer * c.n_layers)()
        for i in range(c.n_layers):
            L = self._layers[i]

            def g(n, i=i):
                return tensors.get(f"blk.{i}.{n}")

            def tp(n):
                return g(n)[0] if g(n) else 0

            def pp(n):
                return _p(g(n)[1]) if g(n) else None
            L.attn_norm, L.ffn_norm = pp("attn_norm"), pp("ffn_norm")
            L.wq_type, L.wq = tp("attn_q"), pp("attn_q")
            L.q_a_type, L.q_a, L.q_a_norm = tp("attn_q_a"), pp("attn_q_a"), pp("attn_q_a_norm")
            L.q_b_type, L.q_b = tp("attn_q_b"), pp("attn_q_b")
            L.kv_a_type, L.kv_a, L.kv_a_norm = tp("attn_kv_a_mqa"), pp("attn_kv_a_mqa"), pp("attn_kv_a_norm")
            L.kv_b_type, L.kv_b = tp("attn_kv_b"), pp("attn_kv_b")
            L.wo_type, L.wo = tp("attn_output"), pp("attn_output")
            moe = g("ffn_gate_inp") is not None
            sfx = "_exps" if moe else ""
            L.gate_type, L.up_type, L.down_type = tp("ffn_gate" + sfx), tp("ffn_up" + sfx), tp("ffn_down" + sfx)
            L.gate, L.up, L.down = pp("ffn_gate" + sfx), pp("ffn_up" + sfx), pp("ffn_down" + sfx)
            L.ffn = c.moe_ffn if moe else c.ffn
            L.router, L.router_bias = pp("ffn_gate_inp"), pp("exp_probs_b.bias")
            L.sh_gate_type, L.sh_up_type = tp("ffn_gate_shexp"), tp("ffn_up_shexp")
            L.sh_down_type = tp("ffn_down_shexp")
            L.sh_gate, L.sh_up, L.sh_down = pp("ffn_gate_shexp"), pp("ffn_up_shexp"), pp("ffn_down_shexp")
            L.sh_ffn = c.shexp_ffn
        M = DsModel()
        M.dim, M.n_layers, M.n_heads, M.nope, M.rope = c.dim, c.n_layers, c.n_heads, c.nope, c.rope_dim
        M.kv_lora, M.q_lora, M.v_head, M.vocab, M.ctx_len = c.kv_lora, c.q_lora, c.v_head, c.vocab, c.ctx_len
        M.eps, M.rope_base, M.attn_scale = c.eps, c.rope_base, c.attn_scale
        M.n_expert, M.n_used, M.gating_sigmoid = c.n_expert, c.n_used, int(c.gating == 2)
        M.weights_norm, M.weights_scale = int(c.weights_norm), c.weights_scale
        M.embd_type, M.token_embd = tensors["token_embd"][0], _p(tensors["token_embd"][1])
        M.output_norm = _p(tensors["output_norm"][1])
        M.output_type, M.output = tensors["output"][0], _p(tensors["output"][1])
        M.layers = self._layers
        M.n_group, M.topk_group = c.n_group, c.topk_group
        self.m = M
        self.cc = np.zeros(c.n_layers * c.ctx_len * c.kv_lora, np.float32)
        self.rc = np.zeros(c.n_layers * c.ctx_len * c.rope_dim, np.float32)

    def step(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self.spec.vocab, np.float32)
        rc = lib().or_deepseek_step(C.byref(self.m), _p(self.cc), _p(self.rc), token, pos, _p(logits))
        assert rc == 0
        return logits
