"""Whole-model decode on the device (include/loom_cuda.h, loom_cuda_model_*).

`ModelSpec` describes a decoder in the reference's tensor naming (GGUF names,
src/gguf/llama.zig:136-200) and shapes; `DeviceModel` holds its tensors on the
GPU and runs the reference's token step (llama.zig:1111-1228) there. The
weights are seeded synthetic tensors generated on the device by the backend's
counter-based generator (the same bytes `oracle.synth` makes on the host), so a
test can build the identical model on both sides.
"""
from __future__ import annotations

import ctypes as C
import zlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from . import _lib
from .device import BLOCK_BYTES, DeviceTensor

F32, Q4_0, Q8_0, Q4_K, Q6_K = 0, 2, 8, 12, 14
BLOCK_ELEMS = {0: 1, 2: 32, 3: 32, 6: 32, 7: 32, 8: 32, 10: 256, 11: 256, 12: 256, 13: 256, 14: 256}


@dataclass
class TensorPlan:
    name: str
    type: int
    rows: int
    cols: int
    planes: int = 1         # 3D expert tensors: [planes][rows][cols]
    fill: str = "synth"     # synth | ones | near_ones
    sigma: float = 1.0      # f32 synth standard deviation
    seed: int = 0

    @property
    def nblk(self) -> int:
        return self.planes * self.rows * self.cols // BLOCK_ELEMS[self.type]

    @property
    def nbytes(self) -> int:
        return self.nblk * BLOCK_BYTES[self.type]


@dataclass
class ModelSpec:
    name: str
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    ctx_len: int
    eps: float = 1e-5
    rope_base: float = 10000.0
    rope_neox: bool = False
    rope_dim: int = 0            # 0: head_dim
    qk_norm: bool = False
    ffn: int = 0                 # dense FFN width (n_expert == 0)
    n_expert: int = 0
    n_used: int = 0
    moe_ffn: int = 0
    types: Dict[str, int] = field(default_factory=dict)
    norms: str = "ones"          # ones | near_ones
    seed: int = 1
    # DeepSeek-V2/V3 (deepseek2 arch): multi-head latent attention and MoE extras
    mla: bool = False
    kv_lora: int = 0
    q_lora: int = 0
    nope: int = 0
    v_head: int = 0
    n_dense: int = 0             # leading dense-FFN layers (ffn wide)
    shexp_ffn: int = 0           # shared expert width (0: none)
    gating: int = 1              # 1 softmax, 2 sigmoid
    weights_norm: bool = True
    weights_scale: float = 1.0
    router_bias: bool = False
    n_group: int = 1
    topk_group: int = 1

    def __post_init__(self):
        if not self.rope_dim:
            self.rope_dim = self.head_dim

    @property
    def attn_scale(self) -> float:
        """MLA softmax scale 1 / sqrt(nope + rope) (deepseek.zig:360, no YaRN)."""
        import math
        return float(np.float32(1.0) / np.float32(math.sqrt(float(self.nope + self.rope_dim))))

    def is_moe_layer(self, i: int) -> bool:
        return self.n_expert > 0 and i >= self.n_dense

    def ty(self, key: str) -> int:
        return self.types[key]

    def plan(self) -> List[TensorPlan]:
        """Every tensor of the model, in a fixed order (the seeds follow the names)."""
        d, qd, kvd = self.dim, self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        out = [TensorPlan("token_embd", self.ty("embd"), self.vocab, d, sigma=0.02),
               TensorPlan("output_norm", F32, 1, d, fill=self.norms),
               TensorPlan("output", self.ty("output"), self.vocab, d)]
        for i in range(self.n_layers):
            p = f"blk.{i}."
            out += [TensorPlan(p + "attn_norm", F32, 1, d, fill=self.norms)]
            if self.mla:
                kd = self.nope + self.rope_dim
                if self.q_lora:
                    out += [TensorPlan(p + "attn_q_a", self.ty("attn_q_a"), self.q_lora, d),
                            TensorPlan(p + "attn_q_a_norm", F32, 1, self.q_lora, fill=self.norms),
                            TensorPlan(p + "attn_q_b", self.ty("attn_q_b"), self.n_heads * kd, self.q_lora)]
                else:
                    out += [TensorPlan(p + "attn_q", self.ty("attn_q"), self.n_heads * kd, d)]
                out += [TensorPlan(p + "attn_kv_a_mqa", self.ty("attn_kv_a_mqa"), self.kv_lora + self.rope_dim, d),
                        TensorPlan(p + "attn_kv_a_norm", F32, 1, self.kv_lora, fill=self.norms),
                        TensorPlan(p + "attn_kv_b", self.ty("attn_kv_b"), self.n_heads * (self.nope + self.v_head),
                                   self.kv_lora),
                        TensorPlan(p + "attn_output", self.ty("attn_output"), d, self.n_heads * self.v_head)]
            else:
                out += [TensorPlan(p + "attn_q", self.ty("attn_q"), qd, d),
                        TensorPlan(p + "attn_k", self.ty("attn_k"), kvd, d),
                        TensorPlan(p + "attn_v", self.ty("attn_v"), kvd, d),
                        TensorPlan(p + "attn_output", self.ty("attn_output"), d, qd)]
            out += [TensorPlan(p + "ffn_norm", F32, 1, d, fill=self.norms)]
            if self.qk_norm:
                out += [TensorPlan(p + "attn_q_norm", F32, 1, self.head_dim, fill="near_ones"),
                        TensorPlan(p + "attn_k_norm", F32, 1, self.head_dim, fill="near_ones")]
            if self.is_moe_layer(i):
                ne, f = self.n_expert, self.moe_ffn
                out += [TensorPlan(p + "ffn_gate_inp", F32, ne, d, sigma=0.02),
                        TensorPlan(p + "ffn_gate_exps", self.ty("ffn_gate"), f, d, planes=ne),
                        TensorPlan(p + "ffn_up_exps", self.ty("ffn_up"), f, d, planes=ne),
                        TensorPlan(p + "ffn_down_exps", self.ty("ffn_down"), d, f, planes=ne)]
                if self.router_bias:
                    out += [TensorPlan(p + "exp_probs_b.bias", F32, 1, ne, sigma=0.05)]
                if self.shexp_ffn:
                    sf = self.shexp_ffn
                    out += [TensorPlan(p + "ffn_gate_shexp", self.ty("ffn_gate"), sf, d),
                            TensorPlan(p + "ffn_up_shexp", self.ty("ffn_up"), sf, d),
                            TensorPlan(p + "ffn_down_shexp", self.ty("ffn_down_shexp"), d, sf)]
            else:
                out += [TensorPlan(p + "ffn_gate", self.ty("ffn_gate"), self.ffn, d),
                        TensorPlan(p + "ffn_up", self.ty("ffn_up"), self.ffn, d),
                        TensorPlan(p + "ffn_down", self.types.get("ffn_down_dense", self.ty("ffn_down")), d,
                                   self.ffn)]
        for t in out:
            t.seed = (self.seed * 0x9E3779B1 + zlib.crc32(t.name.encode())) & 0xFFFFFFFF
        return out

    def weight_bytes(self) -> int:
        return sum(t.nbytes for t in self.plan())


def fill_values(t: TensorPlan) -> np.ndarray:
    """The f32 values of a non-synthetic tensor (norm weights)."""
    n = t.planes * t.rows * t.cols
    if t.fill == "ones":
        return np.ones(n, np.float32)
    rng = np.random.default_rng(t.seed)
    return (1.0 + rng.uniform(-0.25, 0.25, n)).astype(np.float32)


def tiny_llama(ctx_len: int = 256, seed: int = 1) -> ModelSpec:
    """llama-arch, dim 288, 6 layers, 6 heads of 48, FFN 768,
    vocab 32000, every matrix Q4_0, f32 embeddings ~N(0, 0.02), norms 1.0."""
    q = Q4_0
    return ModelSpec("tiny-llama-q4_0", dim=288, n_layers=6, n_heads=6, n_kv_heads=6, head_dim=48, vocab=32000,
                     ctx_len=ctx_len, eps=1e-5, rope_base=10000.0, rope_neox=False, ffn=768,
                     types=dict(embd=F32, output=q, attn_q=q, attn_k=q, attn_v=q, attn_output=q, ffn_gate=q,
                                ffn_up=q, ffn_down=q), seed=seed)


def qwen3_moe(n_layers: int = 48, ctx_len: int = 2048, n_expert: int = 128, vocab: int = 151936,
              seed: int = 3) -> ModelSpec:
    """Qwen3-30B-A3B shape (48 layers, hidden 2048, 32 query /
    4 KV heads of 128, QK-RMSNorm, RoPE NEOX base 1e6, 128 experts top-8 of
    FFN 768, vocab 151936) in the Q4_K_M mix: attn_q/k/output, gate/up and the
    embeddings Q4_K; attn_v, ffn_down and output Q6_K; router and norms f32."""
    return ModelSpec("qwen3-30b-a3b-q4_k_m", dim=2048, n_layers=n_layers, n_heads=32, n_kv_heads=4, head_dim=128,
                     vocab=vocab, ctx_len=ctx_len, eps=1e-6, rope_base=1e6, rope_neox=True, qk_norm=True,
                     n_expert=n_expert, n_used=8, moe_ffn=768,
                     types=dict(embd=Q4_K, output=Q6_K, attn_q=Q4_K, attn_k=Q4_K, attn_v=Q6_K, attn_output=Q4_K,
                                ffn_gate=Q4_K, ffn_up=Q4_K, ffn_down=Q6_K), norms="near_ones", seed=seed)


def deepseek_v2_lite(n_layers: int = 27, ctx_len: int = 4096, n_expert: int = 64, vocab: int = 102400,
                     seed: int = 5) -> ModelSpec:
    """DeepSeek-V2-Lite (deepseek2 / MLA): 27 layers, hidden
    2048, 16 heads, kv_lora 512, rope 64, nope 128, v 128, no q_lora; layer 0
    dense (FFN 10944), then 64 routed experts top-6 of FFN 1408 plus 2 shared
    (one shared FFN of 2816), vocab 102400; softmax gating with renorm.
    Q4_K wherever the width is a multiple of 256; the down projections of
    width 1408 / 10944 / 2816 are Q8_0 (as real Q4_K_M files put them)."""
    return ModelSpec("deepseek-v2-lite-q4_k", dim=2048, n_layers=n_layers, n_heads=16, n_kv_heads=16, head_dim=192,
                     vocab=vocab, ctx_len=ctx_len, eps=1e-6, rope_base=10000.0, rope_neox=False, rope_dim=64,
                     mla=True, kv_lora=512, q_lora=0, nope=128, v_head=128, n_dense=1, ffn=10944,
                     n_expert=n_expert, n_used=6, moe_ffn=1408, shexp_ffn=2816, gating=1, weights_norm=True,
                     types=dict(embd=Q4_K, output=Q6_K, attn_q=Q4_K, attn_kv_a_mqa=Q4_K, attn_kv_b=Q4_K,
                                attn_output=Q4_K, ffn_gate=Q4_K, ffn_up=Q4_K, ffn_down=Q8_0,
                                ffn_down_dense=Q8_0, ffn_down_shexp=Q8_0), seed=seed)


def deepseek_v3(n_layers: int = 61, ctx_len: int = 4096, n_expert: int = 256, vocab: int = 129280, dim: int = 7168,
                n_heads: int = 128, n_dense: int = 3, seed: int = 7) -> ModelSpec:
    """DeepSeek-V3 shape: 61 layers (3 dense, FFN 18432),
    hidden 7168, MLA with 128 heads, q_lora 1536, kv_lora 512; 256 routed
    experts top-8 of FFN 2048, sigmoid gating with selection bias and renorm,
    grouped top-k (8 groups, 4 kept), 1 shared expert; vocab 129280; Q4_K."""
    return ModelSpec("deepseek-v3-q4_k", dim=dim, n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_heads,
                     head_dim=192, vocab=vocab, ctx_len=ctx_len, eps=1e-6, rope_base=10000.0, rope_neox=False,
                     rope_dim=64, mla=True, kv_lora=512, q_lora=1536, nope=128, v_head=128, n_dense=n_dense,
                     ffn=18432, n_expert=n_expert, n_used=8, moe_ffn=2048, shexp_ffn=2048, gating=2,
                     weights_norm=True, weights_scale=2.5, router_bias=True, n_group=8, topk_group=4,
                     types=dict(embd=Q4_K, output=Q4_K, attn_q_a=Q4_K, attn_q_b=Q4_K, attn_kv_a_mqa=Q4_K,
                                attn_kv_b=Q4_K, attn_output=Q4_K, ffn_gate=Q4_K, ffn_up=Q4_K, ffn_down=Q4_K,
                                ffn_down_dense=Q4_K, ffn_down_shexp=Q4_K), seed=seed)


class DeviceModel:
    """A ModelSpec's tensors on the GPU plus the backend's model handle."""

    def __init__(self, spec: ModelSpec, host: Optional[Dict[str, np.ndarray]] = None, exact_order: bool = False,
                 expert_shard: Optional[tuple] = None):
        """expert_shard = (expert0, n_local): this rank holds only those experts of
        every routed layer (expert parallelism after ep_init; the layer's partial
        outputs are summed over the ranks); everything else is replicated."""
        self.spec = spec
        self.t: Dict[str, DeviceTensor] = {}
        e0, nl = expert_shard if expert_shard else (0, spec.n_expert)
        for p in spec.plan():
            if host is not None and p.name in host:
                self.t[p.name] = DeviceTensor.upload(p.type, host[p.name])
            elif p.planes > 1 and expert_shard:
                per = p.nblk // p.planes
                self.t[p.name] = DeviceTensor.synth_range(p.type, e0 * per, nl * per, p.seed, p.sigma)
            elif p.fill == "synth":
                self.t[p.name] = DeviceTensor.synth(p.type, p.nblk, p.seed, p.sigma)
            else:
                self.t[p.name] = DeviceTensor.upload(F32, fill_values(p))
        self._layers = (_lib.ModelLayer * spec.n_layers)()
        h = lambda n: self.t[n].handle if n in self.t else 0  # noqa: E731
        for i in range(spec.n_layers):
            L, p = self._layers[i], f"blk.{i}."
            L.attn_norm, L.ffn_norm = h(p + "attn_norm"), h(p + "ffn_norm")
            L.wq, L.wk, L.wv, L.wo = h(p + "attn_q"), h(p + "attn_k"), h(p + "attn_v"), h(p + "attn_output")
            L.q_norm, L.k_norm = h(p + "attn_q_norm"), h(p + "attn_k_norm")
            L.q_a, L.q_a_norm, L.q_b = h(p + "attn_q_a"), h(p + "attn_q_a_norm"), h(p + "attn_q_b")
            L.kv_a, L.kv_a_norm, L.kv_b = h(p + "attn_kv_a_mqa"), h(p + "attn_kv_a_norm"), h(p + "attn_kv_b")
            if spec.is_moe_layer(i):
                m = L.moe
                m.dim, m.ffn, m.n_expert, m.n_used = spec.dim, spec.moe_ffn, spec.n_expert, spec.n_used
                m.gating, m.weights_norm, m.weights_scale = spec.gating, int(spec.weights_norm), spec.weights_scale
                m.router, m.router_bias = h(p + "ffn_gate_inp"), h(p + "exp_probs_b.bias")
                m.gate, m.up, m.down = h(p + "ffn_gate_exps"), h(p + "ffn_up_exps"), h(p + "ffn_down_exps")
                if spec.shexp_ffn:
                    m.shexp_gate, m.shexp_up = h(p + "ffn_gate_shexp"), h(p + "ffn_up_shexp")
                    m.shexp_down, m.shexp_ffn = h(p + "ffn_down_shexp"), spec.shexp_ffn
                m.expert0, m.n_local = e0, nl
                m.n_group, m.topk_group = spec.n_group, spec.topk_group
                if i + 1 < spec.n_layers and spec.is_moe_layer(i + 1):
                    m.next_router = h(f"blk.{i + 1}.ffn_gate_inp")
            else:
                L.ffn_gate, L.ffn_up, L.ffn_down = h(p + "ffn_gate"), h(p + "ffn_up"), h(p + "ffn_down")
                L.ffn = spec.ffn
        d = _lib.ModelDesc()
        d.dim, d.n_layers, d.n_heads, d.n_kv_heads = spec.dim, spec.n_layers, spec.n_heads, spec.n_kv_heads
        d.head_dim, d.rope_dim, d.vocab, d.ctx_len = spec.head_dim, spec.rope_dim, spec.vocab, spec.ctx_len
        d.eps, d.rope_base, d.attn_logit_mul, d.rope_neox = spec.eps, spec.rope_base, 1.0, int(spec.rope_neox)
        d.exact_order = int(exact_order)
        if spec.mla:
            d.mla, d.kv_lora, d.q_lora, d.nope, d.v_head = 1, spec.kv_lora, spec.q_lora, spec.nope, spec.v_head
            d.mla_scale = spec.attn_scale
        d.token_embd, d.output_norm, d.output = h("token_embd"), h("output_norm"), h("output")
        d.layers = self._layers
        self.desc = d
        hh = C.c_uint64(0)
        _lib.must(_lib.lib().loom_cuda_model_create(C.byref(d), C.byref(hh)), "model_create")
        self.handle = hh.value

    def decode(self, token: int, pos: int, logits: bool = False):
        """One token through the host entry point: returns (next token, logits or None)."""
        nxt = C.c_uint32(0)
        lg = np.empty(self.spec.vocab, np.float32) if logits else None
        _lib.must(_lib.lib().loom_cuda_model_decode(self.handle, token, pos,
                                                    lg.ctypes.data_as(C.c_void_p) if logits else None,
                                                    C.byref(nxt)), "model_decode")
        return nxt.value, lg

    def prefill(self, tokens, pos_base: int = 0, logits: bool = False):
        """Batched prefill of `tokens` at positions pos_base.. (llama.zig stepBatch): returns
        (greedy next token, the last token's logits or None)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        nxt = C.c_uint32(0)
        lg = np.empty(self.spec.vocab, np.float32) if logits else None
        _lib.must(_lib.lib().loom_cuda_model_prefill(self.handle, t.ctypes.data_as(C.c_void_p), t.size, pos_base,
                                                     lg.ctypes.data_as(C.c_void_p) if logits else None,
                                                     C.byref(nxt)), "model_prefill")
        return nxt.value, lg

    def decode_batch(self, tokens, positions, logits: bool = False):
        """One token for each of B sequences (row b: sequence b at positions[b], its own cache;
        llama.zig decodeBatch): returns (next tokens [B], logits [B][vocab] or None)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.uint32))
        assert t.size == p.size
        nxt = np.zeros(t.size, np.uint32)
        lg = np.empty((t.size, self.spec.vocab), np.float32) if logits else None
        _lib.must(_lib.lib().loom_cuda_model_decode_batch(self.handle, t.ctypes.data_as(C.c_void_p),
                                                          p.ctypes.data_as(C.c_void_p), t.size,
                                                          lg.ctypes.data_as(C.c_void_p) if logits else None,
                                                          nxt.ctypes.data_as(C.c_void_p)), "model_decode_batch")
        return nxt, lg

    def step(self, d_token, d_pos, d_logits=None, d_next=None, stream=None) -> None:
        """The step on device buffers (torch cuda tensors: int32 [1])."""
        from .device import _st
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        _lib.must(_lib.lib().loom_cuda_model_step(self.handle, p(d_token), p(d_pos), p(d_logits), p(d_next),
                                                  _st(stream)), "model_step")

    def read_kv(self, layer: int, pos: int):
        sp = self.spec
        kw = sp.kv_lora if sp.mla else sp.n_kv_heads * sp.head_dim
        vw = sp.rope_dim if sp.mla else sp.n_kv_heads * sp.head_dim
        k, v = np.empty(kw, np.float32), np.empty(vw, np.float32)
        _lib.must(_lib.lib().loom_cuda_model_read_kv(self.handle, layer, pos, k.ctypes.data_as(C.c_void_p),
                                                     v.ctypes.data_as(C.c_void_p)), "model_read_kv")
        return k, v

    def error(self) -> int:
        """The fused attention kernel's error word (0: none); re-arms after an error."""
        return int(_lib.lib().loom_cuda_model_error(self.handle))

    def free(self) -> None:
        if self.handle:
            _lib.lib().loom_cuda_model_free(self.handle)
            self.handle = 0
        for t in self.t.values():
            t.free()
        self.t.clear()


def greedy(step, prompt: List[int], n_new: int) -> List[int]:
    """The generation loop: feed the prompt at positions 0..len-1, then take the
    argmax token and feed it back (sampler.zig:7-15 greedy), n_new tokens.
    `step(token, pos)` returns the next token."""
    out: List[int] = []
    nxt = None
    for pos, tok in enumerate(prompt):
        nxt = step(tok, pos)
    pos = len(prompt)
    for _ in range(n_new):
        out.append(nxt)
        if len(out) == n_new:
            break
        nxt = step(nxt, pos)
        pos += 1
    return out
