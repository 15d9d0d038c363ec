"""Test helpers for whole-model decode: the host bytes of a ModelSpec (the same
bytes the device generator makes) and an independent numpy restatement of the
reference's token step, used to pin the oracle's `or_llama_step`."""
from __future__ import annotations

import numpy as np

from loom_b200.model import ModelSpec, fill_values


def host_tensors(spec: ModelSpec, orc) -> dict:
    """name -> (type, numpy array) for every tensor of the spec."""
    out = {}
    for p in spec.plan():
        if p.fill == "synth":
            out[p.name] = (p.type, orc.synth(p.type, p.nblk, p.seed, sigma=p.sigma))
        else:
            out[p.name] = (p.type, fill_values(p))
    return out


def _rope(vec, rope_dim, pos, base, neox):
    """llama.zig:821-858 in float32, pair by pair."""
    f = np.float32
    pairs = [(i, i + rope_dim // 2, 2 * i) for i in range(rope_dim // 2)] if neox else \
        [(i, i + 1, i) for i in range(0, rope_dim - 1, 2)]
    for a_i, b_i, th in pairs:
        exponent = f(th) / f(rope_dim)
        freq = np.power(f(base), -exponent, dtype=np.float32)
        ang = f(pos) * freq
        c, s = np.cos(ang, dtype=np.float32), np.sin(ang, dtype=np.float32)
        a, b = vec[a_i], vec[b_i]
        vec[a_i] = f(a * c) - f(b * s)
        vec[b_i] = f(a * s) + f(b * c)


def _rmsnorm(x, w, eps):
    ss = np.float32(np.sum(x.astype(np.float64) ** 2))
    return (x * np.float32(1.0 / np.sqrt(ss / np.float32(len(x)) + np.float32(eps)))) * w


def numpy_step(spec: ModelSpec, T: dict, orc, kc, vc, token: int, pos: int) -> np.ndarray:
    """llama.zig:1111-1228 for dense or routed layers: matvecs and the MoE layer
    through the oracle's kernels, everything else (norms, RoPE, attention) in
    numpy with float64 sums, so the result agrees with or_llama_step to rounding."""
    d, hd, nh, nkv = spec.dim, spec.head_dim, spec.n_heads, spec.n_kv_heads
    kvd, qd = nkv * hd, nh * hd
    mv = lambda n, x, rows, cols: orc.matvec(T[n][0], T[n][1], x.astype(np.float32), rows, cols)  # noqa: E731
    x = orc.dequant_row(T["token_embd"][0], T["token_embd"][1], token, d).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(np.float32(hd)))
    for li in range(spec.n_layers):
        p = f"blk.{li}."
        h = _rmsnorm(x, T[p + "attn_norm"][1], spec.eps).astype(np.float32)
        q, k, v = mv(p + "attn_q", h, qd, d), mv(p + "attn_k", h, kvd, d), mv(p + "attn_v", h, kvd, d)
        if spec.qk_norm:
            for vec, n, w in ((q, nh, T[p + "attn_q_norm"][1]), (k, nkv, T[p + "attn_k_norm"][1])):
                for hh in range(n):
                    seg = vec[hh * hd:(hh + 1) * hd]
                    vec[hh * hd:(hh + 1) * hd] = _rmsnorm(seg, w, spec.eps)
        for hh in range(nh):
            seg = q[hh * hd:(hh + 1) * hd].copy()
            _rope(seg, spec.rope_dim, pos, spec.rope_base, spec.rope_neox)
            q[hh * hd:(hh + 1) * hd] = seg
        for hh in range(nkv):
            seg = k[hh * hd:(hh + 1) * hd].copy()
            _rope(seg, spec.rope_dim, pos, spec.rope_base, spec.rope_neox)
            k[hh * hd:(hh + 1) * hd] = seg
        kc[li, pos], vc[li, pos] = k, v
        att = np.zeros(qd, np.float32)
        for hh in range(nh):
            g = hh // (nh // nkv)
            K = kc[li, :pos + 1, g * hd:(g + 1) * hd].astype(np.float64)
            V = vc[li, :pos + 1, g * hd:(g + 1) * hd].astype(np.float64)
            s = K @ q[hh * hd:(hh + 1) * hd].astype(np.float64) * float(scale)
            e = np.exp(s - s.max())
            att[hh * hd:(hh + 1) * hd] = (e / e.sum()) @ V
        x = (x + mv(p + "attn_output", att, d, qd)).astype(np.float32)
        h = _rmsnorm(x, T[p + "ffn_norm"][1], spec.eps).astype(np.float32)
        if spec.n_expert:
            y, _ = orc.moe_layer(h[None], T[p + "ffn_gate_inp"][1], T[p + "ffn_gate_exps"], T[p + "ffn_up_exps"],
                                 T[p + "ffn_down_exps"], spec.moe_ffn, spec.n_expert, spec.n_used)
            y = y[0]
        else:
            g_ = mv(p + "ffn_gate", h, spec.ffn, d)
            u_ = mv(p + "ffn_up", h, spec.ffn, d)
            a = (g_ / (np.float32(1) + np.exp(-g_))) * u_
            y = mv(p + "ffn_down", a.astype(np.float32), d, spec.ffn)
        x = (x + y).astype(np.float32)
    h = _rmsnorm(x, T["output_norm"][1], spec.eps).astype(np.float32)
    return mv("output", h, spec.vocab, d)
