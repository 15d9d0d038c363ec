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


def numpy_ds_step(spec: ModelSpec, T: dict, orc, cc, rc, token: int, pos: int) -> np.ndarray:
    """deepseek.zig:1275-1537 / attnLayer :851-1049 in numpy (float64 sums)
    around the oracle's matvecs and dequant: q (direct or q_a -> norm -> q_b),
    kv_a -> normed compressed row + RoPE'd rope row into the caches, W_k
    absorbed into q, softmax over positions in compressed space, W_v once per
    head, output projection; dense FFN or routed MoE + shared expert."""
    d, nh, nope, rope, kvr, vd = spec.dim, spec.n_heads, spec.nope, spec.rope_dim, spec.kv_lora, spec.v_head
    kd = nope + rope
    mv = lambda n, x, rows, cols: orc.matvec(T[n][0], T[n][1], np.asarray(x, np.float32), rows, cols)  # noqa: E731
    x = orc.dequant_row(T["token_embd"][0], T["token_embd"][1], token, d).astype(np.float32)
    for li in range(spec.n_layers):
        p = f"blk.{li}."
        h = _rmsnorm(x, T[p + "attn_norm"][1], spec.eps).astype(np.float32)
        if spec.q_lora:
            qa = _rmsnorm(mv(p + "attn_q_a", h, spec.q_lora, d), T[p + "attn_q_a_norm"][1], spec.eps)
            q = mv(p + "attn_q_b", qa, nh * kd, spec.q_lora)
        else:
            q = mv(p + "attn_q", h, nh * kd, d)
        kv = mv(p + "attn_kv_a_mqa", h, kvr + rope, d)
        cc[li, pos] = _rmsnorm(kv[:kvr], T[p + "attn_kv_a_norm"][1], spec.eps)
        kr = kv[kvr:].copy()
        _rope(kr, rope, pos, spec.rope_base, False)
        rc[li, pos] = kr
        kvb = orc.dequant(T[p + "attn_kv_b"][0], T[p + "attn_kv_b"][1], nh * (nope + vd), kvr).reshape(nh, nope + vd, kvr)
        head_out = np.zeros(nh * vd, np.float32)
        for hh in range(nh):
            qh = q[hh * kd:(hh + 1) * kd].copy()
            qr = qh[nope:].copy()
            _rope(qr, rope, pos, spec.rope_base, False)
            qabs = qh[:nope].astype(np.float64) @ kvb[hh, :nope].astype(np.float64)
            s = (cc[li, :pos + 1].astype(np.float64) @ qabs + rc[li, :pos + 1].astype(np.float64) @ qr) * spec.attn_scale
            e = np.exp(s - s.max())
            cacc = ((e / e.sum()) @ cc[li, :pos + 1].astype(np.float64)).astype(np.float32)
            rows = T[p + "attn_kv_b"][1].reshape(nh * (nope + vd), -1)[hh * (nope + vd) + nope:(hh + 1) * (nope + vd)]
            head_out[hh * vd:(hh + 1) * vd] = orc.matvec(T[p + "attn_kv_b"][0], np.ascontiguousarray(rows), cacc, vd, kvr)
        x = (x + mv(p + "attn_output", head_out, d, nh * vd)).astype(np.float32)
        h = _rmsnorm(x, T[p + "ffn_norm"][1], spec.eps).astype(np.float32)
        if spec.is_moe_layer(li):
            lg = orc.matvec(0, T[p + "ffn_gate_inp"][1], h, spec.n_expert, d)
            bias = T[p + "exp_probs_b.bias"][1] if spec.router_bias else None
            ids, gates = orc.route(lg, spec.n_used, spec.gating, spec.weights_norm, spec.weights_scale, bias=bias,
                                   n_group=spec.n_group, topk_group=spec.topk_group)
            f = spec.moe_ffn
            acc = np.zeros(d, np.float64)
            for e_, gt in zip(ids, gates):
                def plane(n, rows, cols):
                    ty, b = T[p + n]
                    nb = b.size // spec.n_expert
                    return ty, b[int(e_) * nb:(int(e_) + 1) * nb]
                gty, gb = plane("ffn_gate_exps", f, d)
                uty, ub = plane("ffn_up_exps", f, d)
                dty, db = plane("ffn_down_exps", d, f)
                g_ = orc.matvec(gty, gb, h, f, d)
                u_ = orc.matvec(uty, ub, h, f, d)
                acc += float(gt) * orc.matvec(dty, db, ((g_ / (1 + np.exp(-g_))) * u_).astype(np.float32), d, f)
            if spec.shexp_ffn:
                sf = spec.shexp_ffn
                g_, u_ = mv(p + "ffn_gate_shexp", h, sf, d), mv(p + "ffn_up_shexp", h, sf, d)
                acc += mv(p + "ffn_down_shexp", ((g_ / (1 + np.exp(-g_))) * u_).astype(np.float32), d, sf)
            y = acc.astype(np.float32)
        else:
            g_, u_ = mv(p + "ffn_gate", h, spec.ffn, d), mv(p + "ffn_up", h, spec.ffn, d)
            y = mv(p + "ffn_down", ((g_ / (1 + np.exp(-g_))) * u_).astype(np.float32), d, spec.ffn)
        x = (x + y).astype(np.float32)
    h = _rmsnorm(x, T["output_norm"][1], spec.eps).astype(np.float32)
    return mv("output", h, spec.vocab, d)
