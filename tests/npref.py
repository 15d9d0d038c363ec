"""Independent numpy restatement of the reference's block decoders.

Test-only. Written separately from the C++ oracle so the two restatements of
src/gguf/ggml.zig (dequantBlockQ4K :1342, dequantBlockQ6K :1420, dequantRow's
q4_0/q8_0 arms :1830-1848, scaleMinK4 :1332) cross-check each other bit for
bit. numpy float32 multiply and subtract round once each, like Zig's @Vector
ops without contraction.
"""
import numpy as np


def _f16(lo, hi):
    return (lo.astype(np.uint16) | (hi.astype(np.uint16) << 8)).view(np.float16).astype(np.float32)


def _scale_min_k4(s):
    """s: [nb,12] uint8 -> sc, mn: [nb,8] int."""
    s = s.astype(np.int32)
    sc = np.empty((s.shape[0], 8), np.int32)
    mn = np.empty((s.shape[0], 8), np.int32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63
            mn[:, j] = s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc, mn


def dequant_q4k(data, rows, cols):
    b = np.frombuffer(data, np.uint8).reshape(-1, 144)
    d = _f16(b[:, 0], b[:, 1])
    dmin = _f16(b[:, 2], b[:, 3])
    sc, mn = _scale_min_k4(b[:, 4:16])
    qs = b[:, 16:]
    out = np.empty((b.shape[0], 256), np.float32)
    for j in range(4):
        chunk = qs[:, 32 * j:32 * j + 32]
        d1 = d * sc[:, 2 * j].astype(np.float32)
        m1 = dmin * mn[:, 2 * j].astype(np.float32)
        d2 = d * sc[:, 2 * j + 1].astype(np.float32)
        m2 = dmin * mn[:, 2 * j + 1].astype(np.float32)
        out[:, 64 * j:64 * j + 32] = d1[:, None] * (chunk & 0xF).astype(np.float32) - m1[:, None]
        out[:, 64 * j + 32:64 * j + 64] = d2[:, None] * (chunk >> 4).astype(np.float32) - m2[:, None]
    return out.reshape(rows, cols)


def dequant_q6k(data, rows, cols):
    b = np.frombuffer(data, np.uint8).reshape(-1, 210)
    d = _f16(b[:, 208], b[:, 209])
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    out = np.empty((b.shape[0], 256), np.float32)
    for n in range(2):
        ql = b[:, 64 * n:64 * n + 64].astype(np.int32)
        qh = b[:, 128 + 32 * n:128 + 32 * n + 32].astype(np.int32)
        a, bb = ql[:, :32], ql[:, 32:]
        q = [(a & 0xF) | ((qh & 3) << 4), (bb & 0xF) | (((qh >> 2) & 3) << 4),
             (a >> 4) | (((qh >> 4) & 3) << 4), (bb >> 4) | (((qh >> 6) & 3) << 4)]
        for g in range(4):
            for half in range(2):
                s = d * sc[:, 8 * n + half + 2 * g]
                qq = q[g][:, 16 * half:16 * half + 16].astype(np.float32) - np.float32(32)
                out[:, 128 * n + 32 * g + 16 * half:128 * n + 32 * g + 16 * half + 16] = s[:, None] * qq
    return out.reshape(rows, cols)


def dequant_q40(data, rows, cols):
    b = np.frombuffer(data, np.uint8).reshape(-1, 18)
    d = _f16(b[:, 0], b[:, 1])
    qs = b[:, 2:].astype(np.int32)
    lo = ((qs & 0xF) - 8).astype(np.float32) * d[:, None]
    hi = ((qs >> 4) - 8).astype(np.float32) * d[:, None]
    return np.concatenate([lo, hi], axis=1).reshape(rows, cols)


def dequant_q80(data, rows, cols):
    b = np.frombuffer(data, np.uint8).reshape(-1, 34)
    d = _f16(b[:, 0], b[:, 1])
    return (b[:, 2:].view(np.int8).astype(np.float32) * d[:, None]).reshape(rows, cols)


DEQUANT = {12: dequant_q4k, 14: dequant_q6k, 2: dequant_q40, 8: dequant_q80}


def random_blocks(rng, t, rows, cols):
    """Random bytes with one exponent bit of every f16 cleared (ggml.zig:2058-2062),
    so no block scale is NaN/Inf."""
    from oracle.oracle import BLOCK_BYTES, BLOCK_ELEMS
    n = rows * (cols // BLOCK_ELEMS[t]) * BLOCK_BYTES[t]
    data = rng.integers(0, 256, n, dtype=np.uint8)
    data[1::2] &= 0xFB
    return data


def quantize_q40(x):
    """ggml.zig test encoder quantizeQ40 (:1860-1884), one row."""
    out = bytearray()
    for b in range(0, x.size, 32):
        blk = x[b:b + 32].astype(np.float32)
        amax = np.float32(0)
        vmax = np.float32(0)
        for v in blk:
            if abs(v) > amax:
                amax, vmax = np.float32(abs(v)), v
        scale = np.float32(vmax / np.float32(-8.0))
        half = np.float16(scale)
        inv = np.float32(1.0) / scale if scale != 0 else np.float32(0)
        out += half.tobytes()
        for j in range(16):
            lo = int(min(max(int(np.float32(blk[j] * inv + np.float32(8.5))), 0), 15))
            hi = int(min(max(int(np.float32(blk[j + 16] * inv + np.float32(8.5))), 0), 15))
            out.append(lo | (hi << 4))
    return np.frombuffer(bytes(out), np.uint8)


def quantize_q80(x):
    """ggml.zig test encoder quantizeQ80 (:1886-1904), one row."""
    out = bytearray()
    for b in range(0, x.size, 32):
        blk = x[b:b + 32].astype(np.float32)
        amax = np.float32(np.max(np.abs(blk)))
        scale = np.float32(amax / np.float32(127.0))
        out += np.float16(scale).tobytes()
        inv = np.float32(1.0) / scale if scale != 0 else np.float32(0)
        for v in blk:
            p = float(np.float32(v * inv))
            r = np.floor(abs(p) + 0.5) * (1 if p >= 0 else -1)  # @round: half away from zero
            q = int(np.clip(int(r), -127, 127))
            out += np.int8(q).tobytes()
    return np.frombuffer(bytes(out), np.uint8)
