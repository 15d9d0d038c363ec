"""Writes tests/golden/known_answers.json: the reference's own known-answer
tests for the MoE hot path, restated as data (inputs and expected outputs).

Sources (ch4r10t33r/loom):
  src/gguf/ggml.zig:1938-1966  "q4_k dequant with handcrafted block"
  src/gguf/ggml.zig:1968-1977  "q6_k dequant with handcrafted block"
  src/gguf/moe.zig:210-222     "sigmoid gating with selection bias ..."
  src/gguf/moe.zig:224-239     "softmax-topk selects on raw logits ..."
  src/gguf/moe.zig:241-254     "renormalization makes the top-k gates sum to one"
  src/gguf/moe.zig:256-262     "weights_scale multiplies after normalization"
  src/core/tensor.zig:86-91    "softmax sums to one"
  src/engine/sampler.zig:33-36 "argmax finds the max index"

Expected values are the ones the reference tests assert, with the reference
tests' tolerances. Run: python tests/golden/make_golden.py
"""
import json
import math
import os

import numpy as np


def f16_bytes(v):
    return list(np.float16(v).tobytes())


def q4k_block():
    blk = [0] * 144
    blk[0:2] = f16_bytes(1.0)   # d
    blk[2:4] = f16_bytes(0.0)   # dmin
    blk[4:8] = [1, 1, 1, 1]     # sc = 1 for sub-blocks 0..3, min 0
    for i in range(16, 144):
        blk[i] = 0x31           # low nibble 1, high nibble 3
    return blk


def q6k_block():
    blk = [0] * 210
    for i in range(192, 208):
        blk[i] = 1              # scales all 1
    blk[208:210] = f16_bytes(0.5)
    return blk


def sig(x):
    return 1.0 / (1.0 + math.exp(-x))


def main():
    d = math.exp(3.0) + math.exp(2.0)
    g = {
        "source": "ch4r10t33r/loom known-answer tests (see make_golden.py docstring)",
        "dequant": [
            {"name": "q4k_handcrafted", "ref": "src/gguf/ggml.zig:1938", "type": 12, "cols": 256,
             "block": q4k_block(),
             "expect_at": {"0": 1.0, "32": 3.0, "64": 1.0, "96": 3.0, "128": 0.0, "255": 0.0},
             "tol": 1e-4, "matvec_ones": 256.0, "matvec_tol": 1e-2},
            {"name": "q6k_handcrafted", "ref": "src/gguf/ggml.zig:1968", "type": 14, "cols": 256,
             "block": q6k_block(), "expect_all": -16.0, "tol": 1e-4},
        ],
        "route": [
            {"name": "sigmoid_bias", "ref": "src/gguf/moe.zig:210", "logits": [0.0, 1.0, 2.0, 3.0],
             "bias": [10.0, 0.0, 0.0, 0.0], "n_used": 2, "gating": 2, "norm": False, "scale": 1.0,
             "expect_ids": [0, 3], "expect_gates": [sig(0.0), sig(3.0)], "tol": 1e-6},
            {"name": "softmax_topk", "ref": "src/gguf/moe.zig:224", "logits": [0.5, 3.0, 1.0, 2.0],
             "bias": None, "n_used": 2, "gating": 3, "norm": False, "scale": 1.0,
             "expect_ids": [1, 3], "expect_gates": [math.exp(3.0) / d, math.exp(2.0) / d], "tol": 1e-6},
            {"name": "renorm_sum_one", "ref": "src/gguf/moe.zig:241", "logits": [1.0, 2.0, 3.0, 4.0],
             "bias": None, "n_used": 2, "gating": 1, "norm": True, "scale": 1.0,
             "expect_gate_sum": 1.0, "tol": 1e-6},
            {"name": "no_renorm_below", "ref": "src/gguf/moe.zig:251", "logits": [1.0, 2.0, 3.0, 4.0],
             "bias": None, "n_used": 2, "gating": 1, "norm": False, "scale": 1.0,
             "expect_gate_sum_below": 0.95},
            {"name": "scale_after_norm", "ref": "src/gguf/moe.zig:256", "logits": [1.0, 2.0, 3.0, 4.0],
             "bias": None, "n_used": 2, "gating": 1, "norm": True, "scale": 2.5,
             "expect_gate_sum": 2.5, "tol": 1e-5},
        ],
        "softmax": [{"name": "sums_to_one", "ref": "src/core/tensor.zig:86", "x": [1, 2, 3, 4],
                     "expect_sum": 1.0, "tol": 1e-6}],
        "argmax": [{"name": "finds_max_index", "ref": "src/engine/sampler.zig:33", "logits": [-1, 3, 2, 3.5, 0],
                    "expect": 3}],
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")
    with open(path, "w") as f:
        json.dump(g, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
