"""Loads the in-tree CUDA backend library (libloom_cuda.so) and declares the
C ABI of include/loom_cuda.h for ctypes.

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libloom_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "loom_cuda.h")

OK, DECLINED, ERROR = 0, 1, 2


class LoomCudaError(RuntimeError):
    pass


class Weight(C.Structure):  # loom_weight (WeightRef, src/compute/cpu.zig:21)
    _fields_ = [("ggml_type", C.c_int), ("data", C.c_void_p), ("bytes", C.c_size_t)]


class ExpertRef(C.Structure):  # loom_expert (ExpertRef, src/compute/cpu.zig:23)
    _fields_ = [("gate", Weight), ("up", Weight), ("down", Weight), ("weight", C.c_float), ("ffn", C.c_size_t)]


class RoutedCfg(C.Structure):  # loom_routed_cfg (RoutedCfg, src/compute/cpu.zig:61)
    _fields_ = [("n_expert", C.c_size_t), ("n_used", C.c_size_t), ("gating_sigmoid", C.c_int),
                ("weights_norm", C.c_int), ("weights_scale", C.c_float)]


class MoeDesc(C.Structure):  # loom_moe_desc
    _fields_ = [("dim", C.c_size_t), ("ffn", C.c_size_t), ("n_expert", C.c_size_t), ("n_used", C.c_size_t),
                ("gating", C.c_int), ("weights_norm", C.c_int), ("weights_scale", C.c_float),
                ("router", C.c_uint64), ("router_bias", C.c_uint64),
                ("gate", C.c_uint64), ("up", C.c_uint64), ("down", C.c_uint64),
                ("shexp_gate", C.c_uint64), ("shexp_up", C.c_uint64), ("shexp_down", C.c_uint64),
                ("shexp_ffn", C.c_size_t), ("expert0", C.c_size_t), ("n_local", C.c_size_t),
                ("next_router", C.c_uint64), ("n_group", C.c_size_t), ("topk_group", C.c_size_t)]


class ModelLayer(C.Structure):  # loom_model_layer
    _fields_ = [("attn_norm", C.c_uint64), ("wq", C.c_uint64), ("wk", C.c_uint64), ("wv", C.c_uint64),
                ("wo", C.c_uint64), ("q_norm", C.c_uint64), ("k_norm", C.c_uint64), ("ffn_norm", C.c_uint64),
                ("ffn_gate", C.c_uint64), ("ffn_up", C.c_uint64), ("ffn_down", C.c_uint64), ("ffn", C.c_size_t),
                ("moe", MoeDesc), ("q_a", C.c_uint64), ("q_a_norm", C.c_uint64), ("q_b", C.c_uint64),
                ("kv_a", C.c_uint64), ("kv_a_norm", C.c_uint64), ("kv_b", C.c_uint64)]


class ModelDesc(C.Structure):  # loom_model_desc
    _fields_ = [("dim", C.c_size_t), ("n_layers", C.c_size_t), ("n_heads", C.c_size_t), ("n_kv_heads", C.c_size_t),
                ("head_dim", C.c_size_t), ("rope_dim", C.c_size_t), ("vocab", C.c_size_t), ("ctx_len", C.c_size_t),
                ("eps", C.c_float), ("rope_base", C.c_float), ("attn_logit_mul", C.c_float), ("rope_neox", C.c_int),
                ("exact_order", C.c_int), ("token_embd", C.c_uint64), ("output_norm", C.c_uint64), ("output", C.c_uint64),
                ("layers", C.POINTER(ModelLayer)), ("mla", C.c_int), ("kv_lora", C.c_size_t), ("q_lora", C.c_size_t),
                ("nope", C.c_size_t), ("v_head", C.c_size_t), ("mla_scale", C.c_float)]


class GgufTensor(C.Structure):  # loom_gguf_tensor (TensorInfo, src/gguf/gguf.zig:36)
    _fields_ = [("name", C.c_void_p), ("name_len", C.c_size_t), ("n_dims", C.c_uint32),
                ("dims", C.c_uint64 * 8), ("ggml_type", C.c_uint32), ("offset", C.c_uint64)]


class GgufValue(C.Structure):  # loom_gguf_value (MetaKV, src/gguf/gguf.zig:49-72)
    _fields_ = [("key", C.c_void_p), ("key_len", C.c_size_t), ("kind", C.c_int), ("i", C.c_int64),
                ("u", C.c_uint64), ("f", C.c_double), ("str", C.c_void_p), ("str_len", C.c_size_t),
                ("elem_type", C.c_uint32), ("count", C.c_uint64), ("array", C.c_void_p),
                ("span_start", C.c_uint64), ("span_end", C.c_uint64)]


class GgufView(C.Structure):  # loom_gguf_view (Model.resolve's Tensor, src/gguf/llama.zig:259)
    _fields_ = [("ggml_type", C.c_int), ("data", C.c_void_p), ("bytes", C.c_size_t),
                ("ne0", C.c_uint64), ("ne1", C.c_uint64), ("ne2", C.c_uint64)]


class Shard(C.Structure):  # loom_shard
    _fields_ = [("ext", Weight * 4), ("n_ext", C.c_int), ("digest", C.c_uint8 * 32)]


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(loom_(?:cuda|gguf)_\w+)\s*\(", src)))


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise LoomCudaError(f"CUDA backend library not built: {LIB_PATH} (run python -m loom_b200.build)")
    L = C.CDLL(LIB_PATH)
    vp, sz, i, f, u64 = C.c_void_p, C.c_size_t, C.c_int, C.c_float, C.c_uint64
    sig = {
        "loom_cuda_init": (i, [i]),
        "loom_cuda_shutdown": (None, []),
        "loom_cuda_parallel_begin": (None, [sz]),
        "loom_cuda_parallel_end": (None, []),
        "loom_cuda_max_batch": (sz, []),
        "loom_cuda_register_arena": (i, [vp, sz]),
        "loom_cuda_materialize_arenas": (sz, []),
        "loom_cuda_arena_error": (C.c_char_p, []),
        "loom_cuda_take_cmdbuf_count": (sz, []),
        "loom_cuda_kernel_launches": (u64, []),
        "loom_cuda_last_error": (sz, [C.c_char_p, sz]),
        "loom_cuda_clear_weight_cache": (None, []),
        "loom_cuda_matvec": (i, [i, vp, vp, sz, vp, sz, sz]),
        "loom_cuda_matmul": (i, [i, vp, vp, sz, vp, sz, sz, sz]),
        "loom_cuda_dequant_row": (i, [i, vp, vp, sz, sz, sz]),
        "loom_cuda_moe_route": (i, [vp, vp, sz, vp, vp, sz, i, i, f]),
        "loom_cuda_moe_ffn_block": (i, [vp, sz, vp, sz, vp]),
        "loom_cuda_moe_ffn_routed": (i, [vp, sz, vp, vp, Weight, Weight, Weight, vp, sz, sz, RoutedCfg, vp]),
        "loom_cuda_tensor_upload": (i, [i, vp, sz, C.POINTER(u64)]),
        "loom_cuda_tensor_synth": (i, [i, u64, u64, f, C.POINTER(u64)]),
        "loom_cuda_tensor_synth_range": (i, [i, u64, u64, u64, f, C.POINTER(u64)]),
        "loom_cuda_tensor_download": (i, [u64, vp, sz]),
        "loom_cuda_tensor_free": (i, [u64]),
        "loom_cuda_tensor_device_bytes": (sz, [u64]),
        "loom_cuda_moe_forward": (i, [C.POINTER(MoeDesc), vp, sz, vp, vp, vp, vp, vp]),
        "loom_cuda_moe_forward_noalloc": (i, [C.POINTER(MoeDesc), vp, sz, vp, vp, vp]),
        "loom_cuda_reserve": (i, [sz, sz, sz, sz, sz]),
        "loom_cuda_tensor_matmul": (i, [u64, sz, sz, vp, sz, vp, vp]),
        "loom_cuda_sync": (i, []),
        "loom_cuda_force_generic": (i, [i]),
        "loom_cuda_tc_exact": (i, [i]),
        "loom_cuda_last_path": (i, []),
        "loom_cuda_device_error": (i, []),
        "loom_cuda_stack_prepare": (i, [vp, sz, C.POINTER(u64)]),
        "loom_cuda_stack_forward": (i, [u64, vp, vp, vp, vp]),
        "loom_cuda_stack_error": (i, [u64]),
        "loom_cuda_stack_forward_residual": (i, [u64, vp, vp, vp, vp, vp]),
        "loom_cuda_stack_free": (i, [u64]),
        "loom_cuda_stack_trace": (i, [u64, i, vp, sz]),
        "loom_cuda_umma_selftest": (i, [vp, vp, vp, i, i, i]),
        "loom_cuda_tc_profile": (i, [i, vp, sz]),
        "loom_cuda_ep_unique_id": (i, [vp, sz]),
        "loom_cuda_ep_init": (i, [i, i, vp, sz]),
        "loom_cuda_ep_shutdown": (None, []),
        "loom_cuda_ep_rank": (i, []),
        "loom_cuda_ep_size": (i, []),
        "loom_cuda_ep_peer_combine": (i, []),
        "loom_cuda_ep_error": (i, []),
        "loom_cuda_ep_a2a_forward": (i, [C.POINTER(MoeDesc), vp, sz, vp, vp, vp, vp, vp]),
        "loom_cuda_ep_a2a_forward_cap": (i, [C.POINTER(MoeDesc), vp, sz, sz, vp, vp, vp, vp, vp]),
        "loom_cuda_argmax": (i, [vp, sz, vp, vp]),
        "loom_cuda_lm_head_argmax": (i, [C.c_uint64, sz, sz, vp, vp, vp, vp]),
        "loom_cuda_trace_enable": (i, [sz]),
        "loom_cuda_trace_reset": (i, []),
        "loom_cuda_trace_read": (sz, [vp, sz]),
        "loom_cuda_stream": (vp, []),
        "loom_cuda_model_create": (i, [C.POINTER(ModelDesc), C.POINTER(u64)]),
        "loom_cuda_model_step": (i, [u64, vp, vp, vp, vp, vp]),
        "loom_cuda_model_decode": (i, [u64, C.c_uint32, sz, vp, C.POINTER(C.c_uint32)]),
        "loom_cuda_model_read_kv": (i, [u64, sz, sz, vp, vp]),
        "loom_cuda_model_prefill": (i, [u64, vp, sz, sz, vp, C.POINTER(C.c_uint32)]),
        "loom_cuda_model_decode_batch": (i, [u64, vp, vp, sz, vp, vp]),
        "loom_cuda_model_free": (i, [u64]),
        "loom_cuda_model_error": (i, [u64]),
        "loom_cuda_model_trace": (i, [u64, i, vp, sz]),
        "loom_gguf_parse": (vp, [vp, sz]),
        "loom_gguf_open": (vp, [C.c_char_p]),
        "loom_gguf_error": (C.c_char_p, []),
        "loom_gguf_close": (None, [vp]),
        "loom_gguf_version": (C.c_uint32, [vp]),
        "loom_gguf_alignment": (u64, [vp]),
        "loom_gguf_data_offset": (u64, [vp]),
        "loom_gguf_file_size": (u64, [vp]),
        "loom_gguf_image": (vp, [vp]),
        "loom_gguf_n_tensors": (sz, [vp]),
        "loom_gguf_n_meta": (sz, [vp]),
        "loom_gguf_tensor_info": (i, [vp, sz, C.POINTER(GgufTensor)]),
        "loom_gguf_find_tensor": (i, [vp, C.c_char_p, C.POINTER(GgufTensor)]),
        "loom_gguf_meta": (i, [vp, sz, C.POINTER(GgufValue)]),
        "loom_gguf_find_meta": (i, [vp, C.c_char_p, C.POINTER(GgufValue)]),
        "loom_gguf_get_uint": (i, [vp, C.c_char_p, C.POINTER(u64)]),
        "loom_gguf_get_float": (i, [vp, C.c_char_p, C.POINTER(C.c_double)]),
        "loom_gguf_get_string": (i, [vp, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(sz)]),
        "loom_gguf_get_bool": (i, [vp, C.c_char_p, C.POINTER(i)]),
        "loom_gguf_resolve": (i, [vp, C.c_char_p, C.POINTER(GgufView)]),
        "loom_cuda_verify_shards": (i, [C.POINTER(Shard), sz, vp, C.POINTER(sz)]),
        "loom_cuda_sha256_device": (i, [vp, sz, vp]),
        "loom_cuda_tensor_sha256": (i, [u64, u64, u64, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib().loom_cuda_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> int:
    """OK -> OK; DECLINED -> DECLINED (caller decides); ERROR -> raise."""
    if rc == ERROR:
        raise LoomCudaError(f"{what}: {last_error()}")
    return rc


def must(rc: int, what: str) -> None:
    if rc != OK:
        raise LoomCudaError(f"{what}: {'declined' if rc == DECLINED else 'error'}: {last_error()}")
