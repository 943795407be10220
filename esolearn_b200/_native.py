"""ctypes bindings to libscryb200.so (declarations in include/sb_api.h).

The library is the product: there is no Python or CPU fallback.  Importing
this module fails with a clear error when the library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libscryb200.so")

SB_OK = 0
STATUS_NAMES = {0: "SB_OK", 1: "SB_ERR_CUDA", 2: "SB_ERR_NCCL", 3: "SB_ERR_TIMEOUT", 4: "SB_ERR_SHAPE",
                5: "SB_ERR_OOM", 6: "SB_ERR_ARG", 7: "SB_ERR_STATE", 8: "SB_ERR_UNSUPPORTED"}
SB_DTYPE_F32, SB_DTYPE_BF16, SB_DTYPE_F16 = 0, 1, 2
SB_KV_BF16, SB_KV_F32 = 0, 1
SB_W_QKV, SB_W_O, SB_W_GATE, SB_W_UP, SB_W_DOWN, SB_W_LM_HEAD = range(6)
SB_TP_ID_BYTES = 128
SB_F_EMBED, SB_F_NORM_IN, SB_F_NORM_POST, SB_F_NORM_FINAL = range(4)


class SbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class LlamaConfigC(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32),
        ("n_layers", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
        ("max_seq_len", C.c_int32), ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float),
        ("tie_word_embeddings", C.c_int32), ("has_rope_scaling", C.c_int32),
        ("rope_scaling", C.c_double * 4), ("max_batch", C.c_int32), ("page_size", C.c_int32),
        ("kv_dtype", C.c_int32),
    ]


vp = C.c_void_p
i32p = C.POINTER(C.c_int32)
f32p = C.POINTER(C.c_float)

# name -> (restype, argtypes); mirrors include/sb_api.h one to one.
SIGNATURES = {
    "sb_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "sb_abi_version": (C.c_int, []),
    "sb_init": (C.c_int, [C.c_int]),
    "sb_device_info": (C.c_int, [i32p, i32p, i32p, C.POINTER(C.c_size_t)]),
    "sb_alloc": (C.c_int, [C.POINTER(vp), C.c_size_t]),
    "sb_free": (C.c_int, [vp]),
    "sb_memcpy_h2d": (C.c_int, [vp, vp, C.c_size_t, vp]),
    "sb_memcpy_d2h": (C.c_int, [vp, vp, C.c_size_t, vp]),
    "sb_stream_sync": (C.c_int, [vp]),
    "sb_quantize_symmetric_host": (C.c_int, [vp, C.c_size_t, vp, f32p]),
    "sb_quantize_symmetric": (C.c_int, [vp, C.c_size_t, vp, vp, vp]),
    "sb_qweight_create": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(vp)]),
    "sb_qweight_create_tn": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]),
    "sb_qweight_load": (C.c_int, [vp, vp, vp]),
    "sb_qweight_destroy": (C.c_int, [vp]),
    "sb_matmul_i8_f32": (C.c_int, [vp, vp, C.c_int, C.c_int, vp, vp]),
    "sb_matmul_i8_f32_bias": (C.c_int, [vp, vp, C.c_int, C.c_int, vp, vp, vp]),
    "sb_i8_from_vec": (C.c_int, [vp, C.c_size_t, C.POINTER(vp)]),
    "sb_i8_to_vec": (C.c_int, [vp, vp, C.c_size_t]),
    "sb_i8_len": (C.c_int, [vp, C.POINTER(C.c_size_t)]),
    "sb_i8_destroy": (C.c_int, [vp]),
    "sb_i8_matmul_f32": (C.c_int, [vp, vp, C.c_float, C.c_int, C.c_int, C.c_int, vp, vp]),
    "sb_i8_matmul_f32_bias": (C.c_int, [vp, vp, C.c_float, vp, C.c_int, C.c_int, C.c_int, vp, vp]),
    "sb_rmsnorm": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_float, vp, vp]),
    "sb_rope_with_freqs": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, C.c_float, vp, vp]),
    "sb_swiglu": (C.c_int, [vp, vp, C.c_size_t, vp, vp]),
    "sb_argmax_rows": (C.c_int, [vp, C.c_int, C.c_int, vp, vp]),
    "sb_sample_rows": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, vp, vp, vp]),
    "sb_attn_decode_paged": (C.c_int, [vp, vp, vp, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int,
                                       C.c_int, C.c_int, C.c_int, vp, vp]),
    "sb_attn_decode_paged_noalloc": (C.c_int, [vp, vp, vp, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int,
                                               C.c_int, C.c_int, C.c_int, vp, vp]),
    "sb_llama_create": (C.c_int, [C.POINTER(LlamaConfigC), C.POINTER(vp)]),
    "sb_llama_prefill": (C.c_int, [vp, C.c_int, vp, C.c_int]),
    "sb_tp_unique_id": (C.c_int, [vp]),
    "sb_tp_probe_timeout": (C.c_int, [i32p, C.POINTER(C.c_double)]),
    "sb_llama_create_tp": (C.c_int, [C.POINTER(LlamaConfigC), C.c_int, C.c_int, vp, C.POINTER(vp)]),
    "sb_tp_shard_qweight": (C.c_int, [C.POINTER(LlamaConfigC), C.c_int, C.c_int, C.c_int, vp, vp, i32p, i32p]),
    "sb_llama_destroy": (C.c_int, [vp]),
    "sb_llama_init_random": (C.c_int, [vp, C.c_uint64]),
    "sb_llama_load_qweight": (C.c_int, [vp, C.c_int, C.c_int, vp, C.c_float]),
    "sb_llama_get_qweight": (C.c_int, [vp, C.c_int, C.c_int, vp, f32p]),
    "sb_llama_load_f32": (C.c_int, [vp, C.c_int, C.c_int, vp]),
    "sb_llama_load_hf": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(vp), C.POINTER(C.c_int64),
                                   C.c_int64]),
    "sb_llama_load_hf_f32": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, vp, C.c_int64]),
    "sb_llama_reset": (C.c_int, [vp]),
    "sb_llama_forward": (C.c_int, [vp, C.c_int, vp, vp, vp, vp]),
    "sb_llama_forward_seq": (C.c_int, [vp, vp, C.c_int, vp]),
    "sb_llama_sample": (C.c_int, [vp, C.c_int, C.c_float, C.c_int, C.c_float, vp, vp]),
    "sb_llama_set_sampling": (C.c_int, [vp, C.c_int, C.c_float, C.c_int, C.c_float, C.c_int, vp]),
    "sb_llama_clear_sampling": (C.c_int, [vp]),
    "sb_llama_get_rng": (C.c_int, [vp, C.c_int, vp]),
    "sb_llama_generate_greedy": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, vp]),
    "sb_llama_set_trace": (C.c_int, [vp, C.c_int]),
    "sb_llama_get_trace": (C.c_int, [vp, vp]),
    "sb_llama_begin": (C.c_int, [vp, C.c_int, vp, C.c_int]),
    "sb_llama_step": (C.c_int, [vp, C.c_int]),
    "sb_llama_tokens": (C.c_int, [vp, vp, C.c_int, i32p]),
    "sb_llama_stream": (vp, [vp]),
    "sb_llama_profile_step": (C.c_int, [vp, f32p, f32p, f32p, i32p]),
    "sb_llama_step_bytes": (C.c_int, [vp, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "sb_llama_step_launches": (C.c_int, [vp, C.c_int, i32p]),
    "sb_llama_attn_plan": (C.c_int, [vp, C.c_int, i32p, i32p, i32p]),
    "sb_llama_set_timeline": (C.c_int, [vp, C.c_int]),
    "sb_llama_get_timeline": (C.c_int, [vp, vp, C.c_size_t, i32p, i32p]),
}

_lib = None


def lib() -> C.CDLL:
    """Load libscryb200.so once; raise if it is missing (no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libscryb200.so not found at {LIB_PATH}; build it with `python -m esolearn_b200.build` "
            "(the B200 engine has no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().sb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != SB_OK:
        raise SbError(status, last_error())
