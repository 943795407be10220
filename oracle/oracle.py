"""ctypes bindings to liborc.so, the C restatement of the reference CPU path.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Every function here is a
thin numpy wrapper over one ``orc_*`` symbol of scry_oracle.c, which cites the
reference file:line it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liborc.so")
_lib = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


class OrcConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int), ("hidden_size", C.c_int), ("intermediate_size", C.c_int),
        ("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
        ("max_seq_len", C.c_int), ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float),
        ("tie_word_embeddings", C.c_int), ("has_rope_scaling", C.c_int),
        ("rope_scaling", C.c_double * 4),
    ]


def build() -> str:
    """Compile liborc.so with oracle/Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = C.CDLL(_LIB_PATH)
    u64p = C.POINTER(C.c_uint64)
    sig = {
        "orc_rng_u64": (C.c_uint64, [u64p]),
        "orc_rng_f64": (C.c_double, [u64p]),
        "orc_rng_below": (C.c_uint64, [u64p, C.c_uint64]),
        "orc_normal_sample": (C.c_float, [u64p, C.c_float, C.c_float]),
        "orc_normal_vec": (None, [u64p, C.c_size_t, C.c_float, C.c_float, f32p]),
        "orc_normal_vec_at": (None, [C.c_uint64, C.c_uint64, C.c_size_t, C.c_float, C.c_float, f32p]),
        "orc_quantize_symmetric": (C.c_float, [f32p, C.c_size_t, i8p]),
        "orc_dequantize": (None, [i8p, C.c_size_t, C.c_float, f32p]),
        "orc_quantize_grouped": (None, [f32p, C.c_int, C.c_int, C.c_int, i8p, f32p]),
        "orc_matmul_i8_f32": (None, [f32p, i8p, C.c_float, C.c_int, C.c_int, C.c_int, f32p]),
        "orc_matmul_i8_f32_tb": (None, [f32p, i8p, C.c_float, C.c_int, C.c_int, C.c_int, f32p]),
        "orc_matmul_i8_f32_grouped": (None, [f32p, i8p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p]),
        "orc_rmsnorm": (None, [f32p, f32p, C.c_int, C.c_int, C.c_float, f32p]),
        "orc_rope": (None, [f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p, f32p]),
        "orc_scale": (None, [f32p, C.c_size_t, C.c_float, f32p]),
        "orc_swiglu": (None, [f32p, f32p, C.c_size_t, f32p]),
        "orc_softmax": (None, [f32p, C.c_int, C.c_int, f32p]),
        "orc_gemv_trans_b": (None, [f32p, f32p, C.c_int, C.c_int, f32p]),
        "orc_gemv": (None, [f32p, f32p, C.c_int, C.c_int, f32p]),
        "orc_gather_reshape_repeat_kv": (None, [f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p]),
        "orc_compute_rope_freqs": (None, [C.c_int, C.c_float, C.c_void_p, f64p]),
        "orc_argmax": (C.c_int64, [f32p, C.c_size_t]),
        "orc_llama_new_random": (C.c_void_p, [C.POINTER(OrcConfig), C.c_uint64]),
        "orc_llama_new_empty": (C.c_void_p, [C.POINTER(OrcConfig)]),
        "orc_llama_new_uniform": (C.c_void_p, [C.POINTER(OrcConfig), C.c_uint64]),
        "orc_cache_fill": (None, [C.c_void_p, C.c_int, C.c_uint64]),
        "orc_llama_free": (None, [C.c_void_p]),
        "orc_llama_weight": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_float),
                                          C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "orc_llama_lm_head": (C.c_void_p, [C.c_void_p, C.POINTER(C.c_float)]),
        "orc_llama_embed": (C.c_void_p, [C.c_void_p]),
        "orc_llama_norm": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int]),
        "orc_llama_set_scale": (None, [C.c_void_p, C.c_int, C.c_int, C.c_float]),
        "orc_cache_new": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int]),
        "orc_cache_free": (None, [C.c_void_p]),
        "orc_forward_with_cache": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, f32p, C.c_void_p]),
        "orc_generate_greedy": (None, [C.c_void_p, i32p, C.c_int, C.c_int, C.c_int, i32p]),
        "orc_forward_tokens": (None, [C.c_void_p, C.c_void_p, i32p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
        "orc_cache_clone": (C.c_void_p, [C.c_void_p]),
        "orc_cache_truncate": (None, [C.c_void_p, C.c_int]),
        "orc_cache_len": (C.c_int, [C.c_void_p]),
        "orc_sample_token": (C.c_int64, [f32p, C.c_size_t, C.c_float, C.c_size_t, C.c_float, u64p]),
        "orc_set_threads": (None, [C.c_int]),
        "orc_get_threads": (C.c_int, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


# ---- RNG -------------------------------------------------------------------
class Rng:
    """fastrand::Rng restatement (state = seed; wyrand)."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(seed & (2**64 - 1))

    def u64(self) -> int:
        return lib().orc_rng_u64(C.byref(self.state))

    def f64(self) -> float:
        return lib().orc_rng_f64(C.byref(self.state))

    def below(self, n: int) -> int:
        return lib().orc_rng_below(C.byref(self.state), n)

    def normal_vec(self, n: int, mean=0.0, std=0.02) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_normal_vec(C.byref(self.state), n, mean, std, out)
        return out


def normal_vec_at(seed: int, first_draw: int, n: int, mean=0.0, std=0.02) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_normal_vec_at(seed, first_draw, n, mean, std, out)
    return out


def prompt_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """Seeded synthetic prompt: n draws of Rng::usize(0..vocab)."""
    r = Rng(seed)
    return np.array([r.below(vocab) for _ in range(n)], np.int32)


# ---- quantize / ops -------------------------------------------------------
def quantize_symmetric(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32).ravel()
    q = np.empty(w.size, np.int8)
    s = lib().orc_quantize_symmetric(w, w.size, q)
    return q, np.float32(s)


def dequantize(q: np.ndarray, scale) -> np.ndarray:
    q = np.ascontiguousarray(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    lib().orc_dequantize(q, q.size, float(scale), out)
    return out


def quantize_grouped(w: np.ndarray, group: int):
    k, n = w.shape
    w = np.ascontiguousarray(w, np.float32)
    q = np.empty((k, n), np.int8)
    s = np.empty(((k + group - 1) // group, n), np.float32)
    lib().orc_quantize_grouped(w, k, n, group, q, s)
    return q, s


def matmul_i8_f32(a: np.ndarray, q: np.ndarray, scale, m: int, k: int, n: int) -> np.ndarray:
    c = np.empty((m, n), np.float32)
    lib().orc_matmul_i8_f32(np.ascontiguousarray(a, np.float32), np.ascontiguousarray(q, np.int8),
                            float(scale), m, k, n, c)
    return c


def matmul_i8_f32_tb(a, q_t, scale, m, k, n) -> np.ndarray:
    c = np.empty((m, n), np.float32)
    lib().orc_matmul_i8_f32_tb(np.ascontiguousarray(a, np.float32), np.ascontiguousarray(q_t, np.int8),
                               float(scale), m, k, n, c)
    return c


def matmul_i8_f32_grouped(a, q, scales, group, m, k, n) -> np.ndarray:
    c = np.empty((m, n), np.float32)
    lib().orc_matmul_i8_f32_grouped(np.ascontiguousarray(a, np.float32), np.ascontiguousarray(q, np.int8),
                                    np.ascontiguousarray(scales, np.float32), group, m, k, n, c)
    return c


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    d = x.shape[-1]
    rows = x.size // d
    out = np.empty_like(x)
    lib().orc_rmsnorm(x, np.ascontiguousarray(w, np.float32), rows, d, eps, out)
    return out


def rope(x, seq, n_heads, hd, start_pos, freqs_f32) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_rope(x, seq, n_heads, hd, start_pos, np.ascontiguousarray(freqs_f32, np.float32), out)
    return out


def scale(x, s) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_scale(x, x.size, float(s), out)
    return out


def swiglu(g, u) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty_like(g)
    lib().orc_swiglu(g, np.ascontiguousarray(u, np.float32), g.size, out)
    return out


def softmax(x, rows, cols) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_softmax(x, rows, cols, out)
    return out


def gather_reshape_repeat_kv(cache, cached_len, n_kv, n_q, hd) -> np.ndarray:
    out = np.empty(n_q * cached_len * hd, np.float32)
    lib().orc_gather_reshape_repeat_kv(np.ascontiguousarray(cache, np.float32), cached_len, n_kv, n_q, hd, out)
    return out


def compute_rope_freqs(hd: int, theta: float, scaling=None) -> np.ndarray:
    out = np.empty(hd // 2, np.float64)
    if scaling is None:
        lib().orc_compute_rope_freqs(hd, theta, None, out)
    else:
        sc = (C.c_double * 4)(*scaling)
        lib().orc_compute_rope_freqs(hd, theta, C.cast(sc, C.c_void_p), out)
    return out


def argmax(x) -> int:
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().orc_argmax(x, x.size))


def sample_token(logits, temperature, top_k, top_p, rng: Rng) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample_token(logits, logits.size, temperature, top_k, top_p, C.byref(rng.state)))


def set_threads(n: int):
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


# ---- model -----------------------------------------------------------------
def make_config(vocab, hidden, inter, layers, heads, kv_heads, max_seq=4096, eps=1e-5,
                theta=10000.0, tie=False, rope_scaling=None) -> OrcConfig:
    c = OrcConfig()
    c.vocab_size, c.hidden_size, c.intermediate_size = vocab, hidden, inter
    c.n_layers, c.n_heads, c.n_kv_heads, c.max_seq_len = layers, heads, kv_heads, max_seq
    c.rms_norm_eps, c.rope_theta, c.tie_word_embeddings = eps, theta, int(tie)
    if rope_scaling is not None:
        c.has_rope_scaling = 1
        for i, v in enumerate(rope_scaling):
            c.rope_scaling[i] = v
    return c


SLOTS = ("qkv", "o", "gate", "up", "down")


class OracleLlama:
    """Quantized LlamaModel (llama.rs) with a contiguous f32 (or bf16-rounded) cache."""

    def __init__(self, cfg: OrcConfig, seed: int | None = 0, uniform: bool = False):
        """seed None: empty model; uniform: seeded uniform int8 weights (for
        timing the CPU path, no parity meaning); else LlamaModel::new."""
        self.cfg = cfg
        L = lib()
        if seed is None:
            self.h = L.orc_llama_new_empty(C.byref(cfg))
        elif uniform:
            self.h = L.orc_llama_new_uniform(C.byref(cfg), seed)
        else:
            self.h = L.orc_llama_new_random(C.byref(cfg), seed)
        self.hd = cfg.hidden_size // cfg.n_heads

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_llama_free(self.h)
            self.h = None

    def weight(self, layer: int, slot: int):
        """(int8 [K,N] view, scale) of one projection, reference [in,out] layout."""
        s = C.c_float()
        k = C.c_int()
        n = C.c_int()
        p = lib().orc_llama_weight(self.h, layer, slot, C.byref(s), C.byref(k), C.byref(n))
        arr = np.ctypeslib.as_array((C.c_int8 * (k.value * n.value)).from_address(p)).reshape(k.value, n.value)
        return arr, np.float32(s.value)

    def lm_head(self):
        s = C.c_float()
        p = lib().orc_llama_lm_head(self.h, C.byref(s))
        V, h = self.cfg.vocab_size, self.cfg.hidden_size
        return np.ctypeslib.as_array((C.c_int8 * (V * h)).from_address(p)).reshape(V, h), np.float32(s.value)

    def embed(self):
        p = lib().orc_llama_embed(self.h)
        V, h = self.cfg.vocab_size, self.cfg.hidden_size
        return np.ctypeslib.as_array((C.c_float * (V * h)).from_address(p)).reshape(V, h)

    def norm(self, layer: int, which: int):
        p = lib().orc_llama_norm(self.h, layer, which)
        return np.ctypeslib.as_array((C.c_float * self.cfg.hidden_size).from_address(p))

    def set_scale(self, layer: int, slot: int, s: float):
        lib().orc_llama_set_scale(self.h, layer, slot, s)

    def new_cache(self, max_seq: int, kv_bf16: bool = False):
        return OracleCache(self, max_seq, kv_bf16)

    def forward_with_cache(self, cache: "OracleCache", token: int, pos: int, trace: bool = False):
        logits = np.empty(self.cfg.vocab_size, np.float32)
        tr = np.empty((self.cfg.n_layers, self.cfg.hidden_size), np.float32) if trace else None
        lib().orc_forward_with_cache(self.h, cache.h, token, pos, logits,
                                     tr.ctypes.data_as(C.c_void_p) if trace else None)
        return (logits, tr) if trace else logits

    def forward_tokens(self, cache: "OracleCache", tokens, pos0: int, all_logits: bool = False):
        """len(tokens) consecutive forward_with_cache calls (positions pos0, pos0+1, ...),
        evaluated layer by layer; bit-identical to the per-token loop.  Returns the
        last token's logits [V], or every token's [n, V] with all_logits."""
        t = np.ascontiguousarray(tokens, np.int32)
        V = self.cfg.vocab_size
        last = np.empty(V, np.float32)
        allv = np.empty((t.size, V), np.float32) if all_logits else None
        lib().orc_forward_tokens(self.h, cache.h, t, t.size, pos0,
                                 allv.ctypes.data_as(C.c_void_p) if all_logits else None,
                                 last.ctypes.data_as(C.c_void_p))
        return allv if all_logits else last

    def generate_greedy(self, prompt, max_tokens: int, kv_bf16: bool = False) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(max_tokens, np.int32)
        lib().orc_generate_greedy(self.h, prompt, prompt.size, max_tokens, int(kv_bf16), out)
        return out


class OracleCache:
    def __init__(self, model: OracleLlama, max_seq: int, kv_bf16: bool, _handle=None):
        self.model = model
        self.h = _handle if _handle is not None else lib().orc_cache_new(model.h, max_seq, int(kv_bf16))

    def clone(self) -> "OracleCache":
        return OracleCache(self.model, 0, False, _handle=lib().orc_cache_clone(self.h))

    def truncate(self, n: int):
        lib().orc_cache_truncate(self.h, n)

    def fill(self, n: int, seed: int = 0):
        """Seeded K/V values in rows 0..n-1, length n (timing only)."""
        lib().orc_cache_fill(self.h, n, seed)

    def __len__(self) -> int:
        return lib().orc_cache_len(self.h)

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_cache_free(self.h)
            self.h = None


def gemv_trans_b(v, mat_t, k: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_gemv_trans_b(np.ascontiguousarray(v, np.float32), np.ascontiguousarray(mat_t, np.float32), k, n, out)
    return out


def gemv(v, mat, k: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_gemv(np.ascontiguousarray(v, np.float32), np.ascontiguousarray(mat, np.float32), k, n, out)
    return out


def attention_decode(q: np.ndarray, kcache: np.ndarray, vcache: np.ndarray, n_q: int, n_kv: int, hd: int) -> np.ndarray:
    """Decode attention of one token as llama.rs:414-456 composes it.

    q: [n_q*hd] (RoPE'd, pre-scaled); kcache/vcache: [S, n_kv*hd].  Returns [n_q*hd]."""
    S = kcache.shape[0]
    kexp = gather_reshape_repeat_kv(kcache.ravel(), S, n_kv, n_q, hd).reshape(n_q, S, hd)
    vexp = gather_reshape_repeat_kv(vcache.ravel(), S, n_kv, n_q, hd).reshape(n_q, S, hd)
    scores = np.stack([gemv_trans_b(q[h * hd:(h + 1) * hd], kexp[h], hd, S) for h in range(n_q)])
    attn = softmax(scores, n_q, S).reshape(n_q, S)
    return np.concatenate([gemv(attn[h], vexp[h], S, hd) for h in range(n_q)])


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (nearest even), returned as f32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32).reshape(np.shape(x))
