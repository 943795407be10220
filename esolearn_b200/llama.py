"""Host-side mirror of scry-llm's Llama decode API over the B200 engine.

Names and argument meanings follow the reference crate:

* ``LlamaConfig`` / ``RopeScaling``           -- nn/llama.rs:10-139
* ``QuantLlamaB200`` implements ``CausalLM``   -- generate.rs:5-21 (the
  quantized counterpart of ``LlamaModel``, llama.rs:583-1004)
* ``SamplingConfig``, ``generate``, ``sample_token`` -- generate.rs:24-185
* ``quantize_symmetric``                        -- quantize.rs:16-32
* ``QWeight`` + ``matmul_i8_f32``               -- backend/mod.rs:521-557

Every numeric call goes through libscryb200.so (include/sb_api.h).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _native as N


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


# ---------------------------------------------------------------------------
# configuration (llama.rs:10-139)

@dataclass
class RopeScaling:
    factor: float = 32.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


@dataclass
class LlamaConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    max_seq_len: int = 4096
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    tie_word_embeddings: bool = False
    rope_scaling: Optional[RopeScaling] = None

    def head_dim(self) -> int:  # llama.rs:97-99
        return self.hidden_size // self.n_heads

    # Reference presets (llama.rs:46-95).
    @staticmethod
    def llama_1b() -> "LlamaConfig":
        return LlamaConfig(128256, 2048, 8192, 16, 32, 8, 131072, 1e-5, 500000.0, True, RopeScaling())

    @staticmethod
    def llama_3b() -> "LlamaConfig":
        return LlamaConfig(128256, 3072, 8192, 28, 24, 8, 131072, 1e-5, 500000.0, True, RopeScaling())

    @staticmethod
    def llama_8b() -> "LlamaConfig":
        return LlamaConfig(128256, 4096, 14336, 32, 32, 8, 131072, 1e-5, 500000.0, False, RopeScaling())

    # The benchmark shapes (random-init, untied lm_head).
    @staticmethod
    def tiny() -> "LlamaConfig":
        return LlamaConfig(32000, 512, 1376, 8, 8, 8, 4096, 1e-5, 10000.0, False, None)

    @staticmethod
    def llama2_7b_shape() -> "LlamaConfig":
        return LlamaConfig(32000, 4096, 11008, 32, 32, 32, 4096, 1e-5, 10000.0, False, None)

    @staticmethod
    def llama3_8b_shape() -> "LlamaConfig":
        return LlamaConfig(128256, 4096, 14336, 32, 32, 8, 8192, 1e-5, 500000.0, False, None)

    @staticmethod
    def llama3_70b_shape() -> "LlamaConfig":
        return LlamaConfig(128256, 8192, 28672, 80, 64, 8, 8192, 1e-5, 500000.0, False, None)

    def to_c(self, max_seq: int, max_batch: int, page_size: int, kv_dtype: int) -> N.LlamaConfigC:
        c = N.LlamaConfigC()
        c.vocab_size, c.hidden_size, c.intermediate_size = self.vocab_size, self.hidden_size, self.intermediate_size
        c.n_layers, c.n_heads, c.n_kv_heads = self.n_layers, self.n_heads, self.n_kv_heads
        c.max_seq_len = max_seq
        c.rms_norm_eps, c.rope_theta = self.rms_norm_eps, self.rope_theta
        c.tie_word_embeddings = int(self.tie_word_embeddings)
        if self.rope_scaling is not None:
            c.has_rope_scaling = 1
            rs = self.rope_scaling
            for i, v in enumerate((rs.factor, rs.low_freq_factor, rs.high_freq_factor,
                                   float(rs.original_max_position_embeddings))):
                c.rope_scaling[i] = v
        c.max_batch, c.page_size, c.kv_dtype = max_batch, page_size, kv_dtype
        return c


# ---------------------------------------------------------------------------
# quantization and the op-level int8 matmul

def quantize_symmetric(weights: np.ndarray):
    """quantize.rs:16-32 -> (int8 array, scale).  Bit-exact with the reference."""
    w = np.ascontiguousarray(weights, np.float32).ravel()
    q = np.empty(w.size, np.int8)
    s = C.c_float()
    N.check(N.lib().sb_quantize_symmetric_host(_ptr(w), w.size, _ptr(q), C.byref(s)))
    return q.reshape(np.shape(weights)), np.float32(s.value)


class QWeight:
    """An int8 [K,N] weight packed on the device (the I8Storage of this backend)."""

    def __init__(self, q: np.ndarray, scales, group: int = 0, tile_n: int = 0):
        """tile_n: on-device column tile width (0 = the GEMV's choice; 128
        lets products of 5 or more rows run on the tensor cores)."""
        q = np.ascontiguousarray(q, np.int8)
        self.K, self.N = q.shape
        self.group = group
        h = C.c_void_p()
        N.check(N.lib().sb_qweight_create_tn(self.K, self.N, group, tile_n, C.byref(h)))
        self._h = h
        sc = np.ascontiguousarray(np.atleast_1d(np.asarray(scales, np.float32)))
        N.check(N.lib().sb_qweight_load(self._h, _ptr(q), _ptr(sc)))

    def __del__(self):
        if getattr(self, "_h", None) and N._lib is not None:
            N._lib.sb_qweight_destroy(self._h)
            self._h = None


def matmul_i8_f32(a, w: QWeight, out=None, bias=None, stream: int = 0):
    """backend/mod.rs:521-557 on torch CUDA tensors: a [M,K] f32/bf16 -> [M,N] f32."""
    import torch

    assert a.is_cuda and a.is_contiguous() and a.shape[-1] == w.K
    M = a.numel() // w.K
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.float32, device=a.device)
    dt = N.SB_DTYPE_BF16 if a.dtype == torch.bfloat16 else N.SB_DTYPE_F32
    if dt == N.SB_DTYPE_F32:
        assert a.dtype == torch.float32
    st = C.c_void_p(stream or torch.cuda.current_stream(a.device).cuda_stream)
    if bias is None:
        N.check(N.lib().sb_matmul_i8_f32(w._h, C.c_void_p(a.data_ptr()), dt, M, C.c_void_p(out.data_ptr()), st))
    else:
        N.check(N.lib().sb_matmul_i8_f32_bias(w._h, C.c_void_p(a.data_ptr()), dt, M, C.c_void_p(bias.data_ptr()),
                                              C.c_void_p(out.data_ptr()), st))
    return out


class I8Storage:
    """DeviceBackend::I8Storage (backend/mod.rs:15-21): int8 bytes on the
    device with no shape, made by i8_from_vec.  Clones share the storage."""

    def __init__(self, data):
        d = np.ascontiguousarray(np.asarray(data, np.int8).ravel())
        h = C.c_void_p()
        N.check(N.lib().sb_i8_from_vec(_ptr(d), d.size, C.byref(h)))
        self._h = h
        self.n = d.size

    def __len__(self) -> int:
        return self.n

    def __del__(self):
        if getattr(self, "_h", None) and N._lib is not None:
            N._lib.sb_i8_destroy(self._h)
            self._h = None


class B200Backend:
    """The quantized part of MathBackend (backend/mod.rs) over this library,
    with the reference trait's names and arguments: Storage is a torch CUDA
    f32 tensor, I8Storage an I8Storage; every op returns a new tensor."""

    @staticmethod
    def i8_from_vec(data) -> I8Storage:
        return I8Storage(data)

    @staticmethod
    def i8_to_vec(storage: I8Storage) -> np.ndarray:
        out = np.empty(len(storage), np.int8)
        N.check(N.lib().sb_i8_to_vec(storage._h, _ptr(out), out.size))
        return out

    @staticmethod
    def matmul_i8_f32(a, b_q: I8Storage, scale: float, m: int, k: int, n: int, bias=None):
        """backend/mod.rs:521-557: [m,k] f32 . dequant([k,n] int8, scale) (+ bias) -> [m,n] f32."""
        import torch

        assert a.is_cuda and a.dtype == torch.float32 and a.is_contiguous() and a.numel() == m * k
        c = torch.empty((m, n), dtype=torch.float32, device=a.device)
        st = C.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)
        if bias is None:
            N.check(N.lib().sb_i8_matmul_f32(C.c_void_p(a.data_ptr()), b_q._h, float(scale), m, k, n,
                                             C.c_void_p(c.data_ptr()), st))
        else:
            assert bias.is_cuda and bias.dtype == torch.float32 and bias.numel() == n
            N.check(N.lib().sb_i8_matmul_f32_bias(C.c_void_p(a.data_ptr()), b_q._h, float(scale),
                                                  C.c_void_p(bias.data_ptr()), m, k, n, C.c_void_p(c.data_ptr()),
                                                  st))
        return c

    @staticmethod
    def matmul_i8_f32_bias(a, b_q: I8Storage, scale: float, bias, m: int, k: int, n: int):
        return B200Backend.matmul_i8_f32(a, b_q, scale, m, k, n, bias=bias)


class QuantLinear:
    """nn::linear::Linear after quantize_weights() (linear.rs:9-13, 56-95), the
    W8A32 layer every other `quantize` consumer uses (GPT-2's Linear layers;
    Whisper's MLP fc1/fc2, scry-stt checkpoint/mod.rs:184-193):
    forward(input[seq, in]) = matmul_i8_f32_bias(input, q, scale, bias) on the
    device.  The weight is [in, out] as in the reference; the bias defaults to
    zeros like Linear::new.  tile_n 128 sends 5+ rows to the tensor cores."""

    def __init__(self, weight: np.ndarray, bias: Optional[np.ndarray] = None, tile_n: int = 128):
        w = np.ascontiguousarray(weight, np.float32)
        if w.ndim != 2:
            raise N.SbError(4, f"Linear weight must be [in, out], got shape {w.shape}")
        self.in_features, self.out_features = w.shape
        self.weight_q, self.scale = quantize_symmetric(w)  # QuantState (linear.rs:9-13)
        self._w = QWeight(self.weight_q, [self.scale], tile_n=tile_n)
        b = np.zeros(self.out_features, np.float32) if bias is None else np.asarray(bias, np.float32)
        if b.shape != (self.out_features,):
            raise N.SbError(4, f"Linear bias must be [{self.out_features}], got shape {b.shape}")
        self._bias_host = np.ascontiguousarray(b)
        self._bias_dev = None

    def forward(self, x, out=None, stream: int = 0):
        """x: torch CUDA [seq, in] f32 or bf16 -> [seq, out] f32."""
        import torch

        if self._bias_dev is None or self._bias_dev.device != x.device:
            self._bias_dev = torch.from_numpy(self._bias_host).to(x.device)
        return matmul_i8_f32(x.contiguous(), self._w, out=out, bias=self._bias_dev, stream=stream)

    __call__ = forward


# ---------------------------------------------------------------------------
# tensor parallelism (no reference counterpart)

def tp_unique_id() -> bytes:
    """A fresh communicator id for a tensor-parallel model (make it on one rank, send it to the others)."""
    buf = (C.c_uint8 * N.SB_TP_ID_BYTES)()
    N.check(N.lib().sb_tp_unique_id(buf))
    return bytes(buf)


def _cfg_c(config: LlamaConfig):
    return config.to_c(config.max_seq_len, 1, 64, N.SB_KV_BF16)


def tp_shard_shape(config: LlamaConfig, slot: int, rank: int, size: int):
    """(rows, cols) of rank's slice of weight `slot` (SB_W_*, SB_W_LM_HEAD = [V,h]); host only."""
    r, c = C.c_int32(), C.c_int32()
    cfg = _cfg_c(config)
    N.check(N.lib().sb_tp_shard_qweight(C.byref(cfg), slot, rank, size, None, None, C.byref(r), C.byref(c)))
    return r.value, c.value


def tp_shard_qweight(config: LlamaConfig, slot: int, rank: int, size: int, full: np.ndarray) -> np.ndarray:
    """Rank's slice of a full reference int8 tensor, as the engine keeps it (host only, no GPU)."""
    full = np.ascontiguousarray(full, np.int8)
    out = np.empty(tp_shard_shape(config, slot, rank, size), np.int8)
    cfg = _cfg_c(config)
    N.check(N.lib().sb_tp_shard_qweight(C.byref(cfg), slot, rank, size, _ptr(full), _ptr(out), None, None))
    return out


# ---------------------------------------------------------------------------
# the model (CausalLM, generate.rs:5-21)

class LlamaKvCacheHandle:
    """Caller-owned cache handle (LlamaKvCache, kv_cache.rs:134-145).

    The pages live inside the engine; the handle records the sequence slot and
    the number of cached positions, like LlamaLayerKvCache::seq_len."""

    def __init__(self, model: "QuantLlamaB200", max_seq: int, slot: int = 0):
        self.model, self.max_seq, self.slot, self.seq_len = model, max_seq, slot, 0


class QuantLlamaB200:
    """Int8 Llama decode on one B200 (the quantized LlamaModel)."""

    def __init__(self, config: LlamaConfig, *, max_seq: Optional[int] = None, max_batch: int = 1,
                 page_size: int = 64, kv_dtype: str = "bf16", tp_rank: int = 0, tp_size: int = 1,
                 tp_id: Optional[bytes] = None):
        """tp_size > 1: this process is rank tp_rank of a tensor-parallel model
        (one GPU per rank, the current device); every rank passes the same
        tp_id (from tp_unique_id() on one rank) and makes the same calls."""
        self.config = config
        self.max_seq = max_seq or config.max_seq_len
        self.max_batch = max_batch
        self.tp_rank, self.tp_size = tp_rank, tp_size
        kvd = {"bf16": N.SB_KV_BF16, "f32": N.SB_KV_F32}[kv_dtype]
        self.kv_dtype = kv_dtype
        cfg = config.to_c(self.max_seq, max_batch, page_size, kvd)
        self._cfg_c = cfg
        h = C.c_void_p()
        if tp_size > 1:
            if tp_id is None or len(tp_id) != N.SB_TP_ID_BYTES:
                raise N.SbError(6, "tensor parallelism needs the communicator id of tp_unique_id()")
            idb = (C.c_uint8 * N.SB_TP_ID_BYTES).from_buffer_copy(tp_id)
            N.check(N.lib().sb_llama_create_tp(C.byref(cfg), tp_rank, tp_size, idb, C.byref(h)))
        else:
            N.check(N.lib().sb_llama_create(C.byref(cfg), C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) and N._lib is not None:
            N._lib.sb_llama_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    # -- weights --------------------------------------------------------
    @classmethod
    def from_safetensors(cls, config: LlamaConfig, paths, cache: Optional[str] = None, device_quantize: bool = True,
                         **kw) -> "QuantLlamaB200":
        """LlamaModel::from_safetensors (llama.rs:768-958) + quantize_symmetric per projection.
        device_quantize: convert, transpose, fuse and quantize on the GPU
        (sb_llama_load_hf) instead of the host.  cache: a packed-int8 cache
        file, read when it exists, else written from the shards during this
        load (host quantization)."""
        from .safetensors_io import load_into

        m = cls(config, **kw)
        load_into(m, config, paths, cache=cache, device=device_quantize)
        return m

    @classmethod
    def new_random(cls, config: LlamaConfig, seed: int, **kw) -> "QuantLlamaB200":
        """LlamaModel::new (llama.rs:593-680) + quantize_symmetric, on the device."""
        m = cls(config, **kw)
        N.check(N.lib().sb_llama_init_random(m._h, seed))
        return m

    def load_qweight(self, layer: int, slot: int, q: np.ndarray, scale: float):
        q = np.ascontiguousarray(q, np.int8)
        N.check(N.lib().sb_llama_load_qweight(self._h, layer, slot, _ptr(q), float(scale)))

    def get_qweight(self, layer: int, slot: int):
        """(int8 [K,N] in the reference layout, scale); layer -1 = lm_head [V,h].
        Under tensor parallelism: this rank's slice (tp_shard_qweight)."""
        sl = N.SB_W_LM_HEAD if layer < 0 else slot
        shape = tp_shard_shape(self.config, sl, self.tp_rank, self.tp_size)
        q = np.empty(shape, np.int8)
        s = C.c_float()
        N.check(N.lib().sb_llama_get_qweight(self._h, layer, slot, _ptr(q), C.byref(s)))
        return q, np.float32(s.value)

    def load_f32(self, which: int, layer: int, data: np.ndarray):
        d = np.ascontiguousarray(data, np.float32)
        N.check(N.lib().sb_llama_load_f32(self._h, which, layer, _ptr(d)))

    # -- CausalLM ------------------------------------------------------
    def vocab_size(self) -> int:
        return self.config.vocab_size

    def new_kv_cache(self, max_seq: int) -> LlamaKvCacheHandle:
        if max_seq > self.max_seq:
            raise N.SbError(4, f"cache of {max_seq} positions exceeds the engine's {self.max_seq}")
        N.check(N.lib().sb_llama_reset(self._h))
        return LlamaKvCacheHandle(self, max_seq)

    def forward(self, token_ids: Sequence[int]) -> np.ndarray:
        """CausalLM::forward (generate.rs:9, llama.rs:683-700): logits [seq, vocab]
        of every position, as batched prefill chunks (sb_llama_forward_seq).
        Overwrites sequence slot 0's cached positions."""
        t = np.ascontiguousarray(token_ids, np.int32)
        out = np.empty((t.size, self.config.vocab_size), np.float32)
        N.check(N.lib().sb_llama_forward_seq(self._h, _ptr(t), t.size, _ptr(out)))
        return out

    def forward_with_cache(self, token_id: int, pos: int, cache: LlamaKvCacheHandle) -> np.ndarray:
        """forward_with_llama_cache (llama.rs:744-763): logits [vocab] of one token."""
        logits, _ = self.forward_batch([token_id], [pos], slots=[cache.slot])
        cache.seq_len = pos + 1
        return logits[0]

    def forward_batch(self, tokens: Sequence[int], positions: Sequence[int], slots=None, want_logits=True):
        """One decode step of len(tokens) sequences (slot b = row b)."""
        B = len(tokens)
        if slots is not None and list(slots) != list(range(B)):
            raise N.SbError(6, "sequences occupy slots 0..B-1 in order")
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        am = np.empty(B, np.int32)
        lg = np.empty((B, self.config.vocab_size), np.float32) if want_logits else None
        N.check(N.lib().sb_llama_forward(self._h, B, _ptr(t), _ptr(p), _ptr(lg) if want_logits else None, _ptr(am)))
        return lg, am

    def sample(self, config: "SamplingConfig", rngs: Sequence["Rng"]) -> list:
        """sample_token (generate.rs:92-165) on the device for each row of the
        logits the last forward left there (sb_llama_sample); rngs[b]
        advances exactly as Rng.f64() would on the host."""
        st = np.array([r.state for r in rngs], np.uint64)
        out = np.empty(len(rngs), np.int32)
        N.check(N.lib().sb_llama_sample(self._h, len(rngs), float(config.temperature), int(config.top_k),
                                        float(config.top_p), _ptr(st), _ptr(out)))
        for r, v in zip(rngs, st):
            r.state = int(v)
        return out.tolist()

    def set_sampling(self, config: "SamplingConfig", rngs: Sequence["Rng"], max_draws: int | None = None):
        """Make every decode step that step() queues end in sample_token on
        the device for rows 0..len(rngs)-1 (sb_llama_set_sampling): the
        sampled token feeds the next step with no host round trip; rngs[b]'s
        state is copied to the device (rng_states() reads it back)."""
        st = np.array([r.state for r in rngs], np.uint64)
        md = 0x7FFFFFFF if max_draws is None else int(max_draws)
        N.check(N.lib().sb_llama_set_sampling(self._h, len(rngs), float(config.temperature), int(config.top_k),
                                              float(config.top_p), md, _ptr(st)))

    def clear_sampling(self):
        N.check(N.lib().sb_llama_clear_sampling(self._h))

    def rng_states(self, batch: int) -> np.ndarray:
        st = np.empty(batch, np.uint64)
        N.check(N.lib().sb_llama_get_rng(self._h, batch, _ptr(st)))
        return st

    def generate_sampled(self, prompts, config: "SamplingConfig", rngs: Sequence["Rng"],
                         batched_prefill: bool = False) -> np.ndarray:
        """generate() (generate.rs:51-89) with sampling, for equal-length
        prompts, as one device loop: max(1, max_tokens) tokens per prompt,
        [B, n]; rngs[b] ends where sampling on the host would leave it."""
        pr = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        B, n_out = pr.shape[0], max(1, config.max_tokens)
        if len(rngs) != B:
            raise ValueError("generate_sampled: one generator per prompt")
        self.set_sampling(config, rngs, n_out)
        try:
            if batched_prefill:
                self.prefill(pr)
                self.step(n_out - 1)
            else:
                self.begin(pr)
                self.step(pr.shape[1] + n_out - 1)
            out = self.tokens(B, n_out)
            st = self.rng_states(B)
        finally:
            self.clear_sampling()
        for r, v in zip(rngs, st):
            r.state = int(v)
        return out

    def set_trace(self, on: bool):
        N.check(N.lib().sb_llama_set_trace(self._h, int(on)))

    def get_trace(self, batch: int = 1) -> np.ndarray:
        out = np.empty((self.config.n_layers, batch, self.config.hidden_size), np.float32)
        N.check(N.lib().sb_llama_get_trace(self._h, _ptr(out)))
        return out

    def generate_greedy(self, prompts, max_tokens: int, batched_prefill: bool = False) -> np.ndarray:
        """generate (generate.rs:51-89) at temperature 0 for equal-length prompts.
        batched_prefill: run the prompt as chunks of max_batch positions
        (sb_llama_prefill) instead of one position per step."""
        pr = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        out = np.empty((pr.shape[0], max_tokens), np.int32)
        if not batched_prefill:
            N.check(N.lib().sb_llama_generate_greedy(self._h, pr.shape[0], _ptr(pr), pr.shape[1], max_tokens,
                                                     _ptr(out)))
            return out
        self.prefill(pr)
        self.step(max_tokens - 1)
        return self.tokens(pr.shape[0], max_tokens)

    def prefill(self, prompts):
        """Batched prefill (sb_llama_prefill): the sequences are then ready to decode with step()."""
        pr = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        N.check(N.lib().sb_llama_prefill(self._h, pr.shape[0], _ptr(pr), pr.shape[1]))

    # -- benchmark helpers --------------------------------------------------
    def begin(self, prompts):
        pr = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        N.check(N.lib().sb_llama_begin(self._h, pr.shape[0], _ptr(pr), pr.shape[1]))

    def step(self, n: int = 1):
        N.check(N.lib().sb_llama_step(self._h, n))

    def tokens(self, batch: int, max_tokens: int) -> np.ndarray:
        out = np.zeros((batch, max_tokens), np.int32)
        n = C.c_int32()
        N.check(N.lib().sb_llama_tokens(self._h, _ptr(out), max_tokens, C.byref(n)))
        return out[:, : n.value]

    def stream(self) -> int:
        return N.lib().sb_llama_stream(self._h) or 0

    def profile_step(self):
        """One eager step timed per kernel class: (gemv_ms, attn_ms, other_ms, launches)."""
        g, a, o = C.c_float(), C.c_float(), C.c_float()
        n = C.c_int32()
        N.check(N.lib().sb_llama_profile_step(self._h, C.byref(g), C.byref(a), C.byref(o), C.byref(n)))
        return g.value, a.value, o.value, n.value

    def step_launches(self, batch: int = 1) -> int:
        """Kernel launches per decode step (1 = the persistent single-kernel step)."""
        n = C.c_int32()
        N.check(N.lib().sb_llama_step_launches(self._h, batch, C.byref(n)))
        return n.value

    def attn_plan(self, batch: int = 1):
        """(context splits, tensor-map kernel?, chunk) of a step's attention (sb_llama_attn_plan)."""
        s, t, c = C.c_int32(), C.c_int32(), C.c_int32()
        N.check(N.lib().sb_llama_attn_plan(self._h, batch, C.byref(s), C.byref(t), C.byref(c)))
        return s.value, bool(t.value), c.value

    def set_timeline(self, on: bool):
        """Record per-phase, per-CTA %globaltimer stamps in every later persistent step."""
        N.check(N.lib().sb_llama_set_timeline(self._h, int(on)))

    def timeline(self) -> np.ndarray:
        """Stamps of the last persistent step: [phases, ctas, 5] ns (start, input done,
        first and last weight stage ready, end)."""
        p, c = C.c_int32(), C.c_int32()
        N.check(N.lib().sb_llama_get_timeline(self._h, None, 0, C.byref(p), C.byref(c)))
        out = np.zeros((p.value, c.value, 5), np.uint64)
        N.check(N.lib().sb_llama_get_timeline(self._h, _ptr(out), out.size, C.byref(p), C.byref(c)))
        return out

    def step_bytes(self):
        w, kv = C.c_double(), C.c_double()
        N.check(N.lib().sb_llama_step_bytes(self._h, C.byref(w), C.byref(kv)))
        return w.value, kv.value


# ---------------------------------------------------------------------------
# generation (generate.rs:24-185)

@dataclass
class SamplingConfig:
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    max_tokens: int = 128


class Rng:
    """fastrand::Rng (wyrand), used by the sampler's weighted_sample."""

    C0 = 0x2D358DCCAA6C78A5
    C1 = 0x8BB84B93962EACC9
    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        self.state = seed & self.MASK

    def u64(self) -> int:
        self.state = (self.state + self.C0) & self.MASK
        s = self.state
        t = s * (s ^ self.C1)
        return (t & self.MASK) ^ (t >> 64)

    def f64(self) -> float:
        bits = ((1 << 62) - (1 << 52)) + (self.u64() >> 12)
        return float(np.array([bits], np.uint64).view(np.float64)[0]) - 1.0


def argmax_last(logits: np.ndarray) -> int:
    """generate.rs:167-173: the last index among equal maxima."""
    lg = np.asarray(logits)
    return int(len(lg) - 1 - np.argmax(lg[::-1]))


def sample_token(logits: np.ndarray, config: SamplingConfig, rng: Rng) -> int:
    """generate.rs:92-165."""
    n = len(logits)
    if config.temperature < 1e-8:
        return argmax_last(logits)
    scaled = np.asarray(logits, np.float64) / float(np.float32(config.temperature))
    if 0 < config.top_k < n:
        thr = np.sort(scaled)[::-1][config.top_k - 1]
        scaled = np.where(scaled < thr, -np.inf, scaled)
    mx = scaled.max()
    probs = np.exp(scaled - mx)
    s = probs.sum()
    probs = probs / s if s > 0 else np.full(n, 1.0 / n)
    if 0.0 < config.top_p < 1.0:
        order = np.argsort(-probs, kind="stable")
        cum = np.cumsum(probs[order])
        hit = np.nonzero(cum >= float(np.float32(config.top_p)))[0]
        cut = int(hit[0]) + 1 if hit.size else n
        keep = np.zeros(n, bool)
        keep[order[:cut]] = True
        probs = np.where(keep, probs, 0.0)
        s2 = probs.sum()
        if s2 > 0:
            probs = probs / s2
    r = rng.f64()
    cum = 0.0
    for i, p in enumerate(probs):
        cum += p
        if r < cum:
            return i
    return n - 1


def generate(model: QuantLlamaB200, prompt_tokens: Sequence[int], config: SamplingConfig, rng: Rng,
             device_sampling: bool = True, device_loop: bool = True) -> list:
    """generate.rs:51-89.  Greedy runs entirely on the device.  Sampled
    generation runs as one device loop (every step samples on the device and
    feeds its token to the next step) unless device_loop is False, where each
    token is sampled on the device but passes through the host, or
    device_sampling is False or the model is tensor-parallel, where the logits
    come back and sample_token runs on the host."""
    if len(prompt_tokens) == 0:
        raise ValueError("generate: prompt_tokens must not be empty")
    if config.temperature < 1e-8:
        return model.generate_greedy([list(prompt_tokens)], config.max_tokens)[0].tolist()
    if device_sampling and device_loop and model.tp_size == 1:
        return model.generate_sampled([list(prompt_tokens)], config, [rng])[0].tolist()
    max_seq = len(prompt_tokens) + config.max_tokens
    cache = model.new_kv_cache(max_seq)
    V = model.vocab_size()
    on_device = device_sampling and model.tp_size == 1

    def step(tok: int, pos: int, sample: bool):
        if not on_device:
            logits = model.forward_with_cache(tok, pos, cache)
            return sample_token(logits[:V], config, rng) if sample else None
        model.forward_batch([tok], [pos], slots=[cache.slot], want_logits=False)
        cache.seq_len = pos + 1
        return model.sample(config, [rng])[0] if sample else None

    out = []
    for pos, tok in enumerate(prompt_tokens):
        t = step(int(tok), pos, pos == len(prompt_tokens) - 1)
        if t is not None:
            out.append(t)
    for i in range(1, config.max_tokens):
        out.append(step(out[-1], len(prompt_tokens) + i - 1, True))
    return out


def generate_batch(model: QuantLlamaB200, prompts: Sequence[Sequence[int]], config: SamplingConfig,
                   rngs: Sequence[Rng], device_sampling: bool = True, device_loop: bool = True) -> list:
    """generate() (generate.rs:51-89) for several prompts at once, one engine
    row per sequence: sequence b's tokens, and the final state of rngs[b],
    equal generate(model, prompts[b], config, rngs[b]).  Prompts may differ in
    length.  Every row advances one position per step and samples from the
    step of its last prompt token on (max(1, max_tokens) tokens, like the
    reference loop); a row that is done keeps stepping without drawing from
    its generator.  Sampling runs on the device unless device_sampling is
    False or the model is tensor-parallel; prompts of equal length then run
    as one device loop (generate_sampled) unless device_loop is False."""
    B = len(prompts)
    if len(rngs) != B:
        raise ValueError("generate_batch: one generator per prompt")
    if any(len(p) == 0 for p in prompts):
        raise ValueError("generate: prompt_tokens must not be empty")
    if B == 0:
        return []
    if B > model.max_batch:
        raise N.SbError(4, f"generate_batch: {B} prompts exceed the engine's max_batch {model.max_batch}")
    lens = [len(p) for p in prompts]
    n_out = max(1, config.max_tokens)
    if device_sampling and device_loop and model.tp_size == 1 and len(set(lens)) == 1:
        if config.temperature < 1e-8:
            return model.generate_greedy([list(p) for p in prompts], n_out).tolist()
        return model.generate_sampled([list(p) for p in prompts], config, rngs).tolist()
    steps = max(lens) + n_out - 1
    cache = model.new_kv_cache(steps)
    V = model.vocab_size()
    on_device = device_sampling and model.tp_size == 1
    outs = [[] for _ in range(B)]
    for t in range(steps):
        toks = [int(prompts[b][t]) if t < lens[b] else outs[b][-1] for b in range(B)]
        draw = [t >= lens[b] - 1 and len(outs[b]) < n_out for b in range(B)]
        if on_device:
            model.forward_batch(toks, [t] * B, want_logits=False)
            if any(draw):
                # rows that do not sample this step draw from a throwaway state
                got = model.sample(config, [rngs[b] if draw[b] else Rng(0) for b in range(B)])
        else:
            lg, _ = model.forward_batch(toks, [t] * B)
            got = [sample_token(lg[b][:V], config, rngs[b]) if draw[b] else 0 for b in range(B)]
        for b in range(B):
            if draw[b]:
                outs[b].append(int(got[b]))
    cache.seq_len = steps
    return outs


def sample_rows(logits, config: SamplingConfig, rng_states, out=None, stream: int = 0):
    """sample_token (generate.rs:92-165) on the device for every row of a
    torch CUDA [rows, n] f32 tensor (sb_sample_rows).  rng_states: torch
    CUDA int64 [rows] holding the fastrand states (advanced in place, one
    draw per sampled row).  Returns int32 [rows] token ids on the device."""
    import torch

    assert logits.is_cuda and logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
    rows, n = logits.shape
    assert rng_states.is_cuda and rng_states.dtype == torch.int64 and rng_states.numel() == rows
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    st = C.c_void_p(stream or torch.cuda.current_stream(logits.device).cuda_stream)
    N.check(N.lib().sb_sample_rows(C.c_void_p(logits.data_ptr()), rows, n, logits.stride(0),
                                   float(config.temperature), int(config.top_k), float(config.top_p),
                                   C.c_void_p(rng_states.data_ptr()), C.c_void_p(out.data_ptr()), st))
    return out
