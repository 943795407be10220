"""Llama weights from HF safetensors shards, quantized for the B200 engine.

Mirrors LlamaModel::from_safetensors (crates/scry-llm/src/nn/llama.rs:768-958):
every shard is parsed (8-byte little-endian header length, JSON header of
{name: {dtype, shape, data_offsets}}, raw little-endian data), F32 / BF16 /
F16 tensors become f32 exactly (llama.rs:795-808), projection weights stored
by HF as [out, in] are transposed to [in, out] (llama.rs:815-825), q|k|v are
fused column-wise into one [h, q+2kv] matrix (llama.rs:1009-1029) and the
lm_head stays [V, h] (llama.rs:943-948).  Each projection is then quantized
per tensor with quantize_symmetric (quantize.rs:16-32, bit-exact through the
C ABI) -- the int8 wiring the engine runs.  Shards are memory-mapped, so a
tensor is read when it is converted.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterator, Sequence, Tuple

import numpy as np

from . import _native as N
from .llama import LlamaConfig, quantize_symmetric

_DTYPES = {"F32": np.float32, "BF16": np.uint16, "F16": np.float16}


class SafeTensorsShards:
    """Read-only view of the tensors of one or more .safetensors files."""

    def __init__(self, paths: Sequence[str]):
        self._where: Dict[str, Tuple[np.memmap, str, Tuple[int, ...], int, int]] = {}
        for path in paths:
            with open(path, "rb") as f:
                n = int.from_bytes(f.read(8), "little")
                header = json.loads(f.read(n))
            data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)
            for name, info in header.items():
                if name == "__metadata__":
                    continue
                b, e = info["data_offsets"]
                self._where[name] = (data, info["dtype"], tuple(info["shape"]), b, e)

    def names(self):
        return list(self._where)

    def f32(self, name: str) -> np.ndarray:
        """The tensor as f32 (exact for F32, BF16 and F16 sources)."""
        if name not in self._where:
            raise N.SbError(6, f"tensor '{name}' not found in any shard")
        data, dt, shape, b, e = self._where[name]
        if dt not in _DTYPES:
            raise N.SbError(6, f"unsupported dtype {dt} for tensor '{name}'")
        raw = np.frombuffer(data[b:e], dtype=_DTYPES[dt]).reshape(shape)
        if dt == "BF16":
            return (raw.astype(np.uint32) << 16).view(np.float32)
        return raw.astype(np.float32)


def write_safetensors(path: str, tensors: Dict[str, np.ndarray], bf16: Sequence[str] = ()):
    """Write tensors (f32 arrays; names in `bf16` are stored as BF16, rounded
    to nearest even) in the safetensors format."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, np.float32)
        if name in bf16:
            u = a.view(np.uint32)
            raw = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).tobytes()
            dt = "BF16"
        else:
            raw, dt = a.tobytes(), "F32"
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for raw in blobs:
            f.write(raw)


def quantized_llama_tensors(config: LlamaConfig, paths: Sequence[str]) -> Iterator[tuple]:
    """The engine's tensors from HF shards, in load order.

    Yields ("q", layer, slot, int8 [K,N], scale) for every projection (layer
    -1 = lm_head [V,h]) and ("f", which, layer, f32 array) for the embedding
    and norm weights.  Host only."""
    st = SafeTensorsShards(paths)
    h, F = config.hidden_size, config.intermediate_size
    hd = config.head_dim()
    qd, kd = config.n_heads * hd, config.n_kv_heads * hd

    def proj(name, rows, cols):  # HF [out, in] -> [in, out]
        w = st.f32(name)
        if w.shape != (rows, cols):
            raise N.SbError(4, f"tensor '{name}' has shape {w.shape}, expected {(rows, cols)}")
        return np.ascontiguousarray(w.T)

    yield ("f", N.SB_F_EMBED, 0, st.f32("model.embed_tokens.weight"))
    for i in range(config.n_layers):
        p = f"model.layers.{i}"
        q = proj(f"{p}.self_attn.q_proj.weight", qd, h)
        k = proj(f"{p}.self_attn.k_proj.weight", kd, h)
        v = proj(f"{p}.self_attn.v_proj.weight", kd, h)
        qkv = np.concatenate([q, k, v], axis=1)  # fuse_qkv_weights: column concat per row
        yield ("q", i, N.SB_W_QKV) + quantize_symmetric(qkv)
        yield ("q", i, N.SB_W_O) + quantize_symmetric(proj(f"{p}.self_attn.o_proj.weight", h, qd))
        yield ("q", i, N.SB_W_GATE) + quantize_symmetric(proj(f"{p}.mlp.gate_proj.weight", F, h))
        yield ("q", i, N.SB_W_UP) + quantize_symmetric(proj(f"{p}.mlp.up_proj.weight", F, h))
        yield ("q", i, N.SB_W_DOWN) + quantize_symmetric(proj(f"{p}.mlp.down_proj.weight", h, F))
        yield ("f", N.SB_F_NORM_IN, i, st.f32(f"{p}.input_layernorm.weight"))
        yield ("f", N.SB_F_NORM_POST, i, st.f32(f"{p}.post_attention_layernorm.weight"))
    yield ("f", N.SB_F_NORM_FINAL, 0, st.f32("model.norm.weight"))
    head = st.f32("model.embed_tokens.weight" if config.tie_word_embeddings else "lm_head.weight")
    yield ("q", -1, 0) + quantize_symmetric(head)


def load_into(model, config: LlamaConfig, paths: Sequence[str]):
    """Load HF shards into a QuantLlamaB200 (every rank of a tensor-parallel
    model loads the same full tensors and keeps its slice)."""
    for t in quantized_llama_tensors(config, paths):
        if t[0] == "q":
            model.load_qweight(t[1], t[2], t[3], t[4])
        else:
            model.load_f32(t[1], t[2], t[3])


def shard_paths(directory: str) -> list:
    """The .safetensors files of a checkpoint directory, sorted."""
    return sorted(os.path.join(directory, f) for f in os.listdir(directory) if f.endswith(".safetensors"))
