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

Packed-int8 cache: the quantized tensors (int8 [K,N] projections with their
per-tensor scales, f32 embedding and norms) can be written once to a single
safetensors file and loaded from it later without re-quantizing.  Its
metadata records the model configuration, checked on load.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterator, Sequence, Tuple

import numpy as np

from . import _native as N
from .llama import LlamaConfig, quantize_symmetric

_DTYPES = {"F32": np.float32, "BF16": np.uint16, "F16": np.float16, "I8": np.int8}
CACHE_FORMAT = "scry-b200-int8/1"


# bytes per element of the safetensors dtypes (the loader converts F32 / BF16
# / F16 and reads I8; the others are only size-checked)
_ITEMSIZE = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I16": 2, "I8": 1, "U64": 8,
             "U32": 4, "U16": 2, "U8": 1, "BOOL": 1, "F8_E4M3": 1, "F8_E5M2": 1}


def _read_header(path: str):
    """(header dict, header length, file size) of one file; a malformed file
    raises SbError (the reference's loader returns ScryLlmError, error.rs:1-27)."""
    size = os.path.getsize(path)
    if size < 8:
        raise N.SbError(6, f"{path}: {size} bytes, too short for a safetensors header")
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        if n > size - 8:
            raise N.SbError(6, f"{path}: header of {n} bytes runs past the end of the file ({size} bytes)")
        raw = f.read(n)
    try:
        header = json.loads(raw)
    except (UnicodeDecodeError, ValueError) as ex:
        raise N.SbError(6, f"{path}: header is not valid JSON ({ex})") from None
    if not isinstance(header, dict):
        raise N.SbError(6, f"{path}: header is not a map of tensors")
    return header, n, size


def _check_entry(path: str, name: str, info, data_bytes: int):
    """dtype, shape and byte range of one tensor, checked against the file."""
    try:
        dt = info["dtype"]
        shape = tuple(int(d) for d in info["shape"])
        b, e = (int(v) for v in info["data_offsets"])
    except (KeyError, TypeError, ValueError):
        raise N.SbError(6, f"{path}: tensor '{name}' has a malformed entry") from None
    if not isinstance(dt, str) or any(d < 0 for d in shape):
        raise N.SbError(6, f"{path}: tensor '{name}' has a malformed dtype or shape")
    if not 0 <= b <= e <= data_bytes:
        raise N.SbError(6, f"{path}: tensor '{name}' spans bytes [{b}, {e}) of a {data_bytes}-byte data section")
    if dt in _ITEMSIZE and (e - b) != int(np.prod(shape, dtype=np.int64)) * _ITEMSIZE[dt]:
        raise N.SbError(4, f"{path}: tensor '{name}' holds {e - b} bytes, its {dt} shape {list(shape)} needs "
                           f"{int(np.prod(shape, dtype=np.int64)) * _ITEMSIZE[dt]}")
    return dt, shape, b, e


class SafeTensorsShards:
    """Read-only view of the tensors of one or more .safetensors files."""

    def __init__(self, paths: Sequence[str]):
        self._where: Dict[str, Tuple[np.memmap, str, Tuple[int, ...], int, int]] = {}
        self._meta: Dict[str, str] = {}
        for path in paths:
            header, n, size = _read_header(path)
            data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n) if size > 8 + n else np.zeros(0, np.uint8)
            for name, info in header.items():
                if name == "__metadata__":
                    if not isinstance(info, dict):
                        raise N.SbError(6, f"{path}: __metadata__ is not a map")
                    self._meta.update(info)
                    continue
                dt, shape, b, e = _check_entry(path, name, info, size - 8 - n)
                self._where[name] = (data, dt, shape, b, e)

    def names(self):
        return list(self._where)

    def metadata(self) -> dict:
        return dict(self._meta)

    def raw(self, name: str) -> np.ndarray:
        """The tensor in its stored dtype (BF16 as uint16 bits)."""
        if name not in self._where:
            raise N.SbError(6, f"tensor '{name}' not found in any shard")
        data, dt, shape, b, e = self._where[name]
        if dt not in _DTYPES:
            raise N.SbError(6, f"unsupported dtype {dt} for tensor '{name}'")
        return np.frombuffer(data[b:e], dtype=_DTYPES[dt]).reshape(shape)

    def dtype(self, name: str) -> str:
        if name not in self._where:
            raise N.SbError(6, f"tensor '{name}' not found in any shard")
        return self._where[name][1]

    def f32(self, name: str) -> np.ndarray:
        """The tensor as f32 (exact for F32, BF16 and F16 sources)."""
        raw = self.raw(name)
        dt = self._where[name][1]
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


_SB_DTYPE = {"F32": N.SB_DTYPE_F32, "BF16": N.SB_DTYPE_BF16, "F16": N.SB_DTYPE_F16}


def load_hf_device(model, config: LlamaConfig, paths: Sequence[str]):
    """The same wiring as quantized_llama_tensors, done on the device: every
    tensor's bytes go to the GPU as stored (memory-mapped shards, no host
    conversion) and sb_llama_load_hf converts, transposes, fuses q|k|v,
    quantizes and packs them there (bit-exact with the host path).  Every
    rank of a tensor-parallel model passes the full tensors."""
    import ctypes as C

    st = SafeTensorsShards(paths)
    h, F, V = config.hidden_size, config.intermediate_size, config.vocab_size
    hd = config.head_dim()
    qd, kd = config.n_heads * hd, config.n_kv_heads * hd

    def raw(name, shape):
        dt = st.dtype(name)
        if dt not in _SB_DTYPE:
            raise N.SbError(6, f"tensor '{name}': dtype {dt} is not F32, BF16 or F16")
        a = st.raw(name)
        if a.shape != tuple(shape):
            raise N.SbError(4, f"tensor '{name}' has shape {a.shape}, expected {tuple(shape)}")
        return a, _SB_DTYPE[dt]

    def proj(layer, slot, names, rows, cols):
        arrs = [raw(n, (r, cols)) for n, r in zip(names, rows)]
        dts = {d for _, d in arrs}
        if len(dts) != 1:
            raise N.SbError(6, f"tensors {names} mix dtypes")
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a, _ in arrs])
        rr = (C.c_int64 * len(arrs))(*rows)
        N.check(N.lib().sb_llama_load_hf(model._h, layer, slot, dts.pop(), len(arrs), ptrs, rr, cols))

    def f32(which, layer, name, shape):
        a, dt = raw(name, shape)
        N.check(N.lib().sb_llama_load_hf_f32(model._h, which, layer, dt, C.c_void_p(a.ctypes.data), a.size))

    f32(N.SB_F_EMBED, 0, "model.embed_tokens.weight", (V, h))
    for i in range(config.n_layers):
        p = f"model.layers.{i}"
        proj(i, N.SB_W_QKV, [f"{p}.self_attn.{x}_proj.weight" for x in "qkv"], [qd, kd, kd], h)
        proj(i, N.SB_W_O, [f"{p}.self_attn.o_proj.weight"], [h], qd)
        proj(i, N.SB_W_GATE, [f"{p}.mlp.gate_proj.weight"], [F], h)
        proj(i, N.SB_W_UP, [f"{p}.mlp.up_proj.weight"], [F], h)
        proj(i, N.SB_W_DOWN, [f"{p}.mlp.down_proj.weight"], [h], F)
        f32(N.SB_F_NORM_IN, i, f"{p}.input_layernorm.weight", (h,))
        f32(N.SB_F_NORM_POST, i, f"{p}.post_attention_layernorm.weight", (h,))
    f32(N.SB_F_NORM_FINAL, 0, "model.norm.weight", (h,))
    head = "model.embed_tokens.weight" if config.tie_word_embeddings else "lm_head.weight"
    proj(-1, 0, [head], [V], h)


# ---------------------------------------------------------------------------
# packed-int8 cache

_SLOT_NAMES = {N.SB_W_QKV: "qkv", N.SB_W_O: "o", N.SB_W_GATE: "gate", N.SB_W_UP: "up", N.SB_W_DOWN: "down"}
_F_NAMES = {N.SB_F_EMBED: "embed", N.SB_F_NORM_IN: "norm_in", N.SB_F_NORM_POST: "norm_post",
            N.SB_F_NORM_FINAL: "norm_final"}


def _config_meta(config: LlamaConfig) -> str:
    # every field that shapes or identifies the weights (the KV capacity does not)
    fields = {k: (v.__dict__ if hasattr(v, "__dict__") else v) for k, v in vars(config).items() if k != "max_seq_len"}
    return json.dumps(fields, sort_keys=True)


def _cache_layout(config: LlamaConfig):
    """(name, dtype, shape) of every cache entry, in the order
    quantized_llama_tensors yields them (each projection's int8 tensor is
    followed by its scale)."""
    h, F, V = config.hidden_size, config.intermediate_size, config.vocab_size
    hd = config.head_dim()
    qd, kd = config.n_heads * hd, config.n_kv_heads * hd
    shapes = {N.SB_W_QKV: (h, qd + 2 * kd), N.SB_W_O: (qd, h), N.SB_W_GATE: (h, F), N.SB_W_UP: (h, F),
              N.SB_W_DOWN: (F, h)}
    out = [("embed", "F32", (V, h))]
    for i in range(config.n_layers):
        for slot in (N.SB_W_QKV, N.SB_W_O, N.SB_W_GATE, N.SB_W_UP, N.SB_W_DOWN):
            out.append((f"layers.{i}.{_SLOT_NAMES[slot]}.q", "I8", shapes[slot]))
            out.append((f"layers.{i}.{_SLOT_NAMES[slot]}.scale", "F32", (1,)))
        out.append((f"layers.{i}.norm_in", "F32", (h,)))
        out.append((f"layers.{i}.norm_post", "F32", (h,)))
    out.append(("norm_final", "F32", (h,)))
    out.append(("lm_head.q", "I8", (V, h)))
    out.append(("lm_head.scale", "F32", (1,)))
    return out


def _entry_arrays(t) -> list:
    """The cache entries (arrays) of one yielded tensor tuple."""
    if t[0] == "q":
        return [np.ascontiguousarray(t[3], np.int8), np.array([t[4]], np.float32)]
    return [np.ascontiguousarray(t[3], np.float32)]


def write_quantized_cache(config: LlamaConfig, tensors: Iterator[tuple], path: str) -> Iterator[tuple]:
    """Stream `tensors` (quantized_llama_tensors' tuples) into a packed-int8
    cache at `path` while passing each tuple on, so a model can load and
    write the cache in one pass.  Shapes come from the configuration, so the
    header is written first and no tensor is held longer than its write."""
    layout = _cache_layout(config)
    header, off = {}, 0
    for name, dt, shape in layout:
        nbytes = int(np.prod(shape)) * (1 if dt == "I8" else 4)
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    header["__metadata__"] = {"format": CACHE_FORMAT, "config": _config_meta(config)}
    hb = json.dumps(header).encode()
    hb += b" " * (-len(hb) % 8)
    tmp = path + ".partial"
    k = 0
    try:
        with open(tmp, "wb") as f:
            f.write(len(hb).to_bytes(8, "little"))
            f.write(hb)
            for t in tensors:
                for arr in _entry_arrays(t):
                    name, dt, shape = layout[k]
                    if arr.shape != tuple(shape) or (arr.dtype == np.int8) != (dt == "I8"):
                        raise N.SbError(4, f"cache entry '{name}': got {arr.dtype} {arr.shape}, expected {dt} {shape}")
                    f.write(arr.tobytes())
                    k += 1
                yield t
        if k != len(layout):
            raise N.SbError(4, f"cache: {k} of {len(layout)} entries written")
        os.replace(tmp, path)  # only a complete cache ever carries the final name
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)


def cached_llama_tensors(config: LlamaConfig, path: str) -> Iterator[tuple]:
    """quantized_llama_tensors' tuples read back from a packed-int8 cache."""
    st = SafeTensorsShards([path])
    meta = st.metadata()
    if meta.get("format") != CACHE_FORMAT:
        raise N.SbError(6, f"{path}: not a {CACHE_FORMAT} cache")
    if meta.get("config") != _config_meta(config):
        raise N.SbError(4, f"{path}: cache was written for another model configuration")
    yield ("f", N.SB_F_EMBED, 0, st.raw("embed"))
    for i in range(config.n_layers):
        for slot in (N.SB_W_QKV, N.SB_W_O, N.SB_W_GATE, N.SB_W_UP, N.SB_W_DOWN):
            nm = f"layers.{i}.{_SLOT_NAMES[slot]}"
            yield ("q", i, slot, st.raw(nm + ".q"), np.float32(st.raw(nm + ".scale")[0]))
        yield ("f", N.SB_F_NORM_IN, i, st.raw(f"layers.{i}.norm_in"))
        yield ("f", N.SB_F_NORM_POST, i, st.raw(f"layers.{i}.norm_post"))
    yield ("f", N.SB_F_NORM_FINAL, 0, st.raw("norm_final"))
    yield ("q", -1, 0, st.raw("lm_head.q"), np.float32(st.raw("lm_head.scale")[0]))


def load_into(model, config: LlamaConfig, paths: Sequence[str], cache: str = None, device: bool = True):
    """Load HF shards into a QuantLlamaB200 (every rank of a tensor-parallel
    model loads the same full tensors and keeps its slice).  Without a cache
    the conversion and quantization run on the device (device=True, the
    default) or on the host.  With `cache`: read the packed-int8 cache when it
    exists, else quantize the shards on the host and write it on the way."""
    if not cache and device:
        load_hf_device(model, config, paths)
        return
    if cache and os.path.exists(cache):
        tensors = cached_llama_tensors(config, cache)
    elif cache:
        tensors = write_quantized_cache(config, quantized_llama_tensors(config, paths), cache)
    else:
        tensors = quantized_llama_tensors(config, paths)
    for t in tensors:
        if t[0] == "q":
            model.load_qweight(t[1], t[2], t[3], t[4])
        else:
            model.load_f32(t[1], t[2], t[3])


def shard_paths(directory: str) -> list:
    """The .safetensors files of a checkpoint directory, sorted."""
    return sorted(os.path.join(directory, f) for f in os.listdir(directory) if f.endswith(".safetensors"))
