"""Model-load time from a BF16 safetensors checkpoint (LlamaModel::from_safetensors,
llama.rs:768-958) into the int8 engine, next to the reference's published cold
start of 17.54 s for Llama-3.2-1B (bench_results_2026-02-21.md:31).

No checkpoint is on the GPU host, so a synthetic one of the requested shape is
written first (HF tensor names and [out, in] layouts, BF16, shards of at most
2 GB, seeded values); it then sits in the page cache, so the timed load reads
warm files.  Timed, end to end on the host clock: creating the engine
(allocations, RoPE tables, KV pages), opening and memory-mapping the shards,
the upload of every tensor's bytes and their conversion, transposition, q|k|v
fusion, quantize_symmetric and packing on the GPU (sb_llama_load_hf), then one
forward pass (the first token).  --host times the host-quantizing path instead.

    python -m esolearn_b200.load_bench --shape llama_1b [--host] [--dir /tmp/ckpt]
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import tempfile
import time

import numpy as np

from . import _native as N
from .llama import LlamaConfig, QuantLlamaB200

SHARD_BYTES = 2 << 30


def hf_tensors(cfg: LlamaConfig):
    """(name, [out, in] shape) of every checkpoint tensor, in file order."""
    h, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    hd = cfg.head_dim()
    qd, kd = cfg.n_heads * hd, cfg.n_kv_heads * hd
    out = [("model.embed_tokens.weight", (V, h))]
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}"
        out += [(f"{p}.self_attn.q_proj.weight", (qd, h)), (f"{p}.self_attn.k_proj.weight", (kd, h)),
                (f"{p}.self_attn.v_proj.weight", (kd, h)), (f"{p}.self_attn.o_proj.weight", (h, qd)),
                (f"{p}.mlp.gate_proj.weight", (F, h)), (f"{p}.mlp.up_proj.weight", (F, h)),
                (f"{p}.mlp.down_proj.weight", (h, F)), (f"{p}.input_layernorm.weight", (h,)),
                (f"{p}.post_attention_layernorm.weight", (h,))]
    out.append(("model.norm.weight", (h,)))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (V, h)))
    return out


def write_checkpoint(cfg: LlamaConfig, directory: str, seed: int = 0) -> list:
    """Synthetic BF16 checkpoint: N(0, 0.02)-like values (a seeded block of
    bf16 bit patterns repeated through every tensor; norms are 1.0)."""
    rng = np.random.default_rng(seed)
    block = rng.standard_normal(1 << 20, dtype=np.float32) * np.float32(0.02)
    bits = (block.view(np.uint32) >> 16).astype(np.uint16)  # truncated to bf16
    one = np.uint16(0x3F80)
    tensors = hf_tensors(cfg)
    shards, cur, size = [], [], 0
    for name, shape in tensors:
        nb = int(np.prod(shape)) * 2
        if cur and size + nb > SHARD_BYTES:
            shards.append(cur)
            cur, size = [], 0
        cur.append((name, shape))
        size += nb
    shards.append(cur)
    paths = []
    for k, group in enumerate(shards):
        header, off = {}, 0
        for name, shape in group:
            nb = int(np.prod(shape)) * 2
            header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + nb]}
            off += nb
        hb = json.dumps(header).encode()
        hb += b" " * (-len(hb) % 8)
        path = os.path.join(directory, f"model-{k + 1:05d}-of-{len(shards):05d}.safetensors")
        with open(path, "wb") as f:
            f.write(len(hb).to_bytes(8, "little"))
            f.write(hb)
            for name, shape in group:
                n = int(np.prod(shape))
                if len(shape) == 1:
                    f.write(np.full(n, one, np.uint16).tobytes())
                    continue
                for s in range(0, n, bits.size):
                    f.write(bits[: min(bits.size, n - s)].tobytes())
        paths.append(path)
    return paths


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--shape", default="llama_1b", help="a LlamaConfig preset (llama_1b, llama2_7b_shape, ...)")
    ap.add_argument("--dir", default=None, help="where to write the synthetic checkpoint (default: a temp dir)")
    ap.add_argument("--host", action="store_true", help="host-side quantization instead of sb_llama_load_hf")
    ap.add_argument("--max-seq", type=int, default=2048)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)
    cfg = getattr(LlamaConfig, args.shape)()
    N.check(N.lib().sb_init(args.device))
    own = args.dir is None
    d = tempfile.mkdtemp(prefix="scry_ckpt_") if own else args.dir
    try:
        t0 = time.perf_counter()
        paths = write_checkpoint(cfg, d)
        t_write = time.perf_counter() - t0
        nbytes = sum(os.path.getsize(p) for p in paths)
        t0 = time.perf_counter()
        m = QuantLlamaB200.from_safetensors(cfg, paths, max_seq=args.max_seq, device_quantize=not args.host)
        t_load = time.perf_counter() - t0
        t1 = time.perf_counter()
        m.forward_with_cache(1, 0, m.new_kv_cache(args.max_seq))
        t_first = time.perf_counter() - t1
        m.close()
        print(json.dumps({"shape": args.shape, "params": sum(int(np.prod(s)) for _, s in hf_tensors(cfg)),
                          "checkpoint_bytes": nbytes, "shards": len(paths),
                          "quantize": "host" if args.host else "device (sb_llama_load_hf)",
                          "write_s": t_write, "load_s": t_load, "first_token_s": t_first,
                          "cold_to_first_token_s": t_load + t_first, "page_cache": "warm (just written)"}))
    finally:
        if own:
            shutil.rmtree(d, ignore_errors=True)


if __name__ == "__main__":
    main()
