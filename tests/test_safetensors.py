"""Weight loading from HF safetensors shards (LlamaModel::from_safetensors,
llama.rs:768-958): dtype conversion, [out,in] -> [in,out] transposes, the
q|k|v fusion and per-tensor quantization must give exactly the int8 tensors
and scales of the reference wiring."""
import numpy as np
import pytest

import oracle as O
from esolearn_b200 import LlamaConfig
from esolearn_b200 import _native as N
from esolearn_b200.safetensors_io import (SafeTensorsShards, cached_llama_tensors, quantized_llama_tensors,
                                         write_quantized_cache, write_safetensors)


def _cfg(tie=False):
    return LlamaConfig(96, 64, 80, 2, 4, 2, 64, 1e-5, 10000.0, tie, None)


def _hf_weights(c: LlamaConfig, seed: int):
    rng = np.random.default_rng(seed)
    h, F, V = c.hidden_size, c.intermediate_size, c.vocab_size
    hd = c.head_dim()
    qd, kd = c.n_heads * hd, c.n_kv_heads * hd
    w = {"model.embed_tokens.weight": rng.standard_normal((V, h)) * 0.02, "model.norm.weight": 1 + 0.1 * rng.standard_normal(h)}
    for i in range(c.n_layers):
        p = f"model.layers.{i}"
        w[f"{p}.self_attn.q_proj.weight"] = rng.standard_normal((qd, h)) * 0.02
        w[f"{p}.self_attn.k_proj.weight"] = rng.standard_normal((kd, h)) * 0.02
        w[f"{p}.self_attn.v_proj.weight"] = rng.standard_normal((kd, h)) * 0.02
        w[f"{p}.self_attn.o_proj.weight"] = rng.standard_normal((h, qd)) * 0.02
        w[f"{p}.mlp.gate_proj.weight"] = rng.standard_normal((F, h)) * 0.02
        w[f"{p}.mlp.up_proj.weight"] = rng.standard_normal((F, h)) * 0.02
        w[f"{p}.mlp.down_proj.weight"] = rng.standard_normal((h, F)) * 0.02
        w[f"{p}.input_layernorm.weight"] = 1 + 0.1 * rng.standard_normal(h)
        w[f"{p}.post_attention_layernorm.weight"] = 1 + 0.1 * rng.standard_normal(h)
    if not c.tie_word_embeddings:
        w["lm_head.weight"] = rng.standard_normal((V, h)) * 0.02
    return {k: v.astype(np.float32) for k, v in w.items()}


def _write_shards(tmp_path, w):
    names = sorted(w)
    half = len(names) // 2
    proj = [n for n in names if "proj" in n]
    paths = []
    for k, part in enumerate((names[:half], names[half:])):
        path = str(tmp_path / f"model-{k:05d}-of-00002.safetensors")
        write_safetensors(path, {n: w[n] for n in part}, bf16=[n for n in part if n in proj])
        paths.append(path)
    return paths, set(proj)


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("tie", [False, True])
def test_loader_matches_reference_wiring(tmp_path, tie):
    c = _cfg(tie)
    w = _hf_weights(c, 3)
    paths, bf = _write_shards(tmp_path, w)
    src = {n: (_bf16(a) if n in bf else a) for n, a in w.items()}  # what the shards hold
    got = list(quantized_llama_tensors(c, paths))
    q_items = {(t[1], t[2]): (t[3], t[4]) for t in got if t[0] == "q"}
    f_items = {(t[1], t[2]): t[3] for t in got if t[0] == "f"}
    h = c.hidden_size
    for i in range(c.n_layers):
        p = f"model.layers.{i}"
        qkv = np.concatenate([src[f"{p}.self_attn.{x}_proj.weight"].T for x in "qkv"], axis=1)
        ref = {N.SB_W_QKV: qkv, N.SB_W_O: src[f"{p}.self_attn.o_proj.weight"].T,
               N.SB_W_GATE: src[f"{p}.mlp.gate_proj.weight"].T, N.SB_W_UP: src[f"{p}.mlp.up_proj.weight"].T,
               N.SB_W_DOWN: src[f"{p}.mlp.down_proj.weight"].T}
        for slot, wf in ref.items():
            qo, so = O.quantize_symmetric(np.ascontiguousarray(wf))  # quantize.rs:16-32 restated
            qg, sg = q_items[(i, slot)]
            assert qg.shape == wf.shape and sg == so and np.array_equal(qg.ravel(), qo), (i, slot)
        assert np.array_equal(f_items[(N.SB_F_NORM_IN, i)], src[f"{p}.input_layernorm.weight"])
        assert np.array_equal(f_items[(N.SB_F_NORM_POST, i)], src[f"{p}.post_attention_layernorm.weight"])
    head = src["model.embed_tokens.weight" if tie else "lm_head.weight"]
    qo, so = O.quantize_symmetric(head)
    qg, sg = q_items[(-1, 0)]
    assert qg.shape == (c.vocab_size, h) and sg == so and np.array_equal(qg.ravel(), qo)
    assert np.array_equal(f_items[(N.SB_F_EMBED, 0)], src["model.embed_tokens.weight"])


def test_dtype_conversion_is_exact(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((5, 7)).astype(np.float32)
    path = str(tmp_path / "t.safetensors")
    write_safetensors(path, {"x": a, "y": a}, bf16=["y"])
    st = SafeTensorsShards([path])
    assert np.array_equal(st.f32("x"), a)
    assert np.array_equal(st.f32("y"), _bf16(a))
    with pytest.raises(N.SbError):
        st.f32("missing")


@pytest.mark.parametrize("tie", [False, True])
def test_packed_int8_cache_round_trip(tmp_path, tie):
    # Written while the shards are quantized (every tuple passed on
    # unchanged), read back as the same tuples: int8 tensors, scales and f32
    # tensors bit for bit, in the same order.
    c = _cfg(tie)
    paths, _ = _write_shards(tmp_path, _hf_weights(c, 5))
    cache = str(tmp_path / "model.int8.safetensors")
    passed = list(write_quantized_cache(c, quantized_llama_tensors(c, paths), cache))
    direct = list(quantized_llama_tensors(c, paths))
    back = list(cached_llama_tensors(c, cache))
    assert len(passed) == len(direct) == len(back)
    for a, b, r in zip(direct, passed, back):
        assert a[:3] == b[:3] == r[:3]
        assert np.array_equal(a[3], b[3]) and np.array_equal(a[3], r[3])
        assert r[3].dtype == (np.int8 if a[0] == "q" else np.float32)
        if a[0] == "q":
            assert np.float32(a[4]) == np.float32(r[4])


def test_packed_int8_cache_rejects_other_configs_and_partial_writes(tmp_path):
    c = _cfg()
    paths, _ = _write_shards(tmp_path, _hf_weights(c, 6))
    cache = str(tmp_path / "model.int8.safetensors")
    list(write_quantized_cache(c, quantized_llama_tensors(c, paths), cache))
    other = LlamaConfig(96, 64, 80, 2, 4, 2, 64, 1e-5, 500000.0, False, None)
    with pytest.raises(N.SbError) as ei:
        list(cached_llama_tensors(other, cache))
    assert ei.value.code == 4
    # a load that stops half way leaves no file under the cache's name
    half = str(tmp_path / "half.int8.safetensors")
    gen = write_quantized_cache(c, quantized_llama_tensors(c, paths), half)
    for _ in range(3):
        next(gen)
    gen.close()
    import os

    assert not os.path.exists(half) and not os.path.exists(half + ".partial")


def _corrupt(tmp_path, name, mutate):
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    path = str(tmp_path / name)
    write_safetensors(path, {"w": a})
    raw = bytearray(open(path, "rb").read())
    raw = mutate(raw)
    open(path, "wb").write(bytes(raw))
    return path


def _header(raw):
    n = int.from_bytes(raw[:8], "little")
    return n, raw[8:8 + n]


def _with_header(raw, text):
    n, _ = _header(raw)
    h = text.encode()
    h += b" " * (-len(h) % 8)
    return bytearray(len(h).to_bytes(8, "little")) + h + raw[8 + n:]


@pytest.mark.parametrize("case", ["short", "header_past_end", "not_json", "not_a_map", "truncated_data",
                                  "shape_mismatch", "bad_entry"])
def test_malformed_weight_files_raise_clean_errors(tmp_path, case):
    # Host-side fault injection for the weight path: every malformed file is
    # an SbError at open (the reference loader's ScryLlmError), never a crash
    # or a silently misread tensor.
    def mutate(raw):
        n, h = _header(raw)
        if case == "short":
            return raw[:5]
        if case == "header_past_end":
            return bytearray((n + 10_000).to_bytes(8, "little")) + raw[8:]
        if case == "not_json":
            return _with_header(raw, "{not json")
        if case == "not_a_map":
            return _with_header(raw, "[1, 2, 3]")
        if case == "truncated_data":
            return raw[:-8]
        if case == "shape_mismatch":
            return _with_header(raw, h.decode().replace("[3, 4]", "[4, 4]"))
        if case == "bad_entry":
            return _with_header(raw, '{"w": {"dtype": "F32", "shape": [3, 4]}}')
        raise AssertionError(case)

    path = _corrupt(tmp_path, case + ".safetensors", mutate)
    with pytest.raises(N.SbError):
        SafeTensorsShards([path])


@pytest.mark.gpu
def test_allocation_failure_is_an_error_and_the_device_stays_usable():
    # Host-side fault injection for device memory: a KV cache far beyond the
    # GPU's 180 GB (2^27 positions: 275 GB) makes sb_llama_create fail with
    # SB_ERR_OOM, releasing what it had allocated; the device then builds and
    # runs a small model normally.
    from esolearn_b200 import QuantLlamaB200

    N.check(N.lib().sb_init(0))
    c = LlamaConfig(512, 512, 1376, 2, 8, 8, 1 << 27, 1e-5, 10000.0, False, None)
    with pytest.raises(N.SbError) as ei:
        QuantLlamaB200(c, max_seq=1 << 27)
    assert ei.value.code == 5  # SB_ERR_OOM
    small = LlamaConfig(512, 512, 1376, 2, 8, 8, 64, 1e-5, 10000.0, False, None)
    e = QuantLlamaB200.new_random(small, 1, max_seq=64)
    om = O.OracleLlama(O.make_config(512, 512, 1376, 2, 8, 8, 64, 1e-5, 10000.0, False), 1)
    cache, oc = e.new_kv_cache(64), om.new_cache(64, kv_bf16=True)
    for pos, t in enumerate(O.prompt_ids(2, 6, small.vocab_size)):
        lg = e.forward_with_cache(int(t), pos, cache)
        lo = om.forward_with_cache(oc, int(t), pos)
        assert np.abs(lg - lo).max() / np.abs(lo).max() < 1e-3


@pytest.mark.gpu
def test_engine_from_packed_cache_equals_engine_from_shards(tmp_path):
    from esolearn_b200 import QuantLlamaB200

    N.check(N.lib().sb_init(0))
    c = LlamaConfig(512, 512, 1376, 2, 8, 2, 64, 1e-5, 10000.0, False, None)
    paths, _ = _write_shards(tmp_path, _hf_weights(c, 12))
    cache = str(tmp_path / "model.int8.safetensors")
    a = QuantLlamaB200.from_safetensors(c, paths, max_seq=64)
    b = QuantLlamaB200.from_safetensors(c, paths, cache=cache, max_seq=64)  # writes the cache
    d = QuantLlamaB200.from_safetensors(c, [], cache=cache, max_seq=64)     # reads it, no shards
    prompt = O.prompt_ids(6, 8, c.vocab_size)
    ref = a.generate_greedy(prompt, 16).tolist()
    assert b.generate_greedy(prompt, 16).tolist() == ref
    assert d.generate_greedy(prompt, 16).tolist() == ref


@pytest.mark.gpu
def test_engine_from_safetensors_equals_engine_from_tensors(tmp_path):
    # The same weights through from_safetensors and through load_qweight of
    # the directly quantized tensors: identical logits and greedy streams.
    from esolearn_b200 import QuantLlamaB200

    N.check(N.lib().sb_init(0))
    c = LlamaConfig(512, 512, 1376, 2, 8, 2, 64, 1e-5, 10000.0, False, None)
    w = _hf_weights(c, 11)
    paths, _ = _write_shards(tmp_path, w)
    a = QuantLlamaB200.from_safetensors(c, paths, max_seq=64)
    b = QuantLlamaB200(c, max_seq=64)
    for t in quantized_llama_tensors(c, paths):
        (b.load_qweight if t[0] == "q" else b.load_f32)(*t[1:])
    prompt = O.prompt_ids(4, 8, c.vocab_size)
    assert a.generate_greedy(prompt, 16).tolist() == b.generate_greedy(prompt, 16).tolist()
    ca, cb = a.new_kv_cache(64), b.new_kv_cache(64)
    for pos, t in enumerate(prompt):
        assert np.array_equal(a.forward_with_cache(int(t), pos, ca), b.forward_with_cache(int(t), pos, cb))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("tie", [False, True])
def test_device_load_equals_host_quantized_tensors(tmp_path, dtype, tie):
    # sb_llama_load_hf: the checkpoint bytes converted, transposed, fused and
    # quantized on the GPU must give the host path's int8 tensors and scales
    # bit for bit (llama.rs:768-958 wiring + quantize.rs:16-32), for BF16, F16
    # and F32 shards, tied and untied lm_heads.
    from esolearn_b200 import QuantLlamaB200
    from esolearn_b200.safetensors_io import load_hf_device

    N.check(N.lib().sb_init(0))
    c = LlamaConfig(512, 256, 192, 2, 4, 2, 64, 1e-5, 10000.0, tie, None)
    w = _hf_weights(c, 21 + tie)
    if dtype == "f16":
        w = {k: v.astype(np.float16).astype(np.float32) for k, v in w.items()}
    path = str(tmp_path / "model.safetensors")
    if dtype == "f16":  # write F16 tensors directly
        import json
        header, blobs, off = {}, [], 0
        for name, a in w.items():
            raw = a.astype(np.float16).tobytes()
            header[name] = {"dtype": "F16", "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
            blobs.append(raw)
            off += len(raw)
        hb = json.dumps(header).encode()
        hb += b" " * (-len(hb) % 8)
        with open(path, "wb") as f:
            f.write(len(hb).to_bytes(8, "little"))
            f.write(hb)
            for raw in blobs:
                f.write(raw)
    else:
        write_safetensors(path, w, bf16=list(w) if dtype == "bf16" else [])
    e = QuantLlamaB200(c, max_seq=64)
    load_hf_device(e, c, [path])
    for t in quantized_llama_tensors(c, [path]):
        if t[0] != "q":
            continue
        q, s = e.get_qweight(t[1], t[2])
        assert s == t[4], (t[1], t[2])
        assert np.array_equal(q, t[3]), (t[1], t[2], int((q != t[3]).sum()))
    ref = QuantLlamaB200(c, max_seq=64)
    for t in quantized_llama_tensors(c, [path]):
        (ref.load_qweight if t[0] == "q" else ref.load_f32)(*t[1:])
    ce, cr = e.new_kv_cache(64), ref.new_kv_cache(64)
    for pos, tok in enumerate(O.prompt_ids(8, 6, c.vocab_size)):
        assert np.array_equal(e.forward_with_cache(int(tok), pos, ce), ref.forward_with_cache(int(tok), pos, cr))
