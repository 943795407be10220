"""Property-based fuzzing of the host side, in the spirit of the reference's
libfuzzer targets (crates/scry-llm/fuzz/fuzz_targets/: no panic or NaN on
arbitrary small inputs).  CPU only.

* quantize_symmetric (quantize.rs:16-32): the library's host quantizer equals
  the oracle bit for bit on arbitrary f32 arrays, special values included,
  and both follow Rust's float rules where the reference meets non-finite
  weights: f32::max ignores NaN in the absmax fold, f32::clamp keeps NaN, and
  `as i8` turns NaN into 0.
* the safetensors parser: arbitrary bytes and arbitrary headers either parse
  into tensors whose byte ranges fit their shapes, or raise SbError.
* tensor-parallel sharding (host C): for any divisible GQA shape and 1-8
  ranks the shards partition every weight exactly; uneven splits are
  SB_ERR_SHAPE.
"""
import json

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import oracle as O
from esolearn_b200 import _native as N
from esolearn_b200.llama import quantize_symmetric
from esolearn_b200.safetensors_io import SafeTensorsShards

F32 = st.floats(width=32, allow_nan=True, allow_infinity=True, allow_subnormal=True)


def _same(a, b):
    return np.asarray(a, np.float32).tobytes() == np.asarray(b, np.float32).tobytes()


@settings(max_examples=400, deadline=None)
@given(st.lists(F32, min_size=0, max_size=64))
def test_host_quantizer_equals_oracle_on_any_floats(vals):
    w = np.array(vals, np.float32)
    q1, s1 = quantize_symmetric(w)
    q2, s2 = O.quantize_symmetric(w)
    assert np.array_equal(np.ravel(q1), np.ravel(q2))
    assert _same(s1, s2)


@pytest.mark.parametrize("vals,q,scale", [
    # a NaN weight is skipped by the absmax fold and quantizes to 0
    ([float("nan"), 1.0, -3.0], [0, 42, -127], np.float32(3.0) / np.float32(127.0)),
    # one infinite weight: scale inf, inv 0, every product 0 or NaN -> all 0
    ([float("inf"), 1.0, -2.0], [0, 0, 0], np.float32("inf")),
    ([float("-inf"), float("nan")], [0, 0], np.float32("inf")),
    # all NaN: the fold stays 0 -> the zero-weights branch (quantize.rs:19-21)
    ([float("nan"), float("nan")], [0, 0], np.float32(0.0)),
    # subnormal absmax: scale 0 after rounding but absmax != 0, inv = inf
    ([1e-45, -1e-45], [127, -127], np.float32(0.0)),
])
def test_quantizer_known_answers_for_special_values(vals, q, scale):
    w = np.array(vals, np.float32)
    for qq, ss in (quantize_symmetric(w), O.quantize_symmetric(w)):
        assert np.ravel(qq).tolist() == q
        assert _same(ss, scale)


@settings(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.binary(max_size=200))
def test_parser_on_arbitrary_bytes(tmp_path, data):
    path = tmp_path / "x.safetensors"
    path.write_bytes(data)
    try:
        st_ = SafeTensorsShards([str(path)])
    except N.SbError:
        return
    for name in st_.names():
        try:
            st_.raw(name)
        except N.SbError:
            pass


_ENTRY = st.fixed_dictionaries({
    "dtype": st.sampled_from(["F32", "BF16", "F16", "I8", "U8", "F64", "XYZ"]),
    "shape": st.lists(st.integers(-2, 6), max_size=3),
    "data_offsets": st.lists(st.integers(-4, 80), min_size=2, max_size=2),
})


@settings(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.dictionaries(st.text(min_size=1, max_size=4), _ENTRY, max_size=4), st.integers(0, 64))
def test_parser_on_arbitrary_headers(tmp_path, header, data_len):
    h = json.dumps(header).encode()
    path = tmp_path / "h.safetensors"
    path.write_bytes(len(h).to_bytes(8, "little") + h + bytes(data_len))
    try:
        st_ = SafeTensorsShards([str(path)])
    except N.SbError:
        return
    # accepted: every tensor of a convertible dtype reads back with its shape
    for name in st_.names():
        info = header[name]
        if info["dtype"] in ("F32", "BF16", "F16"):
            assert st_.f32(name).shape == tuple(info["shape"])
        elif info["dtype"] == "I8":
            assert st_.raw(name).shape == tuple(info["shape"])


@st.composite
def _tp_case(draw):
    T = draw(st.sampled_from([1, 2, 4, 8]))
    kv = T * draw(st.integers(1, 2))
    heads = kv * draw(st.sampled_from([1, 2, 4]))
    hd = draw(st.sampled_from([2, 4, 8]))
    ffn = T * draw(st.integers(1, 6))
    vocab = T * draw(st.integers(1, 6))
    return T, heads, kv, hd, ffn, vocab


@settings(max_examples=120, deadline=None)
@given(_tp_case(), st.integers(0, 2**31 - 1))
def test_tp_shards_partition_every_weight_of_any_config(case, seed):
    # The host sharder (sb_tp_shard_qweight): column slices of q|k|v (by
    # heads, q, k and v separately), gate and up (by ffn columns); row slices
    # of o, down and the [V, h] lm_head.  Concatenating the T shards the way
    # the algebra says gives back the full tensor, for any divisible shape.
    from esolearn_b200 import LlamaConfig, tp_shard_qweight, tp_shard_shape

    T, heads, kv, hd, ffn, vocab = case
    h = heads * hd
    c = LlamaConfig(vocab, h, ffn, 1, heads, kv, 16, 1e-5, 10000.0, False, None)
    Qf, KVf = heads * hd, kv * hd
    rng = np.random.default_rng(seed)
    shapes = {N.SB_W_QKV: (h, Qf + 2 * KVf), N.SB_W_O: (Qf, h), N.SB_W_GATE: (h, ffn), N.SB_W_UP: (h, ffn),
              N.SB_W_DOWN: (ffn, h), N.SB_W_LM_HEAD: (vocab, h)}
    for slot, shape in shapes.items():
        w = rng.integers(-127, 128, shape, dtype=np.int8)
        parts = [tp_shard_qweight(c, slot, r, T, w) for r in range(T)]
        assert all(p.shape == tp_shard_shape(c, slot, r, T) for r, p in enumerate(parts))
        if slot == N.SB_W_QKV:
            q, k = Qf // T, KVf // T
            re = np.concatenate([np.concatenate([p[:, :q] for p in parts], 1),
                                 np.concatenate([p[:, q:q + k] for p in parts], 1),
                                 np.concatenate([p[:, q + k:] for p in parts], 1)], 1)
        elif slot in (N.SB_W_GATE, N.SB_W_UP):
            re = np.concatenate(parts, 1)
        else:
            re = np.concatenate(parts, 0)
        assert np.array_equal(re, w), slot


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 8), st.integers(1, 12), st.integers(1, 40))
def test_tp_uneven_splits_are_shape_errors(T, heads, ffn):
    from esolearn_b200 import LlamaConfig, tp_shard_shape

    c = LlamaConfig(8 * T, heads * 4, ffn, 1, heads, heads, 16, 1e-5, 10000.0, False, None)
    ok = heads % T == 0 and ffn % T == 0
    try:
        tp_shard_shape(c, N.SB_W_GATE, 0, T)
        tp_shard_shape(c, N.SB_W_O, 0, T)
        assert ok
    except N.SbError as e:
        assert not ok and e.code == 4
