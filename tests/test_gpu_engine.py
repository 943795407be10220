"""GPU parity of the quantized Llama engine (sb_llama_*) against the oracle.

The oracle is the reference decode (llama.rs:744-763) with every projection
through matmul_i8_f32 (cpu.rs:1129-1160) and an f32 KV cache; its bf16-cache
variant rounds K/V to bf16 on append like the engine's default cache.

Bars: weight quantization/packing bit-exact; logits
and per-layer activations within 1e-3 max relative error (f32 accumulate)
against the matching oracle, 2e-2 for the bf16 cache against the f32-cache
reference; greedy token streams identical for >= 32 generated tokens.
"""
import numpy as np
import pytest

import oracle as O
from esolearn_b200 import LlamaConfig, QuantLlamaB200, RopeScaling, SamplingConfig, generate, Rng, argmax_last
from esolearn_b200 import _native as N
from tests.gpu_util import engine_from_oracle, greedy_agreement, orc_config, rel_err, small_config

pytestmark = pytest.mark.gpu
TOL_F32 = 1e-3
TOL_BF16 = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _init():
    N.check(N.lib().sb_init(0))


def _pair(c: LlamaConfig, seed=0, max_seq=512, **kw):
    om = O.OracleLlama(orc_config(c, max_seq), seed)
    return om, engine_from_oracle(om, c, max_seq=max_seq, **kw)


def test_tiny_device_init_equals_reference_weights():
    # BASELINE tiny config, seed 0: LlamaModel::new draw order + quantize_symmetric
    # generated on the GPU must equal the oracle's int8 tensors and scales bit for bit.
    c = LlamaConfig.tiny()
    om = O.OracleLlama(orc_config(c, 256), 0)
    e = QuantLlamaB200.new_random(c, 0, max_seq=256)
    for l in range(c.n_layers):
        for slot in range(5):
            qo, so = om.weight(l, slot)
            qg, sg = e.get_qweight(l, slot)
            assert sg == so, (l, slot)
            assert np.array_equal(qg, qo), (l, slot, int((qg != qo).sum()))
    qo, so = om.lm_head()
    qg, sg = e.get_qweight(-1, 0)
    assert sg == so and np.array_equal(qg, qo)


def test_tied_embeddings_device_init():
    c = small_config(layers=1, tie=True)
    om = O.OracleLlama(orc_config(c, 64), 3)
    e = QuantLlamaB200.new_random(c, 3, max_seq=64)
    qo, so = om.lm_head()
    qg, sg = e.get_qweight(-1, 0)
    assert sg == so and np.array_equal(qg, qo)


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_logits_and_layer_trace(kv):
    c = LlamaConfig.tiny()
    om, e = _pair(c, 0, 256, kv_dtype=kv)
    oc = om.new_cache(256, kv_bf16=(kv == "bf16"))
    rc = om.new_cache(256, kv_bf16=False)
    cache = e.new_kv_cache(256)
    e.set_trace(True)
    toks = O.prompt_ids(1, 24, c.vocab_size)
    for pos, t in enumerate(toks):
        ref, tr = om.forward_with_cache(oc, int(t), pos, trace=True)
        got = e.forward_with_cache(int(t), pos, cache)
        assert rel_err(got, ref) < TOL_F32, pos
        gtr = e.get_trace(1)[:, 0, :]
        for l in range(c.n_layers):
            assert rel_err(gtr[l], tr[l]) < TOL_F32, (pos, l)
        if kv == "bf16":
            pure = om.forward_with_cache(rc, int(t), pos)
            assert rel_err(got, pure) < TOL_BF16


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_greedy_stream_token_exact(kv):
    # BASELINE tiny config: seed 0, 16 uniform prompt ids, 128 greedy tokens.
    c = LlamaConfig.tiny()
    om, e = _pair(c, 0, 256, kv_dtype=kv)
    prompt = O.prompt_ids(0, 16, c.vocab_size)
    ref = om.generate_greedy(prompt, 128, kv_bf16=(kv == "bf16"))
    got = e.generate_greedy(prompt, 128)[0]
    assert got[:32].tolist() == ref[:32].tolist()
    assert got.tolist() == ref.tolist()


def test_generate_api_and_cache_reuse():
    c = small_config(layers=2)
    om, e = _pair(c, 5, 128, kv_dtype="f32")
    prompt = [3, 17, 99, 4]
    ref = om.generate_greedy(np.array(prompt, np.int32), 20).tolist()
    assert generate(e, prompt, SamplingConfig(0.0, 0, 1.0, 20), Rng(1)) == ref
    # same again: the engine resets its cache per generation
    assert generate(e, prompt, SamplingConfig(0.0, 0, 1.0, 20), Rng(2)) == ref
    # token-by-token CausalLM path == device-driven path
    cache = e.new_kv_cache(64)
    toks = []
    for pos, t in enumerate(prompt):
        lg = e.forward_with_cache(t, pos, cache)
    toks.append(argmax_last(lg))
    for i in range(1, 20):
        lg = e.forward_with_cache(toks[-1], len(prompt) + i - 1, cache)
        toks.append(argmax_last(lg))
    assert toks == ref


def test_sampling_matches_oracle_sampler():
    c = small_config(layers=1)
    om, e = _pair(c, 2, 64, kv_dtype="f32")
    cfg = SamplingConfig(0.7, 20, 0.9, 8)
    got = generate(e, [1, 2, 3], cfg, Rng(42))
    oc = om.new_cache(64)
    rng = O.Rng(42)
    out = []
    prompt = [1, 2, 3]
    for pos, t in enumerate(prompt):
        lg = om.forward_with_cache(oc, t, pos)
    out.append(O.sample_token(lg, cfg.temperature, cfg.top_k, cfg.top_p, rng))
    for i in range(1, cfg.max_tokens):
        lg = om.forward_with_cache(oc, out[-1], len(prompt) + i - 1)
        out.append(O.sample_token(lg, cfg.temperature, cfg.top_k, cfg.top_p, rng))
    assert got == out


@pytest.mark.parametrize("desc,cfg", [
    ("gqa4", small_config(h=512, heads=8, kv=2, layers=2)),
    ("hd128", small_config(h=1024, heads=8, kv=8, layers=2, ffn=2816)),
    ("hd128_gqa8", small_config(h=1024, heads=8, kv=1, layers=2, ffn=2816)),
    ("llama3_rope", small_config(h=512, heads=8, kv=4, layers=2, theta=500000.0, scaling=RopeScaling())),
    ("odd_ffn", small_config(h=256, heads=4, kv=4, layers=2, ffn=200)),
])
def test_shapes_greedy_and_logits(desc, cfg):
    om, e = _pair(cfg, 11, 160, kv_dtype="f32")
    prompt = O.prompt_ids(2, 8, cfg.vocab_size)
    ref = om.generate_greedy(prompt, 40)
    got = e.generate_greedy(prompt, 40)[0]
    assert got.tolist() == ref.tolist()
    oc = om.new_cache(160)
    cache = e.new_kv_cache(160)
    for pos, t in enumerate(prompt):
        assert rel_err(e.forward_with_cache(int(t), pos, cache), om.forward_with_cache(oc, int(t), pos)) < TOL_F32


@pytest.mark.parametrize("B", [2, 3, 4])
def test_batched_decode_equals_independent_sequences(B):
    # generate() for B prompts at once must reproduce generate() per sequence.
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 128), 9)
    e = engine_from_oracle(om, c, max_seq=128, max_batch=4, kv_dtype="bf16")
    prompts = np.stack([O.prompt_ids(100 + b, 12, c.vocab_size) for b in range(B)])
    got = e.generate_greedy(prompts, 33)
    for b in range(B):
        assert got[b].tolist() == om.generate_greedy(prompts[b], 33, kv_bf16=True).tolist(), b


@pytest.mark.parametrize("B", [5, 8, 32, 64])
def test_tensor_core_batched_decode_equals_independent_sequences(B):
    # Batches of 5-64 run every projection through the tcgen05 GEMM, chained:
    # the finish of o, gate/up and down also writes the next linear's planes
    # (10 launches per layer); with the attention in one context split (a
    # 128-position cache) the q|k|v epilogue runs inside the attention kernel
    # (9 per layer).  Greedy streams must equal the per-sequence oracle.
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 128), 9)
    e = engine_from_oracle(om, c, max_seq=128, max_batch=max(B, 32), kv_dtype="bf16")
    splits, tmap, _ = e.attn_plan(B)
    assert e.step_launches(B) == 5 + (9 if tmap and splits == 1 else 10) * c.n_layers
    assert e.step_launches(4) == 3 + 5 * c.n_layers
    prompts = np.stack([O.prompt_ids(200 + b, 12, c.vocab_size) for b in range(B)])
    got = e.generate_greedy(prompts, 33)
    for b in range(B):
        assert got[b].tolist() == om.generate_greedy(prompts[b], 33, kv_bf16=True).tolist(), b


@pytest.mark.parametrize("B,max_batch,n_prompt,kv", [(1, 16, 40, 2), (3, 16, 40, 2), (2, 8, 17, 2), (1, 1, 9, 2),
                                                     (3, 16, 40, 8), (2, 8, 17, 8)])
def test_batched_prefill_matches_token_by_token(B, max_batch, n_prompt, kv):
    # sb_llama_prefill runs each prompt as chunks of max_batch positions (one
    # batched step per chunk, rows sharing the sequence's pages; with one
    # query head per kv head the chunk's attention is the prefill kernel);
    # the greedy streams that follow must equal the oracle's token-by-token
    # generate(), except where the oracle's own top two logits lie within the
    # logits tolerance (a near-tie: the prompt's attention sums in another
    # order, which may resolve it either way), after which the row is compared
    # no further; the first generated token's logits are held to 1e-3.
    c = small_config(layers=2, heads=8, kv=kv)
    om = O.OracleLlama(orc_config(c, 128), 9)
    e = engine_from_oracle(om, c, max_seq=128, max_batch=max_batch, kv_dtype="bf16")
    prompts = np.stack([O.prompt_ids(300 + b, n_prompt, c.vocab_size) for b in range(B)])
    got = e.generate_greedy(prompts, 24, batched_prefill=True)
    for b in range(B):
        cache = om.new_cache(128, kv_bf16=True)
        lg = om.forward_tokens(cache, prompts[b], 0)
        ref, logs = [], []
        for j in range(24):
            ref.append(O.argmax(lg))
            logs.append(lg)
            lg = om.forward_with_cache(cache, ref[-1], n_prompt + j)
        greedy_agreement(got[b], ref, logs, TOL_F32)  # raises on a divergence that is no near-tie
    lg, _ = e.forward_batch([int(t) for t in got[:, 0]], [n_prompt] * B)
    for b in range(B):
        cache = om.new_cache(128, kv_bf16=True)
        om.forward_tokens(cache, prompts[b], 0)
        assert rel_err(lg[b], om.forward_with_cache(cache, int(got[b, 0]), n_prompt)) < TOL_F32, b


@pytest.mark.parametrize("desc,cfg,B", [
    ("small_gqa4", small_config(layers=2, heads=8, kv=2), 8),
    ("llama3_8b_shape_1layer", LlamaConfig(128256, 4096, 14336, 1, 32, 8, 8192, 1e-5, 500000.0, False,
                                           RopeScaling()), 8),
])
def test_tensor_core_batch_logits_match_oracle(desc, cfg, B):
    # Every row of a batched step (distinct tokens and histories) against the
    # oracle's forward_with_cache of that sequence alone, f32 cache.
    om = O.OracleLlama(orc_config(cfg, 64), 3)
    e = engine_from_oracle(om, cfg, max_seq=64, max_batch=B, kv_dtype="f32")
    seqs = np.stack([O.prompt_ids(50 + b, 4, cfg.vocab_size) for b in range(B)])
    caches = [om.new_cache(64) for _ in range(B)]
    e.new_kv_cache(64)
    for p in range(seqs.shape[1]):
        lg, am = e.forward_batch(seqs[:, p].tolist(), [p] * B)
        for b in range(B):
            ref = om.forward_with_cache(caches[b], int(seqs[b, p]), p)
            assert rel_err(lg[b], ref) < TOL_F32, (p, b)
            assert int(am[b]) == argmax_last(lg[b]), (p, b)


def test_batch1_runs_the_persistent_step_and_agrees_with_per_op_path():
    # Batch 1 is one persistent-kernel launch per step; batches of 2-4 run the
    # per-operation kernels.  The same sequence decoded in both must give the
    # same tokens and logits within the f32 bar (attention splits differ).
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 128), 5)
    e = engine_from_oracle(om, c, max_seq=128, max_batch=2, kv_dtype="bf16")
    assert e.step_launches(1) == 1
    assert e.step_launches(2) == 3 + 5 * c.n_layers
    toks = O.prompt_ids(7, 20, c.vocab_size)
    cache = e.new_kv_cache(128)
    one = [e.forward_with_cache(int(t), p, cache) for p, t in enumerate(toks)]
    e.new_kv_cache(128)
    for p, t in enumerate(toks):
        lg, _ = e.forward_batch([int(t), int(t)], [p, p])
        assert rel_err(lg[0], one[p]) < TOL_F32, p
        assert np.array_equal(lg[0], lg[1]), p


def test_seven_b_shape_two_layers():
    # Llama-2-7B layer shapes (h 4096, ffn 11008, 32 heads, vocab 32000), 2 layers.
    c = LlamaConfig(32000, 4096, 11008, 2, 32, 32, 4096, 1e-5, 10000.0, False, None)
    om, e = _pair(c, 0, 96, kv_dtype="bf16")
    prompt = O.prompt_ids(0, 16, c.vocab_size)
    ref = om.generate_greedy(prompt, 32, kv_bf16=True)
    got = e.generate_greedy(prompt, 32)[0]
    assert got.tolist() == ref.tolist()


def test_capacity_and_argument_errors():
    c = small_config(layers=1)
    with pytest.raises(N.SbError):
        QuantLlamaB200.new_random(c, seed=0, max_seq=32, max_batch=65)  # above the tensor-core path's 64 rows
    with pytest.raises(N.SbError):  # batches above 4 need 32-aligned hidden / ffn sizes
        QuantLlamaB200.new_random(small_config(h=256, heads=4, kv=4, layers=1, ffn=200), seed=0, max_seq=32,
                                  max_batch=8)
    om, e = _pair(c, 1, 32, kv_dtype="f32")
    with pytest.raises(N.SbError):
        e.generate_greedy(np.zeros(20, np.int32), 20)  # 20 + 20 - 1 > 32 positions
    with pytest.raises(N.SbError):
        e.forward_batch([c.vocab_size], [0])  # token outside the vocabulary
    with pytest.raises(N.SbError):
        e.forward_batch([1], [32])  # position beyond the cache
    # the engine still works afterwards
    assert e.generate_greedy(np.array([1, 2], np.int32), 4).shape == (1, 4)


@pytest.mark.parametrize("max_batch,n", [(8, 37), (64, 150), (1, 12)])
def test_full_sequence_forward_logits(max_batch, n):
    # CausalLM::forward (generate.rs:9, llama.rs:683-700): logits [seq, V] of
    # every position in one call, run as batched prefill chunks (tensor-core
    # linears at 5+ rows; the persistent step at max_batch 1), against the
    # oracle's per-position logits (bf16 cache on both sides).
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 256), 13)
    e = engine_from_oracle(om, c, max_seq=256, max_batch=max_batch, kv_dtype="bf16")
    toks = O.prompt_ids(77, n, c.vocab_size)
    got = e.forward(toks)
    ref = om.forward_tokens(om.new_cache(256, kv_bf16=True), toks, 0, all_logits=True)
    assert got.shape == (n, c.vocab_size)
    for p in range(n):
        assert rel_err(got[p], ref[p]) < TOL_F32, p
    # the engine decodes normally afterwards
    prompt = O.prompt_ids(78, 6, c.vocab_size)
    assert e.generate_greedy(prompt, 8)[0].tolist() == om.generate_greedy(prompt, 8, kv_bf16=True).tolist()
