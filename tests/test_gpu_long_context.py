"""GPU parity at the contexts, batch sizes and head layouts the benchmarks run.

The bench workloads decode with 2048-position contexts at batch 32
(Llama-3-8B shape, 4 query heads per KV head), 1024 at batch 64 (Llama-3-70B
shape, 8 per KV head) and 512-768 at batch 1 (Llama-2-7B shape).  There the
tensor-map attention splits every (sequence, kv head) context over several
CTAs and combines the partial softmax records, and the persistent batch-1 step
spreads many 64-position chunks per layer over the SMs.  These tests run those
paths on models that are small where the oracle pays (hidden size, ffn,
vocabulary, depth) and full-size where the kernels' work split depends on it
(head_dim 128, GQA ratio, context, batch, the 7B and 70B head layouts), and
hold them to the oracle (the reference decode, llama.rs:744-763, with every
projection through matmul_i8_f32) with a bf16-rounded cache like the engine's:

* greedy streams identical for 32 generated tokens on every row -- except
  at a step where the oracle's top two logits lie within the logits tolerance
  of each other (a near-tie: 64 rows x 32 tokens of a random-init model meet
  one now and then), where either token is accepted and the row is compared
  up to that step only (gpu_util.greedy_agreement);
* logits of every row within 1e-3 max relative error, each row at its own
  context length (rows rewound to different steps of their stream);
* the attention plan the engine reports shows that the multi-split path ran.

The oracle processes each long prompt with orc_forward_tokens (bit-identical
to the token-by-token loop, checked in tests/test_oracle.py), and rows share a
common prompt prefix whose cache is computed once and cloned per row; every
row's prompt ends in its own tail, so rows still differ in their KV contents.
"""
import numpy as np
import pytest

import oracle as O
from esolearn_b200 import LlamaConfig
from esolearn_b200 import _native as N
from tests.gpu_util import engine_from_oracle, greedy_agreement, orc_config, rel_err, small_config

pytestmark = pytest.mark.gpu
TOL = 1e-3  # f32 accumulate on both sides, same bf16 cache rounding


@pytest.fixture(scope="module", autouse=True)
def _init():
    N.check(N.lib().sb_init(0))


def _cdiv(a, b):
    return -(-a // b)


def _streams(om, prefix, tails, n_gen, max_seq):
    """Oracle greedy streams and per-step logits of prompts prefix + tails[b]."""
    pc = om.new_cache(max_seq, kv_bf16=True)
    if len(prefix):
        om.forward_tokens(pc, prefix, 0)
    S = len(prefix) + tails.shape[1]
    toks, logs = [], []
    for tail in tails:
        c = pc.clone()
        lg = om.forward_tokens(c, tail, len(prefix))
        t, lgs = [O.argmax(lg)], [lg]
        for j in range(1, n_gen):
            lg = om.forward_with_cache(c, t[-1], S + j - 1)
            t.append(O.argmax(lg))
            lgs.append(lg)
        toks.append(t)
        logs.append(lgs)
    return np.array(toks, np.int32), logs


def _rewound_logits(e, prompts, toks, steps):
    """Engine logits of step steps[b] of row b's stream: the token that step
    consumed at its position, all rows in one batched step (rows at different
    contexts).  Step 0 consumed the last prompt token."""
    S = prompts.shape[1]
    tok = [int(prompts[b, -1]) if j == 0 else int(toks[b, j - 1]) for b, j in enumerate(steps)]
    pos = [S + j - 1 for j in steps]
    lg, am = e.forward_batch(tok, pos)
    return lg, am


CASES = [
    # desc, config, batch, prefix, tail
    ("rep4_hd128_b8_ctx2080", small_config(h=512, heads=4, kv=1, layers=1, ffn=512, vocab=1024, theta=500000.0),
     8, 1984, 64),
    ("rep8_hd128_b32_ctx672", small_config(h=1024, heads=8, kv=1, layers=1, ffn=512, vocab=1024, theta=500000.0),
     32, 576, 64),
    ("rep4_hd128_2kv_b64_ctx1056", small_config(h=1024, heads=8, kv=2, layers=1, ffn=512, vocab=1024,
                                                theta=500000.0), 64, 960, 64),
]


@pytest.mark.parametrize("desc,cfg,B,n_prefix,n_tail", CASES, ids=[c[0] for c in CASES])
def test_long_context_batched_decode_matches_oracle(desc, cfg, B, n_prefix, n_tail):
    max_seq = 2304
    om = O.OracleLlama(orc_config(cfg, max_seq), 21)
    e = engine_from_oracle(om, cfg, max_seq=max_seq, max_batch=B, kv_dtype="bf16")
    splits, tmap, chunk = e.attn_plan(B)
    assert tmap and chunk == 64, (splits, tmap, chunk)
    assert splits > 1, splits  # the split partials and their combine run
    prefix = O.prompt_ids(1000, n_prefix, cfg.vocab_size)
    tails = np.stack([O.prompt_ids(2000 + b, n_tail, cfg.vocab_size) for b in range(B)])
    prompts = np.concatenate([np.broadcast_to(prefix, (B, n_prefix)), tails], 1).astype(np.int32)
    S = prompts.shape[1]
    # each split covers ceil(ctx / splits) positions rounded up to whole
    # 64-position tiles, so at these contexts several splits hold positions
    # (and, where ctx is short of splits * per_split, trailing ones none)
    per_split = _cdiv(_cdiv(S + 31, splits), 64) * 64
    assert S > per_split, (S, splits, per_split)
    n_gen = 32
    # batched prefill (chunks of B positions of one sequence, every row on its
    # pages), then 31 batched decode steps of all B rows
    got = e.generate_greedy(prompts, n_gen, batched_prefill=True)
    ref, ref_logits = _streams(om, prefix, tails, n_gen, max_seq)
    agree = [greedy_agreement(got[b], ref[b], ref_logits[b], TOL) for b in range(B)]
    assert sum(a == n_gen for a in agree) >= B - 2, agree  # near-ties are rare
    # a step's inputs are equal on both sides up to the first disagreement
    steps = [min((7 * b + 3) % n_gen, agree[b]) for b in range(B)]
    lg, am = _rewound_logits(e, prompts, got, steps)
    for b in range(B):
        assert rel_err(lg[b], ref_logits[b][steps[b]]) < TOL, (desc, b, steps[b])
        if steps[b] < agree[b]:
            assert int(am[b]) == int(ref[b][steps[b]]), (desc, b)


@pytest.mark.parametrize("rep", [4, 8])
def test_long_context_persistent_step_gqa(rep):
    # Batch 1 runs the persistent step kernel: one kv head, 4 or 8 query heads
    # of head_dim 128, a 2000-position context = 32 chunks of 64 positions.
    cfg = small_config(h=128 * rep, heads=rep, kv=1, layers=1, ffn=512, vocab=1024, theta=500000.0)
    max_seq = 2304
    om = O.OracleLlama(orc_config(cfg, max_seq), 22)
    e = engine_from_oracle(om, cfg, max_seq=max_seq, max_batch=1, kv_dtype="bf16")
    assert e.step_launches(1) == 1
    splits, tmap, chunk = e.attn_plan(1)
    assert splits == 0 and chunk == 64
    prefix = O.prompt_ids(3000 + rep, 1936, cfg.vocab_size)
    tails = O.prompt_ids(3100 + rep, 64, cfg.vocab_size)[None, :]
    prompt = np.concatenate([prefix, tails[0]]).astype(np.int32)
    got = e.generate_greedy(prompt, 32)[0]
    ref, ref_logits = _streams(om, prefix, tails, 32, max_seq)
    assert greedy_agreement(got, ref[0], ref_logits[0], TOL) == 32
    for j in (0, 17, 31):
        lg, _ = _rewound_logits(e, prompt[None, :], got[None, :], [j])
        assert rel_err(lg[0], ref_logits[0][j]) < TOL, j


def test_seven_b_shape_persistent_step_nine_chunks_per_layer():
    # Llama-2-7B layer shapes, 2 layers: a 520-position prompt spans 9
    # attention chunks of 64 positions per kv head and layer (32 kv heads:
    # 288 units over the SMs), like the 7B bench at contexts 512-768.
    cfg = LlamaConfig(32000, 4096, 11008, 2, 32, 32, 4096, 1e-5, 10000.0, False, None)
    max_seq = 640
    om = O.OracleLlama(orc_config(cfg, max_seq), 0)
    e = engine_from_oracle(om, cfg, max_seq=max_seq, max_batch=1, kv_dtype="bf16")
    assert e.step_launches(1) == 1
    _, _, chunk = e.attn_plan(1)
    prompt = O.prompt_ids(5, 520, cfg.vocab_size)
    assert -(-(len(prompt) + 1) // chunk) >= 9
    got = e.generate_greedy(prompt, 32)[0]
    ref, ref_logits = _streams(om, prompt[:-1], prompt[None, -1:], 32, max_seq)
    assert greedy_agreement(got, ref[0], ref_logits[0], TOL) == 32
    for j in (0, 31):
        lg, _ = _rewound_logits(e, prompt[None, :], got[None, :], [j])
        assert rel_err(lg[0], ref_logits[0][j]) < TOL, j


@pytest.mark.parametrize("B", [1, 8])
def test_seventy_b_head_layout_one_layer(B):
    # Llama-3-70B attention layout: hidden 8192, 64 query / 8 kv heads of 128
    # (8 per kv head), one layer (small ffn and vocabulary keep the oracle
    # cheap).  Batch 1 runs the persistent step, batch 8 the tensor-core
    # linears and the tensor-map attention with context splits.
    from esolearn_b200 import RopeScaling

    cfg = LlamaConfig(1024, 8192, 512, 1, 64, 8, 4096, 1e-5, 500000.0, False, RopeScaling())
    max_seq = 512
    om = O.OracleLlama(orc_config(cfg, max_seq), 23)
    e = engine_from_oracle(om, cfg, max_seq=max_seq, max_batch=B, kv_dtype="bf16")
    if B == 1:
        assert e.step_launches(1) == 1
    else:
        splits, tmap, _ = e.attn_plan(B)
        assert tmap and splits > 1, splits
    n_prompt = 150 if B == 1 else 140
    prompts = np.stack([O.prompt_ids(4000 + b, n_prompt, cfg.vocab_size) for b in range(B)])
    got = e.generate_greedy(prompts, 8, batched_prefill=B > 1)
    ref, ref_logits = _streams(om, np.zeros(0, np.int32), prompts, 8, max_seq)
    agree = [greedy_agreement(got[b], ref[b], ref_logits[b], TOL) for b in range(B)]
    assert sum(a == 8 for a in agree) >= B - 1, agree
    steps = [min((3 * b + 1) % 8, agree[b]) for b in range(B)]
    lg, _ = _rewound_logits(e, prompts, got, steps)
    for b in range(B):
        assert rel_err(lg[b], ref_logits[b][steps[b]]) < TOL, (b, steps[b])


@pytest.mark.parametrize("max_batch,n_prompt", [(64, 600), (16, 203)])
def test_seven_b_head_layout_prefill_attention(max_batch, n_prompt):
    # One query head per kv head (the 7B layout: 32 heads of 128): a batched
    # prefill runs the prefill attention kernel, every chunk of max_batch
    # prompt positions reading each K/V tile once for all its rows under the
    # causal mask (10 chunks of 64 over a 600-position prompt; 203 = 12
    # chunks of 16 plus a ragged tail of 11).  The greedy stream and the
    # logits of the steps after it equal the oracle's token-by-token run.
    cfg = LlamaConfig(1024, 4096, 512, 1, 32, 32, 4096, 1e-5, 10000.0, False, None)
    max_seq = 704
    om = O.OracleLlama(orc_config(cfg, max_seq), 31)
    e = engine_from_oracle(om, cfg, max_seq=max_seq, max_batch=max_batch, kv_dtype="bf16")
    prompt = O.prompt_ids(77, n_prompt, cfg.vocab_size)
    got = e.generate_greedy(prompt, 16, batched_prefill=True)[0]
    ref, ref_logits = _streams(om, prompt[:-1], prompt[None, -1:], 16, max_seq)
    assert greedy_agreement(got, ref[0], ref_logits[0], TOL) == 16
    for j in (0, 9, 15):
        lg, _ = _rewound_logits(e, prompt[None, :], got[None, :], [j])
        assert rel_err(lg[0], ref_logits[0][j]) < TOL, j


def test_one_split_attention_with_fused_projection_epilogue():
    # 32 sequences x 8 kv heads fill the GPU with one context split each, so
    # the batched step runs the tensor-map attention with the q|k|v
    # projection's epilogue inside it (q, RoPE and the new K/V row from the
    # GEMM's int64 sums): 9 launches per layer.  Greedy streams (near-tie
    # rule) and rewound logits against the oracle.
    cfg = small_config(h=1024, heads=16, kv=8, layers=2, ffn=512, vocab=1024, theta=500000.0)
    B, n_prompt, n_gen, max_seq = 32, 70, 16, 128
    om = O.OracleLlama(orc_config(cfg, max_seq), 41)
    e = engine_from_oracle(om, cfg, max_seq=max_seq, max_batch=B, kv_dtype="bf16")
    splits, tmap, _ = e.attn_plan(B)
    assert tmap and splits == 1, splits
    assert e.step_launches(B) == 5 + 9 * cfg.n_layers
    prompts = np.stack([O.prompt_ids(7000 + b, n_prompt, cfg.vocab_size) for b in range(B)])
    got = e.generate_greedy(prompts, n_gen, batched_prefill=True)
    ref, ref_logits = _streams(om, np.zeros(0, np.int32), prompts, n_gen, max_seq)
    agree = [greedy_agreement(got[b], ref[b], ref_logits[b], TOL) for b in range(B)]
    assert sum(a == n_gen for a in agree) >= B - 2, agree
    steps = [min((5 * b + 3) % n_gen, agree[b]) for b in range(B)]
    lg, _ = _rewound_logits(e, prompts, got, steps)
    for b in range(B):
        assert rel_err(lg[b], ref_logits[b][steps[b]]) < TOL, (b, steps[b])
