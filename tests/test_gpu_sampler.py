"""Device sampler (sb_sample_rows / sb_llama_sample) against the oracle's
restatement of sample_token (generate.rs:92-165).

The random stream is integer work (fastrand wyrand states), so the states
after every draw must equal the oracle's bit for bit; the tokens must equal
the oracle's on every draw (sums differ from the reference's left-to-right
order only by rounding, which decides a token only when a draw lands within
f64 rounding of a running sum -- never in these seeded cases).
"""
import numpy as np
import pytest

import oracle as O
from esolearn_b200 import QuantLlamaB200, Rng, SamplingConfig, generate, sample_rows
from esolearn_b200 import _native as N

from gpu_util import engine_from_oracle, orc_config, small_config

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DRAWS = 3  # draws per row from the same logits: the states must advance like the host's


@pytest.fixture(scope="module", autouse=True)
def _init():
    N.check(N.lib().sb_init(0))


def _states(seeds):
    return torch.from_numpy(np.array(seeds, np.uint64).view(np.int64)).cuda()


def _check(logits: np.ndarray, cfg: SamplingConfig, seeds):
    rows, n = logits.shape
    lg = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    st = _states(seeds)
    refs = [O.Rng(s) for s in seeds]
    for d in range(DRAWS):
        got = sample_rows(lg, cfg, st).cpu().numpy()
        want = [O.sample_token(logits[r], cfg.temperature, cfg.top_k, cfg.top_p, refs[r]) for r in range(rows)]
        assert got.tolist() == want, (d, cfg)
        states = st.cpu().numpy().view(np.uint64)
        assert [int(v) for v in states] == [int(r.state.value) for r in refs], (d, cfg)


CONFIGS = [
    SamplingConfig(0.7, 0, 1.0), SamplingConfig(1.0, 50, 1.0), SamplingConfig(0.8, 40, 0.9),
    SamplingConfig(1.5, 0, 0.5), SamplingConfig(1.0, 0, 0.95), SamplingConfig(2.0, 10, 0.5),
    SamplingConfig(0.0, 0, 1.0), SamplingConfig(1.0, 5000, 0.999), SamplingConfig(5.0, 0, 0.3),
]


@pytest.mark.parametrize("n", [97, 32000, 128256])
@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: f"t{c.temperature}_k{c.top_k}_p{c.top_p}")
def test_sampler_matches_oracle(n, cfg):
    rng = np.random.default_rng(n + int(cfg.temperature * 10) + cfg.top_k)
    logits = (rng.standard_normal((6, n)) * 3.0).astype(np.float32)
    _check(logits, cfg, [11 + 1000 * r for r in range(6)])


@pytest.mark.parametrize("cfg", [SamplingConfig(1.0, 7, 1.0), SamplingConfig(1.0, 0, 0.6), SamplingConfig(0.5, 300, 0.8),
                                 SamplingConfig(1.0, 1, 1.0), SamplingConfig(1.0, 0, 0.999999)],
                         ids=lambda c: f"t{c.temperature}_k{c.top_k}_p{c.top_p}")
def test_sampler_ties_and_special_values(cfg):
    # Integer-valued logits tie everywhere: the top-k threshold counts ties
    # with multiplicity and the top-p cut keeps tied values lowest index
    # first; -inf logits, an all -inf row (uniform fallback), and -0 / +0.
    rng = np.random.default_rng(5)
    n = 4099
    rows = [rng.integers(0, 4, n).astype(np.float32), rng.integers(-2, 3, n).astype(np.float32)]
    r = rng.standard_normal(n).astype(np.float32)
    r[rng.random(n) < 0.5] = -np.inf
    rows.append(r)
    rows.append(np.full(n, -np.inf, np.float32))
    z = np.zeros(n, np.float32)
    z[::2] = -0.0
    z[7] = 1.0
    rows.append(z)
    _check(np.stack(rows), cfg, [3, 5, 7, 9, 13])


@pytest.mark.parametrize("n", [1, 2, 5])
def test_sampler_tiny_rows(n):
    rng = np.random.default_rng(n)
    logits = rng.standard_normal((4, n)).astype(np.float32)
    for cfg in (SamplingConfig(1.0, 0, 1.0), SamplingConfig(1.0, 1, 1.0), SamplingConfig(1.0, n, 0.5),
                SamplingConfig(0.0, 0, 1.0)):
        _check(logits, cfg, [1, 2, 3, 4])


def test_sampler_rejects_bad_arguments():
    lg = torch.zeros((2, 8), device="cuda")
    st = _states([1, 2])
    out = torch.empty(2, dtype=torch.int32, device="cuda")
    with pytest.raises(N.SbError):
        sample_rows(lg, SamplingConfig(float("nan"), 0, 1.0), st, out)
    with pytest.raises(N.SbError):
        sample_rows(lg, SamplingConfig(1.0, -1, 1.0), st, out)
    with pytest.raises(N.SbError):
        sample_rows(lg[:, :0].contiguous(), SamplingConfig(1.0, 0, 1.0), st, out)


@pytest.mark.parametrize("cfg", [SamplingConfig(0.7, 20, 0.9, 24), SamplingConfig(1.2, 0, 1.0, 24),
                                 SamplingConfig(0.9, 0, 0.8, 24)],
                         ids=lambda c: f"t{c.temperature}_k{c.top_k}_p{c.top_p}")
def test_generate_device_sampling_equals_host_sampling_and_oracle(cfg):
    # generate() samples on the device (only the token comes back); the
    # stream equals the host sampler's on the same engine logits and the
    # oracle model's generate() with the same seed.
    c = small_config(layers=2)
    om = O.OracleLlama(orc_config(c, 96), 4)
    e = engine_from_oracle(om, c, max_seq=96, max_batch=1, kv_dtype="f32")
    prompt = [5, 9, 2, 7]
    ra, rb = Rng(77), Rng(77)
    dev = generate(e, prompt, cfg, ra)
    host = generate(e, prompt, cfg, rb, device_sampling=False)
    assert dev == host
    assert ra.state == rb.state
    oc = om.new_cache(96)
    rng = O.Rng(77)
    out = []
    for pos, t in enumerate(prompt):
        lg = om.forward_with_cache(oc, t, pos)
    out.append(O.sample_token(lg, cfg.temperature, cfg.top_k, cfg.top_p, rng))
    for i in range(1, cfg.max_tokens):
        lg = om.forward_with_cache(oc, out[-1], len(prompt) + i - 1)
        out.append(O.sample_token(lg, cfg.temperature, cfg.top_k, cfg.top_p, rng))
    assert dev == out
    e.close()


def test_engine_sample_batch_rows_match_oracle():
    # sb_llama_sample over a batch of rows: each row samples from its own
    # logits with its own state, like B independent sample_token calls.
    c = small_config(layers=1)
    e = QuantLlamaB200.new_random(c, 9, max_seq=32, max_batch=4, kv_dtype="f32")
    toks, pos = [3, 1, 4, 1], [0, 0, 0, 0]
    lg, _ = e.forward_batch(toks, pos)
    cfg = SamplingConfig(0.8, 30, 0.9)
    rngs = [Rng(100 + b) for b in range(4)]
    got = e.sample(cfg, rngs)
    refs = [O.Rng(100 + b) for b in range(4)]
    want = [O.sample_token(lg[b], cfg.temperature, cfg.top_k, cfg.top_p, refs[b]) for b in range(4)]
    assert got == want
    assert [r.state for r in rngs] == [int(r.state.value) for r in refs]
    e.close()


def _oracle_sampled(om, prompt, cfg, seed, max_seq):
    """The oracle model's generate() with sampling: tokens and the final state."""
    oc = om.new_cache(max_seq)
    rng = O.Rng(seed)
    for pos, t in enumerate(prompt):
        lg = om.forward_with_cache(oc, int(t), pos)
    out = [O.sample_token(lg, cfg.temperature, cfg.top_k, cfg.top_p, rng)]
    for i in range(1, max(1, cfg.max_tokens)):
        lg = om.forward_with_cache(oc, out[-1], len(prompt) + i - 1)
        out.append(O.sample_token(lg, cfg.temperature, cfg.top_k, cfg.top_p, rng))
    return out, int(rng.state.value)


@pytest.mark.parametrize("B,batched_prefill", [(1, False), (1, True), (3, False), (3, True), (6, False), (6, True)])
def test_device_sampling_loop_matches_oracle(B, batched_prefill):
    # generate() with sampling as one device loop (sb_llama_set_sampling +
    # sb_llama_step): every step samples on the device and feeds its token to
    # the next one.  Batch 1 runs the persistent step kernel, 3 the GEMV graph,
    # 6 the chained tensor-core graph; with batched_prefill the first token is
    # sampled after sb_llama_prefill.  Tokens and generator states equal the
    # oracle model's generate() per sequence.
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 96), 6)
    e = engine_from_oracle(om, c, max_seq=96, max_batch=max(B, 4), kv_dtype="f32")
    cfg = SamplingConfig(0.8, 20, 0.9, 16)
    prompts = np.stack([O.prompt_ids(500 + b, 7, c.vocab_size) for b in range(B)])
    rngs = [Rng(50 + b) for b in range(B)]
    got = e.generate_sampled(prompts, cfg, rngs, batched_prefill=batched_prefill)
    for b in range(B):
        want, state = _oracle_sampled(om, prompts[b], cfg, 50 + b, 96)
        assert got[b].tolist() == want, b
        assert rngs[b].state == state, b
    e.close()


def test_device_sampling_loop_draw_cap_and_state_kept_across_capture():
    # Sampling switched on after sb_llama_begin (the sampled step graph is
    # captured then: its warm-up must leave the sequence state alone), and
    # max_draws = 5: steps after the fifth draw leave the generators as they
    # are.
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 96), 6)
    e = engine_from_oracle(om, c, max_seq=96, max_batch=3, kv_dtype="f32")
    cfg = SamplingConfig(1.1, 0, 0.95, 5)
    prompts = np.stack([O.prompt_ids(600 + b, 6, c.vocab_size) for b in range(3)])
    e.begin(prompts)
    e.set_sampling(cfg, [Rng(90 + b) for b in range(3)], max_draws=5)
    e.step(6 + 12)  # the prompt, then 13 steps: 5 draw, 8 draw nothing
    got = e.tokens(3, 5)
    st = e.rng_states(3)
    e.clear_sampling()
    for b in range(3):
        want, state = _oracle_sampled(om, prompts[b], cfg, 90 + b, 96)
        assert got[b].tolist() == want, b
        assert int(st[b]) == state, b
    e.close()
