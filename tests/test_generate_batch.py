"""generate_batch (several prompts, one engine row each) against generate()
per sequence (generate.rs:51-89).

The CPU tests drive the batching logic through a stand-in model whose
logits are a fixed function of each sequence's own history, so any mix-up
of rows, positions, prompt/sample hand-over or generator draws changes the
streams.  The GPU test runs the real engine.
"""
import hashlib

import numpy as np
import pytest

import oracle as O
from esolearn_b200 import Rng, SamplingConfig, generate, generate_batch, sample_token


class _Cache:
    def __init__(self, model, max_seq):
        self.model, self.max_seq, self.slot, self.seq_len = model, max_seq, 0, 0


class FakeModel:
    """A CausalLM stand-in: logits = hash of the sequence's tokens so far."""

    tp_size = 1

    def __init__(self, vocab=50, max_batch=4, max_seq=64):
        self.vocab, self.max_batch, self.max_seq = vocab, max_batch, max_seq
        self.hist = {}
        self.last = {}

    def vocab_size(self):
        return self.vocab

    def new_kv_cache(self, max_seq):
        assert max_seq <= self.max_seq
        self.hist = {}
        return _Cache(self, max_seq)

    def _logits(self, h):
        d = hashlib.sha256(np.asarray(h, np.int64).tobytes()).digest()
        rng = np.random.default_rng(int.from_bytes(d[:8], "little"))
        return (rng.standard_normal(self.vocab) * 2.0).astype(np.float32)

    def forward_batch(self, tokens, positions, slots=None, want_logits=True):
        out = []
        for b, (t, p) in enumerate(zip(tokens, positions)):
            h = self.hist.setdefault(b, [])
            assert p == len(h), (b, p, len(h))  # positions advance one by one per sequence
            h.append(int(t))
            self.last[b] = self._logits(h)
            out.append(self.last[b])
        return (np.stack(out) if want_logits else None), np.array([int(np.argmax(x)) for x in out])

    def forward_with_cache(self, token, pos, cache):
        return self.forward_batch([token], [pos])[0][0]

    def sample(self, config, rngs):
        return [sample_token(self.last[b], config, r) for b, r in enumerate(rngs)]

    def generate_greedy(self, prompts, max_tokens):
        p = list(np.atleast_2d(prompts)[0])
        return np.array([generate(self, p, SamplingConfig(1.0, 1, 1.0, max_tokens), Rng(0), device_loop=False)])


CONFIGS = [SamplingConfig(0.8, 10, 0.9, 7), SamplingConfig(1.3, 0, 1.0, 5), SamplingConfig(0.0, 0, 1.0, 6),
           SamplingConfig(1.0, 0, 0.5, 0), SamplingConfig(1.0, 3, 1.0, 1)]


@pytest.mark.parametrize("device_sampling", [True, False])
@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: f"t{c.temperature}_k{c.top_k}_p{c.top_p}_n{c.max_tokens}")
def test_generate_batch_equals_generate_per_sequence(cfg, device_sampling):
    m = FakeModel()
    prompts = [[3, 1, 4, 1, 5], [9, 2, 6, 5, 3, 5, 8, 9], [7], [2, 7, 1]]
    rngs = [Rng(10 + b) for b in range(4)]
    got = generate_batch(m, prompts, cfg, rngs, device_sampling=device_sampling)
    for b, p in enumerate(prompts):
        r = Rng(10 + b)
        want = generate(m, p, cfg, r, device_sampling=False)
        assert got[b] == want, (b, got[b], want)
        assert rngs[b].state == r.state, b  # each generator drew exactly its own sequence's samples
        assert len(got[b]) == max(1, cfg.max_tokens)


def test_generate_batch_argument_checks():
    m = FakeModel(max_batch=2)
    with pytest.raises(ValueError):
        generate_batch(m, [[1], []], SamplingConfig(), [Rng(0), Rng(1)])
    with pytest.raises(ValueError):
        generate_batch(m, [[1]], SamplingConfig(), [])
    with pytest.raises(Exception):
        generate_batch(m, [[1], [2], [3]], SamplingConfig(), [Rng(0), Rng(1), Rng(2)])
    assert generate_batch(m, [], SamplingConfig(), []) == []


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [SamplingConfig(0.8, 20, 0.9, 12), SamplingConfig(0.0, 0, 1.0, 12)],
                         ids=["sampled", "greedy"])
def test_engine_generate_batch_reproduces_generate_per_sequence(cfg):
    # One batched engine step per position for 3 ragged prompts, sampling on
    # the device, against generate() of each prompt alone.
    from esolearn_b200 import _native as N
    from gpu_util import engine_from_oracle, orc_config, small_config

    N.check(N.lib().sb_init(0))
    c = small_config(layers=2, heads=8, kv=2)
    om = O.OracleLlama(orc_config(c, 128), 9)
    e = engine_from_oracle(om, c, max_seq=128, max_batch=4, kv_dtype="bf16")
    prompts = [list(O.prompt_ids(300 + b, n, c.vocab_size)) for b, n in enumerate([5, 9, 3])]
    rngs = [Rng(40 + b) for b in range(3)]
    got = generate_batch(e, prompts, cfg, rngs)
    for b, p in enumerate(prompts):
        r = Rng(40 + b)
        assert got[b] == generate(e, p, cfg, r), b
        assert rngs[b].state == r.state, b
    e.close()
