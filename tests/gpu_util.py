"""Shared helpers of the GPU parity tests (they compare libscryb200.so with the oracle)."""
import numpy as np

import oracle as O
from esolearn_b200 import LlamaConfig, QuantLlamaB200
from esolearn_b200 import _native as N


def rel_err(a, b) -> float:
    """Max relative error: max|a - b| / max|b| over the whole tensor."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def orc_config(c: LlamaConfig, max_seq: int):
    sc = None
    if c.rope_scaling is not None:
        r = c.rope_scaling
        sc = (r.factor, r.low_freq_factor, r.high_freq_factor, float(r.original_max_position_embeddings))
    return O.make_config(c.vocab_size, c.hidden_size, c.intermediate_size, c.n_layers, c.n_heads, c.n_kv_heads,
                         max_seq, c.rms_norm_eps, c.rope_theta, c.tie_word_embeddings, sc)


def engine_from_oracle(om: O.OracleLlama, c: LlamaConfig, **kw) -> QuantLlamaB200:
    """A B200 engine holding exactly the oracle's int8 weights, scales and f32 tensors."""
    e = QuantLlamaB200(c, **kw)
    for l in range(c.n_layers):
        for slot in range(5):
            q, s = om.weight(l, slot)
            e.load_qweight(l, slot, q, s)
        e.load_f32(N.SB_F_NORM_IN, l, om.norm(l, 0))
        e.load_f32(N.SB_F_NORM_POST, l, om.norm(l, 1))
    q, s = om.lm_head()
    e.load_qweight(-1, 0, q, s)
    e.load_f32(N.SB_F_EMBED, 0, om.embed())
    e.load_f32(N.SB_F_NORM_FINAL, 0, om.norm(-1, 0))
    return e


def small_config(h=512, layers=2, heads=8, kv=8, ffn=1376, vocab=4096, theta=10000.0, tie=False, scaling=None):
    return LlamaConfig(vocab, h, ffn, layers, heads, kv, 4096, 1e-5, theta, tie, scaling)


def greedy_agreement(got, ref, ref_logits, tol: float = 1e-3) -> int:
    """Number of leading tokens of an engine greedy stream `got` that equal the
    oracle's `ref`.  Every token must match, except where the oracle's own
    logits at that step put the two tokens within `tol` x max|logit| of each
    other (a near-tie that rounding at the logits tolerance may resolve either
    way); the streams are compared up to that step only.  Raises if the streams
    part anywhere else."""
    got, ref = list(got), list(ref)
    for j, (g, r) in enumerate(zip(got, ref)):
        if g == r:
            continue
        lg = np.asarray(ref_logits[j], np.float64)
        gap = abs(lg[r] - lg[g])
        assert gap <= tol * np.abs(lg).max(), (
            f"token {j}: engine {g}, oracle {r}, oracle logit gap {gap:.3e} > {tol} x max|logit|")
        return j
    return len(ref)
