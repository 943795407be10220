"""Pins the CPU oracle against the reference's own unit tests (CPU only).

Each test restates one reference test; the citation names the reference
file:line and the expected values come from that test.  The oracle is the
parity authority for every GPU test, so it is checked first.
"""
import math

import numpy as np
import pytest

import oracle as O


# ---- quantize.rs:42-84 ------------------------------------------------------
def test_quantize_roundtrip_accuracy():
    # quantize.rs:46-65
    w = np.array([i * 0.1 for i in range(-100, 101)], np.float32)
    q, s = O.quantize_symmetric(w)
    rec = O.dequantize(q, s)
    max_abs = np.abs(w).max()
    assert np.abs(w - rec).max() <= max_abs / 127.0 + 1e-6


def test_quantize_zero_weights():
    # quantize.rs:67-73: all zero -> q all 0 and scale exactly 0
    q, s = O.quantize_symmetric(np.zeros(10, np.float32))
    assert (q == 0).all() and s == 0.0


def test_quantize_clamps_to_range():
    # quantize.rs:75-83: exact int8 values
    q, _ = O.quantize_symmetric(np.array([1000.0, -1000.0, 0.0], np.float32))
    assert q.tolist() == [127, -127, 0]


def test_quantize_round_half_away_from_zero():
    # quantize.rs:28 uses f32::round (half away from zero), not round-to-even.
    # absmax 127 -> scale 1, inv 1: 0.5 -> 1, -0.5 -> -1, 2.5 -> 3, -2.5 -> -3.
    w = np.array([127.0, 0.5, -0.5, 2.5, -2.5, 1.49, -126.5], np.float32)
    q, s = O.quantize_symmetric(w)
    assert s == np.float32(1.0)
    assert q.tolist() == [127, 1, -1, 3, -3, 1, -127]


def test_quantize_scale_is_f32_division():
    rng = np.random.default_rng(3)
    w = rng.standard_normal(1000).astype(np.float32) * np.float32(0.02)
    q, s = O.quantize_symmetric(w)
    absmax = np.float32(np.abs(w).max())
    assert s == np.float32(absmax / np.float32(127.0))
    inv = np.float32(np.float32(1.0) / s)
    prod = (w * inv).astype(np.float32)
    expect = np.clip(np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5)), -127, 127).astype(np.int8)
    assert (q == expect).all()


# ---- backend/cpu.rs:1471-1757 --------------------------------------------------
def test_rmsnorm_basic():
    # cpu.rs:1500-1511
    out = O.rmsnorm(np.array([[1, 2, 3, 4]], np.float32), np.ones(4, np.float32), 1e-5)
    rstd = 1.0 / math.sqrt(7.5 + 1e-5)
    for i in range(4):
        assert abs(float(out[0, i]) - (i + 1) * rstd) < 1e-5


def test_swiglu_basic():
    # cpu.rs:1514-1522
    out = O.swiglu(np.array([0.0, 1.0, -1.0], np.float32), np.ones(3, np.float32))
    assert abs(out[0]) < 1e-6
    assert abs(out[1] - 0.7311) < 1e-3
    assert abs(out[2] + 0.2689) < 1e-3


def test_rope_basic():
    # cpu.rs:1539-1548 (theta 1e4, head_dim 4, pos 1; first pair rotates by 1 rad)
    fr = O.compute_rope_freqs(4, 10000.0).astype(np.float32)
    out = O.rope(np.array([1.0, 0.0, 1.0, 0.0], np.float32), 1, 1, 4, 1, fr)
    assert abs(out[0] - 0.5403) < 1e-3
    assert abs(out[1] - 0.8415) < 1e-3


def test_softmax_basic():
    # cpu.rs:1484-1493
    out = O.softmax(np.array([1.0, 2.0, 3.0], np.float32), 1, 3)
    assert abs(out.sum() - 1.0) < 1e-6
    assert out[2] > out[1] > out[0]


def test_gather_reshape_repeat_kv_matches_3step():
    # cpu.rs:1663-1697
    max_seq, n_kv, n_q, hd, cl = 4, 2, 4, 2, 3
    kv_dim = n_kv * hd
    cache = np.arange(max_seq * kv_dim, dtype=np.float32)
    fused = O.gather_reshape_repeat_kv(cache, cl, n_kv, n_q, hd)
    g = cache[: cl * kv_dim].reshape(cl, n_kv, hd).transpose(1, 0, 2)  # [n_kv, cl, hd]
    ref = np.repeat(g, n_q // n_kv, axis=0).ravel()
    assert np.array_equal(fused, ref)


def _f32_matmul(a, b):
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)


def test_matmul_i8_f32_matches_f32_matmul():
    # cpu.rs:1699-1728
    m, k, n = 4, 8, 3
    a = (np.arange(m * k, dtype=np.float32) * np.float32(0.1) - np.float32(1.5)).reshape(m, k)
    b = (np.arange(k * n, dtype=np.float32) * np.float32(0.05) - np.float32(0.6)).reshape(k, n)
    q, s = O.quantize_symmetric(b)
    c = O.matmul_i8_f32(a, q, s, m, k, n)
    tol = np.abs(b).max() / 127.0 * k * 0.5
    assert np.abs(c - _f32_matmul(a, b)).max() < tol


def test_matmul_i8_f32_bias_matches_f32():
    # cpu.rs:1730-1756 (bias added after the int8 product, cpu.rs:554-570)
    m, k, n = 2, 4, 3
    a = (np.arange(m * k, dtype=np.float32) * np.float32(0.1)).reshape(m, k)
    b = (np.arange(k * n, dtype=np.float32) * np.float32(0.05)).reshape(k, n)
    bias = np.array([1.0, 2.0, 3.0], np.float32)
    q, s = O.quantize_symmetric(b)
    c = O.matmul_i8_f32(a, q, s, m, k, n) + bias
    tol = np.abs(b).max() / 127.0 * k * 0.5
    assert np.abs(c - (_f32_matmul(a, b) + bias)).max() < tol


def test_matmul_i8_f32_exact_term_order():
    # cpu.rs:1147-1157: each term is f64 product rounded to f32, summed in f32 in k order.
    rng = np.random.default_rng(0)
    m, k, n = 3, 70, 37
    a = rng.standard_normal((m, k)).astype(np.float32)
    q = rng.integers(-127, 128, (k, n), dtype=np.int8)
    s = np.float32(0.0123)
    c = O.matmul_i8_f32(a, q, s, m, k, n)
    ref = np.zeros((m, n), np.float32)
    for p in range(k):
        term = (a[:, p:p + 1].astype(np.float64) * (q[p:p + 1, :].astype(np.float64) * np.float64(s))).astype(np.float32)
        ref = (ref + term).astype(np.float32)
    assert np.array_equal(c, ref)


def test_matmul_tb_equals_transposed():
    rng = np.random.default_rng(1)
    m, k, n = 2, 64, 45
    a = rng.standard_normal((m, k)).astype(np.float32)
    q = rng.integers(-127, 128, (k, n), dtype=np.int8)
    c1 = O.matmul_i8_f32(a, q, 0.01, m, k, n)
    c2 = O.matmul_i8_f32_tb(a, np.ascontiguousarray(q.T), 0.01, m, k, n)
    assert np.array_equal(c1, c2)


def test_matmul_thread_count_invariant():
    rng = np.random.default_rng(2)
    m, k, n = 2, 300, 1000
    a = rng.standard_normal((m, k)).astype(np.float32)
    q = rng.integers(-127, 128, (k, n), dtype=np.int8)
    t0 = O.get_threads()
    try:
        O.set_threads(1)
        c1 = O.matmul_i8_f32(a, q, 0.01, m, k, n)
        O.set_threads(4)
        c4 = O.matmul_i8_f32(a, q, 0.01, m, k, n)
    finally:
        O.set_threads(t0)
    assert np.array_equal(c1, c4)


def test_grouped_matmul_reduces_to_per_tensor():
    # One group spanning all of K with a column-constant scale equals the per-tensor path.
    rng = np.random.default_rng(4)
    m, k, n = 2, 64, 40
    a = rng.standard_normal((m, k)).astype(np.float32)
    q = rng.integers(-127, 128, (k, n), dtype=np.int8)
    sc = np.full((1, n), 0.01, np.float32)
    c1 = O.matmul_i8_f32(a, q, np.float32(0.01), m, k, n)
    c2 = O.matmul_i8_f32_grouped(a, q, sc, k, m, k, n)
    assert np.array_equal(c1, c2)


def test_quantize_grouped_bounds():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((128, 40)) * 0.02).astype(np.float32)
    for g in (32, 64):
        q, s = O.quantize_grouped(w, g)
        deq = q.astype(np.float32) * np.repeat(s, g, axis=0)
        assert np.abs(deq - w).max() <= np.abs(w).max() / 127.0 + 1e-7
        assert np.abs(q).max() == 127


def test_compute_rope_freqs_llama3_scaling():
    # llama.rs:1035-1067: high-frequency pairs unscaled, low-frequency divided by factor.
    base = O.compute_rope_freqs(128, 500000.0)
    sc = O.compute_rope_freqs(128, 500000.0, (32.0, 1.0, 4.0, 8192.0))
    assert sc[0] == base[0]
    assert abs(sc[-1] - base[-1] / 32.0) < 1e-20


def test_argmax_ties_resolve_to_last():
    # generate.rs:167-173: Iterator::max_by returns the last of equal maxima.
    assert O.argmax(np.array([1.0, 3.0, 2.0, 3.0, 0.0], np.float32)) == 3
    assert O.argmax(np.array([5.0], np.float32)) == 0


# ---- fastrand restatement ---------------------------------------------------------
def test_rng_counter_based_equals_sequential():
    r = O.Rng(7)
    seq = r.normal_vec(1001)
    par = O.normal_vec_at(7, 0, 1001)
    assert np.array_equal(seq, par)
    tail = r.normal_vec(10)
    assert np.array_equal(tail, O.normal_vec_at(7, 2002, 10))


def test_rng_f64_range_and_stats():
    r = O.Rng(0)
    x = np.array([r.f64() for _ in range(20000)])
    assert x.min() >= 0.0 and x.max() < 1.0
    assert abs(x.mean() - 0.5) < 0.01
    z = O.normal_vec_at(0, 0, 200000, 0.0, 0.02)
    assert abs(z.std() - 0.02) < 2e-4 and abs(z.mean()) < 2e-4


def test_rng_below_range():
    r = O.Rng(11)
    v = [r.below(32000) for _ in range(5000)]
    assert min(v) >= 0 and max(v) < 32000


# ---- tests/llama_smoke.rs invariants on the quantized model ---------------------
def _smoke_cfg(**kw):
    base = dict(vocab=32, hidden=16, inter=32, layers=2, heads=4, kv_heads=2, max_seq=64,
                theta=500000.0, tie=True)
    base.update(kw)
    return O.make_config(base["vocab"], base["hidden"], base["inter"], base["layers"], base["heads"],
                         base["kv_heads"], base["max_seq"], 1e-5, base["theta"], base["tie"])


def test_llama_kv_cache_forward_finite():
    # llama_smoke.rs:51-70
    m = O.OracleLlama(_smoke_cfg(), 42)
    cache = m.new_cache(64)
    for pos, tok in enumerate([0, 1, 2, 3]):
        lg = m.forward_with_cache(cache, tok, pos)
        assert lg.shape == (32,) and np.isfinite(lg).all()


def test_llama_generate_deterministic_greedy():
    # llama_smoke.rs:148-168
    m = O.OracleLlama(_smoke_cfg(), 42)
    t1 = m.generate_greedy([0], 5)
    t2 = m.generate_greedy([0], 5)
    assert t1.tolist() == t2.tolist()
    assert all(0 <= t < 32 for t in t1)


@pytest.mark.parametrize("heads,kv", [(4, 4), (4, 2), (4, 1), (8, 2)])
def test_llama_gqa_ratio(heads, kv):
    # llama_smoke.rs:267-305
    cfg = O.make_config(16, heads * 4, 32, 1, heads, kv, 32, 1e-5, 10000.0, True)
    m = O.OracleLlama(cfg, 42)
    cache = m.new_cache(32)
    for pos in range(3):
        assert np.isfinite(m.forward_with_cache(cache, pos, pos)).all()


def test_llama_untied_embeddings():
    # llama_smoke.rs:245-265: untied model draws a separate lm_head
    cfg = _smoke_cfg(layers=1, tie=False)
    m_t = O.OracleLlama(_smoke_cfg(layers=1, tie=True), 42)
    m_u = O.OracleLlama(cfg, 42)
    assert not np.array_equal(m_t.lm_head()[0], m_u.lm_head()[0])
    q_emb, _ = O.quantize_symmetric(m_t.embed())
    assert np.array_equal(m_t.lm_head()[0].ravel(), q_emb)


def test_model_weights_follow_draw_order():
    # llama.rs:593-680: embed first, then layer-0 q, k, v (fused), o, gate, up, down.
    cfg = _smoke_cfg(layers=1, tie=True)
    m = O.OracleLlama(cfg, 42)
    V, h, F = 32, 16, 32
    hd = 4
    qd, kvd = 4 * hd, 2 * hd
    emb = O.normal_vec_at(42, 0, V * h)
    assert np.array_equal(m.embed().ravel(), emb)
    d = 2 * V * h
    qw = O.normal_vec_at(42, d, h * qd).reshape(h, qd); d += 2 * h * qd
    kw = O.normal_vec_at(42, d, h * kvd).reshape(h, kvd); d += 2 * h * kvd
    vw = O.normal_vec_at(42, d, h * kvd).reshape(h, kvd); d += 2 * h * kvd
    fused = np.concatenate([qw, kw, vw], axis=1)
    q, s = O.quantize_symmetric(fused)
    wq, ws = m.weight(0, 0)
    assert np.array_equal(wq.ravel(), q) and ws == s
    ow = O.normal_vec_at(42, d, qd * h); d += 2 * qd * h
    q, s = O.quantize_symmetric(ow)
    assert np.array_equal(m.weight(0, 1)[0].ravel(), q)
    for slot in (2, 3, 4):
        w = O.normal_vec_at(42, d, h * F); d += 2 * h * F
        q, s = O.quantize_symmetric(w)
        assert np.array_equal(m.weight(0, slot)[0].ravel(), q)


def test_kv_bf16_variant_close_to_f32():
    cfg = O.make_config(512, 64, 160, 2, 4, 2, 64, 1e-5, 10000.0, False)
    m = O.OracleLlama(cfg, 0)
    c32, c16 = m.new_cache(16), m.new_cache(16, kv_bf16=True)
    for pos, tok in enumerate([5, 9, 100, 7]):
        a = m.forward_with_cache(c32, tok, pos)
        b = m.forward_with_cache(c16, tok, pos)
        assert np.abs(a - b).max() / np.abs(a).max() < 2e-2


def test_forward_tokens_equals_token_by_token_loop():
    # orc_forward_tokens (test infrastructure for long prompts) must give the
    # logits and cache of consecutive forward_with_cache calls bit for bit,
    # also when continuing a cache; clone + truncate rewinds a sequence.
    cfg = O.make_config(512, 256, 192, 2, 4, 2, 96, 1e-5, 10000.0, False)
    om = O.OracleLlama(cfg, 4)
    toks = O.prompt_ids(9, 60, cfg.vocab_size)
    seq = om.new_cache(96, kv_bf16=True)
    ref = np.stack([om.forward_with_cache(seq, int(t), p) for p, t in enumerate(toks)])
    bat = om.new_cache(96, kv_bf16=True)
    got = np.concatenate([om.forward_tokens(bat, toks[:25], 0, all_logits=True),
                          om.forward_tokens(bat, toks[25:], 25, all_logits=True)])
    assert np.array_equal(got, ref)
    assert len(bat) == 60
    assert np.array_equal(om.forward_tokens(om.new_cache(96), toks[:7], 0),
                          om.forward_tokens(om.new_cache(96), toks[:7], 0, all_logits=True)[-1])
    c = bat.clone()
    c.truncate(40)
    assert len(c) == 40 and len(bat) == 60
    assert np.array_equal(om.forward_with_cache(c, int(toks[40]), 40), ref[40])
    assert np.array_equal(om.forward_with_cache(bat, 5, 60), om.forward_with_cache(seq, 5, 60))
