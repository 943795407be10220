"""Host-side pieces of the measurement harness, on the CPU.

bench.py's workloads must be BASELINE's configurations (shape, batch,
prompt); the clock record must report the throttle reasons that reject a run;
the quantized-linear sweep must cover the configs[1] grid with its stated
byte count; the CPU reference leg must time whole decode steps of the
shape it is given; and the step-timeline summary (the per-phase barrier,
input-stage and work times of the persistent step) must read its stamps
correctly.  None of this needs a GPU.
"""
import time

import bench
from esolearn_b200 import LlamaConfig
from esolearn_b200 import linear_sweep as LS


def _shape(cfg):
    return (cfg.hidden_size, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.intermediate_size, cfg.vocab_size,
            cfg.rope_theta)


def test_workloads_are_the_baseline_configs():
    # Llama-2-7B shape, 512-token prompt, batch 1
    # Llama-3-8B shape with GQA, 2048-token contexts, batch 32
    # Llama-3-70B shape, 1024-token prompts, batch 64
    want = {
        "llama2-7b-bs1": ((4096, 32, 32, 32, 11008, 32000, 10000.0), 1, 512),
        "llama3-8b-bs32": ((4096, 32, 32, 8, 14336, 128256, 500000.0), 32, 2048),
        "llama3-70b-bs64": ((8192, 80, 64, 8, 28672, 128256, 500000.0), 64, 1024),
    }
    assert set(bench.WORKLOADS) == set(want)
    for name, (shape, batch, prompt) in want.items():
        wl = bench.WORKLOADS[name]
        assert _shape(getattr(LlamaConfig, wl["shape"])()) == shape, name
        assert (wl["batch"], wl["prompt"]) == (batch, prompt), name


def _line(ts, sm, mx, hw="Not Active", thermal="Not Active", sw_thermal="Not Active", power="Not Active"):
    # timestamp, index, clocks.sm, clocks.max.sm, power.draw, reasons.active, the four reasons
    return ts, f"2026/01/01 00:00:00.000, 0, {sm}, {mx}, 700.00, 0x0, {hw}, {thermal}, {sw_thermal}, {power}"


def test_clock_record_reports_rejecting_reasons():
    s = bench.ClockSampler(0)
    t0 = time.time()
    s.lines = [_line(t0 - 10, 300, 1965),  # idle, long before the timed region
               _line(t0 + 0.1, 1965, 1965), _line(t0 + 0.2, 1900, 1965, hw="Active"),
               _line(t0 + 0.3, 1965, 1965, power="Active")]
    r = s.summary(t0, t0 + 0.3)
    assert r["samples"] == 3
    assert r["sm_mhz"] == 1965.0 and r["sm_max_mhz"] == 1965.0
    assert r["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_record_without_samples_in_the_region():
    s = bench.ClockSampler(0)
    assert s.summary(0.0, 1.0)["reasons"] == ["unsampled"]
    # a region shorter than the sampling period still reports the latest samples
    t0 = time.time()
    s.lines = [_line(t0 - 5, 1965, 1965), _line(t0 - 4, 1950, 1965)]
    r = s.summary(t0, t0 + 0.01)
    assert r["samples"] == 2 and r["reasons"] == []


def test_sweep_covers_the_configs1_grid():
    assert LS.SHAPES == [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 32000)]
    assert LS.ROWS == [1, 8, 32, 128]
    assert LS.GROUPS == [0, 32, 64]


def test_sweep_byte_count():
    # K*N int8 + f32 scales (one per tensor, or per group of rows and column)
    # + M*K bf16 activations + M*N f32 outputs
    assert LS.algorithmic_bytes(1, 4096, 4096, 0) == 4096 * 4096 + 4 + 2 * 4096 + 4 * 4096
    assert LS.algorithmic_bytes(8, 4096, 11008, 32) == (4096 * 11008 + 4 * 4096 * 11008 // 32 + 2 * 8 * 4096
                                                        + 4 * 8 * 11008)
    assert LS.algorithmic_bytes(128, 11008, 4096, 64) == (11008 * 4096 + 4 * 11008 * 4096 // 64
                                                          + 2 * 128 * 11008 + 4 * 128 * 4096)


def test_cpu_reference_leg_times_whole_steps():
    # a small shape: every layer and the lm_head of each timed step
    shape = LlamaConfig(2048, 256, 512, 2, 4, 2, 64, 1e-5, 10000.0, False, None)
    tok_s, cores, n, sample = bench.cpu_reference_decode(shape, 16, 1, 3)
    assert n == 3 and tok_s > 0 and cores >= 1
    assert "all 2 layers + lm_head" in sample and "contexts 16-19" in sample


def test_step_timeline_summary():
    # A synthetic 1-layer timeline of two CTAs, CTA 1 100 ns behind CTA 0:
    # every phase starts 2 us after the CTA's previous phase ended, spends
    # 3 us on its input stage and 5 us on its work, with the first and last
    # weight stages ready 0.5 and 1.5 us after the input stage.
    import numpy as np

    from esolearn_b200.profile_decode import PHASES, timeline_summary

    P, C = 7, 2  # six phases per layer + lm_head
    t = np.zeros((P, C, 5), dtype=np.int64)
    for p in range(P):
        for c in range(C):
            t[p, c, 0] = 100 * c if p == 0 else t[p - 1, c, 4] + 2000
            t[p, c, 1] = t[p, c, 0] + 3000
            t[p, c, 2] = t[p, c, 1] + 500
            t[p, c, 3] = t[p, c, 1] + 1500
            t[p, c, 4] = t[p, c, 1] + 5000
    r = timeline_summary(t, 1)
    assert PHASES[0] not in r  # the first phase has no barrier before it
    for name in list(PHASES[1:]) + ["lm_head"]:
        got = r[name]
        want = {"barrier": 2.0, "input": 3.0, "work": 5.0, "span": 10.0, "barrier_propagation": 1.9,
                "arrival_lag": 0.05, "start_spread": 0.1, "first_ready": 0.5, "last_ready": 1.5, "after_last": 3.5}
        for k, v in want.items():
            assert abs(got[k] - v) < 1e-9, (name, k, got[k])
    assert abs(r["layers_total"] - 58.1) < 1e-9 and abs(r["per_layer"] - 58.1) < 1e-9
    assert abs(r["step_to_lm_end"] - 68.1) < 1e-9
