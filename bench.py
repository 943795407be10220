"""Decode throughput of the B200 int8 Llama engine (one JSON line on rank 0).

Default workload: Llama-2-7B-shape random-init int8
model (dim 4096, 32 layers, 32 heads, ffn 11008, vocab 32000, RoPE theta 1e4),
seeded 512-token prompt, then greedy decode at batch 1.  --workload
llama3-8b-bs32: Llama-3-8B shape with GQA (32 query /
8 KV heads, ffn 14336, vocab 128256, theta 5e5), 32 sequences with seeded
2048-token prompts.  --workload llama3-70b-bs64:
Llama-3-70B shape (dim 8192, 80 layers, 64 query / 8 KV heads, ffn 28672),
64 sequences with seeded 1024-token prompts.  A step is one decode token of
every sequence: K timed steps follow the prompt and W warm-up steps.

* value      -- decode tokens/s with weights and KV resident in HBM (CUDA
                events on the engine stream around K steps; at batch 1 each
                step is one launch of the persistent decode-step kernel).
* e2e        -- the same metric through the reference-facing C-ABI call
                sb_llama_forward (token id from pinned host memory in, argmax
                token id back to the host, every step).
* roofline   -- HBM bound.  Batch 1: the algorithmic bytes of one launch of
                the persistent step kernel (all int8 weights + the K/V rows
                of the context) divided by its average launch duration (the
                timed region above), against MEASURED_PEAKS.json.  Larger
                batches run a CUDA graph of per-operation kernels (GEMV up to
                4 rows, the tcgen05 GEMM for 5-32): the same step bytes over
                the step time, with the eager per-kernel-class split (linears,
                attention) beside it.
                traffic -- DRAM bytes of one launch from an ncu capture
                (profiles/decode_step_7b_bs1_traffic.json).
* cpu_baseline -- the reference's CPU path (the oracle restatement of
                cpu.rs, every layer of the workload's shape, one sequence)
                timed on this host's cores: 1 warm-up + up to 4 timed steps
                at the workload's context.
* extra      -- (1 GPU, default workload) the metric's other parts measured
                in the same run: "bs32", the Llama-3-8B-shape batch-32 decode
                with 2048-token contexts (value, roofline, e2e, clocks), and
                "quant_linear_sweep", GB/s of every configs[1] cell
                (M in {1, 8, 32, 128}, per-tensor and group-32 scales).

--impl reference times that CPU path alone: W warm-up and K timed decode
steps of the full model (stopped early, and the step count reported, if the
timed loop passes 150 s).  The reference is Rust and cannot be built here;
the oracle restates it operation by operation.
Multi-GPU (torchrun, N ranks): tensor parallelism over the N GPUs -- every
rank holds 1/N of every projection and of the KV heads.  At batch 1 each
rank runs the persistent step kernel, which sums the partial o and down
products and picks the greedy token (the argmax over all ranks' vocabulary
slices) through stores into the other GPUs' memory over NVLink inside the
kernel; larger batches run the per-operation graph with a peer all-reduce
after o and down.  The workload (model,
batch, prompt) is the same at every N ("scaling": "strong"); value is the
job's tokens/s from the slowest rank's CUDA-event time.  --replicas runs N
independent single-GPU replicas instead (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 512
PREFILL_ROWS = 64

WORKLOADS = {
    "llama2-7b-bs1": {"metric": "decode tok/s, 7B-shape int8, bs1", "shape": "llama2_7b_shape", "batch": 1,
                      "prompt": 512, "desc": "llama2-7b-shape int8 decode (BASELINE configs[2])"},
    "llama3-8b-bs32": {"metric": "decode tok/s, 8B-shape GQA int8, bs32", "shape": "llama3_8b_shape", "batch": 32,
                       "prompt": 2048,
                       "desc": "llama3-8b-shape GQA int8 decode, 2048-token bf16 KV context (BASELINE configs[3])"},
    "llama3-70b-bs64": {"metric": "decode tok/s, 70B-shape GQA int8, bs64", "shape": "llama3_70b_shape", "batch": 64,
                        "prompt": 1024,
                        "desc": "llama3-70b-shape GQA int8 decode, 1024-token bf16 KV context (BASELINE configs[4])"},
}


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def read_traffic():
    p = os.path.join(ROOT, "profiles", "decode_step_7b_bs1_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


class ClockSampler:
    """nvidia-smi samples (timestamped) while the timed region runs."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            rows.append((ts, parts))
        inside = [r for r in rows if t0 - 0.15 <= r[0] <= t1 + 0.15] or rows[-3:]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(p[2]) for _, p in inside if p[2].replace(".", "").isdigit()]
        mx = [float(p[3]) for _, p in inside if p[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, p in inside for i in range(4) if p[6 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside)}


def cpu_reference_decode(shape, context: int, warmup: int, steps: int, budget_s: float | None = None):
    """The reference CPU decode (the oracle's operation-by-operation
    restatement of cpu.rs, every layer of the workload's shape) timed on this
    host with all its threads: `warmup` untimed then `steps` timed
    forward_with_cache calls of one sequence at contexts context .. context +
    warmup + steps - 1, greedy-fed.  The K/V cache is filled to `context`
    positions with seeded values instead of running the prompt (the decode
    cost depends on the context length only), and the int8 weights are seeded
    uniform values (the cost does not depend on them).  budget_s stops the
    timed loop early (at least one step).  The reference decodes one sequence
    at a time, so its tok/s is the same at any batch.
    Returns (tok/s, cores, steps timed, sample description)."""
    import oracle as O

    cores = os.cpu_count() or 1
    O.set_threads(cores)
    V, h, F = shape.vocab_size, shape.hidden_size, shape.intermediate_size
    max_seq = context + warmup + steps + 1
    cfg = O.make_config(V, h, F, shape.n_layers, shape.n_heads, shape.n_kv_heads, max_seq, 1e-5, shape.rope_theta,
                        False)
    m = O.OracleLlama(cfg, 0, uniform=True)
    cache = m.new_cache(max_seq, kv_bf16=False)  # the reference's f32 cache
    cache.fill(context, 1)
    tok, pos = 1, context
    for _ in range(warmup):
        tok = O.argmax(m.forward_with_cache(cache, tok, pos))
        pos += 1
    n = 0
    t0 = time.perf_counter()
    while n < steps:
        tok = O.argmax(m.forward_with_cache(cache, tok, pos))
        pos += 1
        n += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    del cache, m
    sample = (f"h{h}/ffn{F}/vocab{V}, all {shape.n_layers} layers + lm_head, {n} timed decode steps after {warmup} "
              f"warm-up at contexts {context}-{pos - 1} (f32 cache), one sequence, {cores} OpenMP threads")
    return n / dt, cores, n, sample


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    from esolearn_b200 import LlamaConfig

    wl = WORKLOADS[args.workload]
    shape = getattr(LlamaConfig, wl["shape"])()
    # bounded so the whole run stays within a few minutes at any shape
    tok_s, cores, n, sample = cpu_reference_decode(shape, args.prompt, args.warmup, args.steps, budget_s=150.0)
    print(json.dumps({
        "impl": "reference", "metric": wl["metric"], "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": n, "warmup": args.warmup, "ms_per_step": 1000.0 / tok_s, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights, f32 activations", "data": "synthetic",
        "config": {"workload": wl["desc"] + " (reference CPU path; one sequence at a time)",
                   "batch": args.batch, "prompt": args.prompt, "context": [args.prompt, args.prompt + args.warmup + n - 1]},
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def measure_decode(wl_name: str, B: int, prompt: int, K: int, W: int, rank: int, world: int, dist, replicas: bool,
                   want_e2e: bool = True, sample_clocks: bool = True):
    """Decode throughput of one workload: build the seeded model on the device,
    prefill the prompts, W warm-up steps, then K timed steps (CUDA events on the
    engine stream, max over ranks) and K steps through sb_llama_forward with
    host buffers (e2e).  Returns the pieces of the JSON line (same on every
    rank after the max-reductions)."""
    import torch

    from esolearn_b200 import LlamaConfig, QuantLlamaB200

    local = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[wl_name]
    cfg = getattr(LlamaConfig, wl["shape"])()
    max_seq = prompt + W + K + 8
    tp = world if (world > 1 and not replicas) else 1
    tp_kw = {}
    if tp > 1:
        from esolearn_b200 import tp_unique_id

        obj = [tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp_kw = {"tp_rank": rank, "tp_size": tp, "tp_id": obj[0]}
    # rows per step: the decoded batch, and up to 64 prompt positions per
    # batched-prefill step (the tensor-core linears take 5-64 rows)
    rows = max(B, PREFILL_ROWS)
    model = QuantLlamaB200.new_random(cfg, seed=0, max_seq=max_seq, max_batch=rows, kv_dtype="bf16", **tp_kw)
    # tensor-parallel ranks decode the same sequences; replicas decode their own
    rng = np.random.default_rng(1000 + (0 if tp > 1 else rank))
    prompts = rng.integers(0, cfg.vocab_size, (B, prompt), dtype=np.int64).astype(np.int32)
    # batched prefill of the prompts (host-timed, includes its syncs), then warm-up steps
    n_warm = min(prompt, rows + prompt % rows)  # every chunk shape the timed prefill uses
    model.prefill(prompts[:, :n_warm])  # captures the step graphs outside the timed prefill
    torch.cuda.synchronize()
    t_pf0 = time.perf_counter()
    model.prefill(prompts)
    t_pf1 = time.perf_counter()
    prefill = {"tok_s": B * prompt / (t_pf1 - t_pf0), "tokens": B * prompt, "ms": (t_pf1 - t_pf0) * 1e3,
               "positions_per_step": rows, "timing": "host wall clock around sb_llama_prefill (synchronous)"}
    model.step(W)
    st = torch.cuda.ExternalStream(model.stream())
    torch.cuda.synchronize()

    clocks = None
    if sample_clocks:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        smi_index = int(vis.split(",")[local]) if vis and vis.split(",")[local].strip().isdigit() else local
        clocks = ClockSampler(smi_index)
        clocks.start()
        time.sleep(0.3)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(st)
    model.step(K)
    e1.record(st)
    e1.synchronize()
    t_wall1 = time.time()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clk = None
    if clocks is not None:
        clk = clocks.summary(t_wall0, t_wall1)
        clocks.stop()
    ctx_mid = prompt + W + K / 2
    wbytes, kv_per_pos = model.step_bytes()
    n_jobs = 1 if tp > 1 else world  # independent decode jobs in the run
    value = n_jobs * B * K / (ms / 1000.0)
    launches_per_step = model.step_launches(B)
    peak, peak_kind = read_peaks()
    step_alg_bytes = wbytes + kv_per_pos * ctx_mid * B
    achieved = step_alg_bytes / (ms / K / 1000.0) / 1e9
    if launches_per_step == 1:
        # one persistent kernel per step: its average launch duration is the step time
        traffic = read_traffic()
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": peak_kind, "kernel": "decode_step_kernel (persistent: every projection + attention)",
                "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
                "traffic_context": traffic.get("context") if traffic else None,
                "algorithmic_bytes_per_launch": step_alg_bytes, "launch_ms": ms / K}
    else:
        # CUDA graph of per-operation kernels: the step bytes over the step
        # time, and an eager pass with one CUDA event pair per kernel class
        prof = [model.profile_step() for _ in range(4)]
        lin_ms = float(np.median([p[0] for p in prof]))
        att_ms = float(np.median([p[1] for p in prof]))
        lin_kernel = "qgm_gemm_kernel (tcgen05)" if B > 4 else "qgemv_kernel"
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": peak_kind, "kernel": f"whole step: {lin_kernel} linears + attention",
                "traffic": None, "algorithmic_bytes_per_step": step_alg_bytes, "step_ms": ms / K,
                "linears": {"bytes": wbytes, "eager_ms": lin_ms, "gbs": wbytes / (lin_ms / 1000.0) / 1e9},
                "attention": {"bytes": kv_per_pos * ctx_mid * B, "eager_ms": att_ms,
                              "gbs": kv_per_pos * ctx_mid * B / (att_ms / 1000.0) / 1e9}}

    # e2e: reference-facing call with host buffers every step (tokens in, argmax out)
    e2e = None
    if want_e2e:
        # Re-decode the timed positions (each step rewrites its own KV row
        # before reading the context), so every e2e step sees the same
        # context length as the matching timed step.
        toks = model.tokens(B, max_seq)
        last = toks[:, -1].copy() if toks.shape[1] else np.zeros(B, np.int32)
        p0 = prompt + W
        pinned_tok = torch.empty(B, dtype=torch.int32).pin_memory()
        for i in range(3):
            model.forward_batch(last.tolist(), [p0 - 3 + i] * B, want_logits=False)
        t0 = time.perf_counter()
        for i in range(K):
            pinned_tok.numpy()[:] = last
            _, am = model.forward_batch(pinned_tok.numpy(), [p0 + i] * B, want_logits=False)
            last = am
        t1 = time.perf_counter()
        e2e_s = t1 - t0
        if dist is not None:
            tt = torch.tensor([e2e_s], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_s = float(tt.item())
        # batch 1 (the persistent step): token and position travel as launch
        # arguments; batches: token, position and prompt length copied per row
        e2e = {"value": n_jobs * B * K / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 8 if B == 1 else 12 * B,
               "d2h_bytes_per_step": 4 * B, "steps": K,
               "api": "sb_llama_forward (token, position in; argmax out; stream-synchronous)"}
    model.close()
    del model
    torch.cuda.synchronize()
    return {"cfg": cfg, "tp": tp, "value": value, "ms": ms, "ctx_mid": ctx_mid, "wbytes": wbytes,
            "launches_per_step": launches_per_step, "prefill": prefill, "roofline": roof, "clocks": clk, "e2e": e2e}


def quant_linear_sweep_summary(iters: int = 5):
    """The quantized-linear sweep on this GPU, compact:
    GB/s (fraction of measured HBM) per (K, N, group, M) cell, M in {1, 8, 32,
    128}, per-tensor scale and groups 32 and 64."""
    from esolearn_b200 import linear_sweep

    peak, kind = read_peaks()
    cells = linear_sweep.run(iters=iters, peak_gbs=peak, groups=[0, 32, 64])
    out = {"timing": f"CUDA events, L2 flushed before each call, median of {iters}",
           "bytes": "K*N int8 + 4*K*N/g scales + 2*M*K bf16 in + 4*M*N f32 out", "peak_gbs": peak,
           "peak_source": kind, "cells": []}
    for r in cells:
        out["cells"].append({"K": r["K"], "N": r["N"], "group": r["group"], "M": r["M"], "us": round(r["us"], 2),
                             "gbs": round(r["gbs"], 1), "frac": round(r["gbs"] / peak, 3),
                             "tflops": round(r["tflops"], 2)})
    return out


def run_ours(args, rank: int, world: int, dist):
    import torch

    from esolearn_b200 import _native as N

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    N.check(N.lib().sb_init(local))
    wl = WORKLOADS[args.workload]
    B, K, W = args.batch, args.steps, args.warmup
    r = measure_decode(args.workload, B, args.prompt, K, W, rank, world, dist, args.replicas, not args.no_e2e)
    tp = r["tp"]
    extra = {}
    if world == 1 and not args.no_extra and args.workload == "llama2-7b-bs1":
        # the metric's other parts, on the same GPU in the same run: batch 32
        # (8B-shape GQA, 2048-token contexts) and the quantized-linear sweep
        wl32 = WORKLOADS["llama3-8b-bs32"]
        r32 = measure_decode("llama3-8b-bs32", wl32["batch"], wl32["prompt"], K, W, rank, world, dist, False, True,
                             sample_clocks=True)
        extra["bs32"] = {"metric": wl32["metric"], "value": r32["value"], "unit": "tok/s",
                         "ms_per_step": r32["ms"] / K, "steps": K, "warmup": W,
                         "config": {"workload": wl32["desc"], "batch": wl32["batch"], "prompt": wl32["prompt"],
                                    "context_mid": r32["ctx_mid"]},
                         "gpu_launches": r32["launches_per_step"] * K, "prefill": r32["prefill"],
                         "roofline": r32["roofline"], "e2e": r32["e2e"], "clocks": r32["clocks"]}
        extra["quant_linear_sweep"] = quant_linear_sweep_summary()
    if rank != 0:
        return
    res = {
        "metric": wl["metric"], "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": r["ms"] / K, "higher_is_better": True, "scaling": "strong" if tp > 1 else "weak",
        "vs_baseline": None,
        "dtype": "int8 weights x f32 activations (exact int32 dp4a products), f32 accumulate; bf16 KV",
        "data": "synthetic: seeded random-init weights (fastrand/Box-Muller N(0,0.02), LlamaModel::new order), "
                "seeded uniform prompt ids",
        "config": {"workload": wl["desc"], "batch": B, "prompt": args.prompt,
                   "context_mid": r["ctx_mid"],
                   "parallelism": (f"tp{tp} (one-shot peer all-reduce over NVLink after o and down)" if tp > 1 else
                                   f"replicas x{world}" if world > 1 else "single GPU"),
                   "l2": f"weights {r['wbytes'] / 1e9:.1f} GB per step >> 126 MB L2 (no flush needed)",
                   "kv_dtype": "bf16",
                   "launch": ("one persistent cooperative kernel per step" if r["launches_per_step"] == 1 else
                              "CUDA graph of per-operation kernels per step, programmatic dependent launch")},
        "gpu_launches": r["launches_per_step"] * K,
        "prefill": r["prefill"],
        "roofline": r["roofline"],
        "clocks": r["clocks"],
    }
    if r["e2e"]:
        res["e2e"] = r["e2e"]
    if not args.no_cpu:
        # bounded sample of the reference CPU path: the full model, 1 warm-up
        # and up to 4 timed steps at the workload's context
        tok_s, cores, n, sample = cpu_reference_decode(r["cfg"], args.prompt, 1, 4, budget_s=30.0)
        res["cpu_baseline"] = {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}
    if extra:
        res["extra"] = extra
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama2-7b-bs1", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=None, help="sequences (default: the workload's)")
    ap.add_argument("--prompt", type=int, default=None, help="prompt length (default: the workload's)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the bs32 workload and the linear sweep (N=1)")
    ap.add_argument("--replicas", action="store_true", help="N>1: independent replicas instead of tensor parallelism")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    args.batch = wl["batch"] if args.batch is None else args.batch
    args.prompt = wl["prompt"] if args.prompt is None else args.prompt
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
