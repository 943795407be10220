"""Standalone quantized-linear sweep: matmul_i8_f32 (backend/mod.rs:521-533)
timed on the device for every cell of the sweep configuration.

Inputs follow the sweep's definition: int8 weights uniform in [-127, 127];
f32 scales per group of 32 or 64 input rows equal to absmax/127 of N(0, 0.02)
source groups (group 0 = one per-tensor scale, the engine's format, packed in
128-column tiles; grouped weights are packed in the GEMV's own tile width for
1-4 rows and in 128-column tiles, which run on the tensor cores, for 5+); bf16 activations
~ N(0, 1); M in {1, 8, 32, 128}; (K, N) in {(4096, 4096), (4096, 11008),
(11008, 4096), (4096, 32000)}; f32 output.

Each cell: 3 warm-up calls, then `iters` calls, each preceded by a 256 MB
write that evicts L2 (126 MB) and a ~0.5 ms device spin during which the host
enqueues the call, timed with CUDA events on the launching stream (the median
is reported).  Algorithmic bytes per call = K*N (int8) + 4*K*N/g
(group scales) + 2*M*K (bf16 in) + 4*M*N (f32 out); FLOPs = 2*M*K*N.  GB/s is
reported against the measured HBM copy bandwidth when a peaks file is given.

    python -m esolearn_b200.linear_sweep [--iters 10] [--peaks MEASURED_PEAKS.json] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from . import _native as N
from .llama import QWeight, matmul_i8_f32

SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 32000)]
ROWS = [1, 8, 32, 128]
GROUPS = [0, 32, 64]


def make_weight(K: int, N_: int, group: int, seed: int, tile_n: int = 128):
    """The sweep's weight for one (K, N, group) cell (QWeight, or a dict of
    them by tile width when tile_n is a tuple)."""
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, (K, N_), dtype=np.int8)
    if group == 0:
        src = rng.standard_normal((K, N_), dtype=np.float32) * np.float32(0.02)
        scales = [np.float32(np.abs(src).max() / np.float32(127.0))]
    else:
        scales = np.empty((K // group, N_), np.float32)
        for g in range(K // group):  # one group of source rows at a time keeps host memory small
            src = rng.standard_normal((group, N_), dtype=np.float32) * np.float32(0.02)
            scales[g] = np.abs(src).max(axis=0) / np.float32(127.0)
    if isinstance(tile_n, tuple):
        return {tn: QWeight(q, scales, group=group, tile_n=tn) for tn in tile_n}
    return QWeight(q, scales, group=group, tile_n=tile_n)


def algorithmic_bytes(M: int, K: int, N_: int, group: int) -> int:
    scale_bytes = 4 * K * N_ // group if group else 4
    return K * N_ + scale_bytes + 2 * M * K + 4 * M * N_


def time_cell(qw: QWeight, M: int, iters: int, flush) -> float:
    """Median device time (s) of one M-row call, L2 flushed before each."""
    import torch

    a = torch.randn(M, qw.K, generator=torch.Generator().manual_seed(M + qw.K)).to(torch.bfloat16).cuda()
    out = torch.empty((M, qw.N), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(3):
        matmul_i8_f32(a, qw, out=out, stream=st.cuda_stream)
    times = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(iters):
        flush.zero_()
        # Keep the GPU busy (~0.5 ms) while the host enqueues the timed call,
        # so the start event does not also time the host's launch path.
        torch.cuda._sleep(1_000_000)
        e0.record(st)
        matmul_i8_f32(a, qw, out=out, stream=st.cuda_stream)
        e1.record(st)
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e-3)
    torch.cuda.synchronize()
    return float(np.median(times))


def run(iters: int = 10, peak_gbs: float | None = None, shapes=SHAPES, rows=ROWS, groups=GROUPS):
    import torch

    N.check(N.lib().sb_init(torch.cuda.current_device()))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    results = []
    for (K, N_) in shapes:
        for group in groups:
            # per-tensor: the engine's 128-column packing; grouped: the GEMV's
            # own tile width for 1-4 rows, 128-column tiles (tensor cores) beyond
            tns = (128,) if group == 0 else (0, 128)
            qws = make_weight(K, N_, group, seed=K * 7 + N_ + group, tile_n=tns)
            for M in rows:
                qw = qws[128] if (group == 0 or M > 4) else qws[0]
                t = time_cell(qw, M, iters, flush)
                b = algorithmic_bytes(M, K, N_, group)
                r = {"K": K, "N": N_, "group": group, "M": M, "us": t * 1e6, "gbs": b / t / 1e9,
                     "tflops": 2.0 * M * K * N_ / t / 1e12}
                if peak_gbs:
                    r["hbm_frac"] = r["gbs"] / peak_gbs
                results.append(r)
            del qws, qw
    return results


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--peaks", default=os.path.join(os.path.dirname(os.path.dirname(__file__)), "MEASURED_PEAKS.json"))
    ap.add_argument("--json", default=None, help="also write the results here")
    ap.add_argument("--rows", type=int, nargs="+", default=ROWS, help="M values (default: 1 8 32 128)")
    ap.add_argument("--groups", type=int, nargs="+", default=GROUPS, help="0 = per-tensor, 32, 64")
    ap.add_argument("--shapes", nargs="+", default=[f"{k}x{n}" for k, n in SHAPES], help="KxN, e.g. 4096x11008")
    args = ap.parse_args()
    shapes = [tuple(int(v) for v in sh.lower().split("x")) for sh in args.shapes]
    peak = None
    if args.peaks and os.path.exists(args.peaks):
        with open(args.peaks) as f:
            peak = float(json.load(f).get("hbm_gbs") or 0) or None
    res = run(args.iters, peak, shapes=shapes, rows=args.rows, groups=args.groups)
    print("| K | N | group | M | µs | GB/s | frac of measured HBM | TFLOP/s |")
    print("|---|---|---|---|---|---|---|---|")
    for r in res:
        frac = f"{r['hbm_frac']:.2f}" if "hbm_frac" in r else "-"
        print(f"| {r['K']} | {r['N']} | {r['group']} | {r['M']} | {r['us']:.1f} | {r['gbs']:.0f} | {frac} | "
              f"{r['tflops']:.2f} |")
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"peak_hbm_gbs": peak, "cells": res}, f, indent=1)


if __name__ == "__main__":
    main()
