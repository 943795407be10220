"""Fixed decode workload for kernel profilers (ncu launch lists and captures).

Builds the llama2-7b-shape int8 model (random init on the device, the same
weights the benchmark uses), optionally with fewer layers, and runs `--steps`
decode steps of `--batch` sequences at context position `--ctx` through
sb_llama_forward, i.e. one replay of the step's CUDA graph per call.  No
prefill is run: the cache rows below `--ctx` hold whatever the engine
initialised them to, which does not change the work any kernel does.

Kernel launches per step: embed, then per layer qkv, attention, o,
gate/up, down, then lm_head and the argmax step (3 + 5 * layers).  The first
call also runs one eager warm-up step before it captures the graph, so a
profiler that should see decode steps at `--ctx` skips one step's launches.

    python -m esolearn_b200.profile_decode --ctx 584 --steps 2
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import time

from . import _native as N
from .llama import LlamaConfig, QuantLlamaB200


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--layers", type=int, default=0, help="layer count (0: the full 32)")
    ap.add_argument("--ctx", type=int, default=584, help="position decoded (context length - 1)")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)

    cfg = LlamaConfig.llama2_7b_shape()
    if args.layers:
        cfg = dataclasses.replace(cfg, n_layers=args.layers)
    N.check(N.lib().sb_init(args.device))
    model = QuantLlamaB200.new_random(cfg, seed=0, max_seq=args.ctx + args.steps + 8, max_batch=args.batch)
    B = args.batch
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        model.forward_batch([1] * B, [args.ctx + i] * B, want_logits=False)
        times.append((time.perf_counter() - t0) * 1e3)
    print(json.dumps({"layers": cfg.n_layers, "batch": B, "ctx": args.ctx, "steps": args.steps,
                      "launches_per_step": 3 + 5 * cfg.n_layers, "host_ms_per_call": times}))


if __name__ == "__main__":
    main()
