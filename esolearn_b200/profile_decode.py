"""Fixed decode workload for kernel profilers (ncu launch lists and captures).

Builds a benchmark-shape int8 model (random init on the device, the same
weights the benchmark uses: --shape llama2_7b_shape or llama3_8b_shape),
optionally with fewer layers, and runs `--steps` decode steps of `--batch`
sequences at context position `--ctx` through sb_llama_forward, i.e. one
replay of the step's CUDA graph per call (one persistent-kernel launch at
batch 1).  No prefill is run: the cache rows below `--ctx` hold whatever the
engine initialised them to, which does not change the work any kernel does.

The first call of a graph-driven batch also runs one eager warm-up step
before it captures the graph, so a profiler that should see decode steps at
`--ctx` skips one step's launches (printed as launches_per_step).

    python -m esolearn_b200.profile_decode --ctx 584 --steps 2
    python -m esolearn_b200.profile_decode --shape llama3_8b_shape --batch 32 --layers 2 --ctx 2068
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
    ap.add_argument("--shape", default="llama2_7b_shape", choices=["llama2_7b_shape", "llama3_8b_shape"])
    ap.add_argument("--layers", type=int, default=0, help="layer count (0: the shape's own)")
    ap.add_argument("--ctx", type=int, default=584, help="position decoded (context length - 1)")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)

    cfg = getattr(LlamaConfig, args.shape)()
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
    print(json.dumps({"shape": args.shape, "layers": cfg.n_layers, "batch": B, "ctx": args.ctx, "steps": args.steps,
                      "launches_per_step": model.step_launches(B), "host_ms_per_call": times}))


if __name__ == "__main__":
    main()
