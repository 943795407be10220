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
    python -m esolearn_b200.profile_decode --ctx 584 --steps 4 --timeline
    torchrun --nproc-per-node 2 -m esolearn_b200.profile_decode --timeline   (tensor parallel, one rank per GPU)

--timeline (batch 1, persistent step; needs the profiling build of the
library, `SB_STEP_TIMELINE=1 python -m esolearn_b200.build --force`) records the step kernel's per-phase
%globaltimer stamps (sb_llama_set_timeline) in the last step and prints, per
phase kind, the mean over layers of: the grid-barrier wait (a CTA's end of the
previous phase to its start of this one, mean over CTAs), the input stage and
the work (mean over CTAs), and the phase's span on the critical path (last
arrival of the previous phase to last arrival of this one), in microseconds.
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
    ap.add_argument("--timeline", action="store_true", help="per-phase timeline of the last persistent step")
    ap.add_argument("--timeline-out", default=None, help="also save the raw stamps [phases, ctas, 5] (.npy)")
    ap.add_argument("--prefill", type=int, default=0,
                    help="instead of decode steps: prefill one prompt of this many seeded tokens (chunks of --batch)")
    args = ap.parse_args(argv)

    cfg = getattr(LlamaConfig, args.shape)()
    if args.layers:
        cfg = dataclasses.replace(cfg, n_layers=args.layers)
    # under torchrun: tensor parallelism over the ranks (one GPU each)
    import os

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    tp_kw = {}
    if world > 1:
        import torch.distributed as dist

        from .llama import tp_unique_id

        args.device = int(os.environ.get("LOCAL_RANK", "0"))
        dist.init_process_group("gloo")
        obj = [tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp_kw = {"tp_rank": rank, "tp_size": world, "tp_id": obj[0]}
    N.check(N.lib().sb_init(args.device))
    max_seq = max(args.ctx + args.steps, args.prefill) + 8
    model = QuantLlamaB200.new_random(cfg, seed=0, max_seq=max_seq, max_batch=args.batch, **tp_kw)
    B = args.batch
    if args.prefill:
        import numpy as np

        prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (1, args.prefill)).astype(np.int32)
        t0 = time.perf_counter()
        model.prefill(prompt)
        print(json.dumps({"shape": args.shape, "layers": cfg.n_layers, "prefill": args.prefill, "chunk": B,
                          "host_ms": (time.perf_counter() - t0) * 1e3}))
        return
    if args.timeline:
        model.set_timeline(True)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        model.forward_batch([1] * B, [args.ctx + i] * B, want_logits=False)
        times.append((time.perf_counter() - t0) * 1e3)
    out = {"shape": args.shape, "layers": cfg.n_layers, "batch": B, "ctx": args.ctx, "steps": args.steps,
           "tp": world, "rank": rank, "launches_per_step": model.step_launches(B), "host_ms_per_call": times}
    if args.timeline:
        ts = model.timeline()
        out["timeline_us"] = timeline_summary(ts, cfg.n_layers)
        if args.timeline_out:
            import numpy as np

            np.save(args.timeline_out if world == 1 else f"{args.timeline_out}.rank{rank}.npy", ts)
    print(json.dumps(out))
    if world > 1:
        model.close()
        import torch.distributed as dist

        dist.destroy_process_group()


PHASES = ("qkv", "attention", "o", "gate_up", "swiglu", "down")


def timeline_summary(ts, n_layers: int) -> dict:
    """Per-phase-kind means (us) of a step timeline [phases, ctas, 5] (ns)."""
    import numpy as np

    t = ts.astype(np.float64)
    P = t.shape[0]
    res = {}
    kinds = [(k, [6 * l + i for l in range(n_layers)]) for i, k in enumerate(PHASES)]
    kinds.append(("lm_head", [6 * n_layers]))
    for name, idx in kinds:
        wait, inp, work, span, r0, r1, tail = [], [], [], [], [], [], []
        prop, lag, spread = [], [], []
        for p in idx:
            if p == 0 or p >= P:
                continue
            wait.append(np.mean(t[p, :, 0] - t[p - 1, :, 4]))
            # the grid barrier before phase p: last arrival -> first start
            # (propagation), last arrival - median arrival (imbalance), and
            # the spread of the start stamps
            prop.append(t[p, :, 0].min() - t[p - 1, :, 4].max())
            lag.append(t[p - 1, :, 4].max() - np.median(t[p - 1, :, 4]))
            spread.append(t[p, :, 0].max() - t[p, :, 0].min())
            inp.append(np.mean(t[p, :, 1] - t[p, :, 0]))
            work.append(np.mean(t[p, :, 4] - t[p, :, 1]))
            span.append(np.max(t[p, :, 4]) - np.max(t[p - 1, :, 4]))
            g = t[p, :, 2] > 0  # CTAs with weight stages in this phase
            if g.any():
                r0.append(np.mean(t[p, g, 2] - t[p, g, 1]))
                r1.append(np.mean(t[p, g, 3] - t[p, g, 1]))
                tail.append(np.mean(t[p, g, 4] - t[p, g, 3]))
        if span:
            res[name] = {"barrier": np.mean(wait) / 1e3, "input": np.mean(inp) / 1e3, "work": np.mean(work) / 1e3,
                         "span": np.mean(span) / 1e3, "barrier_propagation": np.mean(prop) / 1e3,
                         "arrival_lag": np.mean(lag) / 1e3, "start_spread": np.mean(spread) / 1e3}
            if r0:  # input done -> first / last weight stage ready, last stage ready -> phase end
                res[name].update({"first_ready": np.mean(r0) / 1e3, "last_ready": np.mean(r1) / 1e3,
                                  "after_last": np.mean(tail) / 1e3})
    first, last = t[0, :, 0].min(), t[6 * n_layers, :, 4].max()
    res["layers_total"] = (t[6 * n_layers - 1, :, 4].max() - first) / 1e3
    res["per_layer"] = res["layers_total"] / n_layers
    res["step_to_lm_end"] = (last - first) / 1e3
    return res


if __name__ == "__main__":
    main()
