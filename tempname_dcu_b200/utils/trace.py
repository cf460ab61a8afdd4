"""Kernel-time breakdown of training micro-steps (torch.profiler / CUPTI).

    python -m tempname_dcu_b200.utils.trace [--layers L] [--micro 1 | --step] [--chrome out.json] [--ranges]

Runs warm-up micro-steps, then profiles ``--micro`` micro-batches of the GPT
training step and prints the device time per kernel name (sum, count, share),
plus the total device time and the host wall time of the profiled region.
The chrome trace (optional) shows the overlap of streams.  Numbers taken under
the profiler are for shares only, never benchmark values.

Reference parity: the reference records torch.profiler chrome traces per
operator role (python/flux_dcu/worker.py:317-325) and operator event rows
(runtime.py:270-292).
"""
from __future__ import annotations

import argparse
import collections
import json
import time


# Kernel-name buckets for the per-category summary (first match wins).
CATEGORIES = (
    ("fused GEMM -> reduce-scatter", ("gemm_rs_kernel", "gemm_rs_mx_kernel", "rs_reduce_kernel", "rs_advance")),
    ("fused all-gather -> GEMM", ("ag_gemm", "ag_pull", "ag_stage", "ag_advance", "push_advance")),
    ("GEMM (tcgen05)", ("gemm_kernel", "gemm2_kernel", "gemm_mx_kernel")),
    ("attention", ("attn",)),
    ("NCCL", ("nccl",)),
    ("LayerNorm / reductions", ("layernorm", "ln_", "colred", "colsum")),
    ("cross-entropy", ("xent",)),
    ("optimizer", ("adamw", "clip", "norm")),
    ("embedding", ("embedding", "emb::", "embx::", "position", "sort_tokens")),
)


def categorize(kernels):
    """{category: (microseconds, launches)} for [{"name", "us", "count"}]."""
    out = {}
    for k in kernels:
        name = k["name"].lower()
        cat = next((c for c, keys in CATEGORIES if any(key.lower() in name for key in keys)), "other")
        us, n = out.get(cat, (0.0, 0))
        out[cat] = (us + k["us"], n + k["count"])
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--micro", type=int, default=1)
    ap.add_argument("--chrome", default="")
    ap.add_argument("--json", default="")
    ap.add_argument("--step", action="store_true", help="profile one whole optimizer step instead")
    ap.add_argument("--arm", default="flux", help="tensor-parallel arm when launched with torchrun (WORLD_SIZE > 1)")
    ap.add_argument("--graph", action="store_true", help="capture the step as a CUDA graph and profile a replay")
    ap.add_argument("--ranges", action="store_true",
                    help="name every layer's forward / backward (profiler + NVTX ranges) and print their host times")
    args = ap.parse_args(argv)
    import os
    import torch
    from torch.profiler import ProfilerActivity, profile
    from ..models.config import BENCH_CONFIG
    from ..train import Trainer, synthetic_batches
    cfg = dict(BENCH_CONFIG, layers=args.layers)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    group, factory, rank = None, None, 0
    if world > 1:  # one rank per GPU under torchrun; rank 0 prints
        import datetime
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        group, rank = dist.group.WORLD, dist.get_rank()
        if args.arm != "nccl":
            from ..runtime import operator_factory_for
            factory = operator_factory_for(args.arm)
    trainer = Trainer(cfg, args.arm if args.arm != "nccl" else "flux", group, operator_factory=factory,
                      cuda_graph=args.graph, graph_warmup=1)
    (tokens, labels), = synthetic_batches(trainer.config, 1)
    tokens, labels = tokens.cuda(), labels.cuda()
    for _ in range(3 if args.graph else 1):  # graph: eager step, capture + replay, replay
        trainer.step(tokens, labels)
    torch.cuda.synchronize()
    model = trainer.model
    model.trace_ranges = args.ranges and not args.graph
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        t0 = time.perf_counter()
        if args.step or args.graph:
            trainer.step(tokens, labels)
        else:
            for i in range(args.micro):
                model.forward_backward(tokens[i], labels[i], trainer.loss)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    trainer.release_graph()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        if rank != 0:
            dist.destroy_process_group()
            return
    if args.chrome:
        prof.export_chrome_trace(args.chrome)
    per = collections.defaultdict(lambda: [0.0, 0])
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA:
            per[evt.name][0] += evt.device_time_total if hasattr(evt, "device_time_total") else evt.cuda_time_total
            per[evt.name][1] += 1
    total = sum(v[0] for v in per.values())
    rows = sorted(per.items(), key=lambda kv: -kv[1][0])
    what = "one optimizer step" if args.step else f"{args.micro} micro-batch(es)"
    print(f"profiled {what}, {args.layers} layers: device {total / 1e3:.2f} ms, "
          f"host wall {wall * 1e3:.2f} ms")
    for name, (us, n) in rows[:40]:
        print(f"{us / 1e3:10.3f} ms {100 * us / total:6.2f}% x{n:<6d} {name[:110]}")
    cats = categorize([dict(name=k, us=v[0], count=v[1]) for k, v in rows])
    for cat, (us, n) in sorted(cats.items(), key=lambda kv: -kv[1][0]):
        print(f"{us / 1e3:10.3f} ms {100 * us / total:6.2f}% x{n:<6d} [{cat}]")
    if model.trace_ranges:
        ranges = collections.defaultdict(lambda: [0.0, 0])
        for evt in prof.events():
            if evt.name.startswith("tdb/layer"):
                kind = evt.name.rsplit("/", 1)[-1]
                ranges[kind][0] += evt.cpu_time_total
                ranges[kind][1] += 1
        for kind, (us, n) in sorted(ranges.items()):
            print(f"layer {kind}: {n} ranges, host {us / 1e3:.2f} ms total, {us / max(n, 1) / 1e3:.3f} ms each")
    if args.json:
        with open(args.json, "w") as fh:
            json.dump(dict(total_us=total, wall_s=wall, kernels=[dict(name=k, us=v[0], count=v[1])
                                                                  for k, v in rows]), fh, indent=1)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
