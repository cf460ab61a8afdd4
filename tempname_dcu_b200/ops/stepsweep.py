"""Training-step A/B over transport settings, in one process group.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m tempname_dcu_b200.ops.stepsweep \\
        --configs "ag=2;ag=3;ag=3,epi=off;ag=3,embx=off" [--steps K] [--warmup W]

For each configuration (``;``-separated; each a ``,``-separated list of
``ag=-1..3`` fused all-gather variant (-1 automatic), ``rs=0..7`` fused GEMM-RS variant bits,
``epi=on|off`` epilogue reduction, ``embx=on|off`` sparse embedding
exchange, ``wg=N`` weight-gradient overlap on N SMs (0 off); unnamed keys keep the framework default) this builds the GPT-6.7B
tensor-parallel trainer (flux arm, CUDA graph), runs W warm-up steps, times K
steps with CUDA events between two barriers and takes the max over ranks --
the same step and timing as ``bench.py`` -- then drops the trainer before the
next one.  Configurations run in the given order on the same GPUs, so
building the process group and importing the stack is paid once.  Rank 0
prints one JSON line per configuration.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
from datetime import timedelta

KEYS = ("ag", "rs", "epi", "embx", "wg")


def parse_config(text):
    out = {}
    for item in filter(None, (t.strip() for t in text.split(","))):
        key, _, value = item.partition("=")
        if key not in KEYS:
            raise ValueError(f"unknown key {key!r} (expected one of {KEYS})")
        if key in ("ag", "rs", "wg"):
            out[key] = int(value)
        elif value in ("on", "off"):
            out[key] = value == "on"
        else:
            raise ValueError(f"{key} takes on|off")
    return out


def apply(cfg, defaults):
    from .. import runtime
    from ..parallel import allgather, embedding_exchange
    allgather.set_ag_variant(cfg.get("ag", defaults["ag"]))
    runtime.set_rs_variant(cfg.get("rs", defaults["rs"]))
    runtime.set_epilogue_reduction(cfg.get("epi", defaults["epi"]))
    embedding_exchange.set_embedding_exchange(cfg.get("embx", defaults["embx"]))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--configs", required=True)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--wgrad-sms", type=int, default=None,
                    help="default of the wg key (default: the framework's choice for the world size)")
    args = ap.parse_args(argv)
    configs = [parse_config(c) for c in args.configs.split(";") if c.strip()]
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    group = dist.group.WORLD
    from .. import runtime
    from ..models.config import BENCH_CONFIG
    from ..ops import native
    from ..parallel import allgather, embedding_exchange
    from ..train import Trainer, synthetic_batches
    from ..models.gpt import default_wgrad_sms
    if args.wgrad_sms is None:
        args.wgrad_sms = default_wgrad_sms(world)
    lib = native.lib()
    defaults = dict(ag=allgather.ag_variant(), rs=int(lib.tdb_rs_set_variant(-1)),
                    epi=runtime.epilogue_reduction_default(), embx=embedding_exchange.enabled(), wg=args.wgrad_sms)
    tokens = labels = None
    for cfg in configs:
        apply(cfg, defaults)
        trainer = Trainer(dict(BENCH_CONFIG), "flux", group, operator_factory=runtime.operator_factory_for("flux"),
                          cuda_graph=True, graph_warmup=min(2, max(0, args.warmup - 1)),
                          wgrad_sms=cfg.get("wg", defaults["wg"]))
        c = trainer.config
        if tokens is None:
            (th, lh), = synthetic_batches(c, 1, seed=4321)
            tokens, labels = th.to("cuda"), lh.to("cuda")
        for _ in range(args.warmup):
            trainer.step(tokens, labels)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            loss, _ = trainer.step(tokens, labels)
        end.record()
        torch.cuda.synchronize()
        dist.barrier()
        ms = torch.tensor(start.elapsed_time(end) / args.steps, dtype=torch.float64, device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        native.raise_on_status()
        tokens_per_step = c["sequence"] * c["micro_batch"] * c["accumulation_steps"]
        row = dict(config=cfg, effective={k: cfg.get(k, defaults[k]) for k in KEYS}, world=world,
                   steps=args.steps, warmup=args.warmup, ms_per_step=round(float(ms.item()), 3),
                   tokens_per_s=round(tokens_per_step * 1000.0 / float(ms.item()), 1),
                   loss=round(float(loss.item()), 5))
        if rank == 0:
            print(json.dumps(row), flush=True)
        trainer.release_graph()
        del trainer, loss
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
    apply({}, defaults)
    runtime.shutdown_context(group)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
