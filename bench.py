"""Headline benchmark: GPT-6.7B tensor-parallel bf16 training tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|baseline] [--arm ARM]
    # N > 1: python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
    #            --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload (the headline configuration): GPT-6.7B (32 layers, d_model 4096, 32 heads x 128,
FFN 16384 exact GELU, vocab 50257 padded to 50304, pre-LayerNorm, learned
positions, seq 2048), micro-batch 1 x gradient accumulation 8 = 16384 tokens
per optimizer step, bf16 compute with fp32 masters, AdamW, synthetic uniform
tokens, random N(0, 0.02) weights; tensor parallel over the N GPUs (TP=N,
sequence parallel), so total work per step is fixed (strong scaling).

Timing: W untimed warm-up steps; then barrier + synchronize, CUDA events on
the compute stream around exactly K steps, synchronize; the reported step
time is the max over ranks.  Operands (13 GB of weights per step) are far
larger than the 126 MB L2, so no explicit flush is needed between steps.
``e2e`` times the same K steps through the public API (``Trainer.step``) with
the token/label H2D copy from pinned host memory and the loss D2H read inside
every step.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "GPT-6.7B TP8 train tokens/s (max over ranks) at 1/2/4/8 B200; fused-op roofline %"
# Same-box baseline ("same-box baseline" table): the reference
# design on CUDA -- stock PyTorch with cuBLAS GEMMs, SDPA and NCCL all-gather /
# reduce-scatter, `bench.py --impl baseline` -- measured on B200 with this
# script at the same N and config.  vs_baseline divides by the entry for the
# run's N (null where none was measured).
SAME_BOX_BASELINE_TOKENS_PER_S = {1: 16906.14, 2: 27054.36, 4: 36142.31, 8: 38951.11}
# Best published predecessor number (8xH100, GPT-6.7B TP8, 8192 tok/step), context only.
PUBLISHED_MA11_TOKENS_PER_S = 18177.69


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=("ours", "reference", "baseline"))
    p.add_argument("--arm", default="flux")
    p.add_argument("--no-graph", action="store_true", help="issue every kernel from the host (no CUDA graph)")
    p.add_argument("--taco-allgather", action="store_true",
                   help="TACO-compress the fused all-gathers too (peers' rows cross NVLink as H128/E4M3 packets)")
    p.add_argument("--codec-calibration-steps", type=int, default=0,
                   help="TACO arms: observe the codec error on this many first (warm-up) steps, then freeze the "
                        "block masks within --error-budget (must not exceed --warmup)")
    p.add_argument("--error-budget", type=float, default=0.01)
    p.add_argument("--small", action="store_true", help="2-layer smoke configuration (not a headline number)")
    # transport choices (defaults: the framework's); all ranks must agree
    p.add_argument("--ag-variant", type=int, choices=(-1, 0, 1, 2, 3), default=None,
                   help="fused all-gather GEMM row movement: -1 automatic, 0-2 pull, 3 push")
    p.add_argument("--rs-variant", type=int, choices=tuple(range(8)), default=None,
                   help="fused GEMM-RS variant bits: 1 per-tile signals, 2 in-kernel consumer, 4 bulk pushes")
    p.add_argument("--epilogue-reduction", choices=("on", "off"), default=None,
                   help="remote-first BF16 operators reduce their own blocks in the producer epilogue")
    p.add_argument("--wgrad-sms", type=int, default=None,
                   help="overlap the backward's weight-gradient GEMMs with the fused collectives on this many SMs "
                        "(0 off; default: the framework's choice for the run's world size)")
    p.add_argument("--embedding-exchange", choices=("on", "off"), default=None,
                   help="sparse vocabulary-parallel embedding exchange instead of the dense collectives")
    return p.parse_args()


def apply_transport(args):
    """Apply the transport options and return the settings in effect."""
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.parallel import allgather, embedding_exchange
    from tempname_dcu_b200 import runtime
    if args.ag_variant is not None:
        allgather.set_ag_variant(args.ag_variant)
    if args.rs_variant is not None:
        runtime.set_rs_variant(args.rs_variant)
    if args.epilogue_reduction is not None:
        runtime.set_epilogue_reduction(args.epilogue_reduction == "on")
    if args.embedding_exchange is not None:
        embedding_exchange.set_embedding_exchange(args.embedding_exchange == "on")
    lib = native.lib()
    return dict(ag_variant=allgather.ag_variant(), rs_variant=int(lib.tdb_rs_set_variant(-1)),
                epilogue_reduction=runtime.epilogue_reduction_default(),
                embedding_exchange=embedding_exchange.enabled())


class ClockSampler:
    """nvidia-smi samples (200 ms) of this rank's GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"], samples=0)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(smax) if smax else None,
                    reasons=sorted(reasons), samples=len(sm))


def physical_gpu(local_rank):
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


def init_distributed(n):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return world, rank, local


def reference_arm(args):
    """Run the unmodified reference (installed in baseline/_ref) through its
    own public entry point, ``flux_dcu.model.train_window``."""
    root = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(root, "baseline", "_ref"))
    try:
        from flux_dcu.model import train_window  # the reference's own API
    except Exception as exc:  # noqa: BLE001
        return dict(impl="reference", unavailable=f"reference not importable from baseline/_ref: {exc}")
    try:
        import torch.distributed as dist
        group = dist.group.WORLD if dist.is_initialized() else None
        cfg = dict(layers=32, hidden=4096, ffn=16384, heads=32, sequence=2048, micro_batch=1,
                   accumulation_steps=8, vocab=50304, chunk_rows=128)
        train_window(cfg, "flux", group, None, args.warmup, args.steps)
    except Exception as exc:  # noqa: BLE001
        return dict(impl="reference", unavailable=(
            "the reference needs a HIP/DTK PyTorch and hipcc (flux_dcu/model.py train_window, runtime.py:28-29); "
            f"on CUDA B200 its train_window raises {type(exc).__name__}: {exc}"))
    return dict(impl="reference", unavailable="reference returned without a timing record on this platform")


def main():
    args = parse()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world > 1:
            init_distributed(args.gpus)
        line = reference_arm(args)
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(line), flush=True)
        return 0

    import torch
    import torch.distributed as dist
    world, rank, local = init_distributed(args.gpus)
    group = dist.group.WORLD if world > 1 else None
    from tempname_dcu_b200.models.config import BENCH_CONFIG, SMALL_CONFIG, train_flops_per_step
    from tempname_dcu_b200.ops import native
    config = dict(SMALL_CONFIG if args.small else BENCH_CONFIG)
    transport = apply_transport(args) if args.impl == "ours" else None
    if args.impl == "baseline":
        from tempname_dcu_b200.models.torch_baseline import BaselineTrainer as TrainerCls
        trainer = TrainerCls(config, group)
    else:
        from tempname_dcu_b200.train import Trainer, synthetic_batches
        factory = None
        if world > 1:
            from tempname_dcu_b200.runtime import operator_factory_for
            factory = operator_factory_for(args.arm)
        if args.codec_calibration_steps > args.warmup:
            raise SystemExit("--codec-calibration-steps must run inside the warm-up steps")
        from tempname_dcu_b200.models.gpt import default_wgrad_sms
        wgrad_sms = args.wgrad_sms if args.wgrad_sms is not None else default_wgrad_sms(world)
        transport["wgrad_sms"] = wgrad_sms
        trainer = Trainer(config, args.arm, group, operator_factory=factory, cuda_graph=not args.no_graph,
                          graph_warmup=min(2, max(0, args.warmup - 1)), taco_allgather=args.taco_allgather,
                          codec_calibration_steps=args.codec_calibration_steps, error_budget=args.error_budget,
                          wgrad_sms=wgrad_sms)
    from tempname_dcu_b200.train import synthetic_batches
    c = trainer.config
    (tokens_h, labels_h), = synthetic_batches(c, 1, seed=4321)
    tokens_d, labels_d = tokens_h.to("cuda"), labels_h.to("cuda")
    tokens_per_step = c["sequence"] * c["micro_batch"] * c["accumulation_steps"]

    # ---------------- device-timed region
    for _ in range(args.warmup):
        trainer.step(tokens_d, labels_d)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    launches0 = native.launch_count()
    replays0 = getattr(trainer, "graph_replays", 0)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        loss, norm = trainer.step(tokens_d, labels_d)
    end.record()
    torch.cuda.synchronize()
    # host-issued library kernels plus those replayed from the captured step graph
    launches = native.launch_count() - launches0 + \
        getattr(trainer, "graph_kernels", 0) * (getattr(trainer, "graph_replays", 0) - replays0)
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = torch.tensor(start.elapsed_time(end) / args.steps, dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_per_step = float(ms.item())
    final_loss = float(loss.item())

    # ---------------- end-to-end through the public API
    trainer.step(tokens_h, labels_h)[0].item()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        loss_value = trainer.step(tokens_h, labels_h)[0].item()  # H2D inputs + D2H loss every step
    e2e_local = (time.perf_counter() - t0) / args.steps * 1000.0
    e2e = torch.tensor(e2e_local, dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e.item())

    flops = train_flops_per_step(c, 1)
    if rank == 0:
        value = tokens_per_step * 1000.0 / ms_per_step
        line = dict(
            metric=METRIC, value=round(value, 2), unit="tokens/s", n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=round(ms_per_step, 3), higher_is_better=True, scaling="strong",
            vs_baseline=(round(value / SAME_BOX_BASELINE_TOKENS_PER_S[world], 4)
                         if world in SAME_BOX_BASELINE_TOKENS_PER_S and args.impl == "ours" and not args.small
                         else None), dtype="bf16",
            data="synthetic uniform tokens, random-init N(0,0.02) weights",
            impl=args.impl,
            config=dict(model="GPT-6.7B" if not args.small else "GPT-small-2L (smoke)",
                        global_batch=c["micro_batch"] * c["accumulation_steps"], seq_len=c["sequence"],
                        parallelism=f"tp{world}" if world > 1 else "tp1", micro_batch=c["micro_batch"],
                        accumulation_steps=c["accumulation_steps"], vocab=c["vocab"], padded_vocab=c["padded_vocab"],
                        layers=c["layers"], hidden=c["hidden"], ffn=c["ffn"], heads=c["heads"],
                        tokens_per_step=tokens_per_step, arm=args.arm if args.impl == "ours" else None,
                        taco_allgather=bool(args.taco_allgather) if args.impl == "ours" else None,
                        codec_calibration=(dict(steps=args.codec_calibration_steps, error_budget=args.error_budget)
                                           if args.codec_calibration_steps else None),
                        cuda_graph=bool(args.impl == "ours" and not args.no_graph),
                        transport=transport if world > 1 else None,
                        l2="inputs larger than L2 (13 GB of bf16 weights streamed per step); no flush",
                        model_tflops_per_gpu=round(flops / (ms_per_step / 1000.0) / world / 1e12, 1),
                        baseline_ref=dict(
                            same_box=SAME_BOX_BASELINE_TOKENS_PER_S.get(world),
                            same_box_impl="stock PyTorch (cuBLAS, SDPA, NCCL): bench.py --impl baseline",
                            published_ma11_8xh100=PUBLISHED_MA11_TOKENS_PER_S),
                        final_loss=final_loss, e2e_last_loss=loss_value),
            clocks=clocks,
            e2e=dict(value=round(tokens_per_step * 1000.0 / e2e_ms, 2), unit="tokens/s",
                     ms_per_step=round(e2e_ms, 3), h2d_bytes_per_step=int(tokens_h.numel() * 8 * 2),
                     d2h_bytes_per_step=4),
            gpu_launches=int(launches),
        )
        print(json.dumps(line), flush=True)
    if hasattr(trainer, "release_graph"):
        trainer.release_graph()  # graphs holding NCCL work go before the process group
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
