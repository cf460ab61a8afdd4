"""Operator benchmark of the fused GEMM + reduce-scatter against GEMM + NCCL.

    python -m torch.distributed.run --nproc-per-node N -m tempname_dcu_b200.ops.opbench [--iters 50]

For each role of GPT-6.7B (attention-out K = h/N, FC2 K = f/N; M = 2048,
N = 4096) and each arm, times the fused kernel and the unfused baseline
(tcgen05 GEMM, then NCCL reduce_scatter_tensor, then bias + residual) with
CUDA events, max over ranks, and reports the fraction of the fused path's
roofline: max(FLOPs / measured bf16 peak, remote bytes sent per rank / 770
GB/s NVLink peer bandwidth).
"""
from __future__ import annotations

import argparse
import json
import math
import os
from pathlib import Path

NVLINK_GBS = 770.0


def _peak():
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if path.is_file():
        return json.loads(path.read_text()).get("bf16_tflops", 1590.0), "measured"
    return 1590.0, "fallback"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--arms", default="all")
    ap.add_argument("--remote-first", action="store_true", help="produce remote-bound blocks first (training order)")
    ap.add_argument("--tile-n", type=int, default=0, help="fused kernel tile width (128 or 256; 0 = automatic)")
    ap.add_argument("--variant", type=int, default=None, choices=tuple(range(8)),
                    help="fused GEMM-RS variant (bit 0 per-tile signals, bit 1 in-kernel consumer, "
                         "bit 2 bulk TMA pushes)")
    ap.add_argument("--variants", default=None,
                    help="comma-separated fused GEMM-RS variants to time one after another (e.g. 0,4)")
    ap.add_argument("--no-rs", action="store_true", help="skip the fused GEMM-RS timings")
    ap.add_argument("--consumers", default="auto",
                    help="comma list of consumer forms to time for remote-first operators: auto (epilogue reduction "
                         "where eligible), kernel (separate consumer kernel)")
    ap.add_argument("--ag", action="store_true",
                    help="also time the fused all-gather GEMMs (QKV, FC1 shapes) for each row-movement variant")
    ap.add_argument("--ag-variants", default="0,1,2,3",
                    help="comma list of fused all-gather variants to time (0-2 pull, 3 push)")
    ap.add_argument("--selective-mode", default="wire", choices=("wire", "fp8-mma"),
                    help="fp8-mma: the selective arm computes every block as block-scaled FP8 (BF16 on the wire)")
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    group = dist.group.WORLD
    from ..mapping import ARMS, wire_bytes
    from ..planning import make_role
    from ..runtime import FluxB200, set_epilogue_reduction, set_rs_variant, shutdown_context
    if args.variant is not None:
        set_rs_variant(args.variant)
    from . import gemm as G
    from . import kernels as K
    from . import native
    peak, source = _peak()
    m, n, chunk = 2048, 4096, 128
    arms = ARMS if args.arms == "all" else tuple(args.arms.split(","))

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor(s.elapsed_time(e) / args.iters * 1000.0, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rows = []
    for role, k in (("attn", 4096 // world), ("mlp", 16384 // world)):
        gen = torch.Generator(device="cuda").manual_seed(7 + rank)
        x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
        w = (torch.randn((n, k), generator=gen, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
        bias = torch.zeros(n, device="cuda", dtype=torch.bfloat16)
        res = torch.zeros(m // world, n, device="cuda", dtype=torch.bfloat16)
        partial = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        rs_out = torch.empty(m // world, n, device="cuda", dtype=torch.bfloat16)

        def baseline():
            G.linear(x, w, out=partial)
            dist.reduce_scatter_tensor(rs_out, partial)
            K.bias_residual(rs_out, bias, res, out=rs_out)
        base_us = timed(baseline)
        gemm_us = timed(lambda: G.linear(x, w, out=partial))
        flops = 2.0 * m * n * k
        compute_us = flops / (peak * 1e12) * 1e6
        variants = [int(v) for v in args.variants.split(",")] if args.variants else [args.variant]
        consumers = args.consumers.split(",")
        for variant, arm, consumer in ((v, a, c) for v in variants for a in (() if args.no_rs else arms)
                                       for c in consumers):
            if variant is not None:
                set_rs_variant(variant)
            set_epilogue_reduction(consumer == "auto")
            plan = make_role(m, n, k, world, chunk) if arm in ARMS[3:] else None
            mode = args.selective_mode if arm == ARMS[4] else "wire"
            if mode == "fp8-mma":
                plan = make_role(m, n, k, world, chunk, mask=[True] * (m // chunk))
            op = FluxB200(m, n, k, group, arm, chunk_rows=chunk, plan=plan, remote_first=args.remote_first,
                          tile_n=(args.tile_n or None) if mode == "wire" else None, selective_mode=mode)
            us = timed(lambda: op.forward(x, w, bias, res))
            op.enable_phase_profile(True)
            op.forward(x, w, bias, res)
            torch.cuda.synchronize()
            phases = op.phase_summary()
            op.enable_phase_profile(False)
            quant = op.quantized and mode == "wire"
            link_us = wire_bytes(m, n, world, quant) / (NVLINK_GBS * 1e9) * 1e6
            roof = max(compute_us / (2.0 if mode == "fp8-mma" else 1.0), link_us)
            rows.append(dict(role=role, arm=arm, selective_mode=mode, variant=variant, consumer=op.consumer_policy,
                             world=world, m=m, n=n, k=k,
                             fused_us=round(us, 2),
                             gemm_plus_nccl_rs_us=round(base_us, 2), gemm_only_us=round(gemm_us, 2),
                             speedup_vs_nccl=round(base_us / us, 3), roofline_us=round(roof, 2),
                             roofline_fraction=round(roof / us, 3), bound="link" if link_us > compute_us else "compute",
                             wire_bytes_per_rank=wire_bytes(m, n, world, quant), peak_source=source,
                             phases=phases))
    if args.ag:
        from ..parallel.allgather import SymmAgGemm, set_ag_variant
        from ..parallel.tp import TPGroup
        tp = TPGroup(group)
        ml, h = m // world, 4096
        agg = SymmAgGemm(tp, ml, h)
        xl = torch.randn(ml, h, device="cuda").to(torch.bfloat16)
        full = torch.empty(m, h, dtype=torch.bfloat16, device="cuda")
        for role, n_out, mode in (("qkv", 3 * h // world, agg.BIAS), ("fc1", 16384 // world, agg.BIAS_GELU)):
            w = (torch.randn(n_out, h, device="cuda") / 64).to(torch.bfloat16)
            bias = torch.zeros(n_out, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(m, n_out, dtype=torch.bfloat16, device="cuda")
            pre = torch.empty(m, n_out, dtype=torch.bfloat16, device="cuda")

            def nccl():
                dist.all_gather_into_tensor(full, xl)
                if mode == agg.BIAS_GELU:
                    G.linear_gelu(full, w, bias, pre_out=pre, out=out)
                else:
                    G.linear(full, w, bias, out=out)
            base = timed(nccl)
            gemm_only = timed(lambda: G.linear(full, w, bias, out=out))
            flops = 2.0 * m * n_out * h
            link = (world - 1) * ml * h * 2 / (NVLINK_GBS * 1e9) * 1e6
            roof = max(flops / (peak * 1e12) * 1e6, link)
            for variant in (int(v) for v in args.ag_variants.split(",")):
                set_ag_variant(variant)
                us = timed(lambda: agg(xl, w, mode=mode, bias=bias, out=out, full=full,
                                       **({"aux_out": pre} if mode == agg.BIAS_GELU else {})))
                rows.append(dict(role=f"ag_{role}", pull_variant=variant, world=world, m=m, n=n_out, k=h,
                                 fused_us=round(us, 2), nccl_ag_plus_gemm_us=round(base, 2),
                                 gemm_only_us=round(gemm_only, 2), roofline_us=round(roof, 2),
                                 roofline_fraction=round(roof / us, 3), peak_source=source))
            set_ag_variant(0)
        agg.close()
    native.raise_on_status()
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    shutdown_context(group)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
