"""Rooflines of the fused tensor-parallel paths of a GPT training step.

    python -m tempname_dcu_b200.ops.roofline [--world 8] [--taco] [--trace trace.json]
    python -m tempname_dcu_b200.ops.roofline --world 8 --opbench rows.jsonl --step-ms 243.4

For every fused collective+GEMM path of one layer and micro-batch (forward:
QKV and FC1 all-gather -> GEMM, attention-out and FC2 GEMM -> reduce-scatter;
backward: the four mirrored paths; plus the LM head and its data gradient) the
roofline time is the slower of the GEMM at the measured bf16 peak and the
bytes this rank moves over NVLink at the measured peer bandwidth.  With
``--trace`` (the JSON of ``utils/trace.py --step --json``) the measured device
time of the fused kernels is set against the step's fused roofline.

With ``--opbench`` (the JSON lines of ``ops/opbench.py --ag`` at this world
size) the exposed communication of a step is estimated: per fused path, the
fused call's time minus the GEMM alone (what the collective adds), summed over
layers and micro-batches; the backward's paths take the forward row of the
same kind and nearest inner size (the all-gather of the attention-out data
gradient, N = h / W, takes the QKV row; the QKV data-gradient reduce-scatter,
K = 3h / W, the FC2 row).  ``--step-ms`` sets it against a measured step.

Peaks: ``MEASURED_PEAKS.json`` at the repository root when present (bf16 GEMM
burst rate, HBM copy); NVLink 770 GB/s per direction (measured peer copy) --
otherwise the fallbacks below.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

FALLBACK_BF16_TFLOPS = 1590.0
NVLINK_GBS = 770.0
TACO_RATIO = 136 / 256  # H128 packet bytes per BF16 byte


def peaks():
    """(bf16 TFLOP/s, NVLink GB/s, source)."""
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return float(data.get("bf16_tflops", FALLBACK_BF16_TFLOPS)), NVLINK_GBS, "measured"
    return FALLBACK_BF16_TFLOPS, NVLINK_GBS, "fallback"


def fused_paths(config, world, taco=False):
    """Per layer and micro-batch: [{name, flops, link_bytes}] for this rank;
    ``link_bytes`` is what the rank sends (= receives) over NVLink."""
    from ..models.config import validate_config
    c = validate_config(config, world)
    m, h, f = c["sequence"] * c["micro_batch"], c["hidden"], c["ffn"]
    link = (world - 1) * (m // world) * h * 2 * (TACO_RATIO if taco else 1.0)
    rows = []
    for name, n_local in (("qkv", 3 * h // world), ("attn_out", h // world), ("fc1", f // world),
                          ("fc2", f // world)):
        gemm = 2.0 * m * h * n_local  # every path multiplies [m, h]-sized gathered / scattered rows by a shard
        kind = "all-gather -> GEMM" if name in ("qkv", "fc1") else "GEMM -> reduce-scatter"
        back = "GEMM -> reduce-scatter" if name in ("qkv", "fc1") else "all-gather -> GEMM"
        rows.append(dict(name=f"{name}.fwd", kind=kind, flops=gemm, link_bytes=link))
        rows.append(dict(name=f"{name}.dgrad", kind=back, flops=gemm, link_bytes=link))
    return rows


def head_paths(config, world, taco=False):
    """The LM head (tied embedding): all-gather -> GEMM forward and its data
    gradient GEMM -> reduce-scatter, once per micro-batch."""
    from ..models.config import validate_config
    c = validate_config(config, world)
    m, h, v = c["sequence"] * c["micro_batch"], c["hidden"], c["padded_vocab"]
    link = (world - 1) * (m // world) * h * 2 * (TACO_RATIO if taco else 1.0)
    gemm = 2.0 * m * h * (v // world)
    return [dict(name="lm_head.fwd", kind="all-gather -> GEMM", flops=gemm, link_bytes=link),
            dict(name="lm_head.dgrad", kind="GEMM -> reduce-scatter", flops=gemm, link_bytes=link)]


def roofline_us(path, tflops, nvlink_gbs):
    compute = path["flops"] / (tflops * 1e12) * 1e6
    link = path["link_bytes"] / (nvlink_gbs * 1e9) * 1e6
    return max(compute, link), ("link" if link > compute else "compute")


def step_roofline(config, world, taco=False, tflops=None, nvlink_gbs=None):
    """Sum over one optimizer step of the fused paths' roofline times (us)."""
    from ..models.config import validate_config
    c = validate_config(config, world)
    if tflops is None or nvlink_gbs is None:
        tflops, nvlink_gbs, _ = peaks()
    per_layer = sum(roofline_us(p, tflops, nvlink_gbs)[0] for p in fused_paths(c, world, taco))
    head = sum(roofline_us(p, tflops, nvlink_gbs)[0] for p in head_paths(c, world, taco))
    return c["accumulation_steps"] * (c["layers"] * per_layer + head)


# forward rows of ops/opbench.py standing in for each fused path of a layer
_OPBENCH_ROW = {"qkv.fwd": "ag_qkv", "fc1.fwd": "ag_fc1", "attn_out.fwd": "attn", "fc2.fwd": "mlp",
                "qkv.dgrad": "mlp", "fc1.dgrad": "mlp", "attn_out.dgrad": "ag_qkv", "fc2.dgrad": "ag_fc1"}


def exposed_from_opbench(rows, config, world):
    """(per-path list, total us per optimizer step) of fused time minus GEMM
    time, from opbench rows (the fastest fused form of each role, flux arm
    for the reduce-scatters)."""
    from ..models.config import validate_config
    c = validate_config(config, world)
    best = {}
    for r in rows:
        if r.get("world") != world or "fused_us" not in r:
            continue
        if r["role"] in ("attn", "mlp") and r.get("arm") != "flux":
            continue
        if r["role"] not in best or r["fused_us"] < best[r["role"]]["fused_us"]:
            best[r["role"]] = r
    missing = sorted(set(_OPBENCH_ROW.values()) - set(best))
    if missing:
        raise ValueError(f"opbench rows missing for {missing} at world {world}")
    per_path = []
    for path, role in _OPBENCH_ROW.items():
        r = best[role]
        per_path.append(dict(path=path, row=role, fused_us=r["fused_us"], gemm_us=r["gemm_only_us"],
                             exposed_us=max(0.0, r["fused_us"] - r["gemm_only_us"])))
    per_layer = sum(p["exposed_us"] for p in per_path)
    return per_path, c["accumulation_steps"] * c["layers"] * per_layer


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--taco", action="store_true", help="TACO-compressed link bytes")
    ap.add_argument("--trace", default="", help="utils/trace.py --json output of one step at this world size")
    ap.add_argument("--opbench", default="", help="JSON lines of ops/opbench.py --ag at this world size")
    ap.add_argument("--step-ms", type=float, default=0.0, help="measured step time for the exposed fraction")
    args = ap.parse_args(argv)
    from ..models.config import BENCH_CONFIG
    tflops, nvlink, source = peaks()
    print(f"peaks ({source}): bf16 {tflops:.0f} TFLOP/s, NVLink {nvlink:.0f} GB/s per direction")
    print(f"{'path':16s} {'kind':24s} {'GFLOP':>8s} {'link MB':>8s} {'roofline us':>12s}  bound")
    for p in fused_paths(BENCH_CONFIG, args.world, args.taco) + head_paths(BENCH_CONFIG, args.world, args.taco):
        us, bound = roofline_us(p, tflops, nvlink)
        print(f"{p['name']:16s} {p['kind']:24s} {p['flops'] / 1e9:8.1f} {p['link_bytes'] / 1e6:8.2f} {us:12.2f}  {bound}")
    total = step_roofline(BENCH_CONFIG, args.world, args.taco, tflops, nvlink)
    print(f"fused paths per optimizer step: roofline {total / 1e3:.1f} ms")
    if args.trace:
        from ..utils.trace import categorize
        data = json.loads(Path(args.trace).read_text())
        cats = categorize(data["kernels"])
        measured = sum(cats.get(k, (0.0, 0))[0] for k in ("fused GEMM -> reduce-scatter", "fused all-gather -> GEMM"))
        print(f"measured fused kernels: {measured / 1e3:.1f} ms -> {total / measured:.3f} of roofline")
    if args.opbench:
        rows = [json.loads(line) for line in Path(args.opbench).read_text().splitlines() if line.startswith("{")]
        per_path, exposed = exposed_from_opbench(rows, BENCH_CONFIG, args.world)
        for p in per_path:
            print(f"{p['path']:16s} from {p['row']:7s} fused {p['fused_us']:7.1f} us  GEMM {p['gemm_us']:6.1f} us  "
                  f"exposed {p['exposed_us']:6.1f} us")
        line = f"exposed communication per step (layers x micro-batches, LM head excluded): {exposed / 1e3:.1f} ms"
        if args.step_ms > 0:
            line += f" = {exposed / 1e3 / args.step_ms:.2f} of a {args.step_ms:.1f} ms step"
        print(line)


if __name__ == "__main__":
    main()
