"""One torchrun window of the experiment protocol (per rank), plus the
independent references its numerical gates use.

Stages: ``preflight`` (capability probes: BF16 tcgen05 GEMM, NCCL collectives,
peer access, symmetric heap round trip, native codec vs the FP64 oracle),
``calibrate`` (fit and freeze the arrival/selective plan), ``operator``
(five-arm operator windows with the reference's gates, changed-input reuse,
bitwise order invariance, artificial lane-skew diagnostic, timed iterations
and a full-GEMM control) and ``train`` (a full GPT training window).  Each
rank writes ``rank{r}.json``; failures write a row with the traceback first.

Reference parity: python/flux_dcu/worker.py:18-441.  Timing here uses CUDA
events reduced with MAX over ranks.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
from pathlib import Path
import platform
import socket
import traceback

from .mapping import ARMS, BACKEND


# --------------------------------------------------------------------------
# small helpers
# --------------------------------------------------------------------------
def write(path, value):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(".tmp")
    tmp.write_text(json.dumps(value, indent=2, ensure_ascii=False, allow_nan=False) + "\n")
    tmp.replace(path)


def tensor_sha(tensor):
    import torch
    raw = tensor.detach().contiguous().view(-1).view(torch.uint8).cpu()
    return hashlib.sha256(raw.numpy().tobytes()).hexdigest()


def require_all(ok, message, group):
    """Rank-coordinated gate: MIN all-reduce of the local verdict (on the GPU
    for NCCL groups, on the host for gloo)."""
    import torch
    import torch.distributed as dist
    device = "cuda" if dist.is_initialized() and str(dist.get_backend(group)) == "nccl" else "cpu"
    flag = torch.tensor(int(bool(ok)), dtype=torch.int32, device=device)
    if dist.is_initialized():
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) != 1:
        raise RuntimeError(message + " (failed on at least one rank)")


def relative_error(actual, expected):
    import torch
    a, e = actual.float(), expected.float()
    if not bool(torch.isfinite(a).all() and torch.isfinite(e).all()):
        return float("inf")
    return torch.linalg.vector_norm(a - e).item() / max(torch.linalg.vector_norm(e).item(), 1e-12)


# --------------------------------------------------------------------------
# independent references (torch, no native code)
# --------------------------------------------------------------------------
def hadamard(values):
    """Orthonormal H128 over the last dimension (groups of 128) by explicit
    butterflies on reshaped tensors; independent of the device kernels."""
    import torch
    x = values.float().reshape(-1, 128)
    stride = 1
    while stride < 128:
        pairs = x.reshape(-1, 128 // (2 * stride), 2, stride)
        x = torch.stack((pairs[:, :, 0] + pairs[:, :, 1], pairs[:, :, 0] - pairs[:, :, 1]), dim=2).reshape(-1, 128)
        stride *= 2
    return x / math.sqrt(128)


def _e4m3_levels(device):
    import torch
    from .reference import e4m3_decode
    return torch.tensor([e4m3_decode(code) for code in range(127)], dtype=torch.float32, device=device)


def independent_codec(values):
    """TACO round trip (encode + decode) in FP32 torch with nearest-code
    rounding (ties to the even code), returning BF16."""
    import torch
    shape = values.shape
    x = values.float().reshape(-1, 128)
    adaptive = (448.0 / torch.sqrt((x * x).mean(1, keepdim=True) + 1e-6)).clamp(1e-3, 1e3)
    z = hadamard(x * adaptive)
    scale = (z.abs().amax(1, keepdim=True).clamp_min(1e-12) / 448.0).clamp(1e-12, 1e6)
    scaled = (z / scale).clamp(-448, 448)
    levels = _e4m3_levels(values.device)
    mag = scaled.abs().contiguous()
    hi = torch.bucketize(mag, levels).clamp(0, 126)
    lo = (hi - 1).clamp_min(0)
    d_lo, d_hi = mag - levels[lo], levels[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    q = levels[torch.where(pick_hi, hi, lo)] * scaled.sign()
    out = hadamard(q * scale) / adaptive
    return out.reshape(shape).to(torch.bfloat16)


def reduce_reference_sources(sources, rank, quantized, selection_mask=None, chunk_rows=None):
    """Plain ordered BF16 sum and the same sum with the independent codec
    applied to remote contributions (all, or the masked physical blocks)."""
    import torch
    world, rows, _ = sources.shape
    if selection_mask is not None:
        if chunk_rows is None or rows % chunk_rows:
            raise ValueError("masked reference needs an exact chunk size")
        per = rows // chunk_rows
        if len(selection_mask) != world * per:
            raise ValueError("mask needs one bool per physical block")
    plain = torch.zeros_like(sources[0])
    coded = torch.zeros_like(plain)
    for s in range(world):
        plain = (plain + sources[s]).to(torch.bfloat16)
        contrib = sources[s]
        if quantized and s != rank:
            if selection_mask is None:
                contrib = independent_codec(contrib)
            else:
                contrib = contrib.clone()
                for w in range(per):
                    if selection_mask[rank * per + w]:
                        blk = contrib.narrow(0, w * chunk_rows, chunk_rows)
                        blk.copy_(independent_codec(blk))
        coded = (coded + contrib).to(torch.bfloat16)
    return plain, coded


def projection_reference(input_, weight, rank, world, group, quantized, selection_mask=None, chunk_rows=None,
                         b_mn=False):
    """Full GEMM (cuBLAS via torch, a different code path from the operator),
    NCCL all-to-all of the row blocks, then the ordered references."""
    import torch
    import torch.distributed as dist
    partial = (input_ @ (weight if b_mn else weight.t())).contiguous()
    sources = torch.empty_like(partial)
    dist.all_to_all_single(sources.view(-1), partial.view(-1), group=group)
    sources = sources.view(world, partial.shape[0] // world, partial.shape[1])
    return reduce_reference_sources(sources, rank, quantized, selection_mask, chunk_rows)


def mx_projection_reference(input_, weight, rank, world, group, fp8_rows):
    """Reference of the selective arm in fp8-mma mode: the rows of the
    calibrated blocks as the fp32 product of the dequantized block-scaled FP8
    operands (quantized by the torch restatement in ops/mx.py, not by the
    kernel), the other rows as the BF16 product; then the NCCL all-to-all and
    the ordered BF16 sum."""
    import torch
    import torch.distributed as dist
    from .ops import mx
    a, ea = mx.quantize_reference(input_.cpu())
    b, eb = mx.quantize_reference(weight.cpu())
    deq_a = (a.view(a.shape[0], -1, 32) * torch.exp2(ea.float()).unsqueeze(-1)).view_as(a).to(input_.device)
    deq_b = (b.view(b.shape[0], -1, 32) * torch.exp2(eb.float()).unsqueeze(-1)).view_as(b).to(input_.device)
    rows = fp8_rows.bool().repeat_interleave(input_.shape[0] // fp8_rows.numel())[:, None]
    partial = torch.where(rows, (deq_a @ deq_b.t()).to(torch.bfloat16), input_ @ weight.t()).contiguous()
    sources = torch.empty_like(partial)
    dist.all_to_all_single(sources.view(-1), partial.view(-1), group=group)
    sources = sources.view(world, partial.shape[0] // world, partial.shape[1])
    return reduce_reference_sources(sources, rank, False)[0]


# --------------------------------------------------------------------------
# stages
# --------------------------------------------------------------------------
def identity(local_rank):
    import torch
    prop = torch.cuda.get_device_properties(local_rank)
    return dict(host=socket.gethostname(), local_rank=local_rank, device_name=prop.name,
                device_count=torch.cuda.device_count(), torch=torch.__version__, cuda=torch.version.cuda,
                python=platform.python_version(), backend="nccl", sm_count=prop.multi_processor_count,
                total_memory=prop.total_memory, capability=f"{prop.major}.{prop.minor}",
                uuid=str(getattr(prop, "uuid", "unavailable")),
                visibility={k: os.environ.get(k) for k in ("CUDA_VISIBLE_DEVICES",)},
                communication_environment={k: v for k, v in sorted(os.environ.items())
                                           if k.startswith(("NCCL_", "TORCH_NCCL_"))})


def native_checks(group):
    """Native codec vs the FP64 oracle (actual bytes <= 1%, independent <= 2%)."""
    import torch
    from . import reference
    from .ops.codec import codec, packet_bytes
    gen = torch.Generator(device="cuda").manual_seed(9871)
    cases = [torch.zeros(256, device="cuda", dtype=torch.bfloat16),
             torch.randn(256, generator=gen, device="cuda").to(torch.bfloat16)]
    outlier = cases[1].clone()
    outlier[0], outlier[128] = 128.0, -96.0
    cases.append(outlier)
    results = []
    for x in cases:
        packet = torch.empty(packet_bytes(x.numel()), dtype=torch.uint8, device="cuda")
        out = torch.empty_like(x)
        codec().encode(x, packet)
        codec().decode(packet, out)
        torch.cuda.synchronize()
        raw = bytes(packet.cpu().tolist())
        byte_ref = torch.tensor(reference.decode(raw), device="cuda")
        indep = torch.tensor(reference.decode(reference.encode(x.float().cpu().tolist())), device="cuda")
        e_bytes, e_alg = relative_error(out, byte_ref), relative_error(out, indep)
        require_all(bool(torch.isfinite(out).all()) and e_bytes <= 0.01 and e_alg <= 0.02,
                    f"native codec vs FP64 oracle failed: {e_bytes}, {e_alg}", group)
        results.append(dict(actual_packet_reference_relative_l2=e_bytes, independent_codec_relative_l2=e_alg))
    return results


def preflight(config, rank, world, group):
    import torch
    import torch.distributed as dist
    from .ops import gemm as G
    from .ops import native
    from .runtime import initialize_context
    a = (torch.arange(64 * 64, device="cuda", dtype=torch.float32).reshape(64, 64) / 512).to(torch.bfloat16)
    b = a.t().contiguous()
    a8 = torch.nn.functional.pad(a, (0, 0, 0, 64))
    prod = G.linear(a8.contiguous(), b.contiguous())[:64]
    ref = (a.double() @ b.double().t()).to(torch.bfloat16)
    require_all(relative_error(prod, ref) < 0.01, "tcgen05 BF16 GEMM capability check failed", group)
    probes = []
    if world > 1:
        values = torch.full((world * 4,), rank + 1, dtype=torch.bfloat16, device="cuda")
        reduced = torch.empty(4, dtype=torch.bfloat16, device="cuda")
        dist.reduce_scatter_tensor(reduced, values, group=group)
        require_all(torch.equal(reduced, torch.full_like(reduced, world * (world + 1) // 2)),
                    "NCCL BF16 reduce_scatter failed", group)
        ctx = initialize_context(group)
        # symmetric-heap round trip: every rank writes its id into its slot on every peer
        heap = ctx.heap
        probe = torch.full((16,), rank + 1, dtype=torch.int32, device="cuda")
        for r in range(world):
            native.check(native.lib().tdb_memcpy_async(heap.addrs[r] + ctx.recv_off + rank * 64,
                                                       probe.data_ptr(), 64, native.stream_ptr()), "peer copy")
        torch.cuda.synchronize()
        dist.barrier(group=group)
        seen = heap.view(ctx.recv_off, (world, 16), torch.int32)[:, 0].cpu().tolist()
        require_all(seen == list(range(1, world + 1)), f"symmetric heap peer writes failed: {seen}", group)
        heap.zero_(ctx.recv_off, 64 * world)
        torch.cuda.synchronize()
        dist.barrier(group=group)
        probes.append(dict(kind="symmetric_heap_peer_write", passed=True))
    peers = []
    for other in range(torch.cuda.device_count()):
        try:
            peers.append(bool(torch.cuda.can_device_access_peer(rank, other)) if other != rank else True)
        except RuntimeError:
            peers.append(None)
    return dict(capabilities=dict(tcgen05_bf16_gemm=True, bf16_reduce_scatter=world > 1, peer_access=peers,
                                  direct_peer_required=world > 1, transport_lanes=2),
                collective_probes=probes, codec_checks=native_checks(group))


def _timed(fn, iters, group):
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier(group=group)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    local = start.elapsed_time(end) / 1000.0
    value = torch.tensor(local, dtype=torch.float64, device="cuda")
    if dist.is_initialized():
        dist.all_reduce(value, op=dist.ReduceOp.MAX, group=group)
    return float(value.item()), local


def arrival_diagnostic(config, arm, role_plan, input_, weight, group, selective_mode="wire"):
    """Artificial skew: rank 0 delays the signal of the first lane-0 block by
    5e7 cycles; lane-1 blocks consumed before it completes show ready bypass.
    Outputs must stay bitwise equal.  Never part of timed runs."""
    from copy import deepcopy
    import torch
    from .planning import base_order
    from .runtime import FluxB200
    world = config["world_size"]
    m, k = input_.shape
    n = weight.shape[0]
    chunk = config["model"]["chunk_rows"]
    plan = deepcopy(role_plan)
    plan["arrival_order"] = base_order(m, n, k, world, chunk)
    cycles = 50_000_000
    probe = FluxB200(m, n, k, group, arm, chunk_rows=chunk, plan=plan, diagnostic_delay_cycles=cycles,
                     selective_mode=selective_mode)
    probe.validate_next_call = True
    normal = probe.forward(input_, weight).clone()
    delayed, diag = probe.profile_call(input_, weight)
    require_all(torch.equal(normal, delayed), "artificial lane skew changed the output", group)
    first0 = next(item for item in probe.order if item["lane"] == 0)
    pending = first0["physical"]
    pending_rows = [r for r in diag["events"] if r["physical"] == pending]
    overtakes = []
    if pending_rows:
        done = pending_rows[0]["end_ms"]
        overtakes = [r["physical"] for r in diag["events"] if r["lane"] != 0 and r["end_ms"] < done]
    return dict(passed=True, numerical_bitwise_equal=True, artificial=True, delayed_rank=0, delayed_lane=0,
                delayed_physical=pending, delay_cycles=cycles, later_blocks_completed_before_pending=overtakes,
                ready_bypass_observed=bool(overtakes), evidence=diag, ordinary_speedup_claim=False,
                limitation="Artificial skew, receiver-local device timestamps; no cross-rank clock comparison or "
                           "normal-workload speedup claim.")


def operators(config, arm, rank, world, group, out):
    import torch
    from .runtime import FluxB200
    model, timing = config["model"], config["timing"]
    m, n = model["sequence"] * model["micro_batch"], model["hidden"]
    mode = config.get("selective_mode", "wire") if arm == ARMS[4] else "wire"
    results, states, hashes = [], [], []
    for role, k in (("attn", model["hidden"] // world), ("mlp", model["ffn"] // world)):
        gen = torch.Generator(device="cuda").manual_seed(config["seed"] + 173 * rank + k)
        x = torch.randn((m, k), generator=gen, device="cuda", dtype=torch.bfloat16)
        w = (torch.randn((n, k), generator=gen, device="cuda", dtype=torch.bfloat16) / math.sqrt(k)).to(torch.bfloat16)
        hashes += [tensor_sha(x), tensor_sha(w)]
        role_plan = config["execution_plan"]["roles"][role] if arm in ARMS[3:] else None
        mask = role_plan["selective_mask"] if arm == ARMS[4] else None
        op = FluxB200(m, n, k, group, arm, chunk_rows=model["chunk_rows"], plan=role_plan, selective_mode=mode)
        op.validate_next_call = True
        output = op.forward(x, w)
        plain, coded = projection_reference(x, w, rank, world, group, arm != "flux", mask, model["chunk_rows"])
        if mode == "fp8-mma":  # the "codec" reference is the block-scaled FP8 product on the selected blocks
            coded = mx_projection_reference(x, w, rank, world, group, op.mx["mask"])
        e_plain, e_codec = relative_error(output, plain), relative_error(output, coded)
        require_all(e_plain <= (0.05 if arm != "flux" else 0.01) and e_codec <= 0.01,
                    f"{role} full-shape reference failed: BF16={e_plain}, codec={e_codec}", group)
        retained = output.clone()
        x2 = (x * 0.75 + 0.125).to(torch.bfloat16).contiguous()
        op.validate_next_call = True
        changed = op.forward(x2, w)
        _, coded2 = projection_reference(x2, w, rank, world, group, arm != "flux", mask, model["chunk_rows"])
        if mode == "fp8-mma":
            coded2 = mx_projection_reference(x2, w, rank, world, group, op.mx["mask"])
        e_reuse = relative_error(changed, coded2)
        require_all(torch.equal(output, retained) and e_reuse <= 0.01,
                    f"{role} output lifetime / changed-input reuse failed", group)
        bitwise = None
        if arm != "flux":
            other_plan = None
            if arm == ARMS[4]:
                from copy import deepcopy
                from .planning import base_order
                other = arm
                other_plan = deepcopy(role_plan)
                other_plan["arrival_order"] = base_order(m, n, k, world, model["chunk_rows"])
            else:
                other = "flux_taco" if arm == "flux_taco_interleaved" else "flux_taco_interleaved"
            control = FluxB200(m, n, k, group, other, chunk_rows=model["chunk_rows"], plan=other_plan,
                               selective_mode=mode if other == ARMS[4] else "wire")
            bitwise = torch.equal(control.forward(x, w), retained)
            require_all(bitwise, f"{role} order-only output changed; no fair scheduling ablation", group)
        diag = arrival_diagnostic(config, arm, role_plan, x, w, group, mode) if arm in ARMS[3:] else None
        profile = None
        if config.get("profile"):
            _, profile = op.profile_call(x, w)
        for _ in range(timing["operator_warmup"]):
            op.forward(x, w)
        elapsed, local = _timed(lambda: op.forward(x, w), timing["operator_iterations"], group)
        from .ops import gemm as G
        full = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        for _ in range(5):
            G.linear(x, w, out=full)
        gemm_elapsed, _ = _timed(lambda: G.linear(x, w, out=full), timing["operator_iterations"], group)
        state = op.state()
        states.append(state)
        results.append(dict(role=role, elapsed_seconds=elapsed, local_elapsed_seconds=local,
                            timed_iterations=timing["operator_iterations"], correctness_passed=True,
                            bf16_relative_l2=e_plain, codec_reference_relative_l2=e_codec,
                            changed_input_relative_l2=e_reuse, order_bitwise_equal=bitwise,
                            full_gemm_only_seconds=gemm_elapsed, profile=profile, arrival_diagnostic=diag,
                            execution=state))
    digest = hashlib.sha256("".join(hashes).encode()).hexdigest()
    return dict(operator_results=results, operators=states, input_sha256=digest, initialization_sha256=digest)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--config", type=Path, required=True)
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--stage", choices=("preflight", "calibrate", "operator", "train"), required=True)
    ap.add_argument("--arm", choices=ARMS, required=True)
    args = ap.parse_args(argv)
    config = json.loads(args.config.read_text())
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    row = dict(rank=rank, world_size=world, stage=args.stage, arm=args.arm, run_id=config["run_id"], completed=False,
               passed=False, execution_plan_sha256=config.get("execution_plan_sha256"), backend=BACKEND,
               original_cuda_flux=False, cta_level_swizzle=True)
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        if world != config["world_size"]:
            raise ValueError("torchrun world size differs from the frozen configuration")
        if torch.cuda.device_count() <= local:
            raise RuntimeError(f"need a CUDA device for local rank {local}")
        torch.cuda.set_device(local)
        torch.set_num_threads(1)
        if world > 1:
            dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
        group = dist.group.WORLD if world > 1 else None
        if args.stage in ("operator", "train"):
            from .planning import validate_role_plan
            from .experiment.protocol import digest
            bundle = config.get("execution_plan")
            if not bundle or digest(bundle) != config.get("execution_plan_sha256"):
                raise ValueError("missing or changed frozen calibration plan")
            if bundle.get("world_size") != world or bundle.get("transport_lanes") != 2:
                raise ValueError("plan topology mismatch")
            model = config["model"]
            for role, width in (("attn", model["hidden"]), ("mlp", model["ffn"])):
                validate_role_plan(bundle["roles"][role], model["sequence"] * model["micro_batch"], model["hidden"],
                                   width // world, world, model["chunk_rows"])
        row["environment_identity"] = identity(local)
        from .ops import _build, native
        native.lib()
        row["codec_build"] = _build.manifest_for_rows()
        if args.stage == "preflight":
            row.update(preflight(config, rank, world, group))
        elif args.stage == "calibrate":
            from .calibration import calibrate
            row.update(calibrate(config, group, args.out))
        elif args.stage == "operator":
            row["codec_checks"] = native_checks(group)
            row.update(operators(config, args.arm, rank, world, group, args.out))
        else:
            from .runtime import operator_factory_for
            from .train import train_window
            row.update(train_window(config["model"], args.arm, group, config["timing"]["warmup_steps"],
                                    config["timing"]["timed_steps"], seed=config["seed"],
                                    token_seed=config["token_seed"],
                                    operator_factory=operator_factory_for(
                                        args.arm, selective_mode=config.get("selective_mode", "wire"))
                                    if world > 1 else None,
                                    execution_plan=config["execution_plan"] if args.arm in ARMS[3:] else None))
        torch.cuda.synchronize()
        row.update(completed=True, passed=True)
        write(args.out / f"rank{rank}.json", row)
        if world > 1:
            dist.barrier()
            from .runtime import shutdown_context
            shutdown_context(group)
            dist.destroy_process_group()
    except BaseException as exc:
        row.update(completed=False, passed=False, error=str(exc), traceback=traceback.format_exc())
        write(args.out / f"rank{rank}.json", row)
        raise


if __name__ == "__main__":
    main()
