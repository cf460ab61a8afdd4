"""Kernel microbenchmarks with CUDA-event timing.

    python -m tempname_dcu_b200.ops.microbench gemm [--shapes M,N,K:...] [--iters 20]
    python -m tempname_dcu_b200.ops.microbench ncu-gemm M N K [--mode fwd|dgrad|wgrad]
    python -m tempname_dcu_b200.ops.microbench attn [--seq 2048 --heads 32 --mb 1] [--iters 20]
    python -m tempname_dcu_b200.ops.microbench ncu-attn [--impl tc] [--seq 2048 --heads 8]
    python -m tempname_dcu_b200.ops.microbench attn-timeline [--seq 2048 --heads 32]

Each measurement: warm-up launches, then ``iters`` timed launches, each
preceded by a write of a 256 MB buffer (larger than the 126 MB L2) so that
operands come from HBM; CUDA events on the launching stream bracket only the
kernel.  Results are TFLOP/s and the fraction of the measured cuBLAS bf16
peak recorded in MEASURED_PEAKS.json (when present).
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

# GPT-6.7B linear-layer shapes per micro-batch (M = 2048 tokens) at TP=1.
DEFAULT_SHAPES = [
    ("qkv.fwd", 2048, 12288, 4096, "fwd"),
    ("attn_out.fwd", 2048, 4096, 4096, "fwd"),
    ("fc1.fwd", 2048, 16384, 4096, "fwd"),
    ("fc2.fwd", 2048, 4096, 16384, "fwd"),
    ("lm_head.fwd", 2048, 50304, 4096, "fwd"),
    ("fc1.dgrad", 2048, 4096, 16384, "dgrad"),
    ("fc2.dgrad", 2048, 16384, 4096, "dgrad"),
    ("fc1.wgrad", 16384, 4096, 2048, "wgrad"),
    ("fc2.wgrad", 4096, 16384, 2048, "wgrad"),
    ("qkv.tp8.fwd", 2048, 1536, 4096, "fwd"),
    ("attn_out.tp8.fwd", 2048, 4096, 512, "fwd"),
]


def _peaks():
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return data.get("bf16_tflops", 1590.0), data.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def _operands(torch, M, N, K, kind, device):
    g = torch.Generator(device=device).manual_seed(0)
    if kind in ("fwd", "fwd_f32"):      # x[M,K] @ w[N,K]^T
        a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
        b = torch.randn(N, K, device=device, generator=g).to(torch.bfloat16)
    elif kind == "dgrad":  # dy[M,K'] @ w[K',N] where the GEMM is M x N x K
        a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
        b = torch.randn(K, N, device=device, generator=g).to(torch.bfloat16)
    else:                  # dw[M,N] = dy[K,M]^T @ x[K,N]
        a = torch.randn(K, M, device=device, generator=g).to(torch.bfloat16)
        b = torch.randn(K, N, device=device, generator=g).to(torch.bfloat16)
    return a, b


def _ours(gemm, a, b, kind, out):
    if kind == "fwd":
        return lambda: gemm.gemm(a, b, out=out)
    if kind == "wgrad_bf16":  # wgrad operand layouts, bf16 output (layout vs epilogue cost)
        return lambda: gemm.gemm(a, b, a_mn=True, b_mn=True, out=out)
    if kind == "fwd_f32":     # forward operand layouts, fp32 output
        return lambda: gemm.gemm(a, b, out=out, mode=gemm.ACC_F32, beta=0.0)
    if kind == "dgrad":
        return lambda: gemm.gemm(a, b, b_mn=True, out=out)
    return lambda: gemm.gemm(a, b, a_mn=True, b_mn=True, out=out, mode=gemm.ACC_F32, beta=0.0)


def _cublas(torch, a, b, kind, out):
    if kind in ("fwd", "fwd_f32"):
        return lambda: torch.matmul(a, b.t(), out=out)
    if kind == "dgrad":
        return lambda: torch.matmul(a, b, out=out)
    return lambda: torch.matmul(a.t(), b, out=out)


def time_fn(torch, fn, iters, warmup=3, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.add_(1)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    times.sort()
    return times[len(times) // 2]


def _bench_mx(torch, name, M, N, K, iters, flush, peak, source):
    """Block-scaled FP8 GEMM (operands quantized once, outside the timing)
    against the bf16 GEMMs of the same shape; the quantizer is timed apart."""
    from . import gemm, mx
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    qa, sfa = mx.quantize(x)
    qb, sfb = mx.quantize(w)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ours = time_fn(torch, lambda: mx.gemm(qa, sfa, qb, sfb, out=out), iters, flush=flush)
    quant = time_fn(torch, lambda: mx.quantize(x, qa, sfa), iters, flush=flush)
    bf16 = time_fn(torch, lambda: gemm.gemm(x, w, out=out), iters, flush=flush)
    theirs = time_fn(torch, lambda: torch.matmul(x, w.t()), iters, flush=flush)
    mx.gemm(qa, sfa, qb, sfb, out=out)
    ref = mx.dequantize(qa, sfa) @ mx.dequantize(qb, sfb).t()
    err = ((out.float() - ref).norm() / ref.norm()).item()
    flops = 2.0 * M * N * K
    return dict(name=name, M=M, N=N, K=K, kind="mx", ours_ms=ours, quantize_a_ms=quant, ours_bf16_ms=bf16,
                cublas_bf16_ms=theirs, ours_tflops=flops / ours / 1e9, speedup_vs_our_bf16=bf16 / ours,
                speedup_vs_cublas_bf16=theirs / ours, frac_of_bf16_peak=flops / ours / 1e9 / peak,
                rel_err_vs_dequantized=err, peak_source=source)


def bench_gemm(shapes, iters):
    import torch
    from . import gemm, native
    device = torch.device("cuda", 0)
    peak, _, source = _peaks()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
    rows = []
    for name, M, N, K, kind in shapes:
        if kind == "mx":
            rows.append(_bench_mx(torch, name, M, N, K, iters, flush, peak, source))
            print(json.dumps(rows[-1]), flush=True)
            continue
        a, b = _operands(torch, M, N, K, kind, device)
        out_dtype = torch.float32 if kind in ("wgrad", "fwd_f32") else torch.bfloat16
        out = torch.empty(M, N, dtype=out_dtype, device=device)
        ref_out = torch.empty(M, N, dtype=torch.bfloat16, device=device)
        ours = time_fn(torch, _ours(gemm, a, b, kind, out), iters, flush=flush)
        theirs = time_fn(torch, _cublas(torch, a, b, kind, ref_out), iters, flush=flush)
        ref = _cublas(torch, a.float(), b.float(), kind, None)()
        err = ((out.float() - ref).norm() / ref.norm()).item()
        flops = 2.0 * M * N * K
        rows.append(dict(name=name, M=M, N=N, K=K, kind=kind, ours_ms=ours, cublas_ms=theirs,
                         ours_tflops=flops / ours / 1e9, cublas_tflops=flops / theirs / 1e9,
                         frac_of_peak=flops / ours / 1e9 / peak, speedup_vs_cublas=theirs / ours,
                         rel_err=err, peak_source=source))
        print(json.dumps(rows[-1]), flush=True)
    native.raise_on_status()
    return rows


def attn_flops(mb, seq, heads, causal=True):
    """Forward FLOPs of causal attention, head_dim 128 (QK^T and PV, half the square)."""
    flops = 4.0 * mb * heads * seq * seq * 128
    return flops / 2 if causal else flops


def bench_attn(mb, seq, heads, iters):
    import torch
    from . import kernels, native
    device = torch.device("cuda", 0)
    peak, _, source = _peaks()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
    g = torch.Generator(device=device).manual_seed(0)
    qkv = torch.randn(mb * seq, 3 * heads * 128, device=device, generator=g).to(torch.bfloat16)
    out = torch.empty(mb * seq, heads * 128, dtype=torch.bfloat16, device=device)
    lse = torch.empty(mb, heads, seq, dtype=torch.float32, device=device)
    fl = attn_flops(mb, seq, heads)
    rows = []
    for impl in ("tc", "mma"):
        ms = time_fn(torch, lambda: kernels.attention_fwd(qkv, mb, seq, heads, out=out, lse=lse, impl=impl), iters,
                     flush=flush)
        rows.append(dict(op="attn.fwd", impl=impl, mb=mb, seq=seq, heads=heads, ms=ms, tflops=fl / ms / 1e9,
                         frac_of_peak=fl / ms / 1e9 / peak, peak_source=source))
        print(json.dumps(rows[-1]), flush=True)
    dout = torch.randn_like(out)
    dqkv = torch.empty_like(qkv)
    dsum = torch.empty(mb, heads, seq, dtype=torch.float32, device=device)
    kernels.attention_fwd(qkv, mb, seq, heads, out=out, lse=lse)
    for impl in ("tc", "mma"):
        ms = time_fn(torch, lambda: kernels.attention_bwd(qkv, out, dout, lse, mb, seq, heads, dqkv=dqkv, dsum=dsum,
                                                          impl=impl), iters, flush=flush)
        # algorithmic backward FLOPs = 2.5x forward (5 GEMMs); the deterministic
        # two-kernel schedule executes 7
        rows.append(dict(op="attn.bwd", impl=impl, mb=mb, seq=seq, heads=heads, ms=ms, tflops=2.5 * fl / ms / 1e9,
                         frac_of_peak=2.5 * fl / ms / 1e9 / peak, peak_source=source))
        print(json.dumps(rows[-1]), flush=True)
    try:  # library kernel, for context only
        from flash_attn import flash_attn_func
        q, k, v = qkv.reshape(mb, seq, 3, heads, 128).unbind(2)
        ms = time_fn(torch, lambda: flash_attn_func(q, k, v, causal=True), iters, flush=flush)
        rows.append(dict(op="attn.fwd", impl="flash_attn (library)", mb=mb, seq=seq, heads=heads, ms=ms,
                         tflops=fl / ms / 1e9))
        print(json.dumps(rows[-1]), flush=True)
    except Exception as exc:  # noqa: BLE001
        print(json.dumps(dict(op="attn.fwd", impl="flash_attn (library)", unavailable=str(exc)[:200])))
    native.raise_on_status()
    return rows


TIMELINE_EVENTS = ("tma_K", "tma_V", "mma_S", "mma_p_full", "mma_PV", "sm_s_full", "sm_S_loaded", "sm_max_xchg",
                   "sm_P_stored", "sm_pv_done", "sm_p_full")


def attn_timeline(seq, heads):
    """Pipeline timeline of the heaviest forward CTA (clock64 cycles relative
    to its first event) -- a diagnostic of the tcgen05 attention schedule."""
    import ctypes
    import torch
    from . import kernels, native
    lib = native.lib()
    fn = lib.tdb_attn_fwd_tc_timeline
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    device = torch.device("cuda", 0)
    qkv = torch.randn(seq, 3 * heads * 128, device=device).to(torch.bfloat16)
    out = torch.empty(seq, heads * 128, dtype=torch.bfloat16, device=device)
    lse = torch.empty(1, heads, seq, dtype=torch.float32, device=device)
    steps = seq // 128
    tl = torch.zeros(16 * steps, dtype=torch.int64, device=device)
    for _ in range(3):
        kernels.attention_fwd(qkv, 1, seq, heads, out=out, lse=lse)
        native.check(fn(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), lse.data_ptr(), 1, seq, heads,
                        1.0 / 128 ** 0.5, native.stream_ptr(), tl.data_ptr()), "attn timeline")
    torch.cuda.synchronize()
    t = tl.view(steps, 16)[:, :len(TIMELINE_EVENTS)].cpu()
    base = int(t[t > 0].min())
    rows = []
    for j in range(steps):
        row = {name: (int(t[j, k]) - base if int(t[j, k]) else None) for k, name in enumerate(TIMELINE_EVENTS)}
        row["step"] = j
        rows.append(row)
        print(json.dumps(row))
    return rows


def main(argv=None):
    parser = argparse.ArgumentParser()
    sub = parser.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("gemm")
    p.add_argument("--shapes", default="")
    p.add_argument("--iters", type=int, default=20)
    q = sub.add_parser("ncu-gemm", help="a few launches of one GEMM shape (for ncu captures)")
    q.add_argument("M", type=int)
    q.add_argument("N", type=int)
    q.add_argument("K", type=int)
    q.add_argument("--mode", default="fwd", choices=("fwd", "dgrad", "wgrad", "mx"))
    q.add_argument("--launches", type=int, default=3)
    r = sub.add_parser("attn")
    r.add_argument("--mb", type=int, default=1)
    r.add_argument("--seq", type=int, default=2048)
    r.add_argument("--heads", type=int, default=32)
    r.add_argument("--iters", type=int, default=20)
    t = sub.add_parser("ncu-attn", help="a few launches of the attention forward (for ncu captures)")
    t.add_argument("--impl", default="tc", choices=("tc", "mma"))
    t.add_argument("--seq", type=int, default=2048)
    t.add_argument("--heads", type=int, default=8)
    t.add_argument("--launches", type=int, default=3)
    u = sub.add_parser("attn-timeline")
    u.add_argument("--seq", type=int, default=2048)
    u.add_argument("--heads", type=int, default=32)
    args = parser.parse_args(argv)
    if args.cmd == "attn-timeline":
        attn_timeline(args.seq, args.heads)
    elif args.cmd == "attn":
        bench_attn(args.mb, args.seq, args.heads, args.iters)
    elif args.cmd == "ncu-attn":
        import torch
        from . import kernels
        qkv = torch.randn(args.seq, 3 * args.heads * 128, device="cuda").to(torch.bfloat16)
        for _ in range(args.launches):
            kernels.attention_fwd(qkv, 1, args.seq, args.heads, impl=args.impl)
        torch.cuda.synchronize()
    elif args.cmd == "gemm":
        shapes = DEFAULT_SHAPES
        if args.shapes:
            shapes = []
            for item in args.shapes.split(":"):
                M, N, K, *kind = item.split(",")
                shapes.append((item, int(M), int(N), int(K), kind[0] if kind else "fwd"))
        bench_gemm(shapes, args.iters)
    elif args.mode == "mx":
        import torch
        from . import mx
        x = torch.randn(args.M, args.K, device="cuda").to(torch.bfloat16)
        w = torch.randn(args.N, args.K, device="cuda").to(torch.bfloat16)
        qa, sfa = mx.quantize(x)
        qb, sfb = mx.quantize(w)
        out = torch.empty(args.M, args.N, dtype=torch.bfloat16, device="cuda")
        for _ in range(args.launches):
            mx.gemm(qa, sfa, qb, sfb, out=out)
        torch.cuda.synchronize()
    else:
        import torch
        from . import gemm
        a, b = _operands(torch, args.M, args.N, args.K, args.mode, torch.device("cuda", 0))
        out = torch.empty(args.M, args.N, dtype=torch.float32 if args.mode == "wgrad" else torch.bfloat16,
                          device="cuda")
        fn = _ours(gemm, a, b, args.mode, out)
        for _ in range(args.launches):
            fn()
        torch.cuda.synchronize()


if __name__ == "__main__":
    main()
