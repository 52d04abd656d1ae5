"""
Kernel micro-benchmarks:  ``python -m olmo_b200.ops.microbench {gemm,attention,norm,ce,optim} [options]``

Each case is timed with CUDA events on the launching stream after warm-up, with an L2 flush (a write of a buffer larger
than L2) between timed iterations, and reported against the measured peaks in ``MEASURED_PEAKS.json`` when present.
``--once`` runs each kernel a few times without timing, which is the form used under ``ncu``.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from . import check_status
from . import kernels as k


def _peaks() -> dict:
    p = Path(__file__).resolve().parent.parent.parent / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except Exception:
        return {}


_flush = None


def timeit(fn, iters: int = 10, warmup: int = 3) -> float:
    global _flush
    if _flush is None:
        _flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        _flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def bench_gemm(args) -> None:
    peak = _peaks().get("bf16_tflops")
    shapes = [(8192, 12288, 4096), (8192, 4096, 4096), (8192, 22016, 4096), (8192, 4096, 11008), (8192, 100352, 4096)]
    if args.small:
        shapes = [(4096, 8192, 4096)]
    for M, N, K in shapes:
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
        acc = torch.zeros(N, K, device="cuda")
        cases = {
            "fwd  x·Wt": lambda: k.gemm(a, b),
            "dgrad dy·W": lambda: k.gemm(dy, b, b_trans=True),
            "wgrad dyt·x (+= fp32)": lambda: k.gemm(dy, a, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=acc),
        }
        # the library GEMM (cuBLAS through torch) on the same operands and layouts, same process, for comparison only;
        # its weight gradient is a bf16 product (it has no fp32-accumulating epilogue), i.e. it does less work
        out_fwd = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        out_dg = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
        out_wg = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        library = {
            "fwd  x·Wt": lambda: torch.matmul(a, b.t(), out=out_fwd),
            "dgrad dy·W": lambda: torch.matmul(dy, b, out=out_dg),
            "wgrad dyt·x (+= fp32)": lambda: torch.matmul(dy.t(), a, out=out_wg),
        }
        for name, fn in cases.items():
            if args.once:
                for _ in range(3):
                    fn()
                continue
            ms = timeit(fn)
            tf = 2 * M * N * K / ms / 1e9
            frac = f" ({tf / peak:.2f} of measured cuBLAS burst)" if peak else ""
            lib_ms = timeit(library[name])
            print(f"gemm {M}x{N}x{K} {name}: {ms:.3f} ms  {tf:.0f} TFLOP/s{frac}; library GEMM on the same operands "
                  f"{lib_ms:.3f} ms  {2 * M * N * K / lib_ms / 1e9:.0f} TFLOP/s", flush=True)
        del out_fwd, out_dg, out_wg


def bench_attention(args) -> None:
    from . import attention_native as N

    B, T, H, D = (1, 4096, 8, 128) if args.small else (2, 4096, 32, 128)
    qkv = torch.randn(B * T, 3 * H * D, device="cuda", dtype=torch.bfloat16)
    q = qkv[:, : H * D].view(B, T, H, D)
    kk = qkv[:, H * D : 2 * H * D].view(B, T, H, D)
    v = qkv[:, 2 * H * D :].view(B, T, H, D)
    scale = 1 / math.sqrt(D)
    o, lse = N.forward(q, kk, v, True, scale)
    do = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    dq = dqkv[:, : H * D].view(B, T, H, D)
    dk = dqkv[:, H * D : 2 * H * D].view(B, T, H, D)
    dv = dqkv[:, 2 * H * D :].view(B, T, H, D)
    fwd = lambda: N.forward(q, kk, v, True, scale)  # noqa: E731
    bwd = lambda: N.backward(do, q, kk, v, o, lse, dq, dk, dv, True, scale)  # noqa: E731
    if args.once:
        for _ in range(2):
            fwd()
            bwd()
        return
    fl = 4 * B * H * T * T * D / 2
    t1, t2 = timeit(fwd), timeit(bwd)
    print(f"attention causal B{B} T{T} H{H} D{D}: fwd {t1:.3f} ms {fl / t1 / 1e9:.0f} TFLOP/s | bwd {t2:.3f} ms {2.5 * fl / t2 / 1e9:.0f} TFLOP/s")
    try:
        import flash_attn.flash_attn_interface as fai

        t3 = timeit(lambda: fai._flash_attn_forward(q, kk, v, 0.0, scale, True, -1, -1, 0.0, None, False))
        t4 = timeit(lambda: fai._flash_attn_backward(do, q, kk, v, o, lse, dq, dk, dv, 0.0, scale, True, -1, -1, 0.0, None, False))
        print(f"  flash-attn library for comparison: fwd {t3:.3f} ms | bwd {t4:.3f} ms")
    except Exception as e:  # pragma: no cover
        print(f"  flash-attn library unavailable: {e}")


def bench_norm(args) -> None:
    M, D = (8192, 4096)
    bw = _peaks().get("hbm_gbs")
    x, res = torch.randn(M, D, device="cuda", dtype=torch.bfloat16), torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(D, device="cuda", dtype=torch.bfloat16)
    dy = torch.randn_like(x)
    out, rstd, _ = k.norm_fwd(x, w, None, 1e-6, True, residual=res)
    dw = torch.zeros(D, device="cuda")
    cases = {
        "rmsnorm+residual fwd": (lambda: k.norm_fwd(x, w, None, 1e-6, True, residual=res), 3 * M * D * 2),
        "rmsnorm bwd": (lambda: k.norm_bwd(dy, x, w, rstd, None, True, dweight=dw), 3 * M * D * 2),
    }
    h = torch.randn(M, 22016, device="cuda", dtype=torch.bfloat16)
    cases["swiglu fwd"] = (lambda: k.swiglu_fwd(h), M * 11008 * 3 * 2)
    dact = torch.randn(M, 11008, device="cuda", dtype=torch.bfloat16)
    cases["swiglu bwd"] = (lambda: k.swiglu_bwd(dact, h), M * 11008 * 5 * 2)
    # QK-norm + RoPE over the fused projection of the 7B shape (q | k | v, 3 x 4096 columns)
    from .fused_block import rope_tables

    T, hd = 4096, 128
    qkv = torch.randn(M, 3 * D, device="cuda", dtype=torch.bfloat16)
    dqkv = torch.randn_like(qkv)
    cos, sin = rope_tables(T, hd, 500000.0, torch.device("cuda"))
    _, rq, rk = k.qk_norm_rope_fwd(qkv, w, w, cos, sin, T, D, D, hd, 1e-6, 0.0, True, True)
    dwq, dwk = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    cases["qk-norm+rope fwd"] = (lambda: k.qk_norm_rope_fwd(qkv, w, w, cos, sin, T, D, D, hd, 1e-6, 0.0, True, True), 4 * M * D * 2)
    cases["qk-norm+rope bwd"] = (
        lambda: k.qk_norm_rope_bwd(qkv, dqkv, w, w, cos, sin, rq, rk, T, D, D, hd, 0.0, True, True, dwq=dwq, dwk=dwk), 6 * M * D * 2,
    )
    for name, (fn, nbytes) in cases.items():
        if args.once:
            fn()
            continue
        ms = timeit(fn)
        gbs = nbytes / ms / 1e6
        frac = f" ({gbs / bw:.2f} of measured copy bandwidth)" if bw else ""
        print(f"{name}: {ms:.3f} ms  {gbs:.0f} GB/s{frac}")


def bench_ce(args) -> None:
    R, V = (2048 if args.small else 8192), 100352
    bw = _peaks().get("hbm_gbs")
    logits = torch.randn(R, V, device="cuda", dtype=torch.bfloat16)
    labels = torch.randint(0, V, (R,), device="cuda")
    fn = lambda: k.cross_entropy_(logits, labels, -100, 1e-4, 1.0 / R, True)  # noqa: E731
    if args.once:
        fn()
        return
    ms = timeit(fn)
    gbs = 2 * R * V * 2 / ms / 1e6  # algorithmic: read once, write once
    print(f"cross-entropy fwd+bwd {R}x{V}: {ms:.3f} ms  {gbs:.0f} GB/s" + (f" ({gbs / bw:.2f} of measured copy bandwidth)" if bw else ""))


def bench_optim(args) -> None:
    n = 50_000_000 if args.small else 202_391_552
    bw = _peaks().get("hbm_gbs")
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    v.abs_()
    lowp = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    seg_end = torch.tensor([n], device="cuda", dtype=torch.int64)
    seg_wd, seg_lr = torch.tensor([0.1], device="cuda"), torch.tensor([3e-4], device="cuda")
    fn = lambda: k.adamw_flat(p, g, m, v, lowp, seg_end, seg_wd, seg_lr, 0.9, 0.95, 1e-8, 10, None)  # noqa: E731
    if args.once:
        fn()
        return
    ms = timeit(fn)
    gbs = n * (16 + 12 + 2) / ms / 1e6
    print(f"adamw {n} params: {ms:.3f} ms  {gbs:.0f} GB/s" + (f" ({gbs / bw:.2f} of measured copy bandwidth)" if bw else ""))


def bench_decode(args) -> None:
    """Serving kernels at OLMo-2 7B shapes, 32 sequences: the 4-bit GEMM with fused dequantisation (ff_proj: 22016 x 4096),
    the q/k/v post-processing kernel and the window attention kernel (256 of 512 columns live)."""
    from ..inference.w4a16 import QuantLinear

    bw = _peaks().get("hbm_gbs")
    R, d, H, hd, hidden, window, length = 32, 4096, 32, 128, 22016, 512, 256
    torch.manual_seed(0)
    ql = QuantLinear.from_linear_rtn(torch.nn.Linear(d, hidden, bias=False), group=128).cuda()
    x = torch.randn(R, d, device="cuda", dtype=torch.bfloat16)
    cases = {"w4a16 fused gemm 32x22016x4096": (lambda: ql(x), hidden * d // 2 + hidden * (d // 128) * 3)}
    qkv = torch.randn(R, 3 * d, device="cuda", dtype=torch.bfloat16)
    wn = torch.ones(d, device="cuda", dtype=torch.bfloat16)
    from .fused_block import rope_tables

    cos, sin = rope_tables(4096, hd, 500000.0, torch.device("cuda"))
    kc = torch.randn(R, H, window, hd, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn(R, H, window, hd, device="cuda", dtype=torch.bfloat16)
    rope_pos = torch.arange(R, device="cuda") + 200
    col = torch.tensor([length - 1], device="cuda")
    bias = torch.zeros(R, window, device="cuda", dtype=torch.bfloat16)
    cases["decode qkv (qk-norm + rope + cache write) 32x12288"] = (
        lambda: k.decode_qkv(qkv, wn, wn, cos, sin, rope_pos, col, kc, vc, d, d, hd, 1e-6, 0.0, True, True), R * 3 * d * 2 * 2)
    q = torch.randn(R, d, device="cuda", dtype=torch.bfloat16)
    cases["decode attention 32 seqs x 32 heads x 256 columns"] = (
        lambda: k.decode_attention(q, kc, vc, bias, length, hd ** -0.5, H), 2 * R * H * length * hd * 2)
    for name, (fn, nbytes) in cases.items():
        if args.once:
            fn()
            continue
        ms = timeit(fn)
        gbs = nbytes / ms / 1e6
        print(f"{name}: {ms * 1e3:.1f} us  {gbs:.0f} GB/s" + (f" ({gbs / bw:.2f} of measured copy bandwidth)" if bw else ""))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attention", "norm", "ce", "optim", "decode", "all"])
    ap.add_argument("--small", action="store_true", help="small case (for profiler captures)")
    ap.add_argument("--once", action="store_true", help="launch without timing (for profiler captures)")
    args = ap.parse_args()
    table = {"gemm": bench_gemm, "attention": bench_attention, "norm": bench_norm, "ce": bench_ce, "optim": bench_optim, "decode": bench_decode}
    for name, fn in table.items():
        if args.what in (name, "all"):
            fn(args)
    check_status()


if __name__ == "__main__":
    main()
