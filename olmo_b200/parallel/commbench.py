"""
Roofline report for the fused compute + collective launches, at the OLMo-2 7B block shape.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \\
        -m olmo_b200.parallel.commbench [--iters 10] [--tokens 8192]

Two paths are timed on every rank with CUDA events (max over ranks reported), each launch preceded by a barrier so that
all ranks enter together:

* **AG→GEMM**: the four forward GEMMs of one block (``att_proj``, ``attn_out``, ``ff_proj``, ``ff_out``) whose launches
  also gather the *next* block's bf16 parameters from all peers (one slice per GEMM, sized by GEMM duration), against the
  same GEMMs alone, the gather alone (our
  standalone kernel) and NCCL's ``all_gather_into_tensor``.
* **GEMM→RS**: the four input-gradient GEMMs of a block whose launches also reduce-scatter one block's fp32
  gradients (sum over ranks, scale by 1/N, add into the local fp32 shard), against the GEMMs alone, the reduce-scatter
  alone and NCCL's ``reduce_scatter_tensor``.

The roofline of a fused launch pair is the slower of (its FLOPs ÷ the measured cuBLAS bf16 peak) and (the bytes that must
enter this GPU over NVLink ÷ the measured 770 GB/s per direction); the report gives achieved ÷ roofline.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
from types import SimpleNamespace
from typing import Callable, Dict

import torch
import torch.distributed as dist

NVLINK_MEASURED_GBS = 770.0  # peer copy, per direction, measured on this pool
BLOCK_PARAMS_7B = 202_391_552


def _peaks() -> Dict[str, float]:
    p = Path(__file__).resolve().parent.parent.parent / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except Exception:
        return {}


def timed(fn: Callable[[], None], prepare: Callable[[], None], iters: int, warmup: int = 3) -> float:
    """Median device time (ms) of ``fn``; ``prepare`` (flag publication, barrier) runs untimed before each call."""
    times = []
    for i in range(warmup + iters):
        prepare()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= warmup:
            times.append(a.elapsed_time(b))
    times.sort()
    t = torch.tensor([times[len(times) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--tokens", type=int, default=8192, help="rows of the activation matrix (micro-batch 2 x 4096)")
    ap.add_argument("--ag-ctas", type=int, default=None, help="CTAs set aside per gather-carrying launch; 0 = the spare warps of every GEMM CTA (default: engine default)")
    ap.add_argument("--rs-ctas", type=int, default=None, help="communication CTAs per reduce-scatter-carrying launch")
    args = ap.parse_args()

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)

    from olmo_b200 import ops
    from olmo_b200.ops import kernels as k
    from olmo_b200.parallel.peer import PeerComm

    numel = -(-BLOCK_PARAMS_7B // (world * 1024)) * (world * 1024)
    shard = numel // world
    unit = SimpleNamespace(index=0, numel=numel, shard_size=shard, grad=torch.zeros(shard, dtype=torch.float32, device=dev))
    engine = SimpleNamespace(device=dev, shard_world=world, shard_rank=rank, world=world, compute_dtype=torch.bfloat16, units=[unit])
    comm = PeerComm(engine, dist.group.WORLD)
    ctas = comm.comm_ctas if args.ag_ctas is None else args.ag_ctas
    rs_ctas = comm.rs_ctas if args.rs_ctas is None else args.rs_ctas
    comm.full_all.normal_(0, 0.02)
    comm.gfull_all.normal_(0, 1.0)

    M, d, ffn = args.tokens, 4096, 22016
    x = torch.randn(M, d, device=dev, dtype=torch.bfloat16)
    w_att = torch.randn(3 * d, d, device=dev, dtype=torch.bfloat16) * 0.02
    w_ff = torch.randn(ffn, d, device=dev, dtype=torch.bfloat16) * 0.02
    w_ffo = torch.randn(d, ffn // 2, device=dev, dtype=torch.bfloat16) * 0.02
    w_ao = torch.randn(d, d, device=dev, dtype=torch.bfloat16) * 0.02
    dy = torch.randn(M, d, device=dev, dtype=torch.bfloat16)
    act = torch.randn(M, ffn // 2, device=dev, dtype=torch.bfloat16)
    d_h = torch.randn(M, ffn, device=dev, dtype=torch.bfloat16)
    d_qkv = torch.randn(M, 3 * d, device=dev, dtype=torch.bfloat16)
    out_att = torch.empty(M, 3 * d, device=dev, dtype=torch.bfloat16)
    out_ff = torch.empty(M, ffn, device=dev, dtype=torch.bfloat16)
    out_ffo = torch.empty(M, ffn // 2, device=dev, dtype=torch.bfloat16)
    out_ao = torch.empty(M, d, device=dev, dtype=torch.bfloat16)
    nccl_full = torch.empty(numel, device=dev, dtype=torch.bfloat16)
    nccl_shard = torch.randn(shard, device=dev, dtype=torch.bfloat16)
    nccl_gfull = torch.randn(numel, device=dev, dtype=torch.float32)
    nccl_gshard = torch.empty(shard, device=dev, dtype=torch.float32)

    def nothing() -> None:
        pass

    # ---- AG -> GEMM
    from olmo_b200.parallel.peer import BWD_SPANS, FWD_SPANS

    def fwd(with_comm: bool) -> None:
        def kw(name):
            return {"comm": (comm.ag_task(unit, span=FWD_SPANS[name]), ctas)} if with_comm else {}

        k.gemm(x, w_att, out=out_att, **kw("att_proj"))
        k.gemm(x, w_ao, out=out_ao, **kw("attn_out"))
        k.gemm(x, w_ff, out=out_ff, **kw("ff_proj"))
        k.gemm(act, w_ffo, out=out_ao, **kw("ff_out"))

    def fwd_plain() -> None:
        fwd(False)

    def fwd_fused() -> None:
        fwd(True)

    res: Dict[str, float] = {}
    res["fwd_gemms_ms"] = timed(fwd_plain, nothing, args.iters)
    res["fwd_gemms_with_ag_ms"] = timed(fwd_fused, comm.publish_params, args.iters)
    res["ag_alone_ms"] = timed(lambda: comm.launch(comm.ag_task(unit)), comm.publish_params, args.iters)
    res["nccl_ag_ms"] = timed(lambda: dist.all_gather_into_tensor(nccl_full, nccl_shard), nothing, args.iters)

    # ---- GEMM -> RS
    def bwd(with_comm: bool) -> None:
        def kw(name):
            return {"comm": (comm.rs_task(unit, span=BWD_SPANS[name]), rs_ctas)} if with_comm else {}

        k.gemm(dy, w_ffo, b_trans=True, out=out_ffo, **kw("ff_out_dgrad"))
        k.gemm(d_h, w_ff, b_trans=True, out=out_ao, **kw("ff_proj_dgrad"))
        k.gemm(dy, w_ao, b_trans=True, out=out_ao, **kw("attn_out_dgrad"))
        k.gemm(d_qkv, w_att, b_trans=True, out=out_ao, **kw("att_proj_dgrad"))

    def bwd_plain() -> None:
        bwd(False)

    def bwd_fused() -> None:
        bwd(True)

    def open_grads() -> None:
        comm.begin_grad_epoch()
        comm.publish_grads(unit)

    res["bwd_gemms_ms"] = timed(bwd_plain, nothing, args.iters)
    res["bwd_gemms_with_rs_ms"] = timed(bwd_fused, open_grads, args.iters)
    res["rs_alone_ms"] = timed(lambda: comm.launch(comm.rs_task(unit)), open_grads, args.iters)
    res["nccl_rs_ms"] = timed(lambda: dist.reduce_scatter_tensor(nccl_gshard, nccl_gfull), nothing, args.iters)
    ops.check_status()

    peak = _peaks().get("bf16_tflops", 1590.0) * 1e12
    fwd_flops = 2.0 * M * d * (3 * d + d + ffn + ffn // 2)  # the four GEMMs of a block
    bwd_flops = fwd_flops  # their four input-gradient GEMMs
    ag_bytes = (world - 1) * shard * 2.0          # bf16 shards pulled from every peer
    rs_bytes = (world - 1) * shard * 4.0          # this rank's fp32 slice read from every peer
    link = NVLINK_MEASURED_GBS * 1e9
    roof_fwd = max(fwd_flops / peak, ag_bytes / link) * 1e3
    roof_bwd = max(bwd_flops / peak, rs_bytes / link) * 1e3
    res.update(
        world=world, tokens=M, ag_ctas=ctas, rs_ctas=rs_ctas, unit_params=numel,
        ag_bytes_in_per_gpu=ag_bytes, rs_bytes_in_per_gpu=rs_bytes,
        ag_alone_gbs=ag_bytes / res["ag_alone_ms"] / 1e6, rs_alone_gbs=rs_bytes / res["rs_alone_ms"] / 1e6,
        nccl_ag_gbs=ag_bytes / res["nccl_ag_ms"] / 1e6, nccl_rs_gbs=rs_bytes / res["nccl_rs_ms"] / 1e6,
        roofline_fwd_ms=roof_fwd, roofline_bwd_ms=roof_bwd,
        ag_gemm_fraction_of_roofline=roof_fwd / res["fwd_gemms_with_ag_ms"],
        gemm_rs_fraction_of_roofline=roof_bwd / res["bwd_gemms_with_rs_ms"],
        ag_hidden_fraction=1.0 - (res["fwd_gemms_with_ag_ms"] - res["fwd_gemms_ms"]) / res["ag_alone_ms"],
        rs_hidden_fraction=1.0 - (res["bwd_gemms_with_rs_ms"] - res["bwd_gemms_ms"]) / res["rs_alone_ms"],
        peak_source="MEASURED_PEAKS.json" if _peaks() else "fallback",
    )
    if rank == 0:
        print(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
