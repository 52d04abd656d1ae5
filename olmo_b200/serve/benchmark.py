"""
Offline throughput of the generation engine on random-initialised weights of a named architecture:

    python -m olmo_b200.serve.benchmark --family olmo2-1b --requests 64 --prompt-len 128 --max-tokens 64 [--quantize rtn]

Prints one JSON line: generated tokens per second (device-timed between two synchronisations around the whole batch
of requests), time to first token, and the engine's counters.  Prompts are random token ids; ``ignore_eos`` keeps every
request running for exactly ``--max-tokens`` steps so that runs are comparable.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from typing import List


class _IdTokenizer:
    """Token ids are their own text: the benchmark measures the engine, not a vocabulary."""

    pad_token_id = 0
    eos_token_id = None

    def encode(self, s: str, add_special_tokens: bool = False) -> List[int]:
        return [int(t) for t in s.split()]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return ""


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--family", default="olmo2-1b")
    ap.add_argument("--n-layers", type=int, default=None, help="override the depth (for smoke runs)")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--max-batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--quantize", choices=["none", "rtn"], default="none")
    ap.add_argument("--device", default=None)
    ap.add_argument("--kv-cache", choices=["auto", "static", "dynamic"], default="auto")
    ap.add_argument("--window", type=int, default=None, help="static mode: columns per row (default: prompt + completion, rounded up)")
    ap.add_argument("--no-graphs", action="store_true", help="static mode without CUDA graphs")
    ap.add_argument("--no-decode-kernels", action="store_true", help="static mode with the module-level decode step")
    args = ap.parse_args(argv)

    import torch

    from ..config import ModelConfig
    from ..models.olmo import OLMo
    from ..recipes import model_dict
    from .engine import Engine, SamplingParams

    device = torch.device(args.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    spec = model_dict(args.family)
    spec["init_device"] = str(device)  # random weights are drawn on the device: no multi-gigabyte host copy
    if args.n_layers:
        spec["n_layers"] = args.n_layers
    cfg = ModelConfig.new(**spec)
    torch.manual_seed(0)
    model = OLMo(cfg).to(torch.bfloat16 if args.dtype == "bf16" else torch.float32).eval()
    if args.quantize == "rtn":
        from ..inference.quantize import quantize_model

        quantize_model(model, [torch.full((1, 8), cfg.eos_token_id, device=device)], method="rtn")
    window = args.window or min(cfg.max_sequence_length, -(-(args.prompt_len + args.max_tokens + 1) // 128) * 128)
    engine = Engine(model, _IdTokenizer(), max_batch=args.max_batch, device=device, kv_cache=args.kv_cache, window=window,
                    cuda_graphs=False if args.no_graphs else None, decode_kernels=False if args.no_decode_kernels else None)
    gen = torch.Generator().manual_seed(1)
    prompts = [torch.randint(2, cfg.vocab_size, (args.prompt_len,), generator=gen).tolist() for _ in range(args.requests)]
    params = SamplingParams(max_tokens=args.max_tokens, temperature=0.0, ignore_eos=True)

    engine.generate(prompts[: min(2, len(prompts))], SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True))  # warm-up
    # a second warm-up at full width captures the decode graph of the first length bucket outside the timed region
    engine.generate(prompts[: args.max_batch], SamplingParams(max_tokens=2, temperature=0.0, ignore_eos=True))
    for key in engine.stats:
        engine.stats[key] = 0
    if device.type == "cuda":
        torch.cuda.synchronize()
    start = time.perf_counter()
    done = engine.generate(prompts, params)
    if device.type == "cuda":
        torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    generated = sum(len(r.token_ids) for r in done)
    ttft = sorted(r.first_token_at - r.submitted_at for r in done)
    print(json.dumps({
        "metric": "generated_tokens_per_second", "value": generated / elapsed, "family": args.family, "n_layers": cfg.n_layers,
        "dtype": args.dtype, "quantize": args.quantize, "requests": args.requests, "max_batch": args.max_batch,
        "prompt_len": args.prompt_len, "max_tokens": args.max_tokens, "seconds": elapsed,
        "kv_cache": "dynamic" if engine._static is None else "static", "cuda_graphs": bool(engine._static and engine._static.cuda_graphs),
        "graph_replays": 0 if engine._static is None else engine._static.graph_replays,
        "decode_kernels": bool(engine._static and engine._static.fused),
        "ttft_median_s": ttft[len(ttft) // 2], "ttft_max_s": ttft[-1],
        "decode_tokens_per_second": engine.stats["decode_tokens"] / max(engine.stats["decode_seconds"], 1e-9),
        "decode_ms_per_step": 1e3 * engine.stats["decode_seconds"] / max(engine.stats["decode_steps"], 1),
        "prefill_tokens_per_second": engine.stats["prefill_tokens"] / max(engine.stats["prefill_seconds"], 1e-9),
        **{k: (round(v, 4) if k.endswith("_seconds") else int(v)) for k, v in engine.stats.items()},
    }))
    return 0


if __name__ == "__main__":
    sys.exit(main())
