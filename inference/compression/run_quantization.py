#!/usr/bin/env python
"""4-bit (group 128) GPTQ quantisation of a checkpoint with activation ordering.

    python inference/compression/run_quantization.py --pretrained-model CKPT_DIR --quantized-model-dir OUT [--n-samples 128]
        [--calibration-data tokens.npy | text.txt] [--method gptq|rtn] [--seq-len 2048]

``--pretrained-model`` is an unsharded checkpoint folder of this framework.  Calibration samples come from
``--calibration-data``: a token memmap (``.npy``; ``--n-samples`` windows of ``--seq-len`` tokens are drawn from it) or a text
file that is tokenised with the checkpoint's tokenizer (the reference draws them from Wikitext-2 through the ``datasets``
hub, which needs a network).  Without calibration data the method falls back to round-to-nearest.
"""
import argparse
import sys
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


def calibration_samples(source: str, checkpoint_dir: str, n_samples: int, seq_len: int, seed: int = 0):
    import numpy as np
    import torch

    from olmo_b200.config import TrainConfig

    cfg = TrainConfig.load(Path(checkpoint_dir) / "config.yaml", validate_paths=False)
    seq_len = min(seq_len, cfg.model.max_sequence_length)
    if source.endswith(".npy"):
        dtype = np.uint16 if cfg.model.vocab_size <= 65536 else np.uint32
        tokens = np.memmap(source, dtype=dtype, mode="r")
    else:
        from olmo_b200.tokenizer import Tokenizer

        tokens = np.asarray(Tokenizer.from_checkpoint(checkpoint_dir).encode(Path(source).read_text(), add_special_tokens=False), dtype=np.int64)
    if len(tokens) <= seq_len:
        raise SystemExit(f"{source} holds {len(tokens)} tokens; at least {seq_len + 1} are needed")
    rng = np.random.default_rng(seed)
    starts = rng.integers(0, len(tokens) - seq_len, size=n_samples)
    return [torch.from_numpy(np.asarray(tokens[s : s + seq_len], dtype=np.int64))[None] for s in starts]


def main(argv=None) -> Path:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--pretrained-model", required=True, help="unsharded checkpoint folder")
    ap.add_argument("--quantized-model-dir", required=True, help="output folder")
    ap.add_argument("--n-samples", type=int, default=128, help="calibration windows")
    ap.add_argument("--calibration-data", default=None, help="token memmap (.npy) or text file")
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--method", choices=["gptq", "rtn"], default=None)
    ap.add_argument("--group-size", type=int, default=128)
    args = ap.parse_args(argv)
    from olmo_b200.inference.efficiency import run_quantization

    method = args.method or ("gptq" if args.calibration_data else "rtn")
    samples = []
    if method == "gptq":
        if not args.calibration_data:
            raise SystemExit("--method gptq needs --calibration-data")
        print("Getting data.")
        samples = calibration_samples(args.calibration_data, args.pretrained_model, args.n_samples, args.seq_len)
    print(f"Quantizing ({method})")
    tick = time.time()
    out = run_quantization(args.pretrained_model, args.quantized_model_dir, samples, group=args.group_size, method=method)
    print(f"Elapsed time:{(time.time() - tick) / 60:0.2f} minutes.")
    print(f"Saved to {out}")
    return out


if __name__ == "__main__":
    main()
