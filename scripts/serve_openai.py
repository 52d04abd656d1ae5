"""
Serve a checkpoint behind an OpenAI-compatible HTTP API (completions, chat completions, streaming).

    python scripts/serve_openai.py CHECKPOINT_DIR --port 8000 [--dtype bf16] [--quantize rtn|load] [--api-key KEY]
    curl localhost:8000/v1/chat/completions -d '{"messages": [{"role": "user", "content": "Hello"}], "max_tokens": 64}'

The role of the reference's ``scripts/olmo2_modal_openai.py`` (which deploys a third-party server for an OLMo-2
instruct model), on this framework's own engine (``olmo_b200/serve``).
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("checkpoint_dir")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model-name", default=None, help="name reported by /v1/models (default: the checkpoint folder's name)")
    ap.add_argument("--device", default=None)
    ap.add_argument("--dtype", choices=["bf16", "fp16", "fp32"], default="bf16")
    ap.add_argument("--quantize", choices=["none", "rtn", "load"], default="none",
                    help="rtn: 4-bit round-to-nearest on load; load: the folder was written by the quantisation driver")
    ap.add_argument("--tokenizer", default="", help="tokenizer JSON file or identifier (default: from the checkpoint's config)")
    ap.add_argument("--max-batch", type=int, default=32, help="rows decoded together")
    ap.add_argument("--kv-cache", choices=["auto", "static", "dynamic"], default="auto",
                    help="static: preallocated key/value windows and CUDA graphs (default on a GPU for rotary models)")
    ap.add_argument("--window", type=int, default=None,
                    help="static mode: longest prompt + completion per request; sizes the key/value memory (default: the context length)")
    ap.add_argument("--chat-template", default=None,
                    help="Jinja chat template file, or a tokenizer_config.json with a 'chat_template' entry (default: the OLMo-2 instruct layout)")
    ap.add_argument("--max-queue", type=int, default=0, help="answer 429 when this many requests are waiting (0: no limit)")
    ap.add_argument("--api-key", default=None, help="require 'Authorization: Bearer KEY'")
    args = ap.parse_args(argv)

    import torch
    import uvicorn

    from olmo_b200.serve import create_app, load_engine

    device = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    engine = load_engine(args.checkpoint_dir, device=device, dtype=args.dtype if device != "cpu" else "fp32", quantize=args.quantize,
                         max_batch=args.max_batch, tokenizer=args.tokenizer, kv_cache=args.kv_cache, window=args.window)
    engine.max_queue = args.max_queue
    extra = {}
    if args.chat_template:
        from olmo_b200.serve import load_chat_template

        extra["chat_template"] = load_chat_template(args.chat_template)
    app = create_app(engine, model_name=args.model_name or Path(args.checkpoint_dir.rstrip("/")).name, api_key=args.api_key, **extra)
    uvicorn.run(app, host=args.host, port=args.port, log_level="info")
    return 0


if __name__ == "__main__":
    sys.exit(main())
