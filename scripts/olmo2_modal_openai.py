#!/usr/bin/env python
"""An OpenAI-compatible OLMo-2 endpoint as a `modal.com <https://modal.com>`_ app, or as a local process.

The reference's script of this name deploys a third-party inference server inside a Modal container.  This one deploys the
framework's own engine (:mod:`olmo_b200.serve`: continuous batching, fixed-shape decoding from CUDA graphs) behind the same
routes, in the same two ways:

    modal deploy scripts/olmo2_modal_openai.py          # needs the `modal` package and an account; serves `serve()` below
    python scripts/olmo2_modal_openai.py [--port 8000]  # no Modal: the same app under uvicorn on this machine

Settings come from the environment so that both ways read them alike: ``OLMO_SERVE_CHECKPOINT`` (an unsharded checkpoint
folder of this framework; required), ``OLMO_SERVE_MODEL_NAME`` (name reported by ``/v1/models``), ``MODAL_TOKEN`` (the
bearer token clients must send; unset: no authentication), ``OLMO_SERVE_GPU`` (Modal GPU type, default ``B200``).
"""
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

APP_NAME = "olmo-2-openai"
MINUTES = 60


def build_asgi_app():
    """The FastAPI application over a freshly loaded engine (called once per container or process)."""
    import torch

    from olmo_b200.serve import create_app, load_engine

    checkpoint = os.environ.get("OLMO_SERVE_CHECKPOINT")
    if not checkpoint:
        raise SystemExit("set OLMO_SERVE_CHECKPOINT to an unsharded checkpoint folder")
    device = "cuda" if torch.cuda.is_available() else "cpu"
    engine = load_engine(checkpoint, device=device, dtype="bf16" if device == "cuda" else "fp32",
                         max_batch=int(os.environ.get("OLMO_SERVE_MAX_BATCH", "32")))
    name = os.environ.get("OLMO_SERVE_MODEL_NAME") or Path(checkpoint.rstrip("/")).name
    return create_app(engine, model_name=name, api_key=os.environ.get("MODAL_TOKEN") or None)


try:  # the Modal deployment exists only where the package does
    import modal
except ImportError:
    modal = None

IMAGE_SOURCE_DIR = "/opt/olmo"  # where the two packages are copied inside the container image

if modal is not None:
    image = (
        modal.Image.from_registry("nvidia/cuda:12.9.0-devel-ubuntu24.04", add_python="3.12")
        .pip_install("torch", "numpy", "pyyaml", "tokenizers", "fastapi", "uvicorn", "safetensors")
        .add_local_dir(str(ROOT / "olmo_b200"), f"{IMAGE_SOURCE_DIR}/olmo_b200")
        .add_local_dir(str(ROOT / "olmo_data"), f"{IMAGE_SOURCE_DIR}/olmo_data")
    )
    app = modal.App(APP_NAME)

    @app.function(image=image, gpu=os.environ.get("OLMO_SERVE_GPU", "B200"), scaledown_window=5 * MINUTES, timeout=24 * 60 * MINUTES,
                  secrets=[modal.Secret.from_name("olmo-serve")])  # provides OLMO_SERVE_CHECKPOINT and MODAL_TOKEN
    @modal.concurrent(max_inputs=256)
    @modal.asgi_app()
    def serve():
        sys.path.insert(0, IMAGE_SOURCE_DIR)
        return build_asgi_app()


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    args = ap.parse_args(argv)
    import uvicorn

    uvicorn.run(build_asgi_app(), host=args.host, port=args.port, log_level="info")
    return 0


if __name__ == "__main__":
    sys.exit(main())
