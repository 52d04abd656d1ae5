"""Serving: a continuous-batching generation engine and an OpenAI-compatible HTTP front end."""
from .engine import ContextLengthError, Engine, GenerationRequest, QueueFullError, SamplingParams
from .openai_api import create_app, default_chat_template, load_chat_template

__all__ = ["Engine", "SamplingParams", "GenerationRequest", "ContextLengthError", "QueueFullError", "create_app", "default_chat_template", "load_chat_template", "load_engine"]


def load_engine(checkpoint_dir: str, device: str = "cuda", dtype: str = "bf16", quantize: str = "none", max_batch: int = 32,
                tokenizer: str = "", kv_cache: str = "auto", window=None):
    """Engine over a native checkpoint directory (sharded or unsharded) or a directory written by the 4-bit
    quantisation driver; the tokenizer defaults to the one the checkpoint's config names."""
    import torch

    from ..model import OLMo
    from ..tokenizer import Tokenizer

    if quantize == "load":
        from ..inference.efficiency import load_quantized

        model = load_quantized(checkpoint_dir, device=device)
    else:
        model = OLMo.from_checkpoint(checkpoint_dir, device="cpu")
        model = model.to({"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype])
        if quantize == "rtn":
            from ..inference.quantize import quantize_model

            # round-to-nearest needs no statistics; one short sequence drives the layer-by-layer walk
            quantize_model(model, [torch.full((1, 8), model.config.eos_token_id)], method="rtn")
        model = model.to(device)
    tok = Tokenizer.from_file(tokenizer) if tokenizer and tokenizer.endswith(".json") else (
        Tokenizer.from_pretrained(tokenizer) if tokenizer else Tokenizer.from_checkpoint(checkpoint_dir))
    return Engine(model, tok, max_batch=max_batch, device=torch.device(device), kv_cache=kv_cache, window=window)
