"""
Checkpoint converters.

* :func:`write_hf_olmo_checkpoint` — an unsharded OLMo checkpoint directory (``config.yaml`` + ``model.pt`` or
  ``model.safetensors``) becomes a ``transformers`` directory in the ``hf_olmo`` layout: ``config.json``, weights under
  the ``model.`` prefix, tokenizer files (reference: ``hf_olmo/convert_olmo_to_hf.py:34-316``).
* :func:`to_transformers_state_dict` / :func:`write_transformers_checkpoint` — the same checkpoint re-keyed for the
  architectures that ship inside ``transformers`` itself: ``Olmo2ForCausalLM`` for models with QK-norm and
  norm-after-sublayer (reference: ``scripts/convert_olmo2_to_hf.py:64-200``) and ``OlmoForCausalLM`` for the
  non-parametric-LayerNorm generation (reference: ``scripts/convert_olmo_to_hf_new.py:60-200``).

The fused projections are split here: ``att_proj`` rows are ``[q | k | v]``; ``ff_proj`` rows are ``[up | gate]``
(the activation is applied to the second half).
"""
from __future__ import annotations

import json
import logging
import shutil
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import torch

from ..aliases import PathOrStr
from ..config import ActivationType, BlockType, LayerNormType, ModelConfig, TrainConfig

__all__ = [
    "load_unsharded_model_state",
    "write_hf_olmo_checkpoint",
    "to_transformers_state_dict",
    "transformers_config_dict",
    "write_transformers_checkpoint",
]

log = logging.getLogger(__name__)


def load_unsharded_model_state(checkpoint_dir: PathOrStr) -> Dict[str, torch.Tensor]:
    """Full model weights of an unsharded checkpoint directory (safetensors preferred, ``model.pt`` otherwise)."""
    from ..checkpoint import load_state_dict

    return load_state_dict(checkpoint_dir, "model.pt", map_location="cpu")  # picks model.safetensors up when present


def _strip_prefixes(state: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    out = {}
    for key, value in state.items():
        for prefix in ("model.", "module.", "_fsdp_wrapped_module."):
            while key.startswith(prefix):
                key = key[len(prefix) :]
        out[key] = value
    return out


def _copy_tokenizer(config: TrainConfig, out_dir: Path, tokenizer_path: Optional[PathOrStr]) -> None:
    from ..tokenizer import Tokenizer
    from .tokenization import OLMoTokenizerFast

    if tokenizer_path is not None:
        tok = Tokenizer.from_file(tokenizer_path, eos_token_id=config.model.eos_token_id, pad_token_id=config.model.pad_token_id)
    else:
        try:
            tok = Tokenizer.from_train_config(config)
        except Exception as e:  # noqa: BLE001 - a missing vocabulary must not lose the converted weights
            log.warning("tokenizer '%s' could not be resolved (%s); skipping tokenizer files", config.tokenizer.identifier, e)
            return
    fast = OLMoTokenizerFast(
        tokenizer_object=tok.base_tokenizer, truncation=config.tokenizer.truncate_direction, max_length=config.model.max_sequence_length,
        eos_token=tok.decode([tok.eos_token_id], skip_special_tokens=False), pad_token=tok.decode([tok.pad_token_id], skip_special_tokens=False),
    )
    fast.model_input_names = ["input_ids", "attention_mask"]
    fast.save_pretrained(str(out_dir))


def write_hf_olmo_checkpoint(
    checkpoint_dir: PathOrStr, out_dir: Optional[PathOrStr] = None, *, tokenizer_path: Optional[PathOrStr] = None,
    safe_serialization: bool = True, keep_olmo_artifacts: bool = True,
) -> Path:
    """
    Write ``config.json`` + weights (+ tokenizer) so that ``AutoModelForCausalLM.from_pretrained(out_dir)`` works once
    ``hf_olmo`` has been imported.  ``out_dir`` defaults to the checkpoint directory itself.
    """
    from .configuration import OLMoConfig

    src = Path(checkpoint_dir)
    dst = Path(out_dir) if out_dir is not None else src
    dst.mkdir(parents=True, exist_ok=True)
    train_config = TrainConfig.load(src / "config.yaml", validate_paths=False)
    hf_config = OLMoConfig(**{k: v for k, v in train_config.model.asdict().items()})
    hf_config.save_pretrained(str(dst))

    state = {f"model.{k}": v.contiguous() for k, v in _strip_prefixes(load_unsharded_model_state(src)).items()}
    if safe_serialization:
        from safetensors.torch import save_file

        if dst == src and (dst / "model.safetensors").is_file():
            # the OLMo-flavoured file of the same name keeps its content under another name
            (dst / "model.safetensors").rename(dst / "model.olmo.safetensors")
        save_file(state, str(dst / "model.safetensors"), metadata={"format": "pt"})
    else:
        torch.save(state, dst / "pytorch_model.bin")
    _copy_tokenizer(train_config, dst, tokenizer_path)
    if not keep_olmo_artifacts and dst == src:
        for name in ("model.pt", "optim.pt", "train.pt"):
            (dst / name).unlink(missing_ok=True)
    return dst


# --------------------------------------------------------------------- native transformers layouts


def _flavour(cfg: ModelConfig) -> str:
    if cfg.block_type != BlockType.sequential or cfg.activation_type != ActivationType.swiglu:
        raise ValueError("only sequential SwiGLU blocks have a counterpart inside transformers")
    if cfg.alibi or not cfg.rope or cfg.include_bias:
        raise ValueError("the transformers architectures need RoPE, no ALiBi and bias-free linears")
    if cfg.attention_layer_norm and cfg.norm_after:
        if cfg.layer_norm_type != LayerNormType.rms:
            raise ValueError("Olmo2ForCausalLM uses RMSNorm")
        return "olmo2"
    if cfg.attention_layer_norm or cfg.norm_after:
        raise ValueError("QK-norm and norm-after come as a pair in Olmo2ForCausalLM")
    if cfg.layer_norm_type == LayerNormType.rms or cfg.layer_norm_with_affine:
        raise ValueError("OlmoForCausalLM has non-parametric LayerNorm only")
    return "olmo"


def transformers_config_dict(cfg: ModelConfig) -> Dict[str, Any]:
    """``config.json`` contents for the matching in-library architecture."""
    flavour = _flavour(cfg)
    hidden = cfg.mlp_hidden_size if cfg.mlp_hidden_size is not None else cfg.mlp_ratio * cfg.d_model
    out: Dict[str, Any] = dict(
        vocab_size=cfg.embedding_size or cfg.vocab_size, hidden_size=cfg.d_model, intermediate_size=hidden // 2,
        num_hidden_layers=cfg.n_layers, num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.effective_n_kv_heads,
        max_position_embeddings=cfg.max_sequence_length, pad_token_id=cfg.pad_token_id, bos_token_id=None, eos_token_id=cfg.eos_token_id,
        tie_word_embeddings=cfg.weight_tying, rope_theta=float(cfg.rope_theta), attention_bias=False, hidden_act="silu",
        attention_dropout=cfg.attention_dropout, use_cache=True,
    )
    if flavour == "olmo2":
        out.update(model_type="olmo2", architectures=["Olmo2ForCausalLM"], rms_norm_eps=cfg.layer_norm_eps)
    else:
        out.update(model_type="olmo", architectures=["OlmoForCausalLM"], clip_qkv=cfg.clip_qkv)
    return out


def to_transformers_state_dict(state: Dict[str, torch.Tensor], cfg: ModelConfig) -> Dict[str, torch.Tensor]:
    """Re-key (and split) OLMo weights for ``OlmoForCausalLM`` / ``Olmo2ForCausalLM``."""
    flavour = _flavour(cfg)
    state = _strip_prefixes(state)
    head_dim = cfg.d_model // cfg.n_heads
    kv = cfg.effective_n_kv_heads * head_dim
    out: Dict[str, torch.Tensor] = {"model.embed_tokens.weight": state["transformer.wte.weight"]}
    for i in range(cfg.n_layers):
        src, dst = f"transformer.blocks.{i}", f"model.layers.{i}"
        q, k, v = state[f"{src}.att_proj.weight"].split([cfg.d_model, kv, kv], dim=0)
        up, gate = state[f"{src}.ff_proj.weight"].chunk(2, dim=0)
        out[f"{dst}.self_attn.q_proj.weight"] = q.contiguous()
        out[f"{dst}.self_attn.k_proj.weight"] = k.contiguous()
        out[f"{dst}.self_attn.v_proj.weight"] = v.contiguous()
        out[f"{dst}.self_attn.o_proj.weight"] = state[f"{src}.attn_out.weight"]
        out[f"{dst}.mlp.up_proj.weight"] = up.contiguous()
        out[f"{dst}.mlp.gate_proj.weight"] = gate.contiguous()
        out[f"{dst}.mlp.down_proj.weight"] = state[f"{src}.ff_out.weight"]
        if flavour == "olmo2":
            out[f"{dst}.self_attn.q_norm.weight"] = state[f"{src}.q_norm.weight"]
            out[f"{dst}.self_attn.k_norm.weight"] = state[f"{src}.k_norm.weight"]
            out[f"{dst}.post_attention_layernorm.weight"] = state[f"{src}.attn_norm.weight"]
            out[f"{dst}.post_feedforward_layernorm.weight"] = state[f"{src}.ff_norm.weight"]
    if flavour == "olmo2":
        out["model.norm.weight"] = state["transformer.ln_f.weight"]
    out["lm_head.weight"] = state["transformer.wte.weight"] if cfg.weight_tying else state["transformer.ff_out.weight"]
    return out


def write_transformers_checkpoint(
    checkpoint_dir: PathOrStr, out_dir: PathOrStr, *, tokenizer_path: Optional[PathOrStr] = None, dtype: Optional[torch.dtype] = None,
    include_tokenizer: bool = True, safe_serialization: bool = True, fix_eos_token_id: bool = True,
) -> Tuple[Path, str]:
    """Convert an unsharded checkpoint for the in-library architecture; returns ``(out_dir, model_type)``.
    ``fix_eos_token_id``: configs of early OLMo-1 runs carry ``eos_token_id: 0`` although their tokenizer ends documents
    with 50279; the exported files then say 50279 (the reference's converters apply the same correction)."""
    from safetensors.torch import save_file

    src, dst = Path(checkpoint_dir), Path(out_dir)
    dst.mkdir(parents=True, exist_ok=True)
    train_config = TrainConfig.load(src / "config.yaml", validate_paths=False)
    cfg = train_config.model
    config = transformers_config_dict(cfg)
    state = to_transformers_state_dict(load_unsharded_model_state(src), cfg)
    if dtype is not None:
        state = {k: v.to(dtype) for k, v in state.items()}
    config["torch_dtype"] = str(next(iter(state.values())).dtype).replace("torch.", "")
    if cfg.weight_tying:
        state.pop("lm_head.weight")
    eos = cfg.eos_token_id
    if fix_eos_token_id and eos == 0:
        eos = 50279
        config["eos_token_id"] = eos
    (dst / "config.json").write_text(json.dumps(config, indent=2) + "\n")
    if safe_serialization:
        save_file({k: v.contiguous() for k, v in state.items()}, str(dst / "model.safetensors"), metadata={"format": "pt"})
    else:
        torch.save({k: v.contiguous() for k, v in state.items()}, dst / "pytorch_model.bin")
    (dst / "generation_config.json").write_text(
        json.dumps({"_from_model_config": True, "eos_token_id": eos, "pad_token_id": cfg.pad_token_id}, indent=2) + "\n"
    )
    if include_tokenizer:
        if tokenizer_path is not None and Path(tokenizer_path).is_file():
            shutil.copyfile(tokenizer_path, dst / "tokenizer.json")
        else:
            _copy_tokenizer(train_config, dst, None)
    return dst, config["model_type"]
