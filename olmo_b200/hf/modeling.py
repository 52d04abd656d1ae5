"""
``transformers`` model wrapper around :class:`olmo_b200.models.olmo.OLMo`.

Gives OLMo checkpoints the ``PreTrainedModel`` surface (``from_pretrained`` / ``save_pretrained``,
``generate`` through ``GenerationMixin``, gradient-checkpointing toggle, embedding resize, auto-class
registration).  State-dict keys are ``model.transformer.*`` as in the reference's
``hf_olmo/modeling_olmo.py:40-261``, so weight files are interchangeable.
"""
from __future__ import annotations

import logging
from dataclasses import fields
from typing import Callable, List, Optional, Tuple, Union

import torch
from transformers import GenerationMixin, PreTrainedModel
from transformers.modeling_outputs import CausalLMOutputWithPast
from transformers.models.auto import AutoModelForCausalLM

from ..config import ActivationCheckpointingStrategy, ModelConfig
from ..models.olmo import OLMo
from .configuration import OLMoConfig

__all__ = ["OLMoForCausalLM", "create_model_config_from_pretrained_config"]

log = logging.getLogger(__name__)


def create_model_config_from_pretrained_config(config: OLMoConfig) -> ModelConfig:
    """Rebuild the native model config; HF's attention-implementation switch selects flash attention."""
    from ..utils import structured as S

    raw = {f.name: getattr(config, f.name) for f in fields(ModelConfig) if hasattr(config, f.name)}
    model_config = S.build(ModelConfig, raw)
    impl = getattr(config, "_attn_implementation", None) or "eager"
    if impl == "flash_attention_2":
        model_config.flash_attention = True
    elif impl in ("eager", "sdpa"):
        model_config.flash_attention = False
    else:
        raise ValueError(f"Unexpected _attn_implementation {impl}")
    return model_config


class OLMoForCausalLM(PreTrainedModel, GenerationMixin):
    config_class = OLMoConfig
    base_model_prefix = "model"
    _no_split_modules = ["OLMoBlock"]
    _supports_flash_attn_2 = True
    _supports_flash_attn = True
    _supports_sdpa = True
    supports_gradient_checkpointing = True

    def __init__(self, config: OLMoConfig, model: Optional[OLMo] = None, init_params: bool = False):
        super().__init__(config)
        self._gradient_checkpointing_func: Optional[Callable] = None
        self._gradient_checkpointing = False
        if model is None:
            model_config = create_model_config_from_pretrained_config(config)
            model_config.init_device = "cpu"  # weights arrive through load_state_dict; never allocate on the GPU here
            model = OLMo(model_config, init_params=init_params)
        self.model = model
        self.post_init()

    def _init_weights(self, module) -> None:
        """Initialisation belongs to :meth:`OLMo.reset_parameters`; transformers must not overwrite it."""

    # -- gradient checkpointing --------------------------------------------------------------------

    @property
    def gradient_checkpointing(self) -> bool:
        return self._gradient_checkpointing

    @gradient_checkpointing.setter
    def gradient_checkpointing(self, enabled: bool) -> None:
        if self._gradient_checkpointing == enabled:
            return
        # HF has no notion of partial strategies: on means every block is recomputed
        strategy = ActivationCheckpointingStrategy.whole_layer if enabled else None
        self.model.set_activation_checkpointing(strategy, checkpoint_func=self._gradient_checkpointing_func)
        self._gradient_checkpointing = enabled

    # -- forward -----------------------------------------------------------------------------------

    def forward(
        self,
        input_ids: Optional[torch.LongTensor] = None,
        inputs_embeds: Optional[torch.FloatTensor] = None,
        attention_mask: Optional[torch.Tensor] = None,
        attention_bias: Optional[torch.Tensor] = None,
        past_key_values: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None,
        labels: Optional[torch.LongTensor] = None,
        use_cache: Optional[bool] = None,
        output_attentions: Optional[bool] = None,
        output_hidden_states: Optional[bool] = None,
        return_dict: Optional[bool] = None,
        cache_position=None,  # accepted and ignored: positions follow from the cache length
        **unused,
    ) -> Union[Tuple, CausalLMOutputWithPast]:
        if output_attentions:
            raise ValueError("output_attentions is not yet supported in OLMo")
        use_cache = self.config.use_cache if use_cache is None else use_cache
        if return_dict is None:
            return_dict = getattr(self.config, "return_dict", True)
        if past_key_values is not None and not isinstance(past_key_values, (list, tuple)):
            # a transformers Cache object that is still empty carries no state for this model
            past_key_values = None if len(past_key_values) == 0 else list(past_key_values)
        out = self.model.forward(
            input_ids=input_ids, input_embeddings=inputs_embeds, attention_mask=attention_mask, attention_bias=attention_bias,
            past_key_values=past_key_values, use_cache=use_cache, output_hidden_states=output_hidden_states,
        )
        loss = None
        if labels is not None:
            # position t predicts token t+1
            shift_logits = out.logits[..., :-1, :].contiguous().view(-1, self.config.embedding_size)
            shift_labels = labels[..., 1:].contiguous().view(-1).to(shift_logits.device)
            loss = torch.nn.functional.cross_entropy(shift_logits, shift_labels)
        if not return_dict:
            rest = (out.logits,) + tuple(out[1:])
            return (loss,) + rest if loss is not None else rest
        return CausalLMOutputWithPast(loss=loss, logits=out.logits, past_key_values=out.attn_key_values, hidden_states=out.hidden_states)

    @classmethod
    def can_generate(cls) -> bool:
        return True

    def prepare_inputs_for_generation(self, input_ids: torch.LongTensor, past_key_values=None, **kwargs):
        if past_key_values is not None and not isinstance(past_key_values, (list, tuple)):
            past_key_values = None if len(past_key_values) == 0 else past_key_values
        if past_key_values:
            input_ids = input_ids[:, -1:]  # only the newest token needs processing
            mask = kwargs.get("attention_mask")
        inputs = {"input_ids": input_ids, "past_key_values": past_key_values}
        for key in ("attention_mask", "attention_bias"):
            if kwargs.get(key) is not None:
                inputs[key] = kwargs[key]
        inputs["use_cache"] = kwargs.get("use_cache", self.config.use_cache)
        return inputs

    # -- embeddings --------------------------------------------------------------------------------

    def get_input_embeddings(self) -> torch.nn.Module:
        return self.model.transformer.wte

    def set_input_embeddings(self, value: torch.nn.Module) -> None:
        self.model.transformer.wte = value

    def get_output_embeddings(self):
        return self.model.transformer.wte if self.config.weight_tying else self.model.transformer.ff_out

    def set_output_embeddings(self, value: torch.nn.Module) -> None:
        if self.config.weight_tying:
            self.model.transformer.wte = value
        else:
            self.model.transformer.ff_out = value

    def tie_weights(self, *args, **kwargs) -> None:
        """No-op: with ``weight_tying`` the model has no separate output matrix and reads ``wte`` directly."""

    def resize_token_embeddings(self, new_num_tokens: Optional[int] = None, pad_to_multiple_of: Optional[int] = None, **kwargs) -> torch.nn.Embedding:
        """Resize the embedding table (and output head); ``embedding_size`` — not ``vocab_size`` — tracks the new row count."""
        wte = self.get_input_embeddings()
        if new_num_tokens is None and pad_to_multiple_of is None:
            return wte
        rows = wte.weight.shape[0] if new_num_tokens is None else new_num_tokens
        if pad_to_multiple_of is not None:
            rows = -(-rows // pad_to_multiple_of) * pad_to_multiple_of

        def resized(old: torch.Tensor, std: float) -> torch.Tensor:
            new = old.new_empty((rows, old.shape[1]))
            torch.nn.init.normal_(new, mean=0.0, std=std)
            keep = min(rows, old.shape[0])
            new[:keep] = old[:keep]
            return new

        std = float(getattr(self.config, "init_std", 0.02) or 0.02)
        with torch.no_grad():
            new_wte = torch.nn.Embedding(rows, wte.weight.shape[1], device=wte.weight.device, dtype=wte.weight.dtype)
            new_wte.weight.copy_(resized(wte.weight, std))
            self.model.transformer.wte = new_wte
            if not self.config.weight_tying:
                head = self.model.transformer.ff_out
                new_head = torch.nn.Linear(head.in_features, rows, bias=head.bias is not None, device=head.weight.device, dtype=head.weight.dtype)
                new_head.weight.copy_(resized(head.weight, std))
                if head.bias is not None:
                    new_head.bias.zero_()
                    new_head.bias[: min(rows, head.bias.shape[0])] = head.bias[: min(rows, head.bias.shape[0])]
                self.model.transformer.ff_out = new_head
        self.config.embedding_size = rows
        self.model.config.embedding_size = rows
        if rows < self.config.vocab_size:
            log.warning(
                "Resizing token embeddings to size %d, which is less than the vocab size %d defined in the model configuration. "
                "Make sure your tokenizer's vocabulary size is less than or equal to the new token embedding size.", rows, self.config.vocab_size,
            )
        return self.model.transformer.wte


try:
    AutoModelForCausalLM.register(OLMoConfig, OLMoForCausalLM)
except ValueError:
    pass
