"""
``transformers`` configuration class for OLMo checkpoints in the ``hf_olmo`` layout.

Every :class:`olmo_b200.config.ModelConfig` field becomes a config attribute, so a ``config.json``
written by the reference's ``hf_olmo/configuration_olmo.py:14-65`` loads here and vice versa; the
``model_type`` string ("hf_olmo") is the one the reference registered.
"""
from __future__ import annotations

from transformers import AutoConfig, PretrainedConfig

from ..config import ModelConfig
from ..exceptions import OLMoConfigurationError

__all__ = ["OLMoConfig"]


class OLMoConfig(PretrainedConfig):
    model_type = "hf_olmo"
    keys_to_ignore_at_inference = ["past_key_values"]

    def __init__(self, use_cache: bool = False, **kwargs):
        merged = ModelConfig().asdict()
        merged.update(kwargs)
        merged["use_cache"] = use_cache
        merged["architectures"] = merged.get("architectures") or ["OLMoForCausalLM"]
        # enums serialise as their string values so that config.json stays plain JSON
        for key, value in list(merged.items()):
            if hasattr(value, "value") and isinstance(getattr(value, "value"), str):
                merged[key] = value.value
        super().__init__(**merged)
        # newer transformers releases no longer copy every keyword onto the instance
        for key, value in merged.items():
            if key not in self.__dict__:
                try:
                    setattr(self, key, value)
                except AttributeError:
                    pass

    # names the rest of transformers expects
    @property
    def num_attention_heads(self) -> int:
        return self.n_heads

    @property
    def num_hidden_layers(self) -> int:
        return self.n_layers

    @property
    def hidden_size(self) -> int:
        return self.d_model

    @property
    def effective_n_kv_heads(self) -> int:
        if self.n_kv_heads is None:
            return 1 if self.multi_query_attention is True else self.n_heads
        if self.multi_query_attention is None:
            return self.n_kv_heads
        implied = 1 if self.multi_query_attention else self.n_heads
        if self.n_kv_heads != implied:
            raise OLMoConfigurationError("You can't set `multi_query_attention` and `n_kv_heads` at the same time.")
        return implied


try:
    AutoConfig.register("hf_olmo", OLMoConfig)
except ValueError:  # already registered (e.g. the module was imported under two names)
    pass
