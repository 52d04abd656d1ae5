"""Import-path parity with the reference's ``hf_olmo/modeling_olmo.py``: the classes live in :mod:`olmo_b200.hf.modeling`."""
from olmo_b200.hf.modeling import OLMoForCausalLM, create_model_config_from_pretrained_config

__all__ = ["OLMoForCausalLM", "create_model_config_from_pretrained_config"]
