"""Import alias: ``import hf_olmo`` registers the OLMo classes with the ``transformers`` auto classes."""
from olmo_b200.hf import OLMoConfig, OLMoForCausalLM, OLMoTokenizerFast

__all__ = ["OLMoConfig", "OLMoForCausalLM", "OLMoTokenizerFast"]
