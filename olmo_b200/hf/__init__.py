"""HuggingFace ``transformers`` interoperability: config / model / tokenizer classes and checkpoint converters."""
from .configuration import OLMoConfig
from .modeling import OLMoForCausalLM
from .tokenization import OLMoTokenizerFast

__all__ = ["OLMoConfig", "OLMoForCausalLM", "OLMoTokenizerFast"]
