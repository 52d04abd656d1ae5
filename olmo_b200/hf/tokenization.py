"""Fast-tokenizer class registered for :class:`OLMoConfig` (reference: ``hf_olmo/tokenization_olmo_fast.py``)."""
from transformers import AutoTokenizer, PreTrainedTokenizerFast

from .configuration import OLMoConfig

__all__ = ["OLMoTokenizerFast"]


class OLMoTokenizerFast(PreTrainedTokenizerFast):
    """OLMo's tokenizers are plain ``tokenizers`` JSON files; nothing beyond the base class is needed."""


try:
    AutoTokenizer.register(OLMoConfig, fast_tokenizer_class=OLMoTokenizerFast)
except ValueError:
    pass
