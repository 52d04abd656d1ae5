"""Import-path parity with the reference's ``hf_olmo/tokenization_olmo_fast.py``: the class lives in :mod:`olmo_b200.hf.tokenization`."""
from olmo_b200.hf.tokenization import OLMoTokenizerFast

__all__ = ["OLMoTokenizerFast"]
