"""Import-path parity with the reference's ``hf_olmo/configuration_olmo.py``: the class lives in :mod:`olmo_b200.hf.configuration`."""
from olmo_b200.hf.configuration import OLMoConfig

__all__ = ["OLMoConfig"]
