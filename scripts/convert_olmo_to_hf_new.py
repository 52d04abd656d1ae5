#!/usr/bin/env python
"""Unsharded OLMo-1 checkpoint -> ``transformers`` ``OlmoForCausalLM`` directory (reference: ``scripts/convert_olmo_to_hf_new.py``).
Same options as ``convert_olmo2_to_hf.py``; ``clip_qkv`` is carried into ``config.json``."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from convert_olmo2_to_hf import main

if __name__ == "__main__":
    main(expect="olmo")
