#!/usr/bin/env python
"""Unsharded OLMo-1 checkpoint -> ``transformers`` ``OlmoForCausalLM`` directory (reference: ``scripts/convert_olmo_to_hf_new.py``).
Same options as ``convert_olmo2_to_hf.py`` (``--input_dir``, ``--output_dir``, ``--tokenizer_json_path``, ``--no_tokenizer``,
``--no_fix_eos_token_id``, ``--safe_serialization`` / ``--no_safe_serialization``, ``--no_tmp_cleanup``); ``clip_qkv`` is carried
into ``config.json``."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from convert_olmo2_to_hf import main

if __name__ == "__main__":
    main(expect="olmo")
