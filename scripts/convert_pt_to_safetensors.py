#!/usr/bin/env python
"""``X.pt`` -> ``X.safetensors`` in the nested-key flavour that the checkpoint loaders prefer (reference:
``scripts/convert_pt_to_safetensors.py``).  Usage: ``convert_pt_to_safetensors.py FILE.pt [FILE.pt ...]``"""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch

from olmo_b200.safetensors_util import state_dict_to_safetensors_file
from olmo_b200.util import positional_args

if __name__ == "__main__":
    for name in positional_args(__doc__, 1):
        src = Path(name)
        state = torch.load(src, map_location="cpu", weights_only=False)
        dst = src.with_suffix(".safetensors")
        state_dict_to_safetensors_file(state, dst)
        print(dst)
