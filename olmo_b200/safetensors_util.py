"""
Nested state dict <-> flat safetensors file (format of the reference's ``olmo/safetensors_util.py:17-81``).

A leaf's key is ``base64(pickle((path tuple, is_pickled)))``; non-tensor leaves are pickled into uint8 tensors, so
files written by either implementation load in the other.
"""
from __future__ import annotations

import base64
import pickle
from typing import Any, Dict, Optional, Tuple

import torch

from .aliases import PathOrStr

__all__ = ["state_dict_to_safetensors_file", "safetensors_file_to_state_dict", "STKey"]


class STKey(tuple):
    """(path components, value_is_pickled)"""

    def __new__(cls, keys: Tuple, value_is_pickled: bool):
        return super().__new__(cls, (tuple(keys), bool(value_is_pickled)))

    @property
    def keys(self) -> Tuple:
        return self[0]

    @property
    def value_is_pickled(self) -> bool:
        return self[1]


def encode_key(key: STKey) -> str:
    return base64.urlsafe_b64encode(pickle.dumps((key.keys, key.value_is_pickled))).decode("utf-8")


def decode_key(key: str) -> STKey:
    keys, pickled = pickle.loads(base64.urlsafe_b64decode(key))
    return STKey(keys, pickled)


def flatten_dict(d: Dict) -> Dict[STKey, torch.Tensor]:
    out: Dict[STKey, torch.Tensor] = {}

    def walk(node: Any, path: Tuple) -> None:
        if isinstance(node, torch.Tensor):
            out[STKey(path, False)] = node
        elif isinstance(node, dict) and (node or not path):
            for k, v in node.items():
                walk(v, path + (k,))
        else:  # any other leaf, an empty dictionary included (walking into it would lose its key), is stored pickled
            blob = torch.frombuffer(bytearray(pickle.dumps(node)), dtype=torch.uint8)
            out[STKey(path, True)] = blob

    walk(d, ())
    return out


def unflatten_dict(d: Dict[STKey, torch.Tensor]) -> Dict:
    result: Dict = {}
    for key, value in d.items():
        leaf: Any = pickle.loads(value.numpy().data) if key.value_is_pickled else value
        node = result
        for k in key.keys[:-1]:
            node = node.setdefault(k, {})
        node[key.keys[-1]] = leaf
    return result


def state_dict_to_safetensors_file(state_dict: Dict, filename: PathOrStr) -> None:
    import safetensors.torch

    flat = {encode_key(k): v.contiguous() for k, v in flatten_dict(state_dict).items()}
    # The file format stores every tensor on its own and its writer refuses tensors whose memory overlaps (two names for
    # one tensor, overlapping views).  Disjoint slices of one buffer are fine; of overlapping ones all but the first
    # are copied, so what is written is what the caller passed.
    spans = sorted((t.data_ptr(), t.data_ptr() + t.numel() * t.element_size(), name) for name, t in flat.items() if t.numel() > 0)
    reach = -1
    for start, end, name in spans:
        if start < reach:
            flat[name] = flat[name].clone()
        else:
            reach = end  # only tensors that are written in place occupy their range
    safetensors.torch.save_file(flat, str(filename))


def safetensors_file_to_state_dict(filename: PathOrStr, map_location: Optional[str] = None) -> Dict:
    import safetensors.torch

    flat = safetensors.torch.load_file(str(filename), device=map_location or "cpu")
    return unflatten_dict({decode_key(k): v for k, v in flat.items()})
