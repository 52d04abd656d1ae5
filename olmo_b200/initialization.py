"""
Weight initialisation (reference: ``olmo/initialization.py:8-22``).

Unlike the reference, whose values depend on how FSDP happened to shard the flat parameters, each
parameter here can draw from its own generator keyed by ``(seed, parameter name)`` so that a model
initialises to the same weights at any world size (see :func:`param_generator`).
"""
from __future__ import annotations

import hashlib
from typing import Optional, Union

import torch
import torch.nn as nn

__all__ = ["init_normal", "param_generator"]


def param_generator(seed: int, name: str, device: Union[str, torch.device] = "cpu") -> torch.Generator:
    """A generator whose stream is a pure function of ``(seed, name)``."""
    digest = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    g = torch.Generator(device=device)
    g.manual_seed(int.from_bytes(digest, "little") & ((1 << 63) - 1))
    return g


def init_normal(
    module: Union[nn.Linear, nn.Embedding],
    std: float,
    init_cutoff_factor: Optional[float] = None,
    generator: Optional[torch.Generator] = None,
) -> None:
    """``N(0, std)``, truncated at ``±init_cutoff_factor·std`` when a factor is given; zero bias."""
    with torch.no_grad():
        if init_cutoff_factor is not None:
            cutoff = init_cutoff_factor * std
            nn.init.trunc_normal_(module.weight, mean=0.0, std=std, a=-cutoff, b=cutoff, generator=generator)
        else:
            nn.init.normal_(module.weight, mean=0.0, std=std, generator=generator)
        if isinstance(module, nn.Linear) and module.bias is not None:
            nn.init.zeros_(module.bias)
