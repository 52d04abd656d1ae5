"""Shared type aliases (reference: ``olmo/aliases.py:1-7``)."""
from os import PathLike
from typing import Union

__all__ = ["PathOrStr"]

PathOrStr = Union[str, PathLike]
