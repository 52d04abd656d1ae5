"""
Text <-> token ids, on top of the HuggingFace ``tokenizers`` runtime.

Behaviour follows the reference's ``olmo/tokenizer.py:18-198``: the wrapper owns truncation (left or
right, leaving room for the end-of-sequence token), appends EOS exactly once, and defaults the pad
id to the EOS id.  Identifiers are resolved in this order: a file on disk, a file inside a packaged
data tree (``tokenizers/<name>.json`` under any directory :func:`olmo_b200.util.get_data_path`
searches), and finally a HuggingFace Hub name.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import List, Optional, Sequence, Union

from .aliases import PathOrStr
from .config import ModelConfig, TokenizerConfig, TrainConfig, TruncationDirection
from .exceptions import OLMoConfigurationError

__all__ = ["Tokenizer"]


def _runtime():
    try:
        import tokenizers
    except ImportError as e:  # pragma: no cover - the image ships it
        raise OLMoConfigurationError("the 'tokenizers' package is required for text tokenisation") from e
    return tokenizers.Tokenizer


def _packaged_file(identifier: str) -> Optional[Path]:
    from .util import get_data_path

    for candidate in (identifier, os.path.join("tokenizers", identifier), os.path.join("tokenizers", identifier + ".json")):
        try:
            found = get_data_path(candidate)
        except FileNotFoundError:
            continue
        if found.is_file():
            return found
    return None


class Tokenizer:
    """
    :param base_tokenizer: a ``tokenizers.Tokenizer``.
    :param eos_token_id: id appended to every encoded sequence.
    :param pad_token_id: id used for padding (defaults to ``eos_token_id``).
    :param truncate_to: cap on the encoded length, EOS included.
    :param truncate_direction: which end loses tokens when the cap applies.
    """

    def __init__(
        self,
        base_tokenizer,
        eos_token_id: int,
        pad_token_id: Optional[int] = None,
        truncate_to: Optional[int] = None,
        truncate_direction: Union[str, TruncationDirection] = TruncationDirection.right,
    ):
        self.base_tokenizer = base_tokenizer
        self.base_tokenizer.no_truncation()
        self.eos_token_id = eos_token_id
        self.pad_token_id = eos_token_id if pad_token_id is None else pad_token_id
        self.truncate_to = truncate_to
        self.truncate_direction = TruncationDirection(truncate_direction)

    # -- properties ------------------------------------------------------------------------------

    @property
    def vocab_size(self) -> int:
        return self.base_tokenizer.get_vocab_size()

    @property
    def eos_token(self) -> str:
        return self.decode([self.eos_token_id], skip_special_tokens=False)

    @property
    def pad_token(self) -> str:
        return self.decode([self.pad_token_id], skip_special_tokens=False)

    # -- construction ----------------------------------------------------------------------------

    @classmethod
    def from_file(cls, filename: PathOrStr, **kwargs) -> "Tokenizer":
        """Load a ``tokenizer.json`` written by ``tokenizers.Tokenizer.save``."""
        base = _runtime().from_file(str(filename))
        eos = kwargs.pop("eos_token_id", base.get_vocab_size() - 1)
        return cls(base, eos, **kwargs)

    @classmethod
    def from_pretrained(cls, identifier: str, **kwargs) -> "Tokenizer":
        """Fetch ``tokenizer.json`` of a HuggingFace Hub repository (needs network or a warm cache)."""
        base = _runtime().from_pretrained(identifier)
        eos = kwargs.pop("eos_token_id", base.get_vocab_size() - 1)
        return cls(base, eos, **kwargs)

    @classmethod
    def _resolve(cls, identifier: str, model: ModelConfig) -> "Tokenizer":
        ids = dict(eos_token_id=model.eos_token_id, pad_token_id=model.pad_token_id)
        if Path(identifier).is_file():
            tok = cls.from_file(identifier, **ids)
        else:
            packaged = _packaged_file(identifier)
            tok = cls.from_file(packaged, **ids) if packaged is not None else cls.from_pretrained(identifier, **ids)
        if model.vocab_size != tok.vocab_size:
            raise OLMoConfigurationError("vocab size mismatch between config and tokenizer")
        return tok

    @classmethod
    def from_train_config(cls, config: TrainConfig) -> "Tokenizer":
        return cls._resolve(config.tokenizer.identifier, config.model)

    @classmethod
    def from_checkpoint(cls, checkpoint_dir: PathOrStr) -> "Tokenizer":
        """Build the tokenizer named by the ``config.yaml`` stored next to a checkpoint."""
        from .util import resource_path

        config_path = resource_path(str(checkpoint_dir), "config.yaml")
        tokenizer_config = TokenizerConfig.load(config_path, key="tokenizer", validate_paths=False)
        model_config = ModelConfig.load(config_path, key="model", validate_paths=False)
        return cls._resolve(tokenizer_config.identifier, model_config)

    # -- encoding --------------------------------------------------------------------------------

    def add_special_tokens(self, input_ids: List[int]) -> List[int]:
        """Append EOS in place unless the sequence already ends with it."""
        if not input_ids or input_ids[-1] != self.eos_token_id:
            input_ids.append(self.eos_token_id)
        return input_ids

    def num_special_tokens_to_add(self, is_pair: bool = False) -> int:
        return 2 if is_pair else 1

    def _truncate(self, input_ids: List[int], truncate_to: Optional[int], direction: TruncationDirection) -> List[int]:
        if truncate_to is None or len(input_ids) <= truncate_to:
            return input_ids
        if direction == TruncationDirection.left:
            return input_ids[len(input_ids) - truncate_to :]
        return input_ids[:truncate_to]

    def encode(self, input: str, add_special_tokens: bool = True) -> List[int]:
        return self.encode_batch([input], add_special_tokens=add_special_tokens)[0]

    def encode_batch(self, inputs: Sequence[str], add_special_tokens: bool = True) -> List[List[int]]:
        budget = self.truncate_to
        if budget is not None and add_special_tokens:
            budget -= self.num_special_tokens_to_add(False)
        out: List[List[int]] = []
        for enc in self.base_tokenizer.encode_batch(list(inputs)):
            ids = self._truncate(list(enc.ids), budget, self.truncate_direction)
            out.append(self.add_special_tokens(ids) if add_special_tokens else ids)
        return out

    def decode(self, token_ids: List[int], skip_special_tokens: bool = True) -> str:
        return self.base_tokenizer.decode(list(token_ids), skip_special_tokens=skip_special_tokens)
