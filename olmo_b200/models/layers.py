"""
Building blocks of the decoder: norms, rotary embedding, activations, attention-bias tables.

This is the *portable* implementation (plain PyTorch ops; CPU, MPS or CUDA) that defines the exact
math every sm_100a kernel is tested against.  Math follows the reference's ``olmo/model.py:108-408``.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ActivationType, LayerNormType, ModelConfig

__all__ = [
    "BufferCache",
    "Dropout",
    "LayerNormBase",
    "LayerNorm",
    "RMSLayerNorm",
    "RotaryEmbedding",
    "Activation",
    "GELU",
    "ReLU",
    "SwiGLU",
    "causal_attention_bias",
    "get_causal_attention_bias",
    "alibi_attention_bias",
    "autocast_dtype_for",
]


class BufferCache(dict):
    """Device tables (RoPE sin/cos, causal and ALiBi biases) shared by all blocks of one model.

    Kept outside ``nn.Module`` buffers on purpose: wrappers that flatten or shard module state must
    not touch these, and they never enter a state dict.
    """


def autocast_dtype_for(device: torch.device) -> Optional[torch.dtype]:
    """The active autocast dtype for ``device``'s type, or ``None`` when autocast is off."""
    kind = device.type
    try:
        if torch.is_autocast_enabled(kind):
            return torch.get_autocast_dtype(kind)
    except (RuntimeError, TypeError):
        pass
    return None


class Dropout(nn.Dropout):
    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if self.p == 0.0:
            return input
        return F.dropout(input, self.p, self.training, self.inplace)


# ------------------------------------------------------------------------------------------ norms


class LayerNormBase(nn.Module):
    """Common parameter handling of the norm variants.

    ``elementwise_affine=None`` means "follow ``config.layer_norm_with_affine``"; the bias exists only
    when the affine transform does and ``bias_for_layer_norm`` (default: ``include_bias``) is true.
    """

    def __init__(self, config: ModelConfig, *, size: Optional[int] = None, elementwise_affine: Optional[bool] = True):
        super().__init__()
        self.config = config
        self.eps = config.layer_norm_eps
        self.normalized_shape = (size or config.d_model,)
        affine = elementwise_affine if elementwise_affine is not None else config.layer_norm_with_affine
        if affine:
            self.weight = nn.Parameter(torch.ones(self.normalized_shape, device=config.init_device))
            use_bias = config.bias_for_layer_norm if config.bias_for_layer_norm is not None else config.include_bias
            if use_bias:
                self.bias = nn.Parameter(torch.zeros(self.normalized_shape, device=config.init_device))
            else:
                self.register_parameter("bias", None)
        else:
            self.register_parameter("weight", None)
            self.register_parameter("bias", None)

    @classmethod
    def build(cls, config: ModelConfig, size: Optional[int] = None, **kwargs) -> "LayerNormBase":
        kind = config.layer_norm_type
        if kind == LayerNormType.default:
            return LayerNorm(config, size=size, low_precision=False, **kwargs)
        if kind == LayerNormType.low_precision:
            return LayerNorm(config, size=size, low_precision=True, **kwargs)
        if kind == LayerNormType.rms:
            return RMSLayerNorm(config, size=size, **kwargs)
        raise NotImplementedError(f"Unknown LayerNorm type: '{kind}'")

    def reset_parameters(self) -> None:
        if self.weight is not None:
            nn.init.ones_(self.weight)
        if self.bias is not None:
            nn.init.zeros_(self.bias)


class LayerNorm(LayerNormBase):
    """Mean/variance LayerNorm; ``low_precision`` evaluates it in the autocast dtype."""

    def __init__(
        self,
        config: ModelConfig,
        size: Optional[int] = None,
        low_precision: bool = False,
        elementwise_affine: Optional[bool] = None,
    ):
        super().__init__(config, size=size, elementwise_affine=elementwise_affine)
        self.low_precision = low_precision

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.low_precision:
            return F.layer_norm(x, self.normalized_shape, weight=self.weight, bias=self.bias, eps=self.eps)
        target = autocast_dtype_for(x.device)
        w, b = self.weight, self.bias
        if target is not None:
            x = x.to(target)
            w = None if w is None else w.to(target)
            b = None if b is None else b.to(target)
        with torch.autocast(enabled=False, device_type=x.device.type):
            return F.layer_norm(x, self.normalized_shape, weight=w, bias=b, eps=self.eps)


class RMSLayerNorm(LayerNormBase):
    """``x · rsqrt(mean(x²) + eps)`` with fp32 statistics, cast back, then the affine transform."""

    def __init__(self, config: ModelConfig, size: Optional[int] = None, elementwise_affine: Optional[bool] = None):
        super().__init__(config, size=size, elementwise_affine=elementwise_affine)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        with torch.autocast(enabled=False, device_type=x.device.type):
            in_dtype = x.dtype
            xf = x.float()
            xf = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)
            x = xf.to(in_dtype)
        if self.weight is None:
            return x
        return self.weight * x + self.bias if self.bias is not None else self.weight * x


# ------------------------------------------------------------------------------------------- RoPE


class RotaryEmbedding(nn.Module):
    """Rotate-half (GPT-NeoX style) rotary position embedding.

    ``inv_freq_i = θ^(-2i/hd)``; the angle table is ``cat(freqs, freqs)`` so element ``j`` pairs with
    ``j ± hd/2``.  With ``rope_full_precision`` q and k are rotated in fp32 and cast back.
    Queries take the *last* ``query_len`` positions of the key range, which is what makes
    incremental decoding with a KV cache line up.
    """

    def __init__(self, config: ModelConfig, cache: BufferCache):
        super().__init__()
        self.config = config
        self._cache = cache
        # warm the table for the configured context
        self.get_rotary_embedding(config.max_sequence_length, _materialised_device(config))

    def get_rotary_embedding(self, seq_len: int, device: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
        sin, cos = self._cache.get("rope_pos_sin"), self._cache.get("rope_pos_cos")
        if sin is not None and cos is not None and sin.shape[-2] >= seq_len and cos.shape[-2] >= seq_len:
            if sin.device != device:
                sin, cos = sin.to(device), cos.to(device)
                self._cache["rope_pos_sin"], self._cache["rope_pos_cos"] = sin, cos
            return sin[:, :, :seq_len, :], cos[:, :, :seq_len, :]
        with torch.autocast(device.type, enabled=False):
            hd = self.config.d_model // self.config.n_heads
            inv_freq = 1.0 / (self.config.rope_theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float) / hd))
            t = torch.arange(seq_len, device=device, dtype=torch.float)
            freqs = torch.outer(t, inv_freq)
            angles = torch.cat((freqs, freqs), dim=-1)
            sin, cos = angles.sin()[None, None, :, :], angles.cos()[None, None, :, :]
        self._cache["rope_pos_sin"], self._cache["rope_pos_cos"] = sin, cos
        return sin, cos

    @staticmethod
    def rotate_half(x: torch.Tensor) -> torch.Tensor:
        a, b = x.chunk(2, dim=-1)
        return torch.cat((-b, a), dim=-1)

    def apply_rotary_pos_emb(self, sin: torch.Tensor, cos: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        return (t * cos + self.rotate_half(t) * sin).to(t.dtype)

    def forward(self, q: torch.Tensor, k: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        q_, k_ = (q.float(), k.float()) if self.config.rope_full_precision else (q, k)
        with torch.autocast(q.device.type, enabled=False):
            q_len, k_len = q_.shape[-2], k_.shape[-2]
            sin, cos = self.get_rotary_embedding(k_len, q_.device)
            sin, cos = sin.type_as(q_), cos.type_as(q_)
            q_ = self.apply_rotary_pos_emb(sin[:, :, k_len - q_len : k_len, :], cos[:, :, k_len - q_len : k_len, :], q_)
            k_ = self.apply_rotary_pos_emb(sin, cos, k_)
        return q_.type_as(q), k_.type_as(k)


def _materialised_device(config: ModelConfig) -> torch.device:
    if config.init_device is not None and config.init_device != "meta":
        return torch.device(config.init_device)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


# ------------------------------------------------------------------------------------ activations


class Activation(nn.Module):
    """``output_multiplier`` = (output width) / (input width) of the activation."""

    output_multiplier: float = 1.0

    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config

    @classmethod
    def build(cls, config: ModelConfig) -> "Activation":
        if config.activation_type == ActivationType.gelu:
            return GELU(config)
        if config.activation_type == ActivationType.relu:
            return ReLU(config)
        if config.activation_type == ActivationType.swiglu:
            return SwiGLU(config)
        raise NotImplementedError(f"Unknown activation: '{config.activation_type}'")


class GELU(Activation):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.gelu(x)


class ReLU(Activation):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.relu(x)


class SwiGLU(Activation):
    """First half of the input is the *value*, second half the *gate*: ``silu(gate) · value``."""

    output_multiplier = 0.5

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        value, gate = x.chunk(2, dim=-1)
        return F.silu(gate) * value


# -------------------------------------------------------------------------------- attention biases


def causal_attention_bias(seq_len: int, device: torch.device) -> torch.FloatTensor:
    bias = torch.zeros(seq_len, seq_len, device=device, dtype=torch.float)
    bias.masked_fill_(torch.ones_like(bias, dtype=torch.bool).triu_(1), torch.finfo(torch.float).min)
    return bias.view(1, 1, seq_len, seq_len)  # type: ignore[return-value]


def get_causal_attention_bias(cache: BufferCache, seq_len: int, device: torch.device) -> torch.Tensor:
    bias = cache.get("causal_attention_bias")
    if bias is not None and bias.shape[-1] >= seq_len:
        if bias.device != device:
            bias = bias.to(device)
            cache["causal_attention_bias"] = bias
        return bias
    with torch.autocast(device.type, enabled=False):
        bias = causal_attention_bias(seq_len, device)
    cache["causal_attention_bias"] = bias
    return bias


def alibi_attention_bias(seq_len: int, config: ModelConfig, device: torch.device) -> torch.FloatTensor:
    """``-|i-j| / 2^(m_h)`` with ``m_h = h · alibi_bias_max / n_heads`` for head ``h = 1..n_heads``."""
    pos = torch.arange(1 - seq_len, 1, dtype=torch.float, device=device)
    dist_ = -(pos.view(1, 1, 1, seq_len) - pos.view(1, 1, seq_len, 1)).abs()
    m = torch.arange(1, config.n_heads + 1, dtype=torch.float, device=device) * (config.alibi_bias_max / config.n_heads)
    return dist_ * (1.0 / (2 ** m.view(1, config.n_heads, 1, 1)))  # type: ignore[return-value]
