"""
Transformer blocks (reference: ``olmo/model.py:411-1067``).

Two execution paths share these modules and their parameter names:

* the portable path below (plain PyTorch ops, any device) — also the numerical oracle;
* the sm_100a path: when a block's input is a CUDA bf16 tensor, the configuration is one the fused
  kernels cover and the extension is enabled, :meth:`OLMoSequentialBlock.forward` hands the whole
  block to :func:`olmo_b200.ops.fused_block.run_block`, a single autograd node whose forward and
  backward are sequences of hand-written kernels with an explicit list of saved activations.
"""
from __future__ import annotations

import math
from functools import partial
from typing import Callable, Iterable, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ActivationCheckpointingStrategy, BlockType, InitFnType, ModelConfig
from ..initialization import init_normal
from ..torch_util import ensure_finite_
from .layers import (
    Activation,
    BufferCache,
    Dropout,
    LayerNorm,
    LayerNormBase,
    RotaryEmbedding,
    autocast_dtype_for,
    get_causal_attention_bias,
)

__all__ = [
    "StaticKV",
    "OLMoBlock",
    "OLMoSequentialBlock",
    "OLMoLlamaBlock",
    "OLMoBlockGroup",
    "activation_checkpoint_function",
    "should_checkpoint_block",
]

KV = Tuple[torch.Tensor, torch.Tensor]


class StaticKV:
    """Preallocated key/value window of one block for fixed-shape (graph-capturable) decoding.

    ``k`` and ``v`` are ``[rows, kv_heads, window, head_dim]``.  Keys are stored *after* the rotary embedding, rotated
    by their token's index in its own sequence (``rope_pos``: int64 ``[rows]``, the index of the token being decoded),
    so a row's place in the window carries no meaning and rows may be shifted inside it without touching values.
    ``pos`` is a one-element int64 tensor on the device (the column the new token is written to), ``length`` the
    number of leading columns the attention reads (a Python int: one captured graph per distinct value)."""

    __slots__ = ("k", "v", "pos", "length", "rope_pos")

    def __init__(self, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor, length: int, rope_pos: torch.Tensor):
        self.k, self.v, self.pos, self.length, self.rope_pos = k, v, pos, length, rope_pos


def activation_checkpoint_function(cfg: ModelConfig) -> Callable:
    """Non-re-entrant ``torch.utils.checkpoint`` that skips RNG bookkeeping when no dropout is active."""
    from torch.utils.checkpoint import checkpoint

    any_dropout = cfg.attention_dropout != 0.0 or cfg.embedding_dropout != 0.0 or cfg.residual_dropout != 0.0
    return partial(checkpoint, preserve_rng_state=any_dropout, use_reentrant=False)


_PERIODIC = {
    ActivationCheckpointingStrategy.one_in_two: (2, True),
    ActivationCheckpointingStrategy.one_in_three: (3, True),
    ActivationCheckpointingStrategy.one_in_four: (4, True),
    ActivationCheckpointingStrategy.one_in_eight: (8, True),
    ActivationCheckpointingStrategy.two_in_three: (3, False),
    ActivationCheckpointingStrategy.three_in_four: (4, False),
}


def should_checkpoint_block(strategy: Optional[ActivationCheckpointingStrategy], block_idx: int) -> bool:
    """``one_in_k`` checkpoints blocks with ``idx % k == 0``; ``(k-1)_in_k`` the complement."""
    if strategy is None or strategy == ActivationCheckpointingStrategy.fine_grained:
        return False
    if strategy == ActivationCheckpointingStrategy.whole_layer:
        return True
    period, on_zero = _PERIODIC[strategy]
    return (block_idx % period == 0) == on_zero


def _init_std_and_cutoff(config: ModelConfig, *, mitchell: float, megatron: float) -> Tuple[float, Optional[float]]:
    if config.init_fn == InitFnType.normal:
        return config.init_std, config.init_cutoff_factor
    if config.init_fn == InitFnType.mitchell:
        return mitchell, config.init_cutoff_factor or 3.0
    if config.init_fn == InitFnType.full_megatron:
        return megatron, config.init_cutoff_factor or 3.0
    raise NotImplementedError(config.init_fn)


class OLMoBlock(nn.Module):
    """Shared parts of both block types: QK-norm, RoPE, attention dispatch, output projections."""

    def __init__(self, layer_id: int, config: ModelConfig, cache: BufferCache):
        super().__init__()
        assert config.d_model % config.n_heads == 0
        self.layer_id = layer_id
        self.config = config
        self.hidden_size = config.ff_proj_width
        self._cache = cache
        self._activation_checkpoint_fn: Optional[Callable] = None

        self.dropout = Dropout(config.residual_dropout)
        self.k_norm: Optional[LayerNormBase] = None
        self.q_norm: Optional[LayerNormBase] = None
        if config.attention_layer_norm:
            # the norm spans the whole projected vector (all heads jointly), not one head
            self.k_norm = LayerNormBase.build(
                config,
                size=config.head_dim * config.effective_n_kv_heads,
                elementwise_affine=config.attention_layer_norm_with_affine,
            )
            self.q_norm = LayerNormBase.build(config, elementwise_affine=config.attention_layer_norm_with_affine)
        if config.clip_qkv is not None:
            assert config.clip_qkv > 0

        self.act = Activation.build(config)
        act_out = self.act.output_multiplier * self.hidden_size
        assert act_out % 1 == 0
        self.attn_out = nn.Linear(config.d_model, config.d_model, bias=config.include_bias, device=config.init_device)
        self.ff_out = nn.Linear(int(act_out), config.d_model, bias=config.include_bias, device=config.init_device)
        self.ff_out._is_residual = True  # type: ignore[assignment]
        if config.rope:
            self.rotary_emb = RotaryEmbedding(config, cache)

        self.flash_attn_func = None
        self.flash_attn_varlen_func = None
        if config.flash_attention:
            try:
                from flash_attn import flash_attn_func, flash_attn_varlen_func  # type: ignore

                self.flash_attn_func, self.flash_attn_varlen_func = flash_attn_func, flash_attn_varlen_func
            except Exception:
                pass

    # -- initialisation ---------------------------------------------------------------------
    def reset_parameters(self) -> None:
        for norm in (self.k_norm, self.q_norm):
            if norm is not None:
                norm.reset_parameters()
        cfg = self.config
        if cfg.init_fn == InitFnType.mitchell:
            attn_std = 1 / math.sqrt(2 * cfg.d_model * (self.layer_id + 1))
            ff_std = 1 / math.sqrt(2 * self.ff_out.in_features * (self.layer_id + 1))
            cutoff: Optional[float] = cfg.init_cutoff_factor or 3.0
        else:
            attn_std, cutoff = _init_std_and_cutoff(
                cfg, mitchell=0.0, megatron=cfg.init_std / math.sqrt(2.0 * cfg.n_layers)
            )
            ff_std = attn_std
        init_normal(self.attn_out, std=attn_std, init_cutoff_factor=cutoff)
        init_normal(self.ff_out, std=ff_std, init_cutoff_factor=cutoff)

    def set_activation_checkpointing(
        self, strategy: Optional[ActivationCheckpointingStrategy], checkpoint_func: Optional[Callable] = None
    ) -> None:
        if strategy == ActivationCheckpointingStrategy.fine_grained:
            self._activation_checkpoint_fn = checkpoint_func or activation_checkpoint_function(self.config)
        else:
            self._activation_checkpoint_fn = None

    def _maybe_ckpt(self, fn: Callable, *args):
        if self._activation_checkpoint_fn is not None:
            return self._activation_checkpoint_fn(fn, *args)
        return fn(*args)

    # -- attention ----------------------------------------------------------------------------
    @staticmethod
    def _cast_attn_bias(bias: torch.Tensor, input_dtype: torch.dtype) -> torch.Tensor:
        target = autocast_dtype_for(bias.device) or input_dtype
        if bias.dtype != target:
            bias = bias.to(target)
            ensure_finite_(bias, check_neg_inf=True, check_pos_inf=False)
        return bias

    def _scaled_dot_product_attention(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        attn_mask: Optional[torch.Tensor] = None,
        dropout_p: float = 0.0,
        is_causal: bool = False,
        max_doc_len: Optional[int] = None,
        cu_doc_lens: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        """``q`` is ``(B, nh, Tq, hd)``, ``k``/``v`` are ``(B, n_kv, Tk, hd)``; returns ``(B, nh, Tq, hd)``."""
        from ..ops import attention as attn_ops

        if max_doc_len is not None and cu_doc_lens is not None:
            assert attn_mask is None, "attn-mask is currently not supported with document masking"
            B, T, D = q.size(0), q.size(2), q.size(3)
            out = attn_ops.varlen_attention(
                q.transpose(1, 2).reshape(B * T, -1, D),
                k.transpose(1, 2).reshape(B * T, -1, D),
                v.transpose(1, 2).reshape(B * T, -1, D),
                cu_doc_lens,
                max_doc_len,
                dropout_p=dropout_p,
                causal=is_causal,
                library_fn=self.flash_attn_varlen_func,
            )
            return out.view(B, T, -1, D).transpose(1, 2)
        if attn_mask is None and self.config.flash_attention and q.is_cuda and q.dtype in (torch.bfloat16, torch.float16):
            out = attn_ops.flash_attention(
                q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                dropout_p=dropout_p, causal=is_causal, library_fn=self.flash_attn_func,
            )
            return out.transpose(1, 2)
        n_q, n_kv = q.size(1), k.size(1)
        if n_q != n_kv:  # grouped / multi-query: expand kv heads for the generic SDPA
            assert n_q % n_kv == 0
            k = k.repeat_interleave(n_q // n_kv, dim=1, output_size=n_q)
            v = v.repeat_interleave(n_q // n_kv, dim=1, output_size=n_q)
        return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal)

    def attention(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        attention_bias: Optional[torch.Tensor] = None,
        layer_past: Optional[KV] = None,
        use_cache: bool = False,
        max_doc_len: Optional[int] = None,
        cu_doc_lens: Optional[torch.Tensor] = None,
    ) -> Tuple[torch.Tensor, Optional[KV]]:
        B, T, C = q.size()
        cfg = self.config
        dtype = k.dtype
        if self.q_norm is not None and self.k_norm is not None:
            q = self.q_norm(q).to(dtype=dtype)
            k = self.k_norm(k).to(dtype=dtype)
        hd = C // cfg.n_heads
        q = q.view(B, T, cfg.n_heads, hd).transpose(1, 2)
        k = k.view(B, T, cfg.effective_n_kv_heads, hd).transpose(1, 2)
        v = v.view(B, T, cfg.effective_n_kv_heads, hd).transpose(1, 2)
        if isinstance(layer_past, StaticKV):
            return self.attn_out(self._static_window_attention(q, k, v, attention_bias, layer_past).transpose(1, 2).reshape(B, T, C)), None
        if layer_past is not None:
            past_k, past_v = layer_past
            k = torch.cat((past_k, k), dim=-2)
            v = torch.cat((past_v, v), dim=-2)
        present = (k, v) if use_cache else None  # cached keys are pre-RoPE
        q_len, k_len = q.shape[-2], k.shape[-2]
        if cfg.rope:
            q, k = self.rotary_emb(q, k)
        if attention_bias is not None:
            attention_bias = self._cast_attn_bias(attention_bias[:, :, k_len - q_len : k_len, :k_len], dtype)
        att = self._scaled_dot_product_attention(
            q,
            k,
            v,
            attn_mask=attention_bias,
            dropout_p=cfg.attention_dropout if self.training else 0.0,
            is_causal=attention_bias is None,
            max_doc_len=max_doc_len,
            cu_doc_lens=cu_doc_lens,
        )
        att = att.transpose(1, 2).contiguous().view(B, T, C)
        return self.attn_out(att), present

    def _static_window_attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, bias: Optional[torch.Tensor], cache: StaticKV) -> torch.Tensor:
        """One decode step against a :class:`StaticKV` window: rotate the new query/key by the write column, store
        key and value there, attend over the first ``cache.length`` columns under the additive ``bias``
        (``[rows, 1, 1, window]``: padding and not-yet-written columns carry the dtype's minimum).  Every shape is
        fixed and the column arrives as a device tensor, so the step can be captured in a CUDA graph."""
        cfg = self.config
        assert q.shape[2] == 1 and bias is not None, "the static window decodes one token per row under an explicit bias"
        if cfg.rope:
            sin, cos = self.rotary_emb.get_rotary_embedding(cfg.max_sequence_length, q.device)
            # one angle row per sequence: [rows, 1, 1, head_dim]
            sin = sin[0, 0].index_select(0, cache.rope_pos)[:, None, None, :]
            cos = cos[0, 0].index_select(0, cache.rope_pos)[:, None, None, :]
            q_, k_ = (q.float(), k.float()) if cfg.rope_full_precision else (q, k)
            with torch.autocast(q.device.type, enabled=False):
                sin, cos = sin.type_as(q_), cos.type_as(q_)
                q = self.rotary_emb.apply_rotary_pos_emb(sin, cos, q_).type_as(q)
                k = self.rotary_emb.apply_rotary_pos_emb(sin, cos, k_).type_as(k)
        cache.k.index_copy_(2, cache.pos, k.to(cache.k.dtype))
        cache.v.index_copy_(2, cache.pos, v.to(cache.v.dtype))
        n = cache.length
        keys, values = cache.k[:, :, :n].to(q.dtype), cache.v[:, :, :n].to(q.dtype)
        return F.scaled_dot_product_attention(
            q, keys, values, attn_mask=bias[..., :n].to(q.dtype), enable_gqa=q.shape[1] != keys.shape[1]
        )

    def forward(self, x, attention_bias=None, layer_past=None, use_cache=False, max_doc_len=None, cu_doc_lens=None):
        raise NotImplementedError

    @classmethod
    def build(cls, layer_id: int, config: ModelConfig, cache: BufferCache) -> "OLMoBlock":
        if config.block_type == BlockType.sequential:
            return OLMoSequentialBlock(layer_id, config, cache)
        if config.block_type == BlockType.llama:
            return OLMoLlamaBlock(layer_id, config, cache)
        raise NotImplementedError(f"Unknown block type: '{config.block_type}'")


class OLMoSequentialBlock(OLMoBlock):
    """Fused-QKV block.  ``norm_after=False``: ``x + f(norm(x))``; ``norm_after=True``: ``x + norm(f(x))``."""

    def __init__(self, layer_id: int, config: ModelConfig, cache: BufferCache):
        super().__init__(layer_id, config, cache)
        hd = config.head_dim
        self.fused_dims = (config.d_model, config.effective_n_kv_heads * hd, config.effective_n_kv_heads * hd)
        self.att_proj = nn.Linear(config.d_model, sum(self.fused_dims), bias=config.include_bias, device=config.init_device)
        self.ff_proj = nn.Linear(config.d_model, self.hidden_size, bias=config.include_bias, device=config.init_device)
        self.attn_norm = LayerNorm.build(config, size=config.d_model)
        self.ff_norm = LayerNorm.build(config, size=config.d_model)

    def reset_parameters(self) -> None:
        super().reset_parameters()
        self.attn_norm.reset_parameters()
        self.ff_norm.reset_parameters()
        std, cutoff = _init_std_and_cutoff(
            self.config, mitchell=1 / math.sqrt(self.config.d_model), megatron=self.config.init_std
        )
        init_normal(self.att_proj, std, cutoff)
        init_normal(self.ff_proj, std, cutoff)

    def forward(
        self,
        x: torch.Tensor,
        attention_bias: Optional[torch.Tensor] = None,
        layer_past: Optional[KV] = None,
        use_cache: bool = False,
        max_doc_len: Optional[int] = None,
        cu_doc_lens: Optional[torch.Tensor] = None,
    ) -> Tuple[torch.Tensor, Optional[KV]]:
        from ..ops import fused_block

        if fused_block.eligible(self, x, attention_bias, layer_past, use_cache, doc_masking=cu_doc_lens is not None):
            return fused_block.run_block(self, x, max_doc_len=max_doc_len, cu_doc_lens=cu_doc_lens), None

        cfg = self.config
        h = x if cfg.norm_after else self._maybe_ckpt(self.attn_norm, x)
        qkv = self.att_proj(h)
        if cfg.clip_qkv is not None:
            qkv.clamp_(min=-cfg.clip_qkv, max=cfg.clip_qkv)
        q, k, v = qkv.split(self.fused_dims, dim=-1)
        att, cache = self._maybe_ckpt_attention(q, k, v, attention_bias, layer_past, use_cache, max_doc_len, cu_doc_lens)
        if cfg.norm_after:
            att = self._maybe_ckpt(self.attn_norm, att)
        x = x + self.dropout(att)

        residual = x
        h = x if cfg.norm_after else self._maybe_ckpt(self.ff_norm, x)
        h = self.ff_proj(h)
        h = self._maybe_ckpt(self.act, h)
        h = self.ff_out(h)
        if cfg.norm_after:
            h = self._maybe_ckpt(self.ff_norm, h)
        return residual + self.dropout(h), cache

    def _maybe_ckpt_attention(self, q, k, v, bias, layer_past, use_cache, max_doc_len, cu_doc_lens):
        if self._activation_checkpoint_fn is not None:
            return self._activation_checkpoint_fn(
                self.attention, q, k, v, bias, layer_past=layer_past, use_cache=use_cache,
                max_doc_len=max_doc_len, cu_doc_lens=cu_doc_lens,
            )
        return self.attention(
            q, k, v, bias, layer_past=layer_past, use_cache=use_cache, max_doc_len=max_doc_len, cu_doc_lens=cu_doc_lens
        )


class OLMoLlamaBlock(OLMoBlock):
    """Separate q/k/v projections and an explicit ``softmax(QKᵀ/√d + bias)·V`` attention (pre-norm only)."""

    def __init__(self, layer_id: int, config: ModelConfig, cache: BufferCache):
        super().__init__(layer_id, config, cache)
        self.attn_norm = LayerNorm.build(config)
        self.ff_norm = LayerNorm.build(config)
        kv_dim = config.head_dim if config.multi_query_attention else config.d_model
        dev = config.init_device
        self.q_proj = nn.Linear(config.d_model, config.d_model, bias=config.include_bias, device=dev)
        self.k_proj = nn.Linear(config.d_model, kv_dim, bias=config.include_bias, device=dev)
        self.v_proj = nn.Linear(config.d_model, kv_dim, bias=config.include_bias, device=dev)
        self.ff_proj = nn.Linear(config.d_model, self.hidden_size, bias=config.include_bias, device=dev)

    def reset_parameters(self) -> None:
        super().reset_parameters()
        self.attn_norm.reset_parameters()
        self.ff_norm.reset_parameters()
        std, cutoff = _init_std_and_cutoff(
            self.config, mitchell=1 / math.sqrt(self.config.d_model), megatron=self.config.init_std
        )
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.ff_proj):
            init_normal(lin, std, cutoff)

    def _scaled_dot_product_attention(
        self, q, k, v, attn_mask=None, dropout_p=0.0, is_causal=False, max_doc_len=None, cu_doc_lens=None
    ) -> torch.Tensor:
        if max_doc_len is not None or cu_doc_lens is not None:
            raise NotImplementedError(f"attention document masking is not implemented for {type(self).__name__}")
        n_q, n_kv = q.size(1), k.size(1)
        if n_q != n_kv:
            k = k.expand(-1, n_q, -1, -1) if n_kv == 1 else k.repeat_interleave(n_q // n_kv, dim=1)
            v = v.expand(-1, n_q, -1, -1) if n_kv == 1 else v.repeat_interleave(n_q // n_kv, dim=1)
        scores = torch.matmul(q, k.transpose(-2, -1)) / math.sqrt(q.size(-1))
        if is_causal:
            assert attn_mask is None
            q_len, k_len = q.shape[-2], k.shape[-2]
            scores = scores + get_causal_attention_bias(self._cache, k_len, q.device)[:, :, :q_len, :k_len]
        elif attn_mask is not None:
            scores = scores + attn_mask.to(q.dtype)
        probs = F.softmax(scores, dim=-1).to(q.dtype)
        probs = F.dropout(probs, p=dropout_p)
        return torch.matmul(probs, v)

    def forward(
        self,
        x: torch.Tensor,
        attention_bias: Optional[torch.Tensor] = None,
        layer_past: Optional[KV] = None,
        use_cache: bool = False,
        max_doc_len: Optional[int] = None,
        cu_doc_lens: Optional[torch.Tensor] = None,
    ) -> Tuple[torch.Tensor, Optional[KV]]:
        h = self.attn_norm(x)
        q, k, v = self.q_proj(h), self.k_proj(h), self.v_proj(h)
        c = self.config.clip_qkv
        if c is not None:
            q.clamp_(min=-c, max=c)
            k.clamp_(min=-c, max=c)
            v.clamp_(min=-c, max=c)
        att, cache = self.attention(
            q, k, v, attention_bias, layer_past=layer_past, use_cache=use_cache,
            max_doc_len=max_doc_len, cu_doc_lens=cu_doc_lens,
        )
        x = x + self.dropout(att)
        residual = x
        h = self._maybe_ckpt(self.ff_norm, x)
        h = self.ff_proj(h)
        h = self._maybe_ckpt(self.act, h)
        h = self.dropout(self.ff_out(h))
        return residual + h, cache


class OLMoBlockGroup(nn.ModuleList):
    """A run of consecutive blocks treated as one sharding / checkpointing unit."""

    def __init__(self, config: ModelConfig, layer_offset: int, modules: Optional[Iterable[nn.Module]] = None):
        super().__init__(modules)
        self.config = config
        self.layer_offset = layer_offset
        self.activation_checkpointing_strategy: Optional[ActivationCheckpointingStrategy] = None
        self._activation_checkpoint_fn = activation_checkpoint_function(config)

    def forward(
        self,
        x: torch.Tensor,
        attention_bias: Optional[torch.Tensor] = None,
        layers_past: Optional[List[KV]] = None,
        use_cache: bool = False,
        max_doc_len: Optional[int] = None,
        cu_doc_lens: Optional[torch.Tensor] = None,
    ) -> Tuple[torch.Tensor, Optional[List[KV]]]:
        caches: Optional[List[KV]] = [] if use_cache else None
        for i, block in enumerate(self):
            kwargs = dict(
                attention_bias=attention_bias,
                layer_past=None if layers_past is None else layers_past[i],
                use_cache=use_cache,
                max_doc_len=max_doc_len,
                cu_doc_lens=cu_doc_lens,
            )
            if should_checkpoint_block(self.activation_checkpointing_strategy, i + self.layer_offset):
                x, cache = self._activation_checkpoint_fn(block, x, **kwargs)
            else:
                x, cache = block(x, **kwargs)
            if caches is not None:
                assert cache is not None
                caches.append(cache)
        return x, caches

    def reset_parameters(self) -> None:
        for block in self:
            block.reset_parameters()

    def set_activation_checkpointing(
        self, strategy: Optional[ActivationCheckpointingStrategy], checkpoint_func: Optional[Callable] = None
    ) -> None:
        self.activation_checkpointing_strategy = strategy
        for block in self:
            block.set_activation_checkpointing(strategy, checkpoint_func=checkpoint_func)
