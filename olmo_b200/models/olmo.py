"""
The OLMo decoder (reference: ``olmo/model.py:1070-1878``).

Parameter names (``transformer.wte.weight``, ``transformer.blocks.{i}.att_proj.weight``, …) are the
on-disk contract shared with the reference's unsharded checkpoints and its Hugging Face converters.
"""
from __future__ import annotations

import logging
import math
import re
from collections import defaultdict
from fnmatch import fnmatch
from typing import TYPE_CHECKING, Callable, Dict, List, NamedTuple, Optional, Sequence, Set, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..aliases import PathOrStr
from ..config import (
    ActivationCheckpointingStrategy,
    BlockType,
    CheckpointType,
    FSDPWrapStrategy,
    InitFnType,
    ModelConfig,
)
from ..exceptions import OLMoConfigurationError
from ..initialization import init_normal
from ..torch_util import ensure_finite_, get_cumulative_document_lengths
from .blocks import (
    OLMoBlock,
    OLMoBlockGroup,
    activation_checkpoint_function,
    should_checkpoint_block,
)
from .layers import (
    BufferCache,
    Dropout,
    LayerNorm,
    _materialised_device,
    alibi_attention_bias,
    get_causal_attention_bias,
)

if TYPE_CHECKING:
    from ..beam_search import Constraint, FinalSequenceScorer, Sampler

__all__ = ["OLMo", "OLMoOutput", "OLMoGenerateOutput"]

log = logging.getLogger(__name__)


class OLMoOutput(NamedTuple):
    logits: torch.Tensor  # (batch, seq or 1, embedding_size): unnormalised next-token scores
    attn_key_values: Optional[List[Tuple[torch.Tensor, torch.Tensor]]]  # per block, pre-RoPE keys
    hidden_states: Optional[Tuple[torch.Tensor, ...]]  # block inputs + final normed state


class OLMoGenerateOutput(NamedTuple):
    token_ids: torch.LongTensor  # (batch, beam, max_steps); generated tokens only
    scores: torch.FloatTensor  # (batch, beam)


class OLMo(nn.Module):
    def __init__(self, config: ModelConfig, init_params: bool = True):
        super().__init__()
        self.config = config
        self._cache = BufferCache()

        if config.alibi and config.flash_attention:
            raise OLMoConfigurationError("ALiBi is currently not supported with FlashAttention")
        if config.alibi and config.rope:
            raise OLMoConfigurationError("ALiBi and RoPE are mutually exclusive")
        if config.embedding_size is not None and config.embedding_size != config.vocab_size:
            if config.embedding_size < config.vocab_size:
                raise OLMoConfigurationError("embedding size should be at least as big as vocab size")
            if config.embedding_size % 128 != 0:
                import warnings

                warnings.warn("Embedding size is not a multiple of 128! This could hurt throughput performance.", UserWarning)
        if not (0 < config.block_group_size <= config.n_layers and config.n_layers % config.block_group_size == 0):
            raise OLMoConfigurationError("n layers must be divisible by block group size")

        self.activation_checkpointing_strategy: Optional[ActivationCheckpointingStrategy] = None
        self._activation_checkpoint_fn: Callable = activation_checkpoint_function(config)

        dev = config.init_device
        n_emb = config.n_embeddings
        self.transformer = nn.ModuleDict(
            dict(
                wte=nn.Embedding(n_emb, config.d_model, device=dev),
                emb_drop=Dropout(config.embedding_dropout),
                ln_f=LayerNorm.build(config),
            )
        )
        blocks = [OLMoBlock.build(i, config, self._cache) for i in range(config.n_layers)]
        if config.block_group_size > 1:
            g = config.block_group_size
            groups = [OLMoBlockGroup(config, i, blocks[i : i + g]) for i in range(0, config.n_layers, g)]
            self.transformer.update({"block_groups": nn.ModuleList(groups)})
        else:
            self.transformer.update({"blocks": nn.ModuleList(blocks)})
        if not (config.alibi or config.rope):
            self.transformer.update({"wpe": nn.Embedding(config.max_sequence_length, config.d_model, device=dev)})
        if not config.weight_tying:
            self.transformer.update({"ff_out": nn.Linear(config.d_model, n_emb, bias=config.include_bias, device=dev)})
        if config.embedding_layer_norm:
            self.transformer.update({"emb_norm": LayerNorm.build(config)})

        if init_params and config.init_device != "meta":
            self.reset_parameters()
        self._num_fwd_flops: Optional[int] = None
        self._num_bck_flops: Optional[int] = None

        if config.alibi:
            get_causal_attention_bias(self._cache, config.max_sequence_length, _materialised_device(config))
            self.get_alibi_attention_bias(config.max_sequence_length, _materialised_device(config))

    # ------------------------------------------------------------------------------- structure
    def all_blocks(self) -> List[OLMoBlock]:
        if self.config.block_group_size == 1:
            return list(self.transformer.blocks)  # type: ignore[arg-type]
        return [b for g in self.transformer.block_groups for b in g]  # type: ignore[union-attr]

    def set_activation_checkpointing(
        self, strategy: Optional[ActivationCheckpointingStrategy], checkpoint_func: Optional[Callable] = None
    ) -> None:
        self.activation_checkpointing_strategy = strategy
        units = self.transformer.blocks if self.config.block_group_size == 1 else self.transformer.block_groups
        for unit in units:  # type: ignore[union-attr]
            unit.set_activation_checkpointing(strategy, checkpoint_func=checkpoint_func)

    @property
    def device(self) -> torch.device:
        device: torch.device = self.transformer.wte.weight.device  # type: ignore[union-attr]
        return _materialised_device(self.config) if device.type == "meta" else device

    # -------------------------------------------------------------------------- initialisation
    def _top_level_std(self, which: str) -> Tuple[float, Optional[float]]:
        cfg = self.config
        if cfg.init_fn == InitFnType.normal:
            std = (cfg.emb_init_std or cfg.init_std) if which == "wte" else cfg.init_std
            return std, cfg.init_cutoff_factor
        cutoff = cfg.init_cutoff_factor or 3.0
        inv_sqrt_d = 1.0 / math.sqrt(cfg.d_model)
        if cfg.init_fn == InitFnType.mitchell:
            return ((cfg.emb_init_std or inv_sqrt_d) if which == "wte" else inv_sqrt_d), cutoff
        if cfg.init_fn == InitFnType.full_megatron:
            if which == "wte":
                if cfg.emb_init_std is not None:
                    return cfg.emb_init_std, cutoff
                return cfg.init_std * (math.sqrt(cfg.d_model) if cfg.scale_emb_init else 1.0), cutoff
            if which == "wpe":
                return cfg.init_std, cutoff
            return inv_sqrt_d, cutoff  # output head
        raise NotImplementedError(cfg.init_fn)

    def initialisable_modules(self) -> List[nn.Module]:
        """The modules :meth:`reset_parameters` initialises one by one: embeddings, final norm, output projection and
        every block (or block group)."""
        t = self.transformer
        mods: List[nn.Module] = [t.wte]
        for name in ("wpe", "emb_norm", "ff_out"):
            if hasattr(t, name):
                mods.append(getattr(t, name))
        mods.append(t.ln_f)
        mods += list(t.blocks if self.config.block_group_size == 1 else t.block_groups)  # type: ignore[union-attr]
        if self.config.block_group_size > 1:  # a block inside a group can also be addressed on its own
            mods += list(self.all_blocks())
        return mods

    def reset_parameters(self, only: Optional[set] = None, seed: Optional[int] = None) -> None:
        """Initialise the parameters.  ``only`` (ids of modules from :meth:`initialisable_modules`) restricts the call
        to those modules, which lets a sharded engine materialise and initialise one unit at a time.  With ``seed`` every
        module draws from a random stream of its own that is a function of ``(seed, module name)``, so the values do not
        depend on which other modules are initialised in the same call, nor on their order."""
        if only is None:
            log.info("Initializing model parameters...")
        t = self.transformer

        def want(m: nn.Module) -> bool:
            return only is None or id(m) in only

        def reseed(name: str) -> None:
            if seed is not None:
                from ..initialization import param_generator

                s = param_generator(seed, name).initial_seed()
                torch.manual_seed(s)
                if torch.cuda.is_available():
                    torch.cuda.manual_seed(s)

        if want(t.wte):
            reseed("wte")
            init_normal(t.wte, *self._top_level_std("wte"))  # type: ignore[arg-type]
        if hasattr(t, "wpe") and want(t.wpe):
            reseed("wpe")
            init_normal(t.wpe, *self._top_level_std("wpe"))  # type: ignore[arg-type]
        if want(t.ln_f):
            t.ln_f.reset_parameters()  # type: ignore[operator]
        if hasattr(t, "emb_norm") and want(t.emb_norm):
            t.emb_norm.reset_parameters()  # type: ignore[operator]
        if hasattr(t, "ff_out") and want(t.ff_out):
            reseed("ff_out")
            init_normal(t.ff_out, *self._top_level_std("ff_out"))  # type: ignore[arg-type]
        for unit in t.blocks if self.config.block_group_size == 1 else t.block_groups:  # type: ignore[union-attr]
            for block in ([unit] if self.config.block_group_size == 1 else unit):  # type: ignore[union-attr]
                if want(unit) or want(block):
                    reseed(f"block{block.layer_id}")
                    block.reset_parameters()

    # ------------------------------------------------------------------------------ bias tables
    def get_alibi_attention_bias(self, seq_len: int, device: torch.device) -> torch.Tensor:
        bias = self._cache.get("alibi_attention_bias")
        if bias is not None and bias.shape[-1] >= seq_len:
            if bias.device != device:
                bias = bias.to(device)
                self._cache["alibi_attention_bias"] = bias
            return bias
        with torch.autocast(device.type, enabled=False):
            bias = alibi_attention_bias(seq_len, self.config, device)
        self._cache["alibi_attention_bias"] = bias
        return bias

    def _combined_attention_bias(
        self,
        attention_bias: Optional[torch.Tensor],
        attention_mask: Optional[torch.Tensor],
        batch_size: int,
        seq_len: int,
        past_length: int,
        have_past: bool,
        device: torch.device,
    ) -> Optional[torch.Tensor]:
        """Merge the padding mask, a user bias, the causal table and ALiBi into one additive fp32 bias.

        Returns ``None`` on the pretraining path (no mask, no bias, no ALiBi, no cache), which lets the
        attention kernels use their built-in causal mode.
        """
        if attention_mask is not None:
            attention_mask = attention_mask.to(dtype=torch.float).view(batch_size, -1)[:, None, None, :]
            attention_mask = (1.0 - attention_mask) * torch.finfo(attention_mask.dtype).min
        if attention_bias is None and attention_mask is None and not self.config.alibi and not have_past:
            return None
        total = past_length + seq_len
        if attention_bias is None:
            attention_bias = get_causal_attention_bias(self._cache, total, device)
            if self.config.alibi:
                attention_bias = attention_bias + self.get_alibi_attention_bias(total, device)
        elif attention_bias.dtype in (torch.int8, torch.bool):
            attention_bias = attention_bias.to(dtype=torch.float)
            attention_bias.masked_fill_(attention_bias == 0.0, torch.finfo(attention_bias.dtype).min)
        mask_len = seq_len
        if attention_mask is not None:
            mask_len = attention_mask.shape[-1]
        elif have_past:
            mask_len = total
        attention_bias = attention_bias[:, :, :mask_len, :mask_len].to(dtype=torch.float)
        if attention_mask is not None:
            attention_bias = attention_bias + attention_mask
            ensure_finite_(attention_bias, check_neg_inf=True, check_pos_inf=False)
        return attention_bias

    # --------------------------------------------------------------------------------- forward
    def forward(
        self,
        input_ids: torch.LongTensor,
        input_embeddings: Optional[torch.FloatTensor] = None,
        attention_mask: Optional[torch.Tensor] = None,
        attention_bias: Optional[torch.Tensor] = None,
        past_key_values: Optional[Sequence[Tuple[torch.Tensor, torch.Tensor]]] = None,
        use_cache: bool = False,
        last_logits_only: bool = False,
        output_hidden_states: Optional[bool] = None,
        doc_lens: Optional[torch.Tensor] = None,
        max_doc_lens: Optional[Sequence[int]] = None,
    ) -> OLMoOutput:
        """
        :param input_ids: ``(batch, seq)`` token ids.
        :param input_embeddings: optional ``(batch, seq, d_model)`` replacing the embedding lookup.
        :param attention_mask: ``(batch, seq)``; 1 = attend, 0 = padding (HF convention).
        :param attention_bias: ``(batch|1, 1, seq, seq)``; bool/int8 means "may attend", float is added
            to the scores.  Default is causal.
        :param past_key_values: per-block ``(key, value)`` from a previous call (keys are pre-RoPE).
        :param use_cache: also return the per-block keys/values.
        :param last_logits_only: compute logits for the final position only.
        :param doc_lens: ``(batch, max_docs)`` document lengths for intra-document attention masking.
        :param max_doc_lens: longest document of each instance.
        """
        cfg = self.config
        t = self.transformer
        output_hidden_states = bool(output_hidden_states)
        if past_key_values:
            assert len(past_key_values) == cfg.n_layers
        batch_size, seq_len = input_ids.size() if input_embeddings is None else input_embeddings.size()[:2]
        past_length = 0 if past_key_values is None else past_key_values[0][0].size(-2)

        max_doc_len: Optional[int] = None
        cu_doc_lens: Optional[torch.Tensor] = None
        if doc_lens is not None and max_doc_lens is not None:
            max_doc_len = max(max_doc_lens)
            cu_doc_lens = get_cumulative_document_lengths(doc_lens)

        x = t.wte(input_ids) if input_embeddings is None else input_embeddings  # type: ignore[operator]
        if cfg.embedding_layer_norm:
            x = t.emb_norm(x)  # type: ignore[operator]
        if not (cfg.alibi or cfg.rope):
            pos = torch.arange(past_length, past_length + seq_len, dtype=torch.long, device=x.device).unsqueeze(0)
            x = t.wpe(pos) + x  # type: ignore[operator]
        x = t.emb_drop(x)  # type: ignore[operator]

        attention_bias = self._combined_attention_bias(
            attention_bias, attention_mask, batch_size, seq_len, past_length, past_key_values is not None, x.device
        )

        attn_key_values: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = [] if use_cache else None
        all_hidden_states: List[torch.Tensor] = []
        if cfg.block_group_size == 1:
            for idx, block in enumerate(t.blocks):  # type: ignore[arg-type]
                if output_hidden_states:
                    all_hidden_states.append(x)
                kwargs = dict(
                    attention_bias=attention_bias,
                    layer_past=None if past_key_values is None else past_key_values[idx],
                    use_cache=use_cache,
                    max_doc_len=max_doc_len,
                    cu_doc_lens=cu_doc_lens,
                )
                if should_checkpoint_block(self.activation_checkpointing_strategy, idx):
                    x, cache = self._activation_checkpoint_fn(block, x, **kwargs)
                else:
                    x, cache = block(x, **kwargs)
                if attn_key_values is not None:
                    assert cache is not None
                    attn_key_values.append(cache)
        else:
            g = cfg.block_group_size
            for gidx, group in enumerate(t.block_groups):  # type: ignore[arg-type]
                if output_hidden_states:
                    all_hidden_states.append(x)
                x, caches = group(
                    x,
                    attention_bias=attention_bias,
                    layers_past=None if past_key_values is None else past_key_values[gidx * g : (gidx + 1) * g],
                    use_cache=use_cache,
                    max_doc_len=max_doc_len,
                    cu_doc_lens=cu_doc_lens,
                )
                if attn_key_values is not None:
                    assert caches is not None
                    attn_key_values.extend(caches)

        if last_logits_only:
            x = x[:, -1, :].unsqueeze(1)
        x = t.ln_f(x)  # type: ignore[operator]
        if output_hidden_states:
            all_hidden_states.append(x)
        logits = self.output_projection(x)
        return OLMoOutput(
            logits=logits,
            attn_key_values=attn_key_values,
            hidden_states=tuple(all_hidden_states) if output_hidden_states else None,
        )

    def output_projection(self, x: torch.Tensor) -> torch.Tensor:
        """Final-norm output -> logits (tied or untied head, optional ``1/sqrt(d)`` scaling)."""
        if self.config.weight_tying:
            logits = F.linear(x, self.transformer.wte.weight, None)  # type: ignore[union-attr]
        else:
            logits = self.transformer.ff_out(x)  # type: ignore[operator]
        if self.config.scale_logits:
            logits = logits * (1 / math.sqrt(self.config.d_model))
        return logits

    def hidden_before_head(self, input_ids: torch.LongTensor, **kwargs) -> torch.Tensor:
        """Run everything but the output projection; used by the fused LM-head + loss path, which never
        materialises the full logits tensor."""
        head = self.output_projection
        try:
            self.output_projection = lambda x: x  # type: ignore[method-assign, assignment]
            return self.forward(input_ids, **kwargs).logits
        finally:
            self.output_projection = head  # type: ignore[method-assign]

    # ------------------------------------------------------------------------- sharding layout
    def fsdp_units(self, wrap_strategy: Optional[FSDPWrapStrategy] = None) -> List[Tuple[str, List[nn.Module]]]:
        """Partition the modules into the units whose parameters are flattened and sharded together.

        Mirrors what the reference's wrap policies produce (``olmo/model.py:1467-1560``): the last
        entry, ``"root"``, collects whatever no other unit owns.
        """
        t = self.transformer
        big = [("transformer.wte", t.wte)] + ([("transformer.ff_out", t.ff_out)] if hasattr(t, "ff_out") else [])
        units: List[Tuple[str, List[nn.Module]]] = []
        S = FSDPWrapStrategy
        grouped = self.config.block_group_size > 1
        if wrap_strategy in (S.by_block_group, S.by_block_group_and_size) and not grouped:
            raise OLMoConfigurationError(f"'{wrap_strategy}' FSDP wrapping strategy requires block group size greater than 1")
        if wrap_strategy is None:
            pass
        elif wrap_strategy in (S.by_block, S.by_block_and_size):
            for b in self.all_blocks():
                prefix = (
                    f"transformer.blocks.{b.layer_id}"
                    if not grouped
                    else f"transformer.block_groups.{b.layer_id // self.config.block_group_size}.{b.layer_id % self.config.block_group_size}"
                )
                units.append((prefix, [b]))
            if wrap_strategy == S.by_block_and_size:
                units += [(n, [m]) for n, m in big]
        elif wrap_strategy in (S.by_block_group, S.by_block_group_and_size):
            units += [(f"transformer.block_groups.{i}", [g]) for i, g in enumerate(t.block_groups)]  # type: ignore[arg-type]
            if wrap_strategy == S.by_block_group_and_size:
                units += [(n, [m]) for n, m in big]
        elif wrap_strategy == S.size_based:
            # torch's size-based policy wraps sub-trees above 1e8 parameters; blocks and the two
            # vocabulary-sized matrices are the sub-trees that can reach it.
            for b in self.all_blocks():
                if sum(p.numel() for p in b.parameters()) >= 100_000_000:
                    units.append((f"block{b.layer_id}", [b]))
            units += [(n, [m]) for n, m in big if sum(p.numel() for p in m.parameters()) >= 100_000_000]
        elif wrap_strategy in (S.one_in_two, S.one_in_three, S.one_in_four, S.one_in_five):
            c = {S.one_in_two: 2, S.one_in_three: 3, S.one_in_four: 4, S.one_in_five: 5}[wrap_strategy]
            for b in self.all_blocks():
                if b.layer_id % c == 0:
                    units.append((f"block{b.layer_id}", [b]))
        else:
            raise NotImplementedError(wrap_strategy)
        units.append(("root", [self]))
        return units

    def get_fsdp_wrap_policy(self, wrap_strategy: Optional[FSDPWrapStrategy] = None):
        """A ``torch`` FSDP ``auto_wrap_policy`` equivalent to :meth:`fsdp_units` (for API parity)."""
        if wrap_strategy is None:
            return None
        if wrap_strategy == FSDPWrapStrategy.size_based:
            from torch.distributed.fsdp.wrap import size_based_auto_wrap_policy

            return size_based_auto_wrap_policy
        owned = {id(m) for name, mods in self.fsdp_units(wrap_strategy) if name != "root" for m in mods}

        def policy(module: nn.Module, recurse: bool = True, nonwrapped_numel: int = 0) -> bool:
            del nonwrapped_numel
            return True if recurse else id(module) in owned

        return policy

    # --------------------------------------------------------------------------------- counting
    def num_params(self, include_embedding: bool = True) -> int:
        return sum(
            p.numel()
            for n, p in self.named_parameters()
            if include_embedding or (".wte." not in n and ".wpe." not in n)
        )

    @property
    def num_fwd_flops(self) -> int:
        """Forward FLOPs per token: ``2·(non-embedding params) + n_layers·4·d·T``."""
        if not self._num_fwd_flops:
            cfg = self.config
            self._num_fwd_flops = 2 * self.num_params(include_embedding=False) + cfg.n_layers * 4 * cfg.d_model * cfg.max_sequence_length
        return self._num_fwd_flops

    @property
    def num_bck_flops(self) -> int:
        """Backward FLOPs per token: ``4·(all params) + n_layers·8·d·T``."""
        if not self._num_bck_flops:
            cfg = self.config
            self._num_bck_flops = 4 * self.num_params() + cfg.n_layers * 8 * cfg.d_model * cfg.max_sequence_length
        return self._num_bck_flops

    # -------------------------------------------------------------------------------- generate
    def generate(
        self,
        input_ids: torch.LongTensor,
        attention_mask: Optional[torch.Tensor] = None,
        attention_bias: Optional[torch.Tensor] = None,
        max_steps: int = 10,
        beam_size: int = 1,
        per_node_beam_size: Optional[int] = None,
        sampler: Optional["Sampler"] = None,
        min_steps: Optional[int] = None,
        final_sequence_scorer: Optional["FinalSequenceScorer"] = None,
        constraints: Optional[List["Constraint"]] = None,
    ) -> OLMoGenerateOutput:
        """Beam-search decoding with a KV cache; returns only the generated continuation."""
        from ..beam_search import BeamSearch

        search = BeamSearch(
            self.config.eos_token_id,
            max_steps=max_steps,
            beam_size=beam_size,
            per_node_beam_size=per_node_beam_size,
            sampler=sampler,
            min_steps=min_steps,
            final_sequence_scorer=final_sequence_scorer,
            constraints=constraints,
        )
        batch_size, seq_len = input_ids.shape
        if attention_mask is not None:
            assert attention_mask.shape == (batch_size, seq_len)
        if attention_bias is not None:
            assert attention_bias.dim() == 4 and attention_bias.shape[:2] == (batch_size, 1)
            assert seq_len + search.max_steps <= attention_bias.shape[2] == attention_bias.shape[3] <= self.config.max_sequence_length

        n_layers = self.config.n_layers
        generated = 0

        def step(last_predictions: torch.Tensor, state: Dict[str, torch.Tensor]):
            nonlocal generated
            mask, bias = state.get("attention_mask"), state.get("attention_bias")
            if generated > 0:
                past = [(state[f"past_key_{i}"], state[f"past_value_{i}"]) for i in range(n_layers)]
                ids = last_predictions.unsqueeze(1)
                if mask is not None:
                    mask = torch.cat((mask, mask.new_ones((ids.shape[0], 1))), dim=-1)
            else:
                past, ids = None, state["input_ids"]
            generated += 1
            out = self(ids, attention_mask=mask, attention_bias=bias, past_key_values=past, use_cache=True, last_logits_only=True)
            log_probs = F.log_softmax(out.logits[:, -1, :], dim=-1)
            new_state: Dict[str, torch.Tensor] = {}
            for i, (key, value) in enumerate(out.attn_key_values or []):
                new_state[f"past_key_{i}"] = key
                new_state[f"past_value_{i}"] = value
            if mask is not None:
                new_state["attention_mask"] = mask
            if bias is not None:
                new_state["attention_bias"] = bias
            return log_probs, new_state

        state: Dict[str, torch.Tensor] = {"input_ids": input_ids}
        if attention_mask is not None:
            state["attention_mask"] = attention_mask
        if attention_bias is not None:
            state["attention_bias"] = attention_bias
        with torch.no_grad():
            token_ids, scores = search.search(input_ids.new_zeros((batch_size,)), state, step)
        return OLMoGenerateOutput(token_ids=token_ids, scores=scores)  # type: ignore[arg-type]

    # ----------------------------------------------------------------------------- checkpoints
    @classmethod
    def from_checkpoint(
        cls, checkpoint_dir: PathOrStr, device: str = "cpu", checkpoint_type: Optional[CheckpointType] = None
    ) -> "OLMo":
        """Load weights from an unsharded (``model.pt`` / ``model.safetensors``) or sharded checkpoint."""
        from ..util import resource_path

        def has(name: str) -> bool:
            try:
                return resource_path(checkpoint_dir, name).is_file()
            except FileNotFoundError:
                return False

        if checkpoint_type is None:
            unsharded = has("model.pt") or has("model.safetensors")
            checkpoint_type = CheckpointType.unsharded if unsharded else CheckpointType.sharded
        config_path = resource_path(checkpoint_dir, "config.yaml")
        model_config = ModelConfig.load(config_path, key="model", validate_paths=False)
        if checkpoint_type == CheckpointType.unsharded:
            from ..checkpoint import load_state_dict

            model_config.init_device = "cpu"
            model = cls(model_config)
            state_dict = load_state_dict(checkpoint_dir, "model.pt", map_location="cpu")
            model.load_state_dict(model._make_state_dict_compatible(state_dict)[0])
            model = model.to(torch.device(device))
        else:
            from ..checkpoint import load_model_state

            model_config.init_device = device
            model = cls(model_config)
            load_model_state(checkpoint_dir, model)
        return model.eval()

    def _make_state_dict_compatible(
        self, state_dict: Dict[str, torch.Tensor]
    ) -> Tuple[Dict[str, torch.Tensor], Dict[str, Set[str]]]:
        """Rewrite older key layouts in place so that ``load_state_dict`` accepts them.

        Handles: wrapper prefixes (``_fsdp_wrapped_module.``), the legacy single ``norm`` of the
        sequential block (duplicated into ``attn_norm`` and ``ff_norm``), and a different
        ``block_group_size`` (``blocks.N`` <-> ``block_groups.G.I``).  Returns the dict and a map
        ``original key -> {new keys}`` so optimizer state can follow the same renames.
        """
        origin: Dict[str, str] = {}

        def rename(old: str, new: str, clone: bool = False) -> None:
            tensor = state_dict[old] if clone else state_dict.pop(old)
            state_dict[new] = tensor.clone() if clone else tensor
            origin[new] = origin[old] if clone else origin.pop(old)

        for key in list(state_dict):
            origin[key] = key
        for key in list(state_dict):
            stripped = key.replace("_fsdp_wrapped_module.", "")
            if stripped != key:
                rename(key, stripped)

        if self.config.block_type == BlockType.sequential:
            for key in list(state_dict):
                for leaf in ("weight", "bias"):
                    if fnmatch(key, f"transformer.*.norm.{leaf}"):
                        rename(key, key.replace(f"norm.{leaf}", f"ff_norm.{leaf}"), clone=True)
                        rename(key, key.replace(f"norm.{leaf}", f"attn_norm.{leaf}"))

        have = 1
        if "transformer.block_groups.0.0.attn_out.weight" in state_dict:
            have = sum(1 for k in state_dict if fnmatch(k, "transformer.block_groups.0.*.attn_out.weight"))
        want = self.config.block_group_size
        if have != want:
            log.info("Regrouping state dict blocks from group size %d to group size %d", have, want)
            if have > 1:
                for key in list(state_dict):
                    m = re.match(r"transformer\.block_groups\.(\d+)\.(\d+)\.(.*)", key)
                    if m:
                        idx = int(m.group(1)) * have + int(m.group(2))
                        rename(key, f"transformer.blocks.{idx}.{m.group(3)}")
            if want > 1:
                for key in list(state_dict):
                    m = re.match(r"transformer\.blocks\.(\d+)\.(.*)", key)
                    if m:
                        idx = int(m.group(1))
                        rename(key, f"transformer.block_groups.{idx // want}.{idx % want}.{m.group(2)}")

        renames: Dict[str, Set[str]] = defaultdict(set)
        for new, old in origin.items():
            renames[old].add(new)
        return state_dict, renames
