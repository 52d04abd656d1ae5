"""
Training / model configuration schema.

Field names, defaults and enum spellings follow the reference's ``olmo/config.py:67-1365`` so that
its YAML files and ``--dotted.key=value`` overrides load unchanged and so that a ``config.yaml``
written here is accepted by the reference's structured merge (which rejects unknown keys,
``olmo/config.py:137-148``).  Knobs that only exist in this framework (kernel selection, peer-memory
buffers, residency of gathered parameters) therefore live in :class:`B200Runtime`, which is read
from the environment and never serialised into ``config.yaml``.

Loading is done by :mod:`olmo_b200.utils.structured` instead of OmegaConf.
"""
from __future__ import annotations

import os
from copy import deepcopy
from dataclasses import asdict, dataclass, field
from enum import Enum
from glob import glob
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional, Tuple, Type, TypeVar, Union

import numpy as np
import torch

from .aliases import PathOrStr
from .exceptions import OLMoConfigurationError
from .util import StrEnum
from .utils import structured as S

__all__ = [
    "ActivationType",
    "ActivationCheckpointingStrategy",
    "BlockType",
    "LayerNormType",
    "InitFnType",
    "ModelConfig",
    "OptimizerType",
    "OptimizerConfig",
    "SchedulerType",
    "SchedulerUnits",
    "SchedulerConfig",
    "DataConfig",
    "InstanceFilterConfig",
    "CustomDatasetConfig",
    "CustomDatasetCollatorConfig",
    "EvaluatorConfig",
    "EvaluatorType",
    "TokenizerConfig",
    "TrainConfig",
    "PaddingDirection",
    "TruncationDirection",
    "SpeedMonitorConfig",
    "WandbConfig",
    "CompilerConfig",
    "DDPConfig",
    "DistributedStrategy",
    "DDPGradSyncMode",
    "FSDPPrecision",
    "FSDPWrapStrategy",
    "FSDPConfig",
    "ShardingStrategy",
    "SingleGPUConfig",
    "CheckpointType",
    "ShardedCheckpointerType",
    "B200Runtime",
]

C = TypeVar("C", bound="BaseConfig")


def _register_path_resolvers(validate_paths: bool) -> None:
    def path_glob(*patterns: str) -> List[str]:
        found: List[str] = []
        for pattern in patterns:
            hits = sorted(glob(pattern))
            if validate_paths and not hits:
                raise FileNotFoundError(f"{pattern} does not match any files or dirs")
            found += hits
        return found

    def path_choose(*candidates: str) -> str:
        from .util import is_url

        for cand in candidates:
            if is_url(cand) or Path(cand).exists():
                return cand
        if validate_paths:
            raise FileNotFoundError(", ".join(candidates))
        return ""

    def path_last_checkpoint(folder: str) -> str:
        from .util import find_latest_checkpoint

        latest = find_latest_checkpoint(folder)
        if latest is None:
            if validate_paths:
                raise FileNotFoundError(f"Could not find a latest checkpoint at {folder}")
            return ""
        return str(latest)

    def data_mix(name: str, local_glob: str = "") -> List[str]:
        """Token files of a run: the files ``local_glob`` matches when it is given and matches something (a local copy
        of the data), else the packaged list ``data_mixes/<name>.txt`` (the URLs the official run read, in order)."""
        if local_glob:
            hits = sorted(glob(local_glob))
            if hits:
                return hits
        from .data.named_data_mixes import DATA_PATHS

        try:
            return list(DATA_PATHS[name])
        except KeyError:
            if validate_paths:
                raise FileNotFoundError(f"no local files match '{local_glob}' and there is no packaged data mix '{name}'") from None
            return []

    S.register_resolver("path.glob", path_glob)
    S.register_resolver("data.mix", data_mix)
    S.register_resolver("path.choose", path_choose)
    S.register_resolver("path.last_checkpoint", path_last_checkpoint)


class BaseConfig:
    """Mixin giving every config dataclass ``new`` / ``load`` / ``save`` / ``asdict`` / ``update_with``."""

    @classmethod
    def update_legacy_settings(cls, raw: Dict[str, Any]) -> Dict[str, Any]:
        """Rewrite keys whose meaning changed between releases; subclasses override."""
        return raw

    @classmethod
    def new(cls: Type[C], **kwargs: Any) -> C:
        _register_path_resolvers(validate_paths=True)
        raw = S.resolve_interpolations(cls.update_legacy_settings(dict(kwargs)))
        return S.build(cls, raw)

    @classmethod
    def load(
        cls: Type[C],
        path: PathOrStr,
        overrides: Optional[List[str]] = None,
        key: Optional[str] = None,
        validate_paths: bool = True,
    ) -> C:
        """Read a YAML file, apply ``a.b=c`` overrides, resolve interpolations, validate."""
        _register_path_resolvers(validate_paths=validate_paths)
        try:
            with open(str(path)) as f:
                raw = S.load_yaml(f) or {}
        except OSError as e:
            raise OLMoConfigurationError(f"cannot read config {path}: {e}") from e
        if key is not None:
            raw = raw[key]
        if not isinstance(raw, dict):
            raise OLMoConfigurationError(f"top level of {path} must be a mapping")
        raw = cls.update_legacy_settings(raw)
        if overrides:
            raw = S.deep_merge(raw, S.parse_dotlist(overrides))
        # interpolations may refer to schema defaults that the file does not spell out
        defaults = S.to_container(_schema_defaults(cls), enum_to_str=True)
        resolved = S.resolve_interpolations(raw, root=S.deep_merge(defaults, raw))
        return S.build(cls, resolved)

    def save(self, path: PathOrStr) -> None:
        with open(str(path), "w") as f:
            f.write(S.dump_yaml(S.to_container(self)))

    def asdict(self, exclude: Optional[Iterable[str]] = None) -> Dict[str, Any]:
        out = asdict(self)  # type: ignore[call-overload]
        for name in exclude or ():
            out.pop(name, None)
        return out

    def update_with(self: C, **kwargs: Any) -> C:
        clone = deepcopy(self)
        for k, v in kwargs.items():
            setattr(clone, k, v)
        return clone


def _schema_defaults(cls: Type) -> Any:
    try:
        return cls()
    except TypeError:
        return {}


# ------------------------------------------------------------------------------------------ enums


class LayerNormType(StrEnum):
    default = "default"  # torch-equivalent LayerNorm
    low_precision = "low_precision"  # LayerNorm evaluated in the autocast dtype
    rms = "rms"  # RMSNorm, statistics in fp32


class ActivationType(StrEnum):
    gelu = "gelu"
    relu = "relu"
    swiglu = "swiglu"


class BlockType(StrEnum):
    sequential = "sequential"  # fused QKV projection, ``x + attn`` then ``x + mlp``
    llama = "llama"  # separate q/k/v projections, explicit-softmax attention


class InitFnType(StrEnum):
    mitchell = "mitchell"
    normal = "normal"
    kaiming_normal = "kaiming_normal"
    fan_in = "fan_in"
    full_megatron = "full_megatron"


class OptimizerType(StrEnum):
    lionw = "lionw"
    adamw = "adamw"


class SchedulerType(StrEnum):
    cosine_with_warmup = "cosine_with_warmup"
    linear_with_warmup = "linear_with_warmup"
    inverse_sqrt_with_warmup = "inverse_sqrt_with_warmup"
    max_scheduler = "max_scheduler"
    constant = "constant"
    cosine_linear_envelope = "cosine_linear_envelope"
    constant_with_warmup = "constant_with_warmup"


class SchedulerUnits(StrEnum):
    steps = "steps"
    tokens = "tokens"


class PaddingDirection(StrEnum):
    right = "right"
    left = "left"


class TruncationDirection(StrEnum):
    right = "right"
    left = "left"


class EvaluatorType(StrEnum):
    downstream = "downstream"
    lm = "lm"


class DistributedStrategy(StrEnum):
    ddp = "ddp"  # replicated parameters, gradient all-reduce
    fsdp = "fsdp"  # flat-shard engine (parameters, gradients and optimizer state sharded)
    single = "single"  # one device, no process group needed


class DDPGradSyncMode(StrEnum):
    batch = "batch"  # reduce gradients once, on the last micro-batch
    micro_batch = "micro_batch"  # reduce after every micro-batch


class FSDPWrapStrategy(StrEnum):
    by_block = "by_block"
    by_block_and_size = "by_block_and_size"
    by_block_group = "by_block_group"
    by_block_group_and_size = "by_block_group_and_size"
    size_based = "size_based"
    one_in_two = "one_in_two"
    one_in_three = "one_in_three"
    one_in_four = "one_in_four"
    one_in_five = "one_in_five"


class FSDPPrecision(StrEnum):
    pure = "pure"  # gather, compute and reduce in the autocast dtype
    mixed = "mixed"  # gather/compute in the autocast dtype, reduce gradients in fp32


class ShardingStrategy(Enum):
    """Same member names and integer values as ``torch.distributed.fsdp.ShardingStrategy``."""

    FULL_SHARD = 1
    SHARD_GRAD_OP = 2
    NO_SHARD = 3
    HYBRID_SHARD = 4
    _HYBRID_SHARD_ZERO2 = 5


class CheckpointType(StrEnum):
    sharded = "sharded"
    unsharded = "unsharded"
    sharded_ephemeral = "sharded_ephemeral"


class ShardedCheckpointerType(StrEnum):
    torch_new = "torch_new"
    torch_legacy = "torch_legacy"
    local = "local"
    olmo_core = "olmo_core"


class ActivationCheckpointingStrategy(StrEnum):
    whole_layer = "whole_layer"
    one_in_two = "one_in_two"
    one_in_three = "one_in_three"
    one_in_four = "one_in_four"
    one_in_eight = "one_in_eight"
    two_in_three = "two_in_three"
    three_in_four = "three_in_four"
    fine_grained = "fine_grained"


# --------------------------------------------------------------------------------------- dataclasses


@dataclass
class ModelConfig(BaseConfig):
    """Architecture of the decoder. Defaults equal GPT-2 base, like the reference."""

    d_model: int = 768
    n_heads: int = 12
    n_kv_heads: Optional[int] = None  # None -> n_heads (MHA); 1 -> MQA; in between -> GQA
    clip_qkv: Optional[float] = None  # clamp the fused QKV projection to [-v, v]
    n_layers: int = 12
    mlp_ratio: int = 4
    mlp_hidden_size: Optional[int] = None  # output width of ff_proj; SwiGLU halves it
    activation_type: ActivationType = ActivationType.swiglu
    block_type: BlockType = BlockType.sequential
    block_group_size: int = 1
    alibi: bool = False
    alibi_bias_max: float = 8.0
    rope: bool = False
    rope_full_precision: bool = True
    rope_theta: int = 10_000
    flash_attention: bool = False
    attention_dropout: float = 0.1
    multi_query_attention: Optional[bool] = None  # deprecated spelling of n_kv_heads=1
    attention_layer_norm: bool = False  # QK-norm
    residual_dropout: float = 0.1
    embedding_dropout: float = 0.1
    embedding_layer_norm: bool = False
    layer_norm_type: LayerNormType = LayerNormType.default
    layer_norm_with_affine: bool = True
    layer_norm_eps: float = 1e-05
    attention_layer_norm_with_affine: bool = True
    max_sequence_length: int = 1024
    include_bias: bool = True
    bias_for_layer_norm: Optional[bool] = None  # None -> follow include_bias
    scale_logits: bool = False
    vocab_size: int = 50257
    embedding_size: Optional[int] = 50304  # rows of wte / ff_out (padded vocabulary)
    weight_tying: bool = True
    eos_token_id: int = 50256
    pad_token_id: int = 50256
    init_device: Optional[str] = None
    init_fn: InitFnType = InitFnType.normal
    init_std: float = 0.02
    init_cutoff_factor: Optional[float] = None
    precision: Optional[str] = None  # filled in from TrainConfig.precision
    scale_emb_init: bool = False
    emb_init_std: Optional[float] = None
    norm_after: bool = False  # OLMo-2 "reordered norm": x + norm(f(x))

    @property
    def effective_n_kv_heads(self) -> int:
        if self.n_kv_heads is None:
            return 1 if self.multi_query_attention is True else self.n_heads
        if self.multi_query_attention is None:
            return self.n_kv_heads
        implied = 1 if self.multi_query_attention else self.n_heads
        if self.n_kv_heads != implied:
            raise OLMoConfigurationError("You can't set `multi_query_attention` and `n_kv_heads` at the same time.")
        return implied

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def ff_proj_width(self) -> int:
        return self.mlp_hidden_size if self.mlp_hidden_size is not None else self.mlp_ratio * self.d_model

    @property
    def n_embeddings(self) -> int:
        return self.embedding_size or self.vocab_size


@dataclass
class OptimizerConfig(BaseConfig):
    name: OptimizerType = OptimizerType.lionw
    learning_rate: float = 1.0e-4
    weight_decay: float = 0.01
    betas: Tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-5
    no_decay_norm_and_bias: Optional[bool] = None  # deprecated
    selective_updates: bool = False  # skip param/state updates where the gradient is exactly 0
    decay_norm_and_bias: bool = False
    decay_embeddings: bool = False
    metrics_log_interval: Optional[int] = None
    record_update_metrics: bool = False

    def __post_init__(self) -> None:
        self.betas = tuple(self.betas)  # type: ignore[assignment]

    @classmethod
    def update_legacy_settings(cls, raw: Dict[str, Any]) -> Dict[str, Any]:
        if isinstance(raw, dict) and raw.get("name") == "decoupled_lionw":
            raw = {k: v for k, v in raw.items() if k != "eps"}
            raw["name"] = "lionw"
        return raw


@dataclass
class SchedulerConfig(BaseConfig):
    name: SchedulerType = SchedulerType.cosine_with_warmup
    units: SchedulerUnits = SchedulerUnits.steps
    t_warmup: Union[int, float] = 100
    t_max: Optional[Union[int, float]] = None
    alpha_f: float = 0.1
    grad_clip_warmup_steps: Optional[Union[int, float]] = None
    grad_clip_warmup_factor: Optional[float] = None
    warmup_min_lr: Optional[float] = None  # None -> 10% of the target LR


@dataclass
class InstanceFilterConfig(BaseConfig):
    repetition_max_period: int = 13
    repetition_min_period: int = 1
    repetition_max_count: int = 32


@dataclass
class CustomDatasetCollatorConfig(BaseConfig):
    input_id_field: str = "input_ids"
    attention_mask_field: Optional[str] = None
    attention_bias_field: Optional[str] = None
    label_mask_field: Optional[str] = None
    index_field: Optional[str] = None
    instance_mask_field: Optional[str] = None
    doc_lens_field: Optional[str] = None
    metadata_field: Optional[str] = None


@dataclass
class CustomDatasetConfig(BaseConfig):
    name: str
    module: Optional[str] = None
    args: Optional[Dict[str, Any]] = None
    collate_fn: Optional[str] = None
    token_field: Optional[str] = None
    collate_config: Optional[CustomDatasetCollatorConfig] = field(default_factory=CustomDatasetCollatorConfig)


@dataclass
class DataConfig(BaseConfig):
    paths: Optional[List[str]] = None
    memmap_dtype: str = "uint16"
    datasets: Optional[Dict[str, List[str]]] = None
    label_mask_paths: Optional[List[str]] = None
    pad_direction: PaddingDirection = PaddingDirection.right
    generate_attention_mask: bool = False
    generate_doc_lengths: bool = False
    num_workers: int = 0
    drop_last: bool = False
    pin_memory: bool = False
    prefetch_factor: Optional[int] = None
    persistent_workers: bool = False
    timeout: int = 0
    seed: Optional[int] = None
    instance_filter: Optional[InstanceFilterConfig] = None
    custom_dataset: Optional[CustomDatasetConfig] = None

    @property
    def effective_memmap_dtype(self):
        dtype = getattr(np, self.memmap_dtype, None)
        try:
            np.dtype(dtype)
            if dtype is None:
                raise TypeError
        except TypeError as e:
            raise TypeError(f"Value {self.memmap_dtype} is not a valid numpy type") from e
        return dtype


@dataclass
class EvaluatorConfig(BaseConfig):
    label: str
    type: EvaluatorType = EvaluatorType.lm
    data: DataConfig = field(default_factory=DataConfig)
    device_eval_batch_size: Optional[int] = None
    subset_num_batches: Optional[int] = None


@dataclass
class TokenizerConfig(BaseConfig):
    identifier: str = "gpt2"
    truncate_direction: TruncationDirection = TruncationDirection.right


@dataclass
class WandbConfig(BaseConfig):
    project: Optional[str] = None
    entity: Optional[str] = "ai2-llm"
    group: Optional[str] = None
    name: Optional[str] = None
    tags: Optional[List[str]] = field(default_factory=lambda: ["watching"])
    log_artifacts: bool = False
    rank_zero_only: bool = True
    log_interval: int = 1


@dataclass
class SpeedMonitorConfig(BaseConfig):
    window_size: int = 100
    gpu_flops_available: Optional[Union[float, int]] = None  # when set, MFU is logged


@dataclass
class CompilerConfig(BaseConfig):
    """Accepted for config compatibility.  This framework's hot path is hand-written kernels and
    CUDA graphs, so ``compile`` only affects the portable (non-fused) model path."""

    mode: Optional[str] = None
    fullgraph: bool = False
    backend: str = "inductor"
    dynamic: Optional[bool] = None


@dataclass
class DDPConfig(BaseConfig):
    grad_sync_mode: DDPGradSyncMode = DDPGradSyncMode.batch
    find_unused_params: bool = False


@dataclass
class FSDPConfig(BaseConfig):
    use_orig_params: bool = True
    sharding_strategy: ShardingStrategy = ShardingStrategy.FULL_SHARD
    wrapping_strategy: Optional[FSDPWrapStrategy] = None
    precision: Optional[FSDPPrecision] = FSDPPrecision.pure
    hybrid_sharding_num_model_replicas: Optional[int] = None


@dataclass
class SingleGPUConfig(BaseConfig):
    device: str = "auto"

    def get_device(self) -> torch.device:
        if self.device == "auto":
            if torch.cuda.is_available():
                return torch.device("cuda")
            if torch.backends.mps.is_available():
                return torch.device("mps")
            return torch.device("cpu")
        if self.device == "mps" and not torch.backends.mps.is_available():
            raise OLMoConfigurationError("MPS not available.")
        if self.device == "cuda" and not torch.cuda.is_available():
            raise OLMoConfigurationError("CUDA not available.")
        return torch.device(self.device)


@dataclass
class TrainConfig(BaseConfig):
    """Everything ``scripts/train.py`` needs (reference: ``olmo/config.py:947-1315``)."""

    run_name: Optional[str] = None
    seed: int = 6198
    epoch: Optional[int] = None
    dry_run: bool = False
    model: ModelConfig = field(default_factory=ModelConfig)
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    data: DataConfig = field(default_factory=DataConfig)
    restore_dataloader: bool = True
    fast_forward_batches: Optional[int] = None
    evaluators: List[EvaluatorConfig] = field(default_factory=list)
    eval_interval: int = 1000
    tokenizer: TokenizerConfig = field(default_factory=TokenizerConfig)
    save_folder: str = "./"
    remote_save_folder: Optional[str] = None
    canceled_check_interval: int = 50
    save_interval: Optional[int] = 1000
    save_interval_unsharded: Optional[int] = None
    save_interval_ephemeral: Optional[int] = None
    save_num_checkpoints_to_keep: int = -1
    save_num_unsharded_checkpoints_to_keep: int = -1
    save_overwrite: bool = False
    force_save_unsharded: bool = False
    no_pre_train_checkpoint: bool = False
    load_path: Optional[str] = None
    load_path_sharded_checkpointer: Optional[ShardedCheckpointerType] = None
    try_load_latest_save: bool = False
    reset_optimizer_state: bool = False
    reset_trainer_state: bool = False
    sharded_checkpointer: ShardedCheckpointerType = ShardedCheckpointerType.torch_legacy
    new_style_checkpoints: Optional[bool] = None  # deprecated
    max_duration: Union[int, str] = 10000  # steps | "<n>T" tokens | "<n>ep" epochs
    global_train_batch_size: int = 512
    device_train_batch_size: Optional[int] = None  # derived: global // world_size
    device_train_microbatch_size: int = 16
    device_eval_batch_size: int = 16
    eval_subset_num_batches: int = -1
    eval_on_load: bool = False
    device_train_grad_accum: Optional[int] = None  # derived: device batch // micro-batch
    max_grad_norm: Optional[float] = None
    max_grad_norm_ratio: Optional[float] = None
    precision: Optional[str] = None  # "amp_bf16" | "amp_fp16" | "fp32"
    wandb: Optional[WandbConfig] = None
    speed_monitor: SpeedMonitorConfig = field(default_factory=SpeedMonitorConfig)
    console_log_interval: int = 1
    gen1_gc_interval: Optional[int] = 1
    compile: Optional[CompilerConfig] = None
    distributed_strategy: Optional[DistributedStrategy] = DistributedStrategy.fsdp
    fsdp: Optional[FSDPConfig] = field(default_factory=FSDPConfig)
    ddp: Optional[DDPConfig] = None
    single: SingleGPUConfig = field(default_factory=lambda: SingleGPUConfig(device="auto"))
    softmax_auxiliary_loss: bool = False
    auxiliary_loss_multiplier: Optional[float] = 1e-4
    time_limit: Optional[float] = None
    extra_steps_after_cancel: int = 10
    early_stopping_factor: Optional[float] = None
    save_data_indices: bool = True
    python_profiling: bool = False
    torch_profiling: bool = False
    stop_at: Optional[int] = None
    stop_after: Optional[int] = None
    activation_checkpointing: Optional[ActivationCheckpointingStrategy] = None
    fused_loss: Optional[bool] = None
    hf_datasets_cache_dir: Optional[str] = None  # deprecated
    module_outputs_save_steps: Optional[List[int]] = None

    @property
    def autocast_precision(self) -> torch.dtype:
        table = {"amp_bf16": torch.bfloat16, "amp_fp16": torch.float16, "fp32": torch.float32}
        if self.precision not in table:
            raise ValueError(f"Unexpected precision type '{self.precision}'")
        return table[self.precision]

    @property
    def fsdp_reduce_dtype(self) -> torch.dtype:
        """dtype in which sharded gradient reduction accumulates (``mixed`` -> fp32)."""
        if self.fsdp is None:
            raise ValueError("self.fsdp is None!")
        if self.fsdp.precision == FSDPPrecision.mixed or self.fsdp.precision is None:
            return torch.float32
        return self.autocast_precision

    @property
    def fsdp_param_dtype(self) -> torch.dtype:
        """dtype of the gathered (compute) parameters."""
        if self.fsdp is None:
            raise ValueError("self.fsdp is None!")
        return torch.float32 if self.fsdp.precision is None else self.autocast_precision

    @classmethod
    def update_legacy_settings(cls, raw: Dict[str, Any]) -> Dict[str, Any]:
        raw = dict(raw)
        ac = raw.get("activation_checkpointing", None)
        if ac is False:
            raw["activation_checkpointing"] = None
        elif ac is True:
            raw["activation_checkpointing"] = ActivationCheckpointingStrategy.whole_layer.value
        if isinstance(raw.get("optimizer"), dict):
            raw["optimizer"] = OptimizerConfig.update_legacy_settings(raw["optimizer"])
        return raw


# ------------------------------------------------------------------------------ B200 runtime knobs


def _env_flag(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    return default if v is None else v.strip().lower() not in ("0", "false", "no", "off", "")


@dataclass
class B200Runtime:
    """
    Knobs specific to this framework.  They are environment variables, not config keys, so a saved
    ``config.yaml`` stays loadable by the reference.  Each is read where it acts (the module is named); this class
    gathers the ones that select a code path, for logging at start-up (``B200Runtime.from_env()``).

    Execution
      ``OLMO_B200_KERNELS``        use the sm_100a kernel library on CUDA devices (default on; the library being absent
                                   on a GPU machine is an error, not a silent fallback).  ``ops/__init__.py``
      ``OLMO_B200_SCHEDULE``       ``auto`` (default), ``resident`` (every unit stays gathered between uses) or
                                   ``sharded`` (FULL_SHARD proper: block units streamed through slots, gathered in
                                   forward and in backward, reduced per micro-batch).  ``parallel/fsdp.py``
      ``OLMO_B200_FUSED_COMM``     carry all-gathers and reduce-scatters over peer memory inside GEMM launches
                                   (default on when several GPUs share a node; ``0``: NCCL collectives).  ``parallel/fsdp.py``
      ``OLMO_B200_KEEP_ACTS``      ``auto`` (default), ``1`` or ``0``: keep the rotated q/k and SwiGLU outputs of every
                                   block for the backward pass instead of recomputing them; ``auto`` decides after the
                                   first step from the device memory still free.  ``parallel/fsdp.py``
      ``OLMO_B200_ATTENTION``      ``native`` (tcgen05 kernel; other head sizes and lengths are zero-padded onto it) or
                                   ``library`` (the flash-attn package).  ``ops/attention.py``
      ``OLMO_B200_HEAD_CHUNK``     rows of logits materialised at a time by the LM-head + loss path (default 8192).
    Kernel variants (for A/B measurements; the defaults are the fast ones)
      ``OLMO_B200_GEMM_2CTA``      two-CTA ``cta_group::2`` GEMM (default on); ``OLMO_B200_GEMM_TMA_STORE`` its
                                   shared-memory-staged TMA-store epilogue (default on).  ``ops/__init__.py``
      ``OLMO_B200_COMM_CTAS``, ``OLMO_B200_RS_CTAS``, ``OLMO_B200_COMM_STANDALONE_CTAS``   CTAs that carry an all-gather /
                                   a reduce-scatter inside a GEMM launch / in a stand-alone launch (0: chosen from the
                                   sizes).  ``OLMO_B200_RS_SUMSQ`` (default on): gradient-norm partials come out of
                                   the reduce-scatter.  ``parallel/peer.py``
      ``OLMO_B200_WAIT_BUDGET_MS`` time limit of every device-side wait on a peer's flag (default 30000 ms); when it runs
                                   out the kernel records a status word and returns, and the host raises.  ``parallel/peer.py``
      ``OLMO_B200_DECODE_GEMM``    ``auto`` (default), ``native`` or ``library`` for the serving decode projections;
                                   ``OLMO_B200_W4_TARGET_CTAS`` CTAs the 4-bit decode GEMM aims at when it splits K
                                   (default 444).  ``serve/static_cache.py``, ``csrc/w4a16_mma.cu``
    Host side
      ``OLMO_B200_NATIVE_DATA``    ``0`` disables the C++ token reader (byte-range reads from Python instead).
      ``OLMO_B200_NVTX``           ``1`` adds NVTX spans around trainer phases and every block's forward / backward.
      ``OLMO_B200_WRITE_REFERENCE_LAYOUT``  ``1`` with ``sharded_checkpointer: torch_new`` writes sharded checkpoints in the
                                   reference's ``torch_new`` layout.  ``checkpoint.py``
    Shared with the reference: ``OLMO_SHARED_FS``, ``FS_LOCAL_RANK``, ``OLMO_NUM_THREADS``, ``OLMO_NO_SSL``; package data is
    looked up under ``OLMO_DATA_DIR`` first, downloads are cached under ``OLMO_CACHE_DIR``.
    """

    kernels: bool = True
    fused_comm: bool = True
    schedule: str = "auto"
    keep_acts: str = "auto"
    attention: str = "native"
    wait_budget_ms: float = 30000.0

    @classmethod
    def from_env(cls) -> "B200Runtime":
        return cls(
            kernels=_env_flag("OLMO_B200_KERNELS", True),
            fused_comm=_env_flag("OLMO_B200_FUSED_COMM", True),
            schedule=os.environ.get("OLMO_B200_SCHEDULE", "auto").strip().lower(),
            keep_acts=os.environ.get("OLMO_B200_KEEP_ACTS", "auto").strip().lower(),
            attention=os.environ.get("OLMO_B200_ATTENTION", "native").strip().lower(),
            wait_budget_ms=float(os.environ.get("OLMO_B200_WAIT_BUDGET_MS", "30000")),
        )
