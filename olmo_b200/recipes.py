"""
Named training recipes.

The reference ships its model families as hand-maintained YAML files (``configs/official-1124``,
``configs/official-0425``, ``configs/official-0724``, ``configs/tiny``).  Here the architecture and
optimisation hyper-parameters of those families live in two small tables, and the YAML files under
``configs/`` are *generated* from them (``python -m olmo_b200.recipes --write configs``), so that a
family is described once and the launcher, the benchmark and the files on disk cannot drift apart.

Training data is not part of a recipe: the generated files read the token-file list from
``${path.glob:${oc.env:OLMO_DATA_GLOB}}`` when the environment names one, else from the synthetic
token source, and evaluators from ``OLMO_DATA_DIR``.  What a recipe fixes is everything that
determines the compute: shapes, vocabulary, normalisation layout, optimiser, schedule, batch sizes,
sharding.  Sharding defaults are chosen for 180 GB parts (full sharding inside a node, hybrid
sharding beyond it), not copied from the reference's 80 GB settings.
"""
from __future__ import annotations

import argparse
from copy import deepcopy
from pathlib import Path
from typing import Any, Dict, List, Optional

from .config import TrainConfig
from .utils import structured as S

__all__ = ["MODEL_FAMILIES", "RECIPES", "model_dict", "recipe_dict", "recipe_config", "write_configs", "DEFAULT_EVALUATORS"]

# ------------------------------------------------------------------------------------ architectures

_OLMO2_BASE: Dict[str, Any] = dict(
    weight_tying=False, alibi=False, rope=True, rope_theta=500000, flash_attention=True, attention_dropout=0.0,
    include_bias=False, block_type="sequential", layer_norm_type="rms", layer_norm_with_affine=True, layer_norm_eps=1e-6,
    bias_for_layer_norm=False, attention_layer_norm=True, attention_layer_norm_with_affine=True, norm_after=True,
    activation_type="swiglu", residual_dropout=0.0, embedding_dropout=0.0, max_sequence_length=4096,
    vocab_size=100278, embedding_size=100352, eos_token_id=100257, pad_token_id=100277,
    init_device="meta", init_fn="normal", init_std=0.02, init_cutoff_factor=3,
)
_OLMO1_BASE: Dict[str, Any] = dict(
    weight_tying=False, alibi=False, rope=True, flash_attention=True, attention_dropout=0.0, attention_layer_norm=False,
    multi_query_attention=False, include_bias=False, block_type="sequential", layer_norm_type="default",
    layer_norm_with_affine=False, bias_for_layer_norm=False, attention_layer_norm_with_affine=False,
    activation_type="swiglu", residual_dropout=0.0, embedding_dropout=0.0, max_sequence_length=2048,
    vocab_size=50280, embedding_size=50304, eos_token_id=50279, pad_token_id=1, init_device="meta", init_fn="mitchell",
)
_TINY_BASE: Dict[str, Any] = dict(
    mlp_ratio=8, weight_tying=False, alibi=False, rope=True, flash_attention=True, attention_dropout=0.0,
    attention_layer_norm=False, clip_qkv=None, include_bias=False, block_type="sequential", layer_norm_type="rms",
    layer_norm_with_affine=True, layer_norm_eps=1e-6, bias_for_layer_norm=False, attention_layer_norm_with_affine=False,
    activation_type="swiglu", residual_dropout=0.0, embedding_dropout=0.0, max_sequence_length=4096,
    vocab_size=50280, embedding_size=50304, eos_token_id=0, pad_token_id=1, init_device="meta", init_fn="normal",
    init_std=0.02, init_cutoff_factor=3,
)

#: architecture overrides per family member (reference: configs/official-*/ and configs/tiny/)
MODEL_FAMILIES: Dict[str, Dict[str, Any]] = {
    "olmo2-1b": {**_OLMO2_BASE, "d_model": 2048, "n_heads": 16, "n_layers": 16, "mlp_ratio": 8},
    "olmo2-7b": {**_OLMO2_BASE, "d_model": 4096, "n_heads": 32, "n_layers": 32, "mlp_hidden_size": 22016},
    "olmo2-13b": {**_OLMO2_BASE, "d_model": 5120, "n_heads": 40, "n_layers": 40, "mlp_hidden_size": 27648},
    "olmo1-1b": {**_OLMO1_BASE, "d_model": 2048, "n_heads": 16, "n_layers": 16, "mlp_ratio": 8, "weight_tying": True},
    "olmo1-7b": {**_OLMO1_BASE, "d_model": 4096, "n_heads": 32, "n_layers": 32, "mlp_hidden_size": 22016},
    "olmo1-7b-0724": {**_OLMO1_BASE, "d_model": 4096, "n_heads": 32, "n_layers": 32, "mlp_hidden_size": 22016,
                      "clip_qkv": 8.0, "max_sequence_length": 4096},
    "tiny-20m": {**_TINY_BASE, "d_model": 256, "n_heads": 8, "n_layers": 8},
    "tiny-60m": {**_TINY_BASE, "d_model": 512, "n_heads": 8, "n_layers": 8},
    "tiny-150m": {**_TINY_BASE, "d_model": 768, "n_heads": 12, "n_layers": 12},
    "tiny-300m": {**_TINY_BASE, "d_model": 1024, "n_heads": 16, "n_layers": 16},
    "tiny-700m": {**_TINY_BASE, "d_model": 1536, "n_heads": 16, "n_layers": 16},
}

# --------------------------------------------------------------------------------------- evaluators

_CORE_TASKS = [
    "piqa", "hellaswag", "winogrande", "openbook_qa", "boolq", "sciq", "arc_easy", "arc_challenge", "copa",
    "commonsense_qa", "social_iqa",
]
_MMLU_TASKS = [f"mmlu_{g}_{v}" for v in ("var", "mc_5shot", "mc_5shot_test") for g in ("stem", "humanities", "social_sciences", "other")]
_PPL_TASKS = ["basic_arithmetic", "trivia_qa_wiki_ppl", "natural_qs_open_ppl", "arc_easy_ppl"]
#: the in-loop evaluation suite of the OLMo-2 runs
DEFAULT_EVALUATORS: List[str] = _CORE_TASKS + _MMLU_TASKS + _PPL_TASKS

# ------------------------------------------------------------------------------------------ recipes


def _adamw(lr: float, **extra: Any) -> Dict[str, Any]:
    return {"name": "adamw", "learning_rate": lr, "weight_decay": 0.1, "betas": [0.9, 0.95], "metrics_log_interval": 1, **extra}


_OLMO2_OPT = dict(eps=1e-8, decay_norm_and_bias=True, decay_embeddings=False)
_OLMO2_SCHED = {"name": "cosine_with_warmup", "units": "tokens", "t_warmup": 8388608000, "t_max": 5e12, "alpha_f": 0.1, "warmup_min_lr": 0.0}
_OLMO2_LOSS = {"softmax_auxiliary_loss": True, "auxiliary_loss_multiplier": 1e-5, "fused_loss": True}
_TOK_DOLMA2 = "tokenizers/allenai_dolma2.json"
_TOK_NEOX_PII = "tokenizers/allenai_eleuther-ai-gpt-neox-20b-pii-special.json"
_TOK_DOLMA15 = "tokenizers/allenai_gpt-neox-olmo-dolma-v1_5.json"

#: name -> everything that differs from the TrainConfig defaults.  ``file`` is the path under configs/.
RECIPES: Dict[str, Dict[str, Any]] = {
    "OLMo2-1B-stage1": {
        "file": "official-0425/OLMo2-1B-stage1.yaml", "family": "olmo2-1b", "tokenizer": _TOK_DOLMA2,
        "optimizer": _adamw(4.0e-4, **_OLMO2_OPT), "scheduler": _OLMO2_SCHED, **_OLMO2_LOSS,
        "global_train_batch_size": 512, "device_train_microbatch_size": 8, "max_duration": "4e12T",
        "evaluators": DEFAULT_EVALUATORS,
    },
    "OLMo2-7B-stage1": {
        "file": "official-1124/OLMo2-7B-stage1.yaml", "family": "olmo2-7b", "tokenizer": _TOK_DOLMA2,
        "optimizer": _adamw(3.0e-4, **_OLMO2_OPT), "scheduler": _OLMO2_SCHED, **_OLMO2_LOSS,
        "global_train_batch_size": 1024, "device_train_microbatch_size": 2, "max_duration": "1ep",
        "evaluators": DEFAULT_EVALUATORS,
    },
    "OLMo2-7B-stage2": {
        "file": "official-1124/OLMo2-7B-stage2.yaml", "family": "olmo2-7b", "tokenizer": _TOK_DOLMA2, "seed": 42,
        "optimizer": _adamw(0.000061499, **_OLMO2_OPT),
        "scheduler": {"name": "linear_with_warmup", "t_warmup": 0, "alpha_f": 0.0}, **_OLMO2_LOSS,
        "global_train_batch_size": 1024, "device_train_microbatch_size": 2, "max_duration": "50e9T", "stop_at": 11931,
        "load_path": "${oc.env:OLMO_STAGE1_CHECKPOINT,null}", "restore_dataloader": False, "no_pre_train_checkpoint": True,
        "evaluators": DEFAULT_EVALUATORS,
    },
    "OLMo2-13B-stage1": {
        "file": "official-1124/OLMo2-13B-stage1.yaml", "family": "olmo2-13b", "tokenizer": _TOK_DOLMA2,
        "optimizer": _adamw(3.0e-4, **_OLMO2_OPT), "scheduler": _OLMO2_SCHED, **_OLMO2_LOSS,
        "global_train_batch_size": 2048, "device_train_microbatch_size": 2, "max_duration": "1ep",
        "evaluators": DEFAULT_EVALUATORS,
    },
    "OLMo-1B": {
        "file": "official-0724/OLMo-1B.yaml", "family": "olmo1-1b", "tokenizer": _TOK_NEOX_PII,
        "optimizer": _adamw(4.0e-4), "scheduler": {"name": "cosine_with_warmup", "t_warmup": 2000, "alpha_f": 0.1},
        "global_train_batch_size": 2048, "device_train_microbatch_size": 8, "max_duration": 739328,
        "evaluators": _CORE_TASKS,
    },
    "OLMo-7B": {
        "file": "official-0724/OLMo-7B.yaml", "family": "olmo1-7b", "tokenizer": _TOK_NEOX_PII,
        "optimizer": _adamw(3.0e-4),
        "scheduler": {"name": "linear_with_warmup", "t_warmup": 5000, "alpha_f": 0.1, "grad_clip_warmup_steps": 1000},
        "global_train_batch_size": 2048, "device_train_microbatch_size": 2, "max_duration": "2e12T",
        "evaluators": _CORE_TASKS,
    },
    "OLMo-7B-0724": {
        "file": "official-0724/OLMo-7B-0724.yaml", "family": "olmo1-7b-0724", "tokenizer": _TOK_DOLMA15,
        "optimizer": _adamw(3.0e-4, decay_norm_and_bias=True, decay_embeddings=True),
        "scheduler": {"name": "cosine_with_warmup", "units": "tokens", "t_warmup": 10485760000, "t_max": 3e12, "alpha_f": 0.1,
                      "grad_clip_warmup_steps": 2097152000},
        "global_train_batch_size": 1024, "device_train_microbatch_size": 2, "max_duration": "2ep",
        "evaluators": _CORE_TASKS,
    },
}
# The published stage-2 ("mid-training") runs: the same recipe from the stage-1 endpoint with different data-order
# seeds (their weights are averaged afterwards); reference: configs/official-1124/OLMo2-{7B,13B}-stage2-seed*.yaml and
# configs/official-0425/OLMo2-1B-stage2-seed*.yaml.
for _seed in (42, 42069, 666):
    RECIPES[f"OLMo2-7B-stage2-seed{_seed}"] = {
        **deepcopy(RECIPES["OLMo2-7B-stage2"]), "file": f"official-1124/OLMo2-7B-stage2-seed{_seed}.yaml", "seed": _seed,
        "load_path": "${oc.env:OLMO_STAGE1_CHECKPOINT,https://olmo-checkpoints.org/ai2-llm/peteish7/step928646-unsharded}",
    }
    RECIPES[f"OLMo2-1B-stage2-seed{_seed}"] = {
        **deepcopy(RECIPES["OLMo2-7B-stage2"]), "file": f"official-0425/OLMo2-1B-stage2-seed{_seed}.yaml", "family": "olmo2-1b",
        "seed": _seed, "optimizer": _adamw(0.000074487, **_OLMO2_OPT), "global_train_batch_size": 512,
        "device_train_microbatch_size": 4, "max_duration": "50e9T", "stop_at": 23852,
        "load_path": "${oc.env:OLMO_STAGE1_CHECKPOINT,https://olmo-checkpoints.org/ai2-llm/peteish1/step1907359-unsharded/}",
    }
for _seed, _tokens, _stop in ((1110, "100B", 11931), (2662, "100B", 11931), (6209, "100B", 11931), (2662, "300B", 35773)):
    RECIPES[f"OLMo2-13B-stage2-seed{_seed}-{_tokens}"] = {
        **deepcopy(RECIPES["OLMo2-7B-stage2"]), "file": f"official-1124/OLMo2-13B-stage2-seed{_seed}-{_tokens}.yaml",
        "family": "olmo2-13b", "seed": _seed, "optimizer": _adamw(9e-5, **_OLMO2_OPT),
        "scheduler": {"name": "linear_with_warmup", "units": "steps", "t_warmup": 0, "alpha_f": 0.0},
        "global_train_batch_size": 2048, "device_train_microbatch_size": 2, "max_duration": f"{_tokens[:-1]}e9T", "stop_at": _stop,
        "load_path": "${oc.env:OLMO_STAGE1_CHECKPOINT,https://olmo-checkpoints.org/ai2-llm/peteish13/step596057-unsharded}",
    }
# OLMo-7B-0424 is the run OLMo-7B-0724 continued; the two published configs are the same file
RECIPES["OLMo-7B-0424"] = {**deepcopy(RECIPES["OLMo-7B-0724"]), "file": "official-0724/OLMo-7B-0424.yaml"}

for _name, _mb in (("20M", 16), ("60M", 8), ("150M", 4), ("300M", 4), ("700M", 2)):
    RECIPES[f"OLMo-{_name}"] = {
        "file": f"tiny/OLMo-{_name}.yaml", "family": f"tiny-{_name.lower()}", "tokenizer": _TOK_DOLMA15,
        "optimizer": _adamw(6.0e-4, eps=1e-8, decay_norm_and_bias=True, decay_embeddings=True),
        "scheduler": {"name": "cosine_with_warmup", "t_warmup": 5000, "alpha_f": 0.1},
        "global_train_batch_size": 1024, "device_train_microbatch_size": _mb, "max_duration": "1ep", "stop_at": 406934,
        "evaluators": _CORE_TASKS,
    }

# The development runs the official OLMo-2 configs were distilled from (reference: configs/peteish{1,7,13}-{weka,google,
# s3}.yaml, which differ from one another only in storage roots).  One file per size here; the storage root comes from
# OLMO_DATA_GLOB / OLMO_REMOTE_SAVE_FOLDER instead of a file per storage system.
for _size, _official, _extra in (
    ("1", "OLMo2-1B-stage1", {"device_train_microbatch_size": 4, "fsdp": {"sharding_strategy": "SHARD_GRAD_OP", "wrapping_strategy": "by_block_and_size", "precision": "mixed"}}),
    ("7", "OLMo2-7B-stage1", {"activation_checkpointing": "one_in_four"}),
    ("13", "OLMo2-13B-stage1", {}),
):
    RECIPES[f"peteish{_size}"] = {
        **deepcopy(RECIPES[_official]), "file": f"peteish{_size}.yaml",
        "wandb": {"name": "${run_name}", "project": "olmo-medium" if _size != "1" else "olmo-small", "group": "${run_name}"},
        "save_num_checkpoints_to_keep": -1, "save_interval_unsharded": None,
        "remote_save_folder": "${oc.env:OLMO_REMOTE_SAVE_FOLDER,null}", **_extra,
    }

# Mid-training anneal from a stage-1 checkpoint: linear decay to zero over 50B tokens, data position not restored
# (reference: configs/annealing/*.yaml; ``scripts/anneal_config_maker.py`` derives these from a checkpoint's own config).
RECIPES["OLMo2-7B-anneal-example"] = {
    **deepcopy(RECIPES["OLMo2-7B-stage2"]), "file": "annealing/OLMo2-7B-anneal-example.yaml",
}

# The same development runs as the reference files them, one file per storage system (configs/peteish{1,7,13}-{weka,
# google,s3}.yaml): the recipe of the size with that storage's file list (``data_mixes/<name>.txt``) and the few settings in
# which the files differ (epoch vs token budget, cosine horizon, activation checkpointing on the smaller-memory pool).
for _size, _store, _diff in (
    ("1", "google", {"max_duration": "4e12T"}),
    ("1", "weka", {"max_duration": "1ep", "scheduler": {**_OLMO2_SCHED, "t_max": 3e12}}),
    ("7", "google", {}), ("7", "weka", {}), ("7", "s3", {"activation_checkpointing": None}),
    ("13", "google", {"max_duration": "5e12T"}), ("13", "weka", {}), ("13", "s3", {}),
):
    RECIPES[f"peteish{_size}-{_store}"] = {**deepcopy(RECIPES[f"peteish{_size}"]), "file": f"peteish{_size}-{_store}.yaml", **_diff}

# Mid-training ("annealing") runs: linear decay to zero from a stage-1 checkpoint over a token budget, new data order,
# data position not restored.  (reference: configs/annealing/*.yaml; columns: size, file stem, seed, peak lr, tokens,
# stop step, stage-1 checkpoint, activation checkpointing)
_ANNEAL_RUNS = (
    ("1", "peteish1-anneal-from-1907359-50B-nowup-moremath-dclm07-fw2-se-flan-google", 7201, 7.448728958032132e-05, "50e9T", 23852,
     "gs://ai2-llm/checkpoints/OLMo-small/peteish1/step1907359", "one_in_four"),
    ("13", "peteish13-anneal-from-596057-100B-legal-whammy-2-google", 7201, 9e-5, "100e9T", 11931,
     "gs://ai2-llm/checkpoints/OLMo-medium/peteish13-highlr-zlossfix/step596057", None),
    ("13", "peteish13-anneal-from-596057-300B-legal-whammy-2-google", 7201, 9e-5, "300e9T", 35773,
     "gs://ai2-llm/checkpoints/OLMo-medium/peteish13-highlr-zlossfix/step596057", None),
    ("7", "peteish7-anneal-from-477000-100B-moremath-dclm07-fw2-se-flan-google", 7201, 0.00020707, "100e9T", 23852,
     "gs://ai2-llm/checkpoints/OLMo-medium/peteish7/step477000", None),
    ("7", "peteish7-medlr-anneal-from-477000-100B-moremath-dclm07-fw2-se-flan-google", 7201, 0.00041414, "100e9T", 23852,
     "gs://ai2-llm/checkpoints/OLMo-medium/peteish7-medlr/step477000", None),
) + tuple(
    ("7", f"peteish7-weka-anneal-from-928646-50B-nowup_legal-whammy-2_seed{_seed}", _seed, 6.1499e-05, "50e9T", 11931,
     "/weka/oe-training-default/ai2-llm/checkpoints/OLMo-medium/peteish7/step928646", "one_in_four")
    for _seed in (42, 42069, 666)
)
_SIZE_SHAPE = {"1": ("olmo2-1b", 512), "7": ("olmo2-7b", 1024), "13": ("olmo2-13b", 2048)}
for _size, _stem, _seed, _lr, _tokens, _stop, _ckpt, _ac in _ANNEAL_RUNS:
    RECIPES[_stem] = {
        **deepcopy(RECIPES["OLMo2-7B-stage2"]), "file": f"annealing/{_stem}.yaml", "family": _SIZE_SHAPE[_size][0], "seed": _seed,
        "optimizer": _adamw(_lr, **_OLMO2_OPT), "scheduler": {"name": "linear_with_warmup", "units": "steps", "t_warmup": 0, "alpha_f": 0.0},
        "global_train_batch_size": _SIZE_SHAPE[_size][1], "device_train_microbatch_size": 2, "max_duration": _tokens, "stop_at": _stop,
        "load_path": "${oc.env:OLMO_STAGE1_CHECKPOINT," + _ckpt + "}", "activation_checkpointing": _ac,
    }

# "Micro-anneals": the same decay over one pass of a small candidate data source mixed with web text, used to rank data
# sources cheaply (reference: configs/microannealing/*.yaml).  All start from step 928646 of the 7B run except the last.
_MICRO_SOURCES = (
    "automathtext", "bestof-v1", "mathcoder-synthetic", "mathpile", "owm", "pes2o", "reddit-qa-all", "reddit-v1", "se",
    "small-sources-big-dclm", "small-sources-multiadd", "small-sources", "small-sources_x2", "small-sources_x4", "tiny-gsm-inline",
    "tiny-gsm-mind", "tiny-gsm-mind_x2",
)
_MICRO_RUNS = tuple(
    (f"peteish7-weka-microanneal-from928646_{_src}", 6.1499e-05, "/weka/oe-training-default/ai2-llm/checkpoints/OLMo-medium/peteish7/step928646")
    for _src in _MICRO_SOURCES
) + (("peteish7-weka-microanneal-fromMegaMath1.1-5000_nonmath", 3.5726e-05,
      "/weka/oe-training-default/ai2-llm/checkpoints/OLMo-medium/peteish7-weka-anneal-from-928646-50B-megamath_v1.1.yaml/step5000/"),)
for _stem, _lr, _ckpt in _MICRO_RUNS:
    RECIPES[_stem] = {
        **deepcopy(RECIPES["OLMo2-7B-stage2"]), "file": f"microannealing/{_stem}.yaml", "seed": 7201, "optimizer": _adamw(_lr, **_OLMO2_OPT),
        "max_duration": "1ep", "stop_at": None, "load_path": "${oc.env:OLMO_STAGE1_CHECKPOINT," + _ckpt + "}",
        "activation_checkpointing": "one_in_four",
    }

# Training on a user-supplied ``torch.utils.data.Dataset`` instead of token memmaps (reference:
# configs/custom_dataset_example.yaml): ``name`` is ``module.Class`` (or a class name plus ``module``), ``args`` its
# constructor arguments, ``collate_config`` maps the dataset's field names onto the batch keys the trainer reads.
RECIPES["custom-dataset-example"] = {
    **deepcopy(RECIPES["OLMo-20M"]), "file": "custom_dataset_example.yaml", "evaluators": [],
    "data": {
        "paths": None, "num_workers": 0, "prefetch_factor": None, "persistent_workers": False,
        "custom_dataset": {
            "name": "my_package.my_module.MyDataset", "args": {"path": "/data/my-corpus", "sequence_length": 4096},
            "collate_config": {"input_id_field": "token_ids", "label_mask_field": None, "metadata_field": None},
        },
    },
}

#: recipe name -> packaged ``data_mixes/<name>.txt`` when the two differ
_MIX_ALIASES = {
    "OLMo2-7B-stage2": "OLMo2-7B-stage2-seed42", "peteish1": "peteish1-weka", "peteish7": "peteish7-weka", "peteish13": "peteish13-weka",
    "OLMo2-7B-anneal-example": "peteish7-weka-anneal-from-928646-50B-nowup_legal-whammy-2_seed42",
}

_COMMON: Dict[str, Any] = {
    "seed": 6198,
    "dry_run": False,
    "precision": "amp_bf16",
    "max_grad_norm": 1.0,
    "distributed_strategy": "fsdp",
    # one B200 holds a 7B model's full optimiser state; FULL_SHARD inside the node keeps headroom for
    # long micro-batches, and HYBRID_SHARD takes over when the job spans nodes
    "fsdp": {"sharding_strategy": "FULL_SHARD", "wrapping_strategy": "by_block_and_size", "precision": "mixed"},
    "speed_monitor": {"window_size": 1},
    "save_overwrite": False,
    "save_interval": 1000,
    "save_interval_ephemeral": 250,
    "save_num_checkpoints_to_keep": 0,
    "save_interval_unsharded": 1000,
    "save_num_unsharded_checkpoints_to_keep": -1,
    "sharded_checkpointer": "olmo_core",
    "eval_interval": 1000,
    "eval_subset_num_batches": -1,
    "device_eval_batch_size": "${device_train_microbatch_size}",
    "gen1_gc_interval": 1,
    "data": {
        "pad_direction": "right", "num_workers": 8, "drop_last": True, "pin_memory": True, "prefetch_factor": 8,
        "persistent_workers": True, "memmap_dtype": "uint32", "timeout": 0,
        "instance_filter": {"repetition_max_period": 13, "repetition_min_period": 1, "repetition_max_count": 32},
        "paths": "${path.glob:${oc.env:OLMO_DATA_GLOB,/nonexistent/*.npy}}",
    },
}


def model_dict(family: str) -> Dict[str, Any]:
    """Architecture of a family member as a plain mapping (keys of ``ModelConfig``)."""
    try:
        return deepcopy(MODEL_FAMILIES[family])
    except KeyError:
        raise KeyError(f"unknown model family '{family}'; known: {sorted(MODEL_FAMILIES)}") from None


def recipe_dict(name: str) -> Dict[str, Any]:
    """The un-resolved mapping that is written to ``configs/<file>`` for recipe ``name``."""
    try:
        spec = deepcopy(RECIPES[name])
    except KeyError:
        raise KeyError(f"unknown recipe '{name}'; known: {sorted(RECIPES)}") from None
    spec.pop("file")
    out: Dict[str, Any] = {"run_name": name}
    out.update(deepcopy(_COMMON))
    out["model"] = model_dict(spec.pop("family"))
    out["tokenizer"] = {"identifier": spec.pop("tokenizer"), "truncate_direction": "right"}
    if out["model"]["vocab_size"] < 65536:
        out["data"]["memmap_dtype"] = "uint16"
    out["evaluators"] = [{"label": label, "type": "downstream"} for label in spec.pop("evaluators")]
    mix = spec.pop("mix", _MIX_ALIASES.get(name, name))
    if "data" in spec:
        out["data"] = S.deep_merge(out["data"], spec.pop("data"))
    elif mix is not None:
        # a local copy of the data (OLMO_DATA_GLOB) wins; otherwise the packaged list of the files the published run read
        out["data"]["paths"] = "${data.mix:" + mix + ",${oc.env:OLMO_DATA_GLOB,}}"
    out.update(spec)
    return out


def recipe_config(name: str, overrides: Optional[List[str]] = None, validate_paths: bool = False) -> TrainConfig:
    """Build the validated :class:`TrainConfig` of a recipe, with optional ``a.b=c`` overrides."""
    from .config import _register_path_resolvers, _schema_defaults

    _register_path_resolvers(validate_paths=validate_paths)
    raw = recipe_dict(name)
    if overrides:
        raw = S.deep_merge(raw, S.parse_dotlist(overrides))
    defaults = S.to_container(_schema_defaults(TrainConfig), enum_to_str=True)
    return S.build(TrainConfig, S.resolve_interpolations(raw, root=S.deep_merge(defaults, raw)))


def write_configs(folder: Path, names: Optional[List[str]] = None) -> List[Path]:
    """Write the YAML file of every recipe (or of ``names``) below ``folder``; returns the paths."""
    written = []
    for name in names or sorted(RECIPES):
        target = Path(folder) / RECIPES[name]["file"]
        target.parent.mkdir(parents=True, exist_ok=True)
        header = (
            f"# {name}: generated by `python -m olmo_b200.recipes --write <dir>`; edit olmo_b200/recipes.py, not this file.\n"
            "# Token files: data.paths is the packaged list of the files the published run read (olmo_data/data_mixes/);\n"
            "# set OLMO_DATA_GLOB (e.g. '/data/dolma/**/*.npy') to train on a local copy, or override data.paths.\n"
        )
        target.write_text(header + S.dump_yaml(recipe_dict(name)))
        written.append(target)
    return written


def main(argv: Optional[List[str]] = None) -> None:
    ap = argparse.ArgumentParser(description="List the named recipes or regenerate their YAML files.")
    ap.add_argument("--write", metavar="DIR", help="write every recipe's YAML file below DIR")
    ap.add_argument("--show", metavar="NAME", help="print one recipe as YAML")
    args = ap.parse_args(argv)
    if args.write:
        for p in write_configs(Path(args.write)):
            print(p)
    elif args.show:
        print(S.dump_yaml(recipe_dict(args.show)))
    else:
        for name in sorted(RECIPES):
            print(f"{name:20s} {RECIPES[name]['family']:14s} configs/{RECIPES[name]['file']}")


if __name__ == "__main__":
    main()
