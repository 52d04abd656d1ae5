"""Typed config engine: YAML quirks, overrides, interpolation, resolvers, legacy rewrites, recipes."""
import os
from pathlib import Path

import pytest

from olmo_b200.config import (
    ActivationCheckpointingStrategy,
    CheckpointType,
    DistributedStrategy,
    ModelConfig,
    OptimizerType,
    SchedulerType,
    ShardingStrategy,
    TrainConfig,
)
from olmo_b200.exceptions import OLMoConfigurationError
from olmo_b200.recipes import MODEL_FAMILIES, RECIPES, recipe_config, write_configs
from olmo_b200.utils import structured as S


def write(tmp_path, text, name="c.yaml"):
    p = tmp_path / name
    p.write_text(text)
    return p


def test_yaml_scalars_follow_yaml_1_1_floats():
    raw = S.load_yaml("a: 3e-4\nb: 1e5\nc: 5e12\nd: 4e12T\ne: 739_328\nf: null\ng: off\n")
    assert raw["a"] == pytest.approx(3e-4) and isinstance(raw["a"], float)
    assert raw["b"] == 1e5 and isinstance(raw["c"], float)
    assert raw["d"] == "4e12T"
    assert raw["f"] is None


def test_load_with_overrides_and_interpolation(tmp_path):
    p = write(
        tmp_path,
        """
run_name: demo
model:
  d_model: 64
  n_heads: 4
  n_layers: 2
optimizer:
  learning_rate: 3e-4
scheduler:
  name: linear_with_warmup
device_train_microbatch_size: 4
device_eval_batch_size: ${device_train_microbatch_size}
save_folder: /tmp/${run_name}/ckpt
wandb:
  name: ${run_name}
""",
    )
    cfg = TrainConfig.load(p, overrides=["model.n_layers=3", "optimizer.name=lionw", "max_duration=2ep", "global_train_batch_size=16"])
    assert cfg.model.d_model == 64 and cfg.model.n_layers == 3
    assert cfg.optimizer.name == OptimizerType.lionw and cfg.optimizer.learning_rate == pytest.approx(3e-4)
    assert cfg.scheduler.name == SchedulerType.linear_with_warmup
    assert cfg.device_eval_batch_size == 4
    assert cfg.save_folder == "/tmp/demo/ckpt" and cfg.wandb.name == "demo"
    assert cfg.max_duration == "2ep" and cfg.global_train_batch_size == 16


def test_unknown_keys_and_bad_values_are_rejected(tmp_path):
    with pytest.raises(OLMoConfigurationError):
        TrainConfig.load(write(tmp_path, "not_a_field: 1\n"))
    with pytest.raises(OLMoConfigurationError):
        TrainConfig.load(write(tmp_path, "model:\n  d_model: lots\n"))
    with pytest.raises(OLMoConfigurationError):
        TrainConfig.load(write(tmp_path, "optimizer:\n  name: sgd\n"))
    with pytest.raises(OLMoConfigurationError):
        TrainConfig.load(write(tmp_path, "run_name: x\n"), overrides=["model.nope=1"])
    with pytest.raises(OLMoConfigurationError):
        TrainConfig.load(tmp_path / "missing.yaml")


def test_env_and_path_resolvers(tmp_path, monkeypatch):
    for name in ("a.npy", "b.npy"):
        (tmp_path / name).write_bytes(b"")
    monkeypatch.setenv("MY_GLOB", str(tmp_path / "*.npy"))
    monkeypatch.delenv("NOT_SET_ANYWHERE", raising=False)
    p = write(
        tmp_path,
        """
run_name: ${oc.env:NOT_SET_ANYWHERE,fallback}
data:
  paths: ${path.glob:${oc.env:MY_GLOB}}
load_path: ${path.choose:/definitely/not/here,%s}
""" % tmp_path,
    )
    cfg = TrainConfig.load(p)
    assert cfg.run_name == "fallback"
    assert cfg.data.paths == [str(tmp_path / "a.npy"), str(tmp_path / "b.npy")]
    assert cfg.load_path == str(tmp_path)
    with pytest.raises(FileNotFoundError):
        TrainConfig.load(write(tmp_path, "data:\n  paths: ${path.glob:/definitely/not/here/*.npy}\n", "d.yaml"))
    cfg = TrainConfig.load(tmp_path / "d.yaml", validate_paths=False)
    assert cfg.data.paths == []

    (tmp_path / "run" / "step10").mkdir(parents=True)
    (tmp_path / "run" / "step200").mkdir()
    (tmp_path / "run" / "step200-unsharded").mkdir()
    cfg = TrainConfig.load(write(tmp_path, "load_path: ${path.last_checkpoint:%s}\n" % (tmp_path / "run"), "e.yaml"))
    assert os.path.basename(cfg.load_path).startswith("step200")


def test_legacy_settings_are_rewritten(tmp_path):
    cfg = TrainConfig.load(write(tmp_path, "activation_checkpointing: true\noptimizer:\n  name: decoupled_lionw\n  eps: 1e-8\n"))
    assert cfg.activation_checkpointing == ActivationCheckpointingStrategy.whole_layer
    assert cfg.optimizer.name == OptimizerType.lionw
    cfg = TrainConfig.load(write(tmp_path, "activation_checkpointing: false\n"))
    assert cfg.activation_checkpointing is None


def test_save_load_round_trip_and_helpers(tmp_path):
    cfg = TrainConfig(model=ModelConfig(d_model=32, n_heads=2, n_layers=1), run_name="rt")
    cfg.fsdp.sharding_strategy = ShardingStrategy.HYBRID_SHARD
    cfg.save(tmp_path / "out.yaml")
    again = TrainConfig.load(tmp_path / "out.yaml", validate_paths=False)
    assert again == cfg
    only_model = ModelConfig.load(tmp_path / "out.yaml", key="model")
    assert only_model == cfg.model
    clone = cfg.update_with(run_name="other")
    assert clone.run_name == "other" and cfg.run_name == "rt"
    d = cfg.asdict(exclude=["model"])
    assert "model" not in d and d["run_name"] == "rt"
    made = ModelConfig.new(d_model=16, n_heads=2)
    assert made.d_model == 16
    assert cfg.distributed_strategy in (DistributedStrategy.fsdp, None) or isinstance(cfg.distributed_strategy, DistributedStrategy)
    assert CheckpointType("sharded") == CheckpointType.sharded


def test_model_config_derived_quantities():
    m = ModelConfig(d_model=128, n_heads=8, n_kv_heads=2, n_layers=2)
    assert m.effective_n_kv_heads == 2
    assert ModelConfig(d_model=128, n_heads=8, multi_query_attention=True).effective_n_kv_heads == 1
    assert ModelConfig(d_model=128, n_heads=8).effective_n_kv_heads == 8
    with pytest.raises(OLMoConfigurationError):
        ModelConfig(d_model=128, n_heads=8, multi_query_attention=True, n_kv_heads=2).effective_n_kv_heads


def test_dotlist_parsing_types():
    got = S.parse_dotlist(["a.b=1", "a.c=2.5", "x=null", "y=[1,2]", "z=true", "s=hello world", "t=1e-5"])
    assert got == {"a": {"b": 1, "c": 2.5}, "x": None, "y": [1, 2], "z": True, "s": "hello world", "t": 1e-5}
    assert S.deep_merge({"a": {"b": 1, "c": 2}}, {"a": {"c": 3}}) == {"a": {"b": 1, "c": 3}}


@pytest.mark.parametrize("name", sorted(RECIPES))
def test_every_recipe_builds(name):
    cfg = recipe_config(name)
    fam = MODEL_FAMILIES[RECIPES[name]["family"]]
    assert cfg.model.d_model == fam["d_model"] and cfg.model.n_layers == fam["n_layers"]
    assert cfg.model.d_model % cfg.model.n_heads == 0
    assert cfg.global_train_batch_size % cfg.device_train_microbatch_size == 0
    assert cfg.device_eval_batch_size == cfg.device_train_microbatch_size
    assert cfg.run_name == name


def test_recipe_overrides_and_written_files(tmp_path):
    cfg = recipe_config("OLMo2-7B-stage1", ["model.n_layers=2", "optimizer.learning_rate=1e-3"])
    assert cfg.model.n_layers == 2 and cfg.optimizer.learning_rate == pytest.approx(1e-3)
    assert cfg.model.mlp_hidden_size == 22016 and cfg.softmax_auxiliary_loss and cfg.fused_loss
    paths = write_configs(tmp_path)
    assert len(paths) == len(RECIPES)
    for p in paths:
        loaded = TrainConfig.load(p, validate_paths=False)
        assert loaded == recipe_config(loaded.run_name)


def test_committed_config_files_match_the_recipes():
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent / "configs"
    for name, spec in RECIPES.items():
        on_disk = TrainConfig.load(root / spec["file"], validate_paths=False)
        assert on_disk == recipe_config(name), f"configs/{spec['file']} is stale: rerun python -m olmo_b200.recipes --write configs"


def test_official_config_resolves_tokenizer_data_mix_and_evaluators_from_package_data(monkeypatch):
    """No environment variable: the tokenizer file, the ordered list of the run's token files and the evaluation sets
    come from the ``olmo_data`` package."""
    import torch

    from olmo_b200.eval import build_evaluator
    from olmo_b200.launch import derive_batch_sizes
    from olmo_b200.tokenizer import Tokenizer

    monkeypatch.delenv("OLMO_DATA_GLOB", raising=False)
    monkeypatch.delenv("OLMO_DATA_DIR", raising=False)
    root = Path(__file__).resolve().parent.parent
    cfg = TrainConfig.load(root / "configs" / "official-1124" / "OLMo2-7B-stage1.yaml", validate_paths=False)
    assert len(cfg.data.paths) == 1122 and cfg.data.paths[0].startswith("http") and cfg.data.paths[0].endswith(".npy")
    derive_batch_sizes(cfg, 1)
    tok = Tokenizer.from_train_config(cfg)
    assert tok.vocab_size == 100278 and tok.eos_token_id == 100257
    labels = [e.label for e in cfg.evaluators]
    assert len(labels) == 27
    for ec in cfg.evaluators:
        if ec.label in ("piqa", "arc_easy", "mmlu_stem_var", "basic_arithmetic"):
            ev = build_evaluator(cfg, ec, tok, torch.device("cpu"))
            assert len(ev.eval_loader.dataset) > 0
    # a local copy of the data takes precedence over the packaged list
    monkeypatch.setenv("OLMO_DATA_GLOB", str(root / "test_fixtures" / "*.gz"))
    local = TrainConfig.load(root / "configs" / "official-1124" / "OLMo2-7B-stage1.yaml", validate_paths=False)
    assert local.data.paths and all(p.endswith(".gz") for p in local.data.paths)


def test_named_data_mixes_and_checkpoint_tables_are_packaged():
    from olmo_b200.data.named_data_mixes import DATA_PATHS, resolve_mix

    assert {"dolma17", "dolma17_flan_sep_rulebased", "olmoe-mix-0924"} <= set(DATA_PATHS)
    assert len(DATA_PATHS["dolma17"]) == 1033
    assert resolve_mix("olmoe-mix-0924", "s3://bucket/")[0].startswith("s3://bucket/")
    root = Path(__file__).resolve().parent.parent / "configs"
    for rel in ("official-1124/OLMo-2-1124-7B.csv", "official-1124/OLMo-2-1124-13B.csv", "official-0425/OLMo-2-0425-1B.csv", "official-0724/OLMo-7B-0724.csv"):
        assert (root / rel).is_file(), rel


def test_development_anneal_and_micro_anneal_recipes_are_generated():
    from olmo_b200.recipes import RECIPES, recipe_config

    files = {spec["file"] for spec in RECIPES.values()}
    assert sum(f.startswith("annealing/peteish") for f in files) == 8 and sum(f.startswith("microannealing/") for f in files) == 18
    assert {f"peteish{n}-{s}.yaml" for n, s in (("1", "google"), ("1", "weka"), ("7", "google"), ("7", "weka"), ("7", "s3"), ("13", "google"),
                                                ("13", "weka"), ("13", "s3"))} <= files
    repo = Path(__file__).resolve().parent.parent
    assert all((repo / "configs" / f).is_file() for f in files), "run `python -m olmo_b200.recipes --write configs`"
    micro = recipe_config("peteish7-weka-microanneal-from928646_owm")
    assert micro.max_duration == "1ep" and micro.stop_at is None and micro.seed == 7201 and micro.restore_dataloader is False
    assert micro.optimizer.learning_rate == pytest.approx(6.1499e-05) and micro.load_path.endswith("peteish7/step928646") and len(micro.data.paths) == 25
    big = recipe_config("peteish13-anneal-from-596057-300B-legal-whammy-2-google")
    assert big.model.d_model == 5120 and big.stop_at == 35773 and big.max_duration == "300e9T" and big.global_train_batch_size == 2048
    assert recipe_config("peteish1-weka").scheduler.t_max == 3e12 and recipe_config("peteish7-s3").activation_checkpointing is None


def test_unknown_key_names_the_nearest_field():
    with pytest.raises(OLMoConfigurationError, match=r"Key 'optimizer.learning_rat' is not in struct OptimizerConfig; did you mean 'optimizer.learning_rate'\?"):
        TrainConfig.new(optimizer={"learning_rat": 1e-3})
    with pytest.raises(OLMoConfigurationError) as e:
        TrainConfig.new(zzz_nothing_like_it=1)
    assert "did you mean" not in str(e.value)


def test_random_overrides_round_trip_through_dotlist_and_yaml(tmp_path):
    """Property test over the whole schema: random values for randomly chosen scalar fields (at any depth, every scalar
    type the schema has: int, float, bool, str, enums and their Optional forms), given as dotted command-line overrides,
    land in the right field with the right type, survive ``save`` + ``load``, and leave every other field at its default."""
    import dataclasses
    import typing
    from enum import Enum

    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    from olmo_b200.utils import structured as S

    def scalar_fields(cls, prefix=""):
        hints = S._hints(cls)
        for f in dataclasses.fields(cls):
            if not f.init:
                continue
            tp = hints[f.name]
            args = [a for a in typing.get_args(tp) if a is not type(None)] if typing.get_origin(tp) is typing.Union else [tp]
            optional = type(None) in typing.get_args(tp)
            if len(args) != 1:
                continue
            inner = args[0]
            if dataclasses.is_dataclass(inner):
                if not optional:  # optional sub-configs default to None; setting one field would create the rest
                    yield from scalar_fields(inner, f"{prefix}{f.name}.")
            elif inner in (int, float, bool, str) or (isinstance(inner, type) and issubclass(inner, Enum)):
                yield f"{prefix}{f.name}", inner, optional

    fields = list(scalar_fields(TrainConfig))
    assert len(fields) > 100 and {tp for _, tp, _ in fields} >= {int, float, bool, str}
    defaults = TrainConfig.new().asdict()

    def value_for(tp, optional):
        if isinstance(tp, type) and issubclass(tp, Enum):
            base = st.sampled_from(list(tp))
        else:
            base = {int: st.integers(0, 10**9), bool: st.booleans(),
                    float: st.one_of(st.floats(1e-9, 1e9, allow_nan=False), st.sampled_from([0.0, 1e-5, 3e-4, 0.95, 1.0])),
                    str: st.text(alphabet="abcdefgh_-/.XYZ", min_size=1, max_size=12).filter(lambda t: t.strip("-. ") == t and not t[0].isdigit())}[tp]
        return st.one_of(st.none(), base) if optional else base

    picks = st.lists(st.sampled_from(fields), min_size=1, max_size=6, unique_by=lambda f: f[0]).flatmap(
        lambda chosen: st.tuples(*[st.tuples(st.just(name), st.just(tp), value_for(tp, opt)) for name, tp, opt in chosen]))

    def lookup(tree, dotted):
        for part in dotted.split("."):
            tree = tree[part]
        return tree

    def plain(v):
        return v.value if isinstance(v, Enum) else v

    @settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.too_slow, HealthCheck.function_scoped_fixture])
    @given(picks)
    def check(chosen):
        overrides = []
        for name, tp, value in chosen:
            text = "null" if value is None else repr(value) if tp is float else str(plain(value)).lower() if tp is bool else str(plain(value))
            overrides.append(f"{name}={text}")
        cfg = TrainConfig.new(**S.parse_dotlist(overrides))
        path = tmp_path / "cfg.yaml"
        cfg.save(path)
        again = TrainConfig.load(path, validate_paths=False)
        for tree in (cfg.asdict(), again.asdict()):
            for name, tp, value in chosen:
                got = plain(lookup(tree, name))
                assert got == plain(value) and (value is None or type(got) is type(plain(value))), (name, got, value)
        touched = {name for name, _, _ in chosen}
        for name, _, _ in fields:
            if name not in touched:
                assert plain(lookup(again.asdict(), name)) == plain(lookup(defaults, name)), name

    check()


def test_every_runtime_environment_variable_is_documented():
    """The docstring of ``B200Runtime`` is the list of this framework's environment variables: every ``OLMO_B200_*`` name
    read anywhere in the package (Python or device code) appears there, and it names none that nothing reads."""
    import re
    from pathlib import Path

    from olmo_b200.config import B200Runtime

    pkg = Path(__file__).resolve().parent.parent / "olmo_b200"
    read = set()
    for path in list(pkg.rglob("*.py")) + list((pkg / "csrc").rglob("*.cu")) + list((pkg / "csrc").rglob("*.cuh")):
        text = path.read_text()
        if path.name == "config.py":
            text = text.replace(B200Runtime.__doc__ or "", "")
        read |= set(re.findall(r"OLMO_B200_[A-Z0-9_]+", text))
    documented = set(re.findall(r"OLMO_B200_[A-Z0-9_]+", B200Runtime.__doc__ or ""))
    read.discard("OLMO_B200_RESHARD")  # older spelling of OLMO_B200_SCHEDULE=sharded, honoured but not advertised
    assert read - documented == set(), f"undocumented: {sorted(read - documented)}"
    assert documented - read == set(), f"documented but never read: {sorted(documented - read)}"
