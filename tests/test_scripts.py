"""User-facing scripts: data preparation, dataloader replay / inspection, ladder laws, storage housekeeping, comparisons."""
import gzip
import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
SCRIPTS = ROOT / "scripts"


def load_script(name: str):
    spec = importlib.util.spec_from_file_location(f"script_{name}", SCRIPTS / f"{name}.py")
    module = importlib.util.module_from_spec(spec)
    sys.path.insert(0, str(SCRIPTS))
    try:
        spec.loader.exec_module(module)
    finally:
        sys.path.remove(str(SCRIPTS))
    return module


@pytest.fixture(scope="module")
def tokenizer_json(tmp_path_factory):
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    words = [f"w{i}" for i in range(40)] + ["<|user|>", "<|assistant|>", "hello", "there", "ok"]
    vocab = {w: i for i, w in enumerate(words)}
    vocab["<unk>"] = len(vocab)
    vocab["<pad>"] = len(vocab)
    vocab["<eos>"] = len(vocab)
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.add_special_tokens(["<eos>", "<pad>"])
    path = tmp_path_factory.mktemp("tok") / "tokenizer.json"
    tok.save(str(path))
    return path, vocab


def test_prepare_memmap_dataset_round_trip(tmp_path, tokenizer_json):
    path, vocab = tokenizer_json
    docs = [" ".join(f"w{(i + j) % 40}" for j in range(5 + i % 7)) for i in range(30)]
    src = tmp_path / "docs"
    src.mkdir()
    with gzip.open(src / "a.json.gz", "wt") as f:
        f.write("\n".join(json.dumps({"text": d}) for d in docs[:20]))
    (src / "b.jsonl").write_text("\n".join(json.dumps({"text": d}) for d in docs[20:]))
    mod = load_script("prepare_memmap_dataset")
    total = mod.main([str(src), "-o", str(tmp_path / "out"), "--tokenizer", str(path), "--max-tokens", "64", "--validate", "--paths-per-worker", "2"])
    files = sorted((tmp_path / "out").glob("*.npy"))
    assert len(files) >= 2  # the 64-token cap forces several parts
    tokens = np.concatenate([np.memmap(f, dtype=np.uint16, mode="r") for f in files])
    assert len(tokens) == total == sum(len(d.split()) + 1 for d in docs)
    assert int((tokens == vocab["<eos>"]).sum()) == 30
    assert all(np.memmap(f, dtype=np.uint16, mode="r").shape[0] <= 64 for f in files)
    # and the training dataset reads them
    from olmo_b200.data import MemMapDataset

    ds = MemMapDataset(*files, chunk_size=8)
    assert len(ds) == sum(np.memmap(f, dtype=np.uint16, mode="r").shape[0] // 8 for f in files)


def test_prepare_tulu_data_masks_only_assistant_turns(tmp_path, tokenizer_json):
    path, vocab = tokenizer_json
    convs = [
        {"messages": [{"role": "user", "content": "hello there"}, {"role": "assistant", "content": "ok w1"}]},
        {"messages": [{"role": "user", "content": "hello"}]},  # no assistant turn: dropped
    ]
    src = tmp_path / "c.jsonl"
    src.write_text("\n".join(json.dumps(c) for c in convs))
    mod = load_script("prepare_tulu_data")
    kept = mod.main([str(tmp_path / "out"), "--source", str(src), "-t", str(path), "-s", "16", "--eos", str(vocab["<eos>"]), "--pad", str(vocab["<pad>"])])
    assert kept == 1
    ids = np.memmap(tmp_path / "out" / "input_ids.npy", dtype=np.uint16, mode="r")
    mask = np.memmap(tmp_path / "out" / "label_mask.npy", dtype=np.bool_, mode="r")
    assert len(ids) == len(mask) == 16 and ids[0] == vocab["<eos>"]
    trained = [int(t) for t, m in zip(ids, mask) if m]
    assert trained == [vocab["ok"], vocab["w1"], vocab["<eos>"]]
    assert ids[-1] == vocab["<pad>"] and not mask[-1]


@pytest.fixture()
def tiny_run(tmp_path):
    from olmo_b200.config import DataConfig, ModelConfig, TrainConfig

    files = []
    for i in range(2):
        f = tmp_path / f"part{i}.npy"
        arr = np.memmap(f, dtype=np.uint16, mode="w+", shape=(512,))
        arr[:] = np.arange(i * 512, (i + 1) * 512) % 1000
        arr.flush()
        files.append(str(f))
    cfg = TrainConfig(
        run_name="tiny", model=ModelConfig(max_sequence_length=16, vocab_size=1000, embedding_size=1024, pad_token_id=0, eos_token_id=1),
        data=DataConfig(paths=files, num_workers=0, drop_last=True, pin_memory=False, prefetch_factor=None, persistent_workers=False),
        global_train_batch_size=4, device_train_microbatch_size=2, seed=11, save_folder=str(tmp_path / "run"),
    )
    (tmp_path / "run").mkdir()
    cfg.save(tmp_path / "run" / "config.yaml")
    return tmp_path / "run", cfg


def test_run_dataloader_and_inspect_agree(tiny_run, capsys):
    run, cfg = tiny_run
    replay = load_script("run_dataloader")
    from olmo_b200.config import TrainConfig

    out = run / "batches"
    out.mkdir()
    n = replay.main(TrainConfig.load(run / "config.yaml"), out, world_size=2, rank=1, max_batches=5, batches_per_file=3)
    assert n == 5
    files = sorted(out.glob("input_ids-*.npy"))
    assert [f.name for f in files] == ["input_ids-0000000-0000003.npy", "input_ids-0000003-0000005.npy"]
    first = np.load(files[0])
    assert first.shape == (3, 2, 16) and first.dtype == np.uint16  # 3 batches, 2 sequences per rank

    inspect = load_script("inspect_train_data")
    inspect.main([str(run), "1", "1", "3", "--world_size", "2", "--no_data_indices", "--ids"])
    printed = capsys.readouterr().out
    # the replayed batches of rank 1 at steps 1 and 3 are exactly what the inspector derives
    for step, batch in ((1, first[0]), (3, first[2])):
        for ex, row in enumerate(batch):
            assert f"[step={step}, rank=1, example={ex}," in printed
            assert str(row.tolist()) in printed

    # with recorded indices the same examples come back
    (run / "data-indices").mkdir()
    index_of = {}
    from olmo_b200.data import build_memmap_dataset

    ds = build_memmap_dataset(cfg, cfg.data)
    for i in range(len(ds)):
        index_of[tuple(ds[i]["input_ids"].tolist())] = i
    with gzip.open(run / "data-indices" / "rank1.tsv.gz", "wt") as f:
        f.write("1\t" + "\t".join(str(index_of[tuple(int(t) for t in row)]) for row in first[0]) + "\n")
    inspect.main([str(run), "1", "1", "--ids"])
    printed = capsys.readouterr().out
    for row in first[0]:
        assert str(row.tolist()) in printed

    # anchored at a checkpoint's trainer state: step 3 follows the two batches the checkpoint of step 2 had consumed
    (run / "step2" / "train").mkdir(parents=True)
    torch.save({"global_step": 2, "epoch": 0, "global_train_examples_seen_this_epoch": 8}, run / "step2" / "train" / "rank0.pt")
    inspect.main([str(run), "1", "3", "--world_size", "2", "--no_data_indices", "--ids", "--checkpoint_num", "2"])
    printed = capsys.readouterr().out
    for row in first[2]:
        assert str(row.tolist()) in printed
    with pytest.raises(SystemExit):
        inspect.main([str(run), "1", "2", "--world_size", "2", "--no_data_indices", "--ids", "--checkpoint_num", "2"])
    assert inspect.remount(["/weka/data/a.npy", "/other/b.npy"], [["weka://", "/weka/"]]) == ["weka://data/a.npy", "/other/b.npy"]


def test_ladder_power_laws_and_node_counts():
    from olmo_b200.ladder import batch_size_for, ladder_config, learning_rate_for, node_counts, parse_length, parse_size, size_for_model

    assert parse_size("150M") == 150_000_000 and parse_size("7b") == 7_000_000_000
    assert parse_length("2xC", 10**9) == 40 * 10**9 and parse_length("5B", 1) == 5 * 10**9 and parse_length("3T", 1) == 3 * 10**12
    with pytest.raises(ValueError):
        parse_length("5Q", 1)
    assert batch_size_for(150_000_000) == 192 and batch_size_for(10**9) == 704
    assert learning_rate_for(108_000_000) == pytest.approx(0.0047)
    assert learning_rate_for(864_000_000) == pytest.approx(0.0047 / 2)
    cfg = ladder_config("1B", "1xC", "t")
    assert cfg.global_train_batch_size == 704 and cfg.max_duration == f"{20 * 10**9}T"
    assert cfg.scheduler.t_warmup == round(10**9 / (704 * 2048)) and str(cfg.distributed_strategy) == "ddp"
    assert cfg.global_train_batch_size % cfg.device_train_microbatch_size == 0
    assert str(ladder_config("7B", "1xC", "t").distributed_strategy) == "fsdp"
    assert node_counts(cfg, 8) == [11, 1]
    total, non_emb = size_for_model("150M")
    assert 150e6 < non_emb < total < 200e6
    out = subprocess.run([sys.executable, str(SCRIPTS / "ladder.py"), "size", "--model", "300M"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and len(out.stdout.split()) == 2


def test_named_data_mixes(tmp_path, monkeypatch):
    from olmo_b200.data.named_data_mixes import DATA_PATHS, register_mix, resolve_mix

    (tmp_path / "data_mixes").mkdir()
    (tmp_path / "data_mixes" / "toy.txt").write_text("# comment\npart/a.npy\n\npart/b.npy  # trailing\n")
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))
    assert DATA_PATHS["toy"] == ["part/a.npy", "part/b.npy"] and "toy" in list(DATA_PATHS)
    assert resolve_mix("toy", "s3://bucket/root/") == ["s3://bucket/root/part/a.npy", "s3://bucket/root/part/b.npy"]
    register_mix("mem", ["x.npy"])
    assert DATA_PATHS["mem"] == ["x.npy"]
    with pytest.raises(KeyError):
        DATA_PATHS["nope"]


def test_storage_cleaner_and_compare(tmp_path, capsys):
    cleaner = load_script("storage_cleaner")
    root = tmp_path / "runs"
    for run, steps in (("good", [100, 200, 300]), ("dead", [0]), ("empty", [])):
        (root / run).mkdir(parents=True)
        (root / run / "config.yaml").write_text("run_name: x\n")
        for s in steps:
            (root / run / f"step{s}").mkdir()
            (root / run / f"step{s}" / "model.pt").write_bytes(b"x" * 10)
    assert sorted(Path(r).name for r in cleaner.clean(str(root), 0, dry_run=True)) == ["dead", "empty"]
    assert (root / "dead").exists()
    cleaner.main(["clean", str(root)])
    assert sorted(p.name for p in root.iterdir()) == ["good"]
    n = cleaner.main(["move", str(root / "good"), str(tmp_path / "moved"), "--keep-latest", "2"])
    assert n == 3 and sorted(p.name for p in (tmp_path / "moved").iterdir()) == ["config.yaml", "step200", "step300"]

    # archives are runs too; one entry can be moved on its own; a move can remove its source
    import shutil

    arch_root = tmp_path / "archived"
    arch_root.mkdir()
    shutil.make_archive(str(arch_root / "good"), "gztar", root_dir=root, base_dir="good")
    (root / "stale").mkdir()
    (root / "stale" / "config.yaml").write_text("run_name: y\nwandb:\n  entity: ai2\n  project: olmo\n  name: stale-run\n")
    shutil.make_archive(str(arch_root / "stale"), "zip", root_dir=root / "stale")
    (arch_root / "notes").mkdir()
    (arch_root / "notes" / "readme.txt").write_text("not a run")
    assert cleaner.archive_entries(str(arch_root / "good.tar.gz"), None) == ["config.yaml", "step100", "step200", "step300"]
    assert sorted(Path(r).name for r in cleaner.clean(str(arch_root), 0, dry_run=True)) == ["stale.zip"]
    assert cleaner.clean(str(arch_root), 0, dry_run=True, max_archive_size=1) == []
    with pytest.raises(SystemExit):
        cleaner.clean(str(arch_root), 0, dry_run=True, ignore_non_runs=False)
    cleaner.main(["clean", str(arch_root)])
    assert sorted(p.name for p in arch_root.iterdir()) == ["good.tar.gz", "notes"]
    n = cleaner.main(["--temp-dir", str(tmp_path), "move", str(arch_root / "good.tar.gz"), str(tmp_path / "one"), "--entry", "step300"])
    assert n == 1 and (tmp_path / "one" / "step300" / "model.pt").exists() and (arch_root / "good.tar.gz").exists()
    n = cleaner.main(["move", str(root / "stale"), str(tmp_path / "by_wandb"), "--append-wandb-path", "--remove-src"])
    assert (tmp_path / "by_wandb" / "ai2" / "olmo" / "stale-run" / "config.yaml").exists() and not (root / "stale").exists()
    cleaner.main(["move", str(arch_root / "good.tar.gz"), str(tmp_path / "kept_archive")])
    assert (tmp_path / "kept_archive" / "good.tar.gz").exists()
    cleaner.main(["--temp-dir", str(tmp_path), "move", str(arch_root / "good.tar.gz"), str(tmp_path / "unpacked"), "--store-unarchived", "--remove-src"])
    assert (tmp_path / "unpacked" / "step200" / "model.pt").exists() and not (arch_root / "good.tar.gz").exists()

    cmp_state = load_script("compare_model_state")
    a = {"w": torch.ones(3), "only_a": torch.zeros(1), "nest": {"v": torch.ones(2)}}
    b = {"w": torch.ones(3) * 1.5, "nest": {"v": torch.ones(2)}}
    bad = cmp_state.compare(cmp_state.flatten("", a, {}), cmp_state.flatten("", b, {}), top=5, rtol=0.0)
    assert bad == 2
    assert "only in base:    only_a" in capsys.readouterr().out

    traces_a, traces_b = tmp_path / "ta", tmp_path / "tb"
    for folder, scale in ((traces_a, 1.0), (traces_b, 1.0)):
        folder.mkdir()
        for i in range(3):
            torch.save(torch.full((4,), float(i)) * scale, folder / f"model.transformer.blocks.{i}_0_output.pt")
    torch.save(torch.full((4,), 9.0), traces_b / "model.transformer.blocks.1_0_output.pt")
    proc = subprocess.run([sys.executable, str(SCRIPTS / "compare_module_outputs.py"), str(traces_a), str(traces_b)], capture_output=True, text=True, timeout=300)
    assert proc.returncode == 1 and "first divergence: model.transformer.blocks.1_0_output.pt" in proc.stdout


def test_wandb_helpers_parse_and_diff():
    mod = load_script("compare_wandb_configs")
    assert mod.parse_run_path("https://wandb.ai/ai2/olmo/runs/abc123?x=1") == "ai2/olmo/abc123"
    assert mod.parse_run_path("ai2/olmo/abc123") == "ai2/olmo/abc123"
    rows = list(mod.diff({"a": 1, "m": {"x": [1, 2]}, "save_folder": "p"}, {"a": 2, "m": {"x": [1, 3]}, "save_folder": "q"}))
    assert rows == [("a", 1, 2), ("m.x.1", 2, 3)]


def test_anneal_config_maker_and_olmo_alias(tmp_path):
    mod = load_script("anneal_config_maker")
    out = tmp_path / "anneal.yaml"
    mod.main(["--base", "OLMo2-7B-stage1", "--load-path", "/ckpt/step928646", "--start-lr", "6.1499e-05", "--tokens", "50e9", "--name", "anneal",
              "--seed", "42", "--data-glob", str(tmp_path / "*.npy"), "-o", str(out)])
    from olmo_b200.config import SchedulerType, TrainConfig

    cfg = TrainConfig.load(out, validate_paths=False)
    assert cfg.stop_at == 11931 and cfg.max_duration == "50000000000T" and cfg.seed == 42
    assert cfg.scheduler.name == SchedulerType.linear_with_warmup and cfg.scheduler.alpha_f == 0.0 and cfg.scheduler.t_warmup == 0
    assert cfg.optimizer.learning_rate == pytest.approx(6.1499e-05) and cfg.load_path == "/ckpt/step928646"
    assert cfg.restore_dataloader is False and cfg.no_pre_train_checkpoint is True and cfg.model.d_model == 4096

    # code written against the reference's package name resolves to this framework
    import olmo.optim
    from olmo.config import TrainConfig as AliasedConfig
    from olmo.model import OLMo as AliasedOLMo

    import olmo_b200.models.olmo
    import olmo_b200.optim

    assert AliasedConfig is TrainConfig and AliasedOLMo is olmo_b200.models.olmo.OLMo and olmo.optim is olmo_b200.optim


def test_release_helper_stamps_and_extracts_notes(tmp_path):
    mod = load_script("release")
    changelog = tmp_path / "CHANGELOG.md"
    changelog.write_text(
        "# Changelog\n\n## Unreleased\n\n### Added\n\n- new thing\n\n### Fixed\n\n- a bug\n\n## [v0.1.0] - 2024-01-01\n\n### Changed\n\n- old change\n")
    assert mod.stamp(changelog, "0.2.0", today="2024-02-02") is True
    assert mod.stamp(changelog, "0.2.0") is False  # idempotent
    text = changelog.read_text()
    assert text.index("## Unreleased") < text.index("## [v0.2.0] - 2024-02-02") < text.index("### Added") < text.index("## [v0.1.0]")
    notes = mod.notes(changelog, "v0.2.0")
    assert notes.startswith("## What's new") and "### Added 🎉" in notes and "### Fixed ✅" in notes and "- a bug" in notes
    assert "old change" not in notes
    assert "### Changed ⚠️" in mod.notes(changelog, "v0.1.0")
    with pytest.raises(RuntimeError):
        mod.notes(changelog, "v9.9.9")
    # the repository's own changelog parses and can be stamped with the package version
    copy = tmp_path / "repo-changelog.md"
    copy.write_text((ROOT / "CHANGELOG.md").read_text())
    assert mod.stamp(copy, mod.package_version()) is True
    assert "- " in mod.notes(copy, f"v{mod.package_version()}")


def test_add_code_eval_writes_ppl_documents(tmp_path, monkeypatch):
    datasets = pytest.importorskip("datasets")
    rows = [{"task_id": f"T/{i}", "prompt": f"def f{i}():\n", "canonical_solution": f"    return {i}\n", "entry_point": f"f{i}"} for i in range(3)]
    datasets.Dataset.from_list(rows).save_to_disk(str(tmp_path / "hf_datasets" / "openai_humaneval" / "none" / "test"))
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))
    mod = load_script("add_code_eval")
    assert mod.main([str(tmp_path / "out"), "--dataset", "openai_humaneval", "--split", "test"]) == 0
    with gzip.open(tmp_path / "out" / "openai_humaneval_test.jsonl.gz", "rt") as f:
        docs = [json.loads(line) for line in f]
    assert [d["id"] for d in docs] == ["T/0", "T/1", "T/2"]
    assert docs[1]["text"] == "def f1():\n    return 1\n" and docs[1]["metadata"] == {"entry_point": "f1"}
    # the files feed the offline pipeline's perplexity task
    from olmo_b200.eval.offline import construct_task

    class Tok:
        eos_token_id = 0

        def encode(self, s, add_special_tokens=False):
            return [1 + (ord(c) % 50) for c in s]

    task = construct_task("ppl", Tok(), {"files": [str(tmp_path / "out" / "openai_humaneval_test.jsonl.gz")]})
    assert [text for _, text in task.documents(Tok())] == [d["text"] for d in docs]


def test_flops_figure_renders_an_svg(tmp_path):
    mod = load_script("flops_by_perf_figure")
    flops = mod.training_flops("OLMo2-1B-stage1", 4e12)
    assert 2.5e22 < flops < 6e22  # about 6·N·D for 1.5 B parameters and 4 T tokens, attention on top
    points = tmp_path / "points.csv"
    points.write_text("model,flops,score,group\nA-1B,OLMo2-1B-stage1:4e12,43.5,ours\nB-7B,1.8e23,61.0,ours\nC,9e22,55.2,others\n")
    assert mod.main([str(points), str(tmp_path / "fig.svg"), "--title", "FLOPs vs score"]) == 0
    svg = (tmp_path / "fig.svg").read_text()
    assert svg.startswith("<svg") and svg.count("<circle") == 3 + 2 and "A-1B" in svg and "others" in svg and "10^23" in svg
    import xml.dom.minidom

    xml.dom.minidom.parseString(svg)  # well-formed


def test_ci_data_pipeline_smoke_command(tmp_path):
    """The command the CI workflow runs on the committed fixtures."""
    proc = subprocess.run(
        [sys.executable, str(SCRIPTS / "prepare_memmap_dataset.py"), str(ROOT / "test_fixtures" / "sample-docs.json.gz"), "-o", str(tmp_path / "tokens"),
         "--tokenizer", str(ROOT / "test_fixtures" / "word-tokenizer.json"), "--validate", "--ack-deprecated"],
        capture_output=True, text=True, timeout=300,
    )
    assert proc.returncode == 0, proc.stderr[-2000:]
    files = list((tmp_path / "tokens").rglob("*.npy"))
    assert files and sum(np.memmap(f, dtype=np.uint16, mode="r").shape[0] for f in files) == 2765 + 48  # words + one end token per document


def test_launch_scripts_parse_and_pick_the_node_layout(tmp_path):
    launch = SCRIPTS / "launch"
    for script in sorted(launch.glob("*.sh")) + [SCRIPTS / "test_entrypoint.sh"]:
        assert subprocess.run(["bash", "-n", str(script)], capture_output=True).returncode == 0, script
    # the scheduler entry script maps the scheduler's variables and hands over to the single- or multi-node script
    fake = tmp_path / "launch"
    fake.mkdir()
    (fake / "beaker.sh").write_text((launch / "beaker.sh").read_text())
    for name in ("single_node.sh", "multi_node.sh"):
        (fake / name).write_text(f'#!/usr/bin/env bash\necho "{name} $NNODES $NODE_RANK $MASTER_ADDR $@"\n')
    for f in fake.iterdir():
        f.chmod(0o755)
    env = {"PATH": os.environ["PATH"], "HOME": str(tmp_path), "AWS_CONFIG": "[default]"}
    one = subprocess.run(["bash", str(fake / "beaker.sh"), "c.yaml", "--x=1"], capture_output=True, text=True, env=env)
    assert one.stdout.strip() == "single_node.sh 1 0 127.0.0.1 c.yaml --x=1" and (tmp_path / ".aws" / "config").read_text().strip() == "[default]"
    env.update(BEAKER_REPLICA_COUNT="4", BEAKER_REPLICA_RANK="2", BEAKER_LEADER_REPLICA_HOSTNAME="node0")
    many = subprocess.run(["bash", str(fake / "beaker.sh"), "c.yaml"], capture_output=True, text=True, env=env)
    assert many.stdout.strip() == "multi_node.sh 4 2 node0 c.yaml"


def test_model_size_breakdown_and_config_starter(tmp_path):
    from olmo_b200.config import ModelConfig, TrainConfig
    from olmo_b200.models.olmo import OLMo

    sizes_mod = load_script("show_model_size")
    cfg = TrainConfig(model=ModelConfig(d_model=64, n_heads=4, n_layers=3, mlp_ratio=4, vocab_size=200, embedding_size=256, weight_tying=False,
                                        max_sequence_length=32, include_bias=False, init_device="cpu"))
    sizes = sizes_mod.count(cfg)
    real = OLMo(cfg.model, init_params=False)
    assert cfg.model.n_layers == 3 and sizes["total"] == real.num_params() and sizes["non_embedding"] == real.num_params(include_embedding=False)
    assert sizes["embedding"] + sizes["head"] + sizes["other"] + sizes["blocks"] * sizes["block"] == sizes["total"] and sizes["head"] == 256 * 64
    plans = [sizes_mod.memory_plan(sizes, n) for n in (1, 2, 4, 8)]
    assert plans[0]["resident"] == pytest.approx(18 * sizes["total"] / 1e9)
    assert all(a["resident"] > b["resident"] and b["sharded"] < b["resident"] for a, b in zip(plans, plans[1:]))

    starter = load_script("init_config")
    plain = starter.main(tmp_path / "plain.yaml", ["model.d_model=96"])
    assert plain.model.d_model == 96 and TrainConfig.load(tmp_path / "plain.yaml", validate_paths=False).model.d_model == 96
    recipe = starter.main(tmp_path / "r.yaml", ["seed=11"], recipe="OLMo2-1B-stage1")
    assert recipe.seed == 11 and recipe.model.d_model == 2048 and (tmp_path / "r.yaml").is_file()
    from olmo_b200.exceptions import OLMoCliError

    with pytest.raises(OLMoCliError):
        starter.main(tmp_path / "x.yaml", [], recipe="no-such-recipe")


def test_split_gz_by_size_and_by_lines(tmp_path):
    split = load_script("split_gz")
    src = tmp_path / "in"
    src.mkdir()
    for name, n in (("a.json.gz", 10), ("b.json.gz", 3)):
        with gzip.open(src / name, "wt") as f:
            for i in range(n):
                f.write(json.dumps({"i": i, "pad": "x" * 20}) + "\n")
    (src / "notes.txt").write_text("skip me")
    line = len(json.dumps({"i": 0, "pad": "x" * 20}) + "\n")
    written = split.split_directory(str(src), str(tmp_path / "out"), ".json.gz", ".jsonl.gz", size_limit=4 * line, workers=1)
    assert [Path(p).name for p in written] == ["a_0000.jsonl.gz", "a_0001.jsonl.gz", "a_0002.jsonl.gz", "b_0000.jsonl.gz"]
    back = []
    for p in written[:3]:
        with gzip.open(p, "rt") as f:
            back += [json.loads(x)["i"] for x in f]
    assert back == list(range(10))
    assert split.main(["--input_dir", str(src), "--output_dir", str(tmp_path / "out2"), "--input_ext", ".json.gz", "--lines", "5"]) == 3
    assert split.main([str(src / "a.json.gz"), str(tmp_path / "single"), "--lines", "4"]) == 3 and (tmp_path / "single_0002.json.gz").is_file()


def _token_dir(root, name, sizes):
    d = root / name
    d.mkdir(parents=True)
    for i, n in enumerate(sizes):
        np.zeros(n, dtype=np.uint32).tofile(d / f"part-{i:02d}.npy")
    (d / "notes.txt").write_text("ignored")
    return str(d)


def test_mix_builder_and_config_makers(tmp_path, capsys):
    from olmo_b200.config import TrainConfig
    from olmo_b200.data import mix_builder as mb

    web = _token_dir(tmp_path, "web", [1000] * 10)      # 10 k tokens
    math = _token_dir(tmp_path, "math", [500, 700, 300])  # 1.5 k tokens
    assert mb.parse_source("s3://b/x/=0.25") == mb.Source("s3://b/x/", fraction=0.25)
    assert mb.parse_source("s3://b/x/=2B").tokens == 2e9 and mb.parse_source("/d/x=x2").repeat == 2 and mb.parse_source("s3://b/k=v/").prefix == "s3://b/k=v/"
    with pytest.raises(ValueError):
        mb.Source("x", fraction=1.5)
    paths, rows = mb.build_mix([f"{web}=0.3", math, f"{math}=x2", f"{web}=2500"], seed=3)
    assert [r["files"] for r in rows] == [3, 3, 6, 3] and [r["tokens"] for r in rows] == [3000, 1500, 3000, 3000]
    assert rows[0]["available"] == 10000 and abs(sum(r["share"] for r in rows) - 1) < 1e-9
    again, _ = mb.build_mix([f"{web}=0.3", math, f"{math}=x2", f"{web}=2500"], seed=3)
    other, _ = mb.build_mix([f"{web}=0.3"], seed=4)
    assert again == paths and all(p.endswith(".npy") for p in paths) and other != paths[:3]
    with pytest.raises(ValueError, match="repeat"):
        mb.build_mix([f"{math}=5000"])
    with pytest.raises(FileNotFoundError):
        mb.build_mix([str(tmp_path / "nothing")])
    table = mb.examine(paths)
    assert {Path(r["source"]).name: r["tokens"] for r in table} == {"web": 6000, "math": 4500}
    assert mb.human_count(1.5e9) == "1.50B" and mb.human_count(12) == "12"

    micro = load_script("microanneal_config_maker")
    out = tmp_path / "micro.yaml"
    micro.main(["--name", "candidate", "-o", str(out), "--source", math, "--source", f"{web}=0.2"])
    cfg = TrainConfig.load(out, validate_paths=False)
    assert len(cfg.data.paths) == 5 and cfg.seed == 7201 and cfg.max_duration == "3500T" and cfg.optimizer.learning_rate == pytest.approx(6.1499e-05)
    assert cfg.scheduler.alpha_f == 0.0 and cfg.restore_dataloader is False and cfg.model.d_model == 4096
    capsys.readouterr()
    micro.main(["--examine", str(out)])
    printed = capsys.readouterr().out
    assert "math" in printed and "web" in printed and "total" in printed
    big = load_script("peteish7_config_maker")
    big.main(["--name", "anneal", "--tokens", "50e9", "-o", str(tmp_path / "anneal.yaml"), "--source", web])
    cfg = TrainConfig.load(tmp_path / "anneal.yaml", validate_paths=False)
    assert cfg.stop_at == 11931 and cfg.seed == 42 and len(cfg.data.paths) == 10


def test_memmap_preparation_reads_remote_sources_through_a_cache(tmp_path):
    """Documents listed under a remote prefix are copied into the cache folder once and tokenised from there."""
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    from olmo_b200 import util

    vocab = {f"w{i}": i for i in range(20)}
    vocab["<eos>"] = 20
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="w0"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.save(str(tmp_path / "tok.json"))

    class Store(util.StorageBackend):
        def __init__(self):
            self.blobs, self.reads = {}, 0

        def file_size(self, url):
            return len(self.blobs[url])

        def get_bytes_range(self, url, start, num):
            self.reads += 1
            return self.blobs[url][start : start + num]

        def list_files(self, url):
            return sorted(k for k in self.blobs if k.startswith(url.rstrip("/") + "/"))

    store = Store()
    import io

    buf = io.BytesIO()
    with gzip.GzipFile(fileobj=buf, mode="wb") as f:
        f.write(b'{"text": "w1 w2 w3"}\n{"text": "w4 w5"}\n')
    store.blobs["mem://bucket/docs/a.json.gz"] = buf.getvalue()
    store.blobs["mem://bucket/docs/readme.txt"] = b"not documents"
    util.register_storage_backend("mem", store)
    try:
        prep = load_script("prepare_memmap_dataset")
        assert prep.list_sources(["mem://bucket/docs"]) == ["mem://bucket/docs/a.json.gz"]
        args = ["mem://bucket/docs", "-o", str(tmp_path / "out"), "--tokenizer", str(tmp_path / "tok.json"), "--eos-token-id", "20",
                "--cache-dir", str(tmp_path / "cache"), "--max-tokens", "64"]
        assert prep.main(args) == 7  # five words and an end-of-text token after each of the two documents
        reads = store.reads
        assert prep.main([*args[:2], str(tmp_path / "out2"), *args[3:]]) == 7 and store.reads == reads  # served from the cache
        assert len(list((tmp_path / "cache").rglob("*a.json.gz"))) == 1
    finally:
        util._BACKENDS.pop("mem", None)


def test_ladder_power_law_fit_recovers_a_known_law():
    pytest.importorskip("scipy")
    from olmo_b200.ladder import fit_power_law, ladder_fit, parse_run_name, power_law, size_for_model

    assert parse_run_name("baseline2-300M-5xC") == ("baseline2", "300M", "5xC")
    with pytest.raises(ValueError):
        parse_run_name("not a run")
    xs = [1.5e8, 3e8, 7.5e8, 1e9, 7e9]
    ys = [power_law(x, 420.0, -0.3, 1.8) for x in xs]
    a, b, c = fit_power_law(xs, ys)
    assert abs(b + 0.3) < 1e-3 and abs(c - 1.8) < 1e-3 and abs(a / 420.0 - 1) < 2e-2
    sizes = {s: size_for_model(s)[1] for s in ("150M", "300M", "750M", "1B")}
    results = {f"base-{s}-2xC": power_law(n, 50.0, -0.2, 2.0) for s, n in sizes.items()}
    fit = ladder_fit(results, by="size", hold_out=1)
    held = [p for p in fit["points"] if p["held_out"]]
    assert len(held) == 1 and held[0]["run"] == "base-1B-2xC" and abs(held[0]["predicted"] - held[0]["loss"]) < 1e-2


@pytest.mark.parametrize("run, env", [
    ("peteish1", {"STORAGE": "google"}),
    ("peteish7", {"STORAGE": "s3"}),
    ("peteish7-medlr", {}),
    ("peteish13", {"NNODES": "4", "REMOTE_ROOT": "gs://bucket/checkpoints"}),
    ("peteish13-medlr", {}),
    ("peteish13-highlr", {}),
    ("peteish7-lr-anneal", {"START_STEP": "477000", "START_LR": "2.1e-4", "LOAD_PATH": "/ckpt/step477000", "ANNEAL_TOKENS": "50e9"}),
    ("anneal", {"CONFIG": "configs/annealing/OLMo2-7B-anneal-example.yaml", "SEED": "42"}),
    ("tiny", {"SIZE": "60M"}),
])
def test_published_run_launcher_builds_a_valid_command(run, env, tmp_path):
    """The launcher's dry run prints the command of a published run; its config exists and every override it passes is
    a key of the configuration schema (the settings come from ``scripts/beaker/peteish/*.sh`` and ``scripts/augusta/*.sh``)."""
    from olmo_b200.config import TrainConfig
    from olmo_b200.util import clean_opt

    full_env = {**os.environ, "DRY_RUN": "1", "CHECKPOINT_ROOT": str(tmp_path), **env}
    full_env.pop("BEAKER_REPLICA_COUNT", None)
    out = subprocess.run(["bash", str(SCRIPTS / "launch" / "published_runs.sh"), run, "--global_train_batch_size=64"], env=full_env, cwd=ROOT,
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    words = out.stdout.split("\n")[:-1]
    assert words[0].endswith("launch/beaker.sh") and Path(words[0]).is_file()
    config, overrides = words[1], words[2:]
    assert Path(config).is_file() and overrides[-1] == "--global_train_batch_size=64"
    cfg = TrainConfig.load(config, [clean_opt(o) for o in overrides], validate_paths=False)
    assert cfg.run_name == run and cfg.save_folder == f"{tmp_path}/{run}" and cfg.try_load_latest_save and cfg.global_train_batch_size == 64
    if env.get("NNODES"):
        assert str(cfg.fsdp.sharding_strategy).endswith("HYBRID_SHARD") and cfg.fsdp.hybrid_sharding_num_model_replicas == 4
        assert cfg.remote_save_folder == f"gs://bucket/checkpoints/{run}/"
    if run == "peteish7-lr-anneal":
        assert cfg.max_duration == 477000 + round(50e9 / (1024 * 4096)) and cfg.stop_at == cfg.max_duration + 10
        assert cfg.scheduler.t_warmup == 477000 and cfg.scheduler.alpha_f == 0 and cfg.load_path == "/ckpt/step477000"
    if run == "anneal":
        assert cfg.seed == 42 and cfg.no_pre_train_checkpoint


def test_published_run_launcher_rejects_unknown_runs():
    out = subprocess.run(["bash", str(SCRIPTS / "launch" / "published_runs.sh"), "peteish99"], env={**os.environ, "DRY_RUN": "1"}, cwd=ROOT,
                         capture_output=True, text=True)
    assert out.returncode == 2 and "unknown run" in out.stderr


def test_every_script_answers_help(tmp_path):
    """``--help`` prints a usage text and exits 0 for every entry point under ``scripts/``, and does nothing else: no
    file appears in the working directory (one script used to write a config named ``--help``), the changelog is not
    stamped, no service is contacted."""
    from concurrent.futures import ThreadPoolExecutor

    changelog = (ROOT / "CHANGELOG.md").read_text()

    def ask(script):
        out = subprocess.run([sys.executable, str(script), "--help"], capture_output=True, text=True, cwd=tmp_path, timeout=600)
        if out.returncode != 0 or not out.stdout.strip():
            return script.name, out.returncode, out.stderr.strip().splitlines()[-1:] or out.stdout[-200:]
        return None

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        failures = [f for f in pool.map(ask, sorted(SCRIPTS.glob("*.py"))) if f is not None]
    assert not failures, failures
    assert list(tmp_path.iterdir()) == [] and (ROOT / "CHANGELOG.md").read_text() == changelog


def test_positional_args_helper(capsys):
    from olmo_b200.util import positional_args

    assert positional_args("doc", 2, ["a", "b", "--flag"]) == ["a", "b", "--flag"]
    with pytest.raises(SystemExit) as e:
        positional_args("the usage", 2, ["a"])
    assert e.value.code == 2 and "the usage" in capsys.readouterr().err
    with pytest.raises(SystemExit) as e:
        positional_args("the usage", 0, ["-h"])
    assert e.value.code == 0 and "the usage" in capsys.readouterr().out


def test_mix_builder_properties():
    """Property test of the data-mix builder on random sources: a fraction or token target is met by whole files and
    overshoots by less than one file, a repetition of ``k + f`` holds every file ``k`` or ``k + 1`` times, the same seed
    gives the same mix, asking for more than a source holds is refused, and the shares sum to one."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    from olmo_b200.data.mix_builder import Source, build_mix

    files = st.lists(st.integers(1, 500), min_size=1, max_size=12)

    @settings(max_examples=80, deadline=None)
    @given(sizes_a=files, sizes_b=files, fraction=st.floats(0.05, 1.0), repeat=st.floats(1.0, 3.5), seed=st.integers(0, 1000))
    def check(sizes_a, sizes_b, fraction, repeat, seed):
        a = Source("mem://a", fraction=fraction, files=[(f"mem://a/{i:03d}.npy", 4 * n) for i, n in enumerate(sizes_a)])
        b = Source("mem://b", repeat=repeat, files=[(f"mem://b/{i:03d}.npy", 4 * n) for i, n in enumerate(sizes_b)])
        paths, rows = build_mix([a, b], bytes_per_token=4, seed=seed)
        again, _ = build_mix([a, b], bytes_per_token=4, seed=seed)
        assert paths == again
        size_of = dict(a.files + b.files)
        got_a = [p for p in paths if p.startswith("mem://a/")]
        got_b = [p for p in paths if p.startswith("mem://b/")]
        assert len(set(got_a)) == len(got_a)  # a fraction never takes a file twice
        tokens_a, target_a = sum(size_of[p] // 4 for p in got_a), fraction * sum(sizes_a)
        assert tokens_a >= min(target_a, sum(sizes_a)) - 1e-6
        assert tokens_a - target_a < max(sizes_a) + 1e-6  # overshoot: less than one (the last) file
        whole = int(repeat)
        counts = {p: got_b.count(p) for p, _ in b.files}
        assert set(counts.values()) <= {whole, whole + 1}
        tokens_b = sum(size_of[p] // 4 for p in got_b)
        assert tokens_b >= repeat * sum(sizes_b) - 1e-6 or all(c == whole + 1 for c in counts.values())
        assert rows[0]["tokens"] == tokens_a and rows[1]["tokens"] == tokens_b
        assert sum(r["share"] for r in rows) == pytest.approx(1.0)

    check()
    with pytest.raises(ValueError, match="use repeat"):
        build_mix([Source("mem://a", tokens=1000, files=[("mem://a/0.npy", 400)])], bytes_per_token=4)
