"""End-to-end plumbing on CPU: a tiny decoder trains for a few AdamW steps and its checkpoints round-trip."""
import math
from pathlib import Path

import pytest
import torch
from torch.utils.data import DataLoader

from olmo_b200.config import (
    ActivationType, DistributedStrategy, LayerNormType, ModelConfig, OptimizerConfig, OptimizerType, SchedulerConfig,
    SchedulerType, TrainConfig,
)
from olmo_b200.data import DataCollator, IterableDataset, SyntheticTokenDataset
from olmo_b200.launch import build_trainer, derive_batch_sizes


def tiny_train_config(tmp_path, **model_overrides) -> TrainConfig:
    model = ModelConfig(
        d_model=64, n_heads=4, n_layers=2, mlp_hidden_size=256, activation_type=ActivationType.swiglu, rope=True,
        layer_norm_type=LayerNormType.default, layer_norm_with_affine=False, include_bias=False, vocab_size=250,
        embedding_size=256, max_sequence_length=32, eos_token_id=249, pad_token_id=249, weight_tying=False,
        attention_dropout=0.0, residual_dropout=0.0, embedding_dropout=0.0, init_device="cpu",
    )
    for k, v in model_overrides.items():
        setattr(model, k, v)
    cfg = TrainConfig(
        model=model,
        optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=4e-3, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8),
        scheduler=SchedulerConfig(name=SchedulerType.constant),
        save_folder=str(tmp_path), save_overwrite=True, global_train_batch_size=8, device_train_microbatch_size=4,
        precision="fp32", distributed_strategy=DistributedStrategy.single, max_grad_norm=1.0, max_duration=20,
        save_data_indices=False, console_log_interval=100, softmax_auxiliary_loss=True,
    )
    derive_batch_sizes(cfg, world_size=1)
    return cfg


def make_loader(cfg: TrainConfig, n=128) -> DataLoader:
    ds = SyntheticTokenDataset(n, cfg.model.max_sequence_length, 16, cfg.model.eos_token_id, seed=1, mean_doc_len=0)
    it = IterableDataset(ds, cfg.global_train_batch_size, seed=0, world_size=1, rank=0, fs_local_rank=0, num_threads=0)
    return DataLoader(it, batch_size=cfg.device_train_batch_size, collate_fn=DataCollator.from_train_config(cfg))


def test_loss_decreases_and_checkpoint_round_trip(tmp_path):
    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path)
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    losses = []
    batches = iter(trainer.train_loader)
    for _ in range(8):
        trainer.global_step += 1
        trainer.global_train_examples_seen_this_epoch += cfg.global_train_batch_size
        trainer.global_train_tokens_seen += cfg.global_train_batch_size * cfg.model.max_sequence_length
        losses.append(trainer.train_step(next(batches))["train/CrossEntropyLoss"])
    assert losses[-1] < losses[0] - 0.2, losses
    assert all(math.isfinite(x) for x in losses)

    path, _ = trainer.save_checkpoint()  # unsharded-world "sharded" format
    upath, _ = trainer.save_unsharded_checkpoint()
    before = {n: p.detach().clone() for n, p in trainer.dist_model.engine.named_parameters_for_optimizer()}
    m_before = {n: trainer.optim.state[p]["exp_avg"].clone() for n, p in trainer.dist_model.engine.named_parameters_for_optimizer()}
    next_loss = trainer.train_step(next(batches))["train/CrossEntropyLoss"]

    for load in (path, upath):
        cfg2 = tiny_train_config(tmp_path)
        t2 = build_trainer(cfg2, device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
        t2.restore_checkpoint(load)
        assert t2.global_step == 8
        for n, p in t2.dist_model.engine.named_parameters_for_optimizer():
            assert torch.equal(p.detach(), before[n]), n
            assert torch.allclose(t2.optim.state[p]["exp_avg"], m_before[n]), n
        it2 = iter(t2.train_loader)  # data position restored: the next batch is batch #9
        again = t2.train_step(next(it2))["train/CrossEntropyLoss"]
        assert abs(again - next_loss) < 1e-5


def test_trainer_eval_runs_a_downstream_task(tmp_path, monkeypatch):
    """``Trainer.eval`` drives a multiple-choice task end to end: request batches through the model, the ranked
    classification metric, and the metric key the reference logs under (``olmo/eval/evaluator.py:31-45``)."""
    datasets = pytest.importorskip("datasets")
    from olmo_b200.config import EvaluatorConfig, EvaluatorType
    from olmo_b200.eval import build_downstream_evaluator

    class CharTokenizer:
        pad_token_id = 0
        eos_token_id = 1

        def encode(self, s, add_special_tokens=True):
            return [ord(c) for c in s] + ([self.eos_token_id] if add_special_tokens else [])

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(i) for i in ids if i > 1)

    rows = [{"goal": f"goal {i}", "sol1": "ab" * (1 + i % 3), "sol2": "cd" * (1 + i % 2), "label": i % 2} for i in range(6)]
    datasets.Dataset.from_list(rows).save_to_disk(str(tmp_path / "hf_datasets" / "piqa" / "plain_text" / "validation"))
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "run")
    cfg.device_eval_batch_size = 4
    cfg.eval_subset_num_batches = -1
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    ev_cfg = EvaluatorConfig(label="piqa", type=EvaluatorType.downstream)
    evaluator = build_downstream_evaluator(cfg, ev_cfg, CharTokenizer(), torch.device("cpu"), is_unit_test=True)
    assert len(evaluator.eval_loader.dataset) == 12  # two continuations per document
    trainer.evaluators = [evaluator]
    results = trainer.eval()
    assert list(results) == ["eval/downstream/piqa_len_norm"]

    # the same number computed by hand: length-normalised continuation log-likelihood, argmax per document
    model = trainer.dist_model.module if hasattr(trainer.dist_model, "module") else trainer.model
    model.eval()
    ds = evaluator.eval_loader.dataset
    scores = {}
    with torch.no_grad():
        for i in range(len(ds)):
            item = ds[i]
            ids = torch.as_tensor(item["query"]).unsqueeze(0)
            logp = torch.log_softmax(model(ids).logits[0].float(), dim=-1)
            ctx_len, cont = int(item["ctx_len"]), torch.as_tensor(item["continuation"])
            lp = logp[ctx_len - 1 : ctx_len - 1 + len(cont)].gather(1, cont.unsqueeze(1)).sum()
            scores.setdefault(int(item["doc_id"]), {})[int(item["cont_id"])] = (float(lp) / int(item["cont_str_len"]), int(item["label_id"]))
    correct = [max(conts, key=lambda c: conts[c][0]) == next(iter(conts.values()))[1] for conts in scores.values()]
    assert results["eval/downstream/piqa_len_norm"] == pytest.approx(sum(correct) / len(correct))

    # a subset limit caps the number of batches
    evaluator.subset_num_batches = 1
    seen = []
    monkeypatch.setattr(evaluator, "compute_metrics", lambda: seen.append(len(evaluator.eval_metric.scores)) or {})
    trainer.eval()
    assert seen == [4]


def test_sharded_checkpoint_of_the_reference_layout_is_unsharded_offline(tmp_path):
    """A ``model_and_optim/`` folder in torch's distributed-checkpoint format plus ``train/rank0.pt`` (what the
    reference's ``torch_new`` sharded checkpointer writes, ``olmo/checkpoint.py:99-144,892-966``) becomes an unsharded
    checkpoint that a trainer restores, optimizer moments included."""
    import importlib.util

    import torch.distributed.checkpoint as dcp

    from olmo_b200.checkpoint import is_torch_dcp_checkpoint

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "a")
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    batches = iter(trainer.train_loader)
    for _ in range(3):
        trainer.global_step += 1
        trainer.global_train_examples_seen_this_epoch += cfg.global_train_batch_size
        trainer.global_train_tokens_seen += cfg.global_train_batch_size * cfg.model.max_sequence_length
        trainer.train_step(next(batches))
    named = list(trainer.dist_model.engine.named_parameters_for_optimizer())
    model_state = {n: p.detach().clone() for n, p in named}
    optim_state = {
        "state": {n: {k: v.detach().clone() for k, v in trainer.optim.state[p].items()} for n, p in named},
        "param_groups": [{**{k: v for k, v in g.items() if k not in ("params", "param_names")}, "params": list(g["param_names"])} for g in trainer.optim.param_groups],
    }
    src = tmp_path / "step3"
    (src / "train").mkdir(parents=True)
    # the writer flattens nested mappings into dotted keys, exactly as it does for sharded state dicts
    dcp.save({"model": model_state, "optim": optim_state}, storage_writer=dcp.FileSystemWriter(str(src / "model_and_optim")), no_dist=True)
    torch.save(trainer.trainer_state_dict(), src / "train" / "rank0.pt")
    cfg.save(src / "config.yaml")
    assert is_torch_dcp_checkpoint(src) and not is_torch_dcp_checkpoint(tmp_path)

    spec = importlib.util.spec_from_file_location("unshard_script", str(__import__("pathlib").Path(__file__).resolve().parent.parent / "scripts" / "unshard.py"))
    unshard = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(unshard)
    from olmo_b200.config import ShardedCheckpointerType

    out = tmp_path / "step3-unsharded"
    unshard.main(src, out, ShardedCheckpointerType.torch_new)
    loaded = torch.load(out / "model.pt", map_location="cpu")
    assert set(loaded) == set(model_state) and all(torch.equal(loaded[n], model_state[n]) for n in loaded)

    cfg2 = tiny_train_config(tmp_path / "b")
    t2 = build_trainer(cfg2, device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
    t2.restore_checkpoint(str(out))
    assert t2.global_step == 3
    for n, p in t2.dist_model.engine.named_parameters_for_optimizer():
        assert torch.equal(p.detach(), model_state[n]), n
        assert torch.allclose(t2.optim.state[p]["exp_avg_sq"], optim_state["state"][n]["exp_avg_sq"]), n
    expect = trainer.train_step(next(batches))["train/CrossEntropyLoss"]
    again = t2.train_step(next(iter(t2.train_loader)))["train/CrossEntropyLoss"]
    assert abs(again - expect) < 1e-5


def test_checkpoints_are_exported_to_the_reference_sharded_layout(tmp_path):
    """``scripts/export_sharded.py`` turns an unsharded checkpoint and a flat-shard checkpoint of this framework into the
    reference's ``torch_new`` layout; the result is detected as such, holds every tensor under the key the layout
    prescribes, and a trainer resumes from it with the same weights, moments, step and next loss."""
    import importlib.util
    from pathlib import Path

    from torch.distributed.checkpoint import FileSystemReader

    from olmo_b200.checkpoint_compat import detect_layout
    from olmo_b200.config import CheckpointType, ShardedCheckpointerType, TrainConfig

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "a")
    cfg.save_overwrite = True
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    batches = iter(trainer.train_loader)
    for _ in range(3):
        trainer.global_step += 1
        trainer.global_train_examples_seen_this_epoch += cfg.global_train_batch_size
        trainer.global_train_tokens_seen += cfg.global_train_batch_size * cfg.model.max_sequence_length
        trainer.train_step(next(batches))
    unsharded, _ = trainer.save_checkpoint(CheckpointType.unsharded)
    sharded, _ = trainer.save_checkpoint(CheckpointType.sharded)
    named = dict(trainer.dist_model.engine.named_parameters_for_optimizer())

    spec = importlib.util.spec_from_file_location("export_sharded", str(Path(__file__).resolve().parent.parent / "scripts" / "export_sharded.py"))
    export = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(export)
    for source, name in ((unsharded, "export-a"), (sharded, "export-b")):
        out = export.main(source, tmp_path / name, world_size=2)
        assert detect_layout(out) == "torch_new" and (out / "train" / "rank1.pt").is_file()
        assert TrainConfig.load(out / "config.yaml", validate_paths=False).sharded_checkpointer == ShardedCheckpointerType.torch_new
        keys = set(FileSystemReader(str(out / "model_and_optim")).read_metadata().state_dict_metadata)
        some = next(iter(named))
        assert {f"model.{some}", f"optim.state.{some}.exp_avg", f"optim.state.{some}.exp_avg_sq"} <= keys
        cfg2 = tiny_train_config(tmp_path / f"resume-{name}")
        t2 = build_trainer(cfg2, device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
        t2.restore_checkpoint(str(out))
        assert t2.global_step == 3
        for n, p in t2.dist_model.engine.named_parameters_for_optimizer():
            assert torch.equal(p.detach(), named[n].detach()), n
            assert torch.equal(t2.optim.state[p]["exp_avg"], trainer.optim.state[named[n]]["exp_avg"]), n
    expect = trainer.train_step(next(batches))["train/CrossEntropyLoss"]
    again = t2.train_step(next(iter(t2.train_loader)))["train/CrossEntropyLoss"]
    assert abs(again - expect) < 1e-5
    model_only = export.main(unsharded, tmp_path / "weights", model_only=True)
    assert not any(k.startswith("optim.") for k in FileSystemReader(str(model_only / "model_and_optim")).read_metadata().state_dict_metadata)


@pytest.mark.parametrize("kind", ["sharded", "unsharded"])
def test_failing_upload_leaves_no_checkpoint_behind_and_a_retry_succeeds(tmp_path, monkeypatch, kind):
    """The remote store rejects the second file of a checkpoint.  The save raises, the step's folder does not appear under
    its final name (only the ``-tmp`` one exists, which the next attempt clears), nothing is registered as the latest
    checkpoint, and once the store works again the same step is saved and restores."""
    import olmo_b200.checkpoint as ckpt_mod
    from olmo_b200.config import CheckpointType
    from olmo_b200.exceptions import OLMoNetworkError

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "run")
    cfg.remote_save_folder = "s3://bucket/run"
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    trainer.global_step = 1
    trainer.train_step(next(iter(trainer.train_loader)))
    uploaded, calls = [], {"n": 0}

    def flaky_upload(source, target, save_overwrite=False):
        calls["n"] += 1
        if calls["n"] == 2:
            raise OLMoNetworkError(f"simulated outage while writing {target}")
        uploaded.append(str(target))

    monkeypatch.setattr(ckpt_mod, "upload", flaky_upload)
    which = CheckpointType.sharded if kind == "sharded" else CheckpointType.unsharded
    with pytest.raises(OLMoNetworkError, match="simulated outage"):
        trainer.save_checkpoint(which)
    name = "step1" if kind == "sharded" else "step1-unsharded"
    folder = tmp_path / "run" / name
    assert not folder.exists() and (tmp_path / "run" / f"{name}-tmp").exists()
    assert not (tmp_path / "run" / ("latest" if kind == "sharded" else "latest-unsharded")).exists()
    assert (trainer.checkpoints if kind == "sharded" else trainer.unsharded_checkpoints) == []

    calls["n"] = 100  # the store is back
    remote, local = trainer.save_checkpoint(which)  # with a remote folder the remote location comes first
    assert Path(local) == folder and folder.is_dir() and not (tmp_path / "run" / f"{name}-tmp").exists()
    assert remote == f"s3://bucket/run/{name}" and any(t.endswith("config.yaml") for t in uploaded)
    cfg2 = tiny_train_config(tmp_path / "again")
    t2 = build_trainer(cfg2, device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
    t2.restore_checkpoint(str(folder))
    assert t2.global_step == 1


def test_reference_layout_can_be_written_during_training(tmp_path, monkeypatch):
    """With ``sharded_checkpointer: torch_new`` and the opt-in switch, the trainer's sharded checkpoints are written in the
    reference's ``torch_new`` layout, and resumed from, by the named checkpointer; without the switch the same setting
    writes the flat-shard format."""
    from olmo_b200.checkpoint import FlatShardCheckpointer, TorchNewStyleShardedCheckpointer, build_sharded_checkpointer
    from olmo_b200.checkpoint_compat import detect_layout
    from olmo_b200.config import CheckpointType, ShardedCheckpointerType

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "run")
    cfg.sharded_checkpointer = ShardedCheckpointerType.torch_new
    assert isinstance(build_sharded_checkpointer(cfg), FlatShardCheckpointer)
    monkeypatch.setenv("OLMO_B200_WRITE_REFERENCE_LAYOUT", "1")
    assert isinstance(build_sharded_checkpointer(cfg), TorchNewStyleShardedCheckpointer)
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    batches = iter(trainer.train_loader)
    for _ in range(2):
        trainer.global_step += 1
        trainer.train_step(next(batches))
    folder, _ = trainer.save_checkpoint(CheckpointType.sharded)
    assert detect_layout(folder) == "torch_new" and (Path(folder) / "train" / "rank0.pt").is_file() and (Path(folder) / "config.yaml").is_file()
    named = dict(trainer.dist_model.engine.named_parameters_for_optimizer())
    cfg2 = tiny_train_config(tmp_path / "again")
    cfg2.sharded_checkpointer = ShardedCheckpointerType.torch_new
    t2 = build_trainer(cfg2, device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
    t2.restore_checkpoint(str(folder))
    assert t2.global_step == 2
    for n, p in t2.dist_model.engine.named_parameters_for_optimizer():
        assert torch.equal(p.detach(), named[n].detach()), n
        assert torch.equal(t2.optim.state[p]["exp_avg_sq"], trainer.optim.state[named[n]]["exp_avg_sq"]), n
    monkeypatch.delenv("OLMO_B200_WRITE_REFERENCE_LAYOUT")
    t3 = build_trainer(tiny_train_config(tmp_path / "third"), device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
    t3.restore_checkpoint(str(folder))  # the flat-shard checkpointer detects the foreign layout
    assert t3.global_step == 2


def test_unshard_and_convert_pipeline_runs_stage_by_stage(tmp_path):
    """``scripts/s3_unshard_to_hf.py`` on local "buckets": fetch, unshard, convert, upload; a second call picks up from the
    unsharded stage; the converted weights load in ``transformers`` and reproduce the trainer's logits."""
    import importlib.util

    import transformers

    from olmo_b200.config import CheckpointType

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "run")
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    trainer.global_step = 1
    trainer.train_step(next(iter(trainer.train_loader)))
    sharded, _ = trainer.save_checkpoint(CheckpointType.sharded)
    spec = importlib.util.spec_from_file_location("s3_unshard_to_hf", str(Path(__file__).resolve().parent.parent / "scripts" / "s3_unshard_to_hf.py"))
    tool = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tool)
    work = tmp_path / "work"
    tool.main(["--sharded_bucket", str(sharded), "--unsharded_bucket", str(tmp_path / "bucket" / "unsharded"), "--hf_bucket", str(tmp_path / "bucket" / "hf"),
               "--local_dir", str(work), "--checkpoint_style", "transformers", "--model_only", "--quiet"])
    assert (work / "sharded" / "metadata.yaml").is_file() and (work / "unsharded" / "model.pt").is_file()
    assert (tmp_path / "bucket" / "unsharded" / "model.pt").is_file() and (tmp_path / "bucket" / "hf" / "config.json").is_file()
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path / "bucket" / "hf"), torch_dtype=torch.float32, attn_implementation="eager").eval()
    ids = torch.randint(0, cfg.model.vocab_size - 1, (1, 12))
    with torch.no_grad():
        want = trainer.model(ids).logits
        torch.testing.assert_close(hf(ids).logits[..., : want.shape[-1]], want[..., : hf.config.vocab_size], rtol=1e-4, atol=1e-4)
    shutil_target = tmp_path / "bucket" / "hf2"
    tool.main(["--already_unsharded", "--hf_bucket", str(shutil_target), "--local_dir", str(work), "--hf_olmo", "--cleanup_local_dir", "--quiet"])
    assert (shutil_target / "config.json").is_file() and not work.exists()
    with pytest.raises(SystemExit):
        tool.main(["--hf_bucket", str(tmp_path / "x")])


def test_training_resumes_from_a_torch_legacy_sharded_checkpoint(tmp_path):
    """``rank{r}.pt`` files holding ``ShardedTensor`` pickles (the reference's default sharded layout,
    ``olmo/checkpoint.py:969-1453``), written here by two gloo ranks from a trainer's full state, are detected by
    ``Trainer.restore_checkpoint`` and resumed from on one rank: weights, moments, step count and the next loss agree."""
    import os
    import socket
    import subprocess
    import sys
    from pathlib import Path

    torch.manual_seed(0)
    cfg = tiny_train_config(tmp_path / "a")
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    batches = iter(trainer.train_loader)
    for _ in range(3):
        trainer.global_step += 1
        trainer.global_train_examples_seen_this_epoch += cfg.global_train_batch_size
        trainer.global_train_tokens_seen += cfg.global_train_batch_size * cfg.model.max_sequence_length
        trainer.train_step(next(batches))
    named = list(trainer.dist_model.engine.named_parameters_for_optimizer())
    wrapped = {n: n.replace("transformer.blocks.", "transformer.blocks._fsdp_wrapped_module.") for n, _ in named}  # FSDP's name noise
    source = {
        "model": {wrapped[n]: p.detach().clone() for n, p in named},
        "optim": {
            "state": {wrapped[n]: {k: v.detach().clone() for k, v in trainer.optim.state[p].items()} for n, p in named},
            "param_groups": [{**{k: v for k, v in g.items() if k not in ("params", "param_names")},
                              "params": [wrapped[n] for n in g["param_names"]], "param_names": [wrapped[n] for n in g["param_names"]]}
                             for g in trainer.optim.param_groups],
        },
        "trainer": trainer.trainer_state_dict(),
    }
    torch.save(source, tmp_path / "source.pt")
    legacy = tmp_path / "step3"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    worker = Path(__file__).resolve().parent / "ref_layout_worker.py"
    proc = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
         str(worker), "--source", str(tmp_path / "source.pt"), "--out", str(legacy)],
        stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=300, env=dict(os.environ),
    )
    assert proc.returncode == 0, proc.stdout[-3000:]
    cfg.save(legacy / "config.yaml")

    cfg2 = tiny_train_config(tmp_path / "b")
    t2 = build_trainer(cfg2, device=torch.device("cpu"), train_loader=make_loader(cfg2), with_evaluators=False)
    t2.restore_checkpoint(str(legacy))
    assert t2.global_step == 3
    for n, p in t2.dist_model.engine.named_parameters_for_optimizer():
        assert torch.equal(p.detach(), source["model"][wrapped[n]]), n
        assert torch.allclose(t2.optim.state[p]["exp_avg_sq"], source["optim"]["state"][wrapped[n]]["exp_avg_sq"]), n
    expect = trainer.train_step(next(batches))["train/CrossEntropyLoss"]
    again = t2.train_step(next(iter(t2.train_loader)))["train/CrossEntropyLoss"]
    assert abs(again - expect) < 1e-5

    # the named checkpointers: the legacy one reads (restore and unshard) and refuses to write; the olmo_core one says what it needs
    from olmo_b200.checkpoint import OlmoCoreCheckpointer, TorchLegacyShardedCheckpointer
    from olmo_b200.exceptions import OLMoCheckpointError

    reader = TorchLegacyShardedCheckpointer(cfg2)
    model_state, optim_state, trainer_state = reader.unshard_checkpoint(legacy)
    assert trainer_state["global_step"] == 3 and set(model_state) == set(wrapped) and optim_state is not None
    cfg3 = tiny_train_config(tmp_path / "c")
    t3 = build_trainer(cfg3, device=torch.device("cpu"), train_loader=make_loader(cfg3), with_evaluators=False)
    assert reader.restore_checkpoint(legacy, t3.dist_model, t3.optim)["global_step"] == 3
    for n, p in t3.dist_model.engine.named_parameters_for_optimizer():
        assert torch.equal(p.detach(), source["model"][wrapped[n]]), n
    with pytest.raises(OLMoCheckpointError, match="read-only"):
        reader.save_checkpoint(tmp_path / "nope", t3.dist_model, t3.optim, {})
    with pytest.raises(OLMoCheckpointError, match="olmo_core"):
        OlmoCoreCheckpointer(cfg2).unshard_checkpoint(legacy)


def test_fused_or_portable_is_decided_when_the_engine_is_built(tmp_path):
    """Runs whose batches the fused kernel sequence cannot take (padding masks, module-output traces, document masking
    with heads wider than 128) get the portable path from the start; the rest keep the fused one."""
    from olmo_b200.launch import needs_portable_path

    cfg = tiny_train_config(tmp_path)
    assert needs_portable_path(cfg) is None
    cfg.data.generate_doc_lengths = True
    assert needs_portable_path(cfg) is None  # head dimension <= 128: covered by the native attention kernels
    cfg.model.d_model, cfg.model.n_heads = 512, 2
    assert "128" in needs_portable_path(cfg)
    cfg.model.n_heads = 8
    cfg.data.generate_doc_lengths = False
    cfg.data.generate_attention_mask = True
    assert "mask" in needs_portable_path(cfg)
    cfg.data.generate_attention_mask = False
    cfg.module_outputs_save_steps = [3]
    assert "hooks" in needs_portable_path(cfg)


def test_kept_activation_decision_follows_free_memory(monkeypatch):
    """``OLMO_B200_KEEP_ACTS=auto``: the extra activations are kept only when they fit in the memory still free after the
    first step with a margin (the decision itself needs no GPU: the memory query is replaced)."""
    from types import SimpleNamespace

    from olmo_b200.ops.fused_block import spec_from_config
    from olmo_b200.parallel.fsdp import FlatShardEngine
    from olmo_b200.recipes import recipe_config

    cfg = recipe_config("OLMo2-7B-stage1").model
    spec = spec_from_config(cfg)
    tokens, blocks = 2 * 4096, cfg.n_layers
    extra = (spec.Wq + spec.Wk + cfg.ff_proj_width // 2) * 2 * tokens * blocks  # bytes of rotated q/k + SwiGLU output
    assert 9.5e9 < extra < 11e9
    total = 192 << 30
    for free, expect in [(extra + (13 << 30), True), (extra + (11 << 30), False), (4 << 30, False)]:
        engine = SimpleNamespace(model=SimpleNamespace(config=cfg), device=torch.device("cpu"), keep_recomputable=None)
        monkeypatch.setattr(torch.cuda, "mem_get_info", lambda device=None, f=free: (f, total))
        FlatShardEngine._decide_keep_recomputable(engine, tokens, spec, blocks)
        assert engine.keep_recomputable is expect, (free, expect)
