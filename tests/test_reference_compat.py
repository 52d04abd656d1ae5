"""Unsharded checkpoints written by this framework load into the unmodified reference package (installed under
``baseline/_ref`` for the benchmark's reference arm) and give the same logits there; the trainer and optimizer files
carry the keys the reference's loaders read (``olmo/train.py`` trainer_state_dict, ``olmo/checkpoint.py``
FullCheckpointer).  Skipped where the reference is not installed."""
import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from test_train_cpu import make_loader, tiny_train_config

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref" / "olmo" / "model.py"

pytestmark = pytest.mark.skipif(not REF.is_file(), reason="reference package not installed under baseline/_ref")


@pytest.mark.parametrize("flavour", ["olmo1", "olmo2"])
def test_reference_loads_our_unsharded_checkpoint(tmp_path, flavour):
    from olmo_b200.launch import build_trainer

    torch.manual_seed(0)
    overrides = {}
    if flavour == "olmo2":
        overrides = dict(layer_norm_type="rms", layer_norm_with_affine=True, attention_layer_norm=True,
                         attention_layer_norm_with_affine=True, norm_after=True, rope_theta=500000, layer_norm_eps=1e-6)
    cfg = tiny_train_config(tmp_path / "run", **overrides)
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=make_loader(cfg), with_evaluators=False)
    batches = iter(trainer.train_loader)
    for _ in range(2):
        trainer.global_step += 1
        trainer.global_train_examples_seen_this_epoch += cfg.global_train_batch_size
        trainer.global_train_tokens_seen += cfg.global_train_batch_size * cfg.model.max_sequence_length
        trainer.train_step(next(batches))
    ckpt, _ = trainer.save_unsharded_checkpoint()
    ids = torch.randint(0, 16, (2, 12))
    trainer.model.eval()
    with torch.no_grad():
        ours = trainer.dist_model(ids).logits.float()

    model_fields = {k: (v.value if hasattr(v, "value") else v) for k, v in cfg.model.asdict().items()}
    (tmp_path / "model.json").write_text(json.dumps(model_fields))
    (tmp_path / "ids.json").write_text(json.dumps(ids.tolist()))
    proc = subprocess.run(
        [sys.executable, str(Path(__file__).with_name("ref_compat_child.py")), str(tmp_path / "model.json"), str(ckpt), str(tmp_path / "ids.json")],
        capture_output=True, text=True, timeout=600,
    )
    assert proc.returncode == 0, proc.stderr[-3000:]
    got = json.loads(proc.stdout.strip().splitlines()[-1])
    torch.testing.assert_close(torch.tensor(got["logits"]), ours, rtol=1e-4, atol=1e-4)
    # what the reference's restore path reads from train.pt / optim.pt
    for key in ("global_step", "global_train_examples_seen_this_epoch", "global_train_tokens_seen", "epoch", "checkpoints",
                "unsharded_checkpoints", "ephemeral_checkpoints", "rng", "world_size"):
        assert key in got["trainer_keys"], key
    assert got["optim_keys"] == ["param_groups", "state"]
    n_params = len(list(trainer.model.parameters()))
    assert got["n_optim_state"] == n_params
    assert sum(g["params"] for g in got["param_groups"]) == n_params
