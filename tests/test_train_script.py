"""The training entry point as a user runs it: ``scripts/train.py CONFIG.yaml --dotted=overrides`` on CPU with token files,
an in-loop perplexity evaluator, periodic sharded and unsharded checkpoints with retention, then a second invocation that
resumes from the latest checkpoint and continues the data order."""
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent.parent

CONFIG = """
run_name: script-test
seed: 7
model:
  d_model: 64
  n_heads: 4
  n_layers: 2
  mlp_hidden_size: 256
  weight_tying: false
  rope: true
  flash_attention: false
  include_bias: false
  layer_norm_type: rms
  layer_norm_with_affine: true
  attention_layer_norm: true
  norm_after: true
  max_sequence_length: 32
  vocab_size: 250
  embedding_size: 256
  eos_token_id: 249
  pad_token_id: 249
  init_device: meta
  init_std: 0.05
optimizer:
  name: adamw
  learning_rate: 2.0e-3
  weight_decay: 0.1
  betas: [0.9, 0.95]
  metrics_log_interval: 2
scheduler:
  name: cosine_with_warmup
  t_warmup: 2
  alpha_f: 0.1
precision: fp32
distributed_strategy: fsdp
fsdp:
  sharding_strategy: FULL_SHARD
  wrapping_strategy: by_block
  precision: pure
global_train_batch_size: 8
device_train_microbatch_size: 4
max_duration: 12
max_grad_norm: 1.0
softmax_auxiliary_loss: true
save_interval: 4
save_num_checkpoints_to_keep: 2
save_interval_unsharded: 6
save_num_unsharded_checkpoints_to_keep: 1
save_interval_ephemeral: null
console_log_interval: 2
eval_interval: 6
device_eval_batch_size: 4
eval_subset_num_batches: 2
speed_monitor:
  window_size: 2
data:
  paths: ${path.glob:%(data)s/train-*.npy}
  memmap_dtype: uint16
  num_workers: 0
  drop_last: true
  pin_memory: false
  prefetch_factor: null
  persistent_workers: false
  timeout: 0
evaluators:
  - label: val
    type: lm
    data:
      datasets:
        held-out: ["%(data)s/val-0.npy"]
      memmap_dtype: uint16
      num_workers: 0
      drop_last: true
      pin_memory: false
      prefetch_factor: null
      persistent_workers: false
"""


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run(args, cwd, nproc=2, timeout=900):
    """Two gloo ranks through torchrun, so that the sharded-checkpoint branches of the training loop run."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2", WANDB_MODE="disabled", OLMO_SHARED_FS="1")
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(key, None)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "scripts" / "train.py"), *args]
    return subprocess.run(cmd, cwd=cwd, env=env, capture_output=True, text=True, timeout=timeout)


def test_train_script_end_to_end_and_resume(tmp_path):
    data = tmp_path / "data"
    data.mkdir()
    rng = np.random.default_rng(0)
    for name, n in (("train-0", 4096), ("train-1", 4096), ("val-0", 1024)):
        arr = np.memmap(data / f"{name}.npy", dtype=np.uint16, mode="w+", shape=(n,))
        arr[:] = rng.integers(0, 16, n)  # low-entropy tokens: the loss must fall quickly
        arr.flush()
    cfg = tmp_path / "config.yaml"
    cfg.write_text(CONFIG % {"data": str(data)})
    run_dir = tmp_path / "run"

    first = run([str(cfg), f"--save_folder={run_dir}", "--stop_at=8"], tmp_path)
    out = first.stdout + first.stderr
    assert first.returncode == 0, out[-4000:]
    assert "Training complete" in out
    losses = [float(x) for x in re.findall(r"train/CrossEntropyLoss=([0-9.]+)", out)]
    assert len(losses) >= 3 and losses[-1] < losses[0], losses
    assert re.search(r"eval/val/CrossEntropyLoss|eval/held-out/CrossEntropyLoss", out), out[-3000:]
    assert (run_dir / "config.yaml").is_file()
    names = sorted(p.name for p in run_dir.iterdir())
    # sharded checkpoints at 4 and 8 (the step-0 pre-train checkpoint rotated out by the keep-2 rule); the unsharded one
    # written at step 6 gave way (keep 1) to the final unsharded checkpoint of step 8
    assert "step8" in names and "step4" in names and "step0" not in names, names
    assert "step8-unsharded" in names and "step6-unsharded" not in names, names
    assert (run_dir / "latest").exists() and (run_dir / "latest-unsharded").exists()
    assert (run_dir / "step8" / "config.yaml").is_file() and (run_dir / "train_data" / "global_indices.npy").is_file()

    # (without stop_at the loop runs to max_duration + 10 steps, as the reference's does)
    second = run([str(cfg), f"--save_folder={run_dir}", "--try_load_latest_save=true", "--save_overwrite", "--stop_at=12"], tmp_path)
    out2 = second.stdout + second.stderr
    assert second.returncode == 0, out2[-4000:]
    assert "Resuming from" in out2 and "Training complete" in out2
    steps = [int(x) for x in re.findall(r"\[step=(\d+)/12", out2)]
    assert steps and min(steps) > 8 and max(steps) == 12, steps  # continued after the restored step, up to max_duration
    names = sorted(p.name for p in run_dir.iterdir())
    assert "step12" in names and "step12-unsharded" in names and "step8-unsharded" not in names, names
    assert len([n for n in names if re.fullmatch(r"step\d+", n)]) == 2, names

    # the final unsharded checkpoint loads as a plain model and still predicts the low-entropy data well
    from olmo_b200.models.olmo import OLMo

    model = OLMo.from_checkpoint(run_dir / "step12-unsharded").eval()
    ids = torch.from_numpy(np.asarray(np.memmap(data / "val-0.npy", dtype=np.uint16, mode="r")[:128]).astype(np.int64)).view(4, 32)
    with torch.no_grad():
        logits = model(ids).logits
    loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))
    assert float(loss) < 4.5  # ln(250) = 5.5 at initialisation; the data has ln(16) = 2.8 of entropy


def test_fixture_configs_train_from_the_repository_root(tmp_path):
    """``test_fixtures/train_tiny.yaml`` and ``train_tiny_with_evaluator.yaml`` run as committed (fixture tokenizer and token
    file, CPU, one epoch of ten batches), and an epoch that does not divide into whole batches is explained instead of
    tripping a bare assertion."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2")
    for name, expect_eval in (("train_tiny.yaml", False), ("train_tiny_with_evaluator.yaml", True)):
        env["OLMO_TINY_SAVE_FOLDER"] = str(tmp_path / name)
        proc = subprocess.run([sys.executable, "scripts/train.py", f"test_fixtures/{name}"], cwd=ROOT, env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True, timeout=600)
        assert proc.returncode == 0, proc.stdout[-3000:]
        assert "Training complete" in proc.stdout and (tmp_path / name / "step4-unsharded" / "model.pt").is_file()
        assert ("eval/sample-docs/Perplexity" in proc.stdout) == expect_eval
        losses = [float(x) for x in re.findall(r"train/CrossEntropyLoss=([0-9.]+)", proc.stdout)]
        assert len(losses) == 10 and losses[-1] < losses[0]
    env["OLMO_TINY_SAVE_FOLDER"] = str(tmp_path / "short")
    proc = subprocess.run([sys.executable, "scripts/train.py", "test_fixtures/train_tiny.yaml", "--data.drop_last=false"], cwd=ROOT, env=env,
                          stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=600)
    assert proc.returncode != 0 and "data.drop_last=true" in proc.stdout
