"""The ``inference/`` entry points (paths and options of the reference) on a tiny checkpoint: quantise, benchmark
predictor over stdin/stdout, both with the plain predictor and with the serving engine."""
import importlib.util
import io
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from olmo_b200.config import ModelConfig, TokenizerConfig, TrainConfig
from olmo_b200.models.olmo import OLMo

ROOT = Path(__file__).resolve().parent.parent


def load(rel: str):
    spec = importlib.util.spec_from_file_location(rel.replace("/", "_"), str(ROOT / rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture()
def checkpoint(tmp_path):
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    vocab = {f"t{i}": i for i in range(94)}
    vocab["<pad>"], vocab["<eos>"] = 94, 95
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="t0"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.add_special_tokens(["<pad>", "<eos>"])
    tok.save(str(tmp_path / "tok.json"))
    torch.manual_seed(0)
    cfg = ModelConfig(d_model=64, n_heads=4, n_layers=2, mlp_ratio=2, vocab_size=96, embedding_size=128, max_sequence_length=32, weight_tying=False,
                      include_bias=False, eos_token_id=95, pad_token_id=94, init_device="cpu", rope=True, alibi=False, flash_attention=False)
    model = OLMo(cfg)
    ckpt = tmp_path / "step0-unsharded"
    ckpt.mkdir()
    TrainConfig(model=cfg, tokenizer=TokenizerConfig(identifier=str(tmp_path / "tok.json"))).save(ckpt / "config.yaml")
    torch.save(model.state_dict(), ckpt / "model.pt")
    return ckpt


def test_quantise_then_serve_prompts_over_stdio(tmp_path, checkpoint, monkeypatch, capsys):
    quantise = load("inference/compression/run_quantization.py")
    tokens = tmp_path / "calibration.npy"
    np.random.default_rng(0).integers(0, 94, size=4000, dtype=np.uint16).tofile(tokens)
    out = quantise.main(["--pretrained-model", str(checkpoint), "--quantized-model-dir", str(tmp_path / "q"), "--n-samples", "4",
                         "--calibration-data", str(tokens), "--seq-len", "16", "--group-size", "32"])
    assert (out / "quantized.pt").is_file() and (out / "config.yaml").is_file()
    rtn = quantise.main(["--pretrained-model", str(checkpoint), "--quantized-model-dir", str(tmp_path / "q_rtn"), "--group-size", "32"])
    assert torch.load(rtn / "quantized.pt", weights_only=False)["act_order"] is False
    with pytest.raises(SystemExit):
        quantise.main(["--pretrained-model", str(checkpoint), "--quantized-model-dir", str(tmp_path / "x"), "--method", "gptq"])

    layout = load("inference/compression/olmo_gptq_class.py").OLMoGPTQForCausalLM
    assert layout.inside_layer_modules == [["att_proj"], ["attn_out"], ["ff_proj"], ["ff_out"]] and layout.layers_block_name == "transformer.blocks"

    bench = load("inference/efficiency/run_efficiency_benchmark.py")
    for extra in ([], ["--quantized-model-dir", str(out)], ["--vllm"]):
        monkeypatch.setattr(sys, "stdin", io.StringIO(json.dumps(["t1 t2 t3", "t4 t5"]) + "\n" + json.dumps(["t6"]) + "\n"))
        capsys.readouterr()
        served = bench.main(["--pretrained-model-dir", str(checkpoint), "--max-new-tokens", "3", *extra])
        lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("[")]
        assert served == 2 and [len(x) for x in lines] == [2, 1] and all(isinstance(s, str) for x in lines for s in x), extra
