"""HuggingFace interoperability: auto classes, save/load round trip, and exact agreement between this model and the
architectures that ship inside ``transformers`` after conversion (an independent implementation of the same maths)."""
import json
from pathlib import Path

import pytest
import torch

transformers = pytest.importorskip("transformers")

import hf_olmo  # noqa: E402,F401  (registers the auto classes)
from olmo_b200.config import ModelConfig, TokenizerConfig, TrainConfig  # noqa: E402
from olmo_b200.hf import OLMoConfig, OLMoForCausalLM  # noqa: E402
from olmo_b200.hf.convert import to_transformers_state_dict, transformers_config_dict, write_hf_olmo_checkpoint, write_transformers_checkpoint  # noqa: E402
from olmo_b200.models.olmo import OLMo  # noqa: E402

OLMO2 = dict(d_model=64, n_heads=4, n_layers=2, mlp_hidden_size=256, vocab_size=120, embedding_size=128, max_sequence_length=64,
             weight_tying=False, include_bias=False, rope=True, rope_theta=500000, flash_attention=False, layer_norm_type="rms",
             layer_norm_with_affine=True, layer_norm_eps=1e-6, bias_for_layer_norm=False, attention_layer_norm=True,
             attention_layer_norm_with_affine=True, norm_after=True, eos_token_id=119, pad_token_id=118, init_device="cpu", init_std=0.05)
OLMO1 = dict(d_model=64, n_heads=4, n_layers=2, mlp_hidden_size=256, vocab_size=120, embedding_size=128, max_sequence_length=64,
             weight_tying=False, include_bias=False, rope=True, flash_attention=False, layer_norm_type="default",
             layer_norm_with_affine=False, attention_layer_norm=False, clip_qkv=0.5, eos_token_id=119, pad_token_id=118,
             init_device="cpu", init_fn="mitchell")


def native(kwargs):
    torch.manual_seed(0)
    m = OLMo(ModelConfig(**kwargs))
    m.reset_parameters()
    with torch.no_grad():  # make the norm weights non-trivial
        for n, p in m.named_parameters():
            if "norm" in n or "ln_f" in n:
                p.uniform_(0.5, 1.5)
    return m.eval()


def save_unsharded(model: OLMo, folder):
    folder.mkdir(parents=True, exist_ok=True)
    TrainConfig(model=model.config, tokenizer=TokenizerConfig(identifier="missing-tokenizer.json")).save(folder / "config.yaml")
    torch.save(model.state_dict(), folder / "model.pt")
    return folder


@pytest.mark.parametrize("kwargs,cls_name", [(OLMO2, "Olmo2ForCausalLM"), (OLMO1, "OlmoForCausalLM")])
def test_converted_weights_reproduce_logits_in_transformers(tmp_path, kwargs, cls_name):
    model = native(kwargs)
    out_dir, model_type = write_transformers_checkpoint(save_unsharded(model, tmp_path / "ckpt"), tmp_path / "hf")
    assert json.loads((out_dir / "config.json").read_text())["architectures"] == [cls_name]
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(out_dir), torch_dtype=torch.float32, attn_implementation="eager").eval()
    assert type(hf).__name__ == cls_name
    ids = torch.randint(0, 118, (2, 17))
    with torch.no_grad():
        ours = model(ids).logits
        theirs = hf(ids).logits
    torch.testing.assert_close(ours, theirs, rtol=2e-4, atol=2e-4)
    # greedy continuations agree as well (KV cache paths of both implementations)
    with torch.no_grad():
        gen_hf = hf.generate(ids, max_new_tokens=5, do_sample=False, attention_mask=torch.ones_like(ids), pad_token_id=118)
        gen_ours = OLMoForCausalLM(OLMoConfig(**model.config.asdict()), model=model).generate(
            ids, max_new_tokens=5, do_sample=False, attention_mask=torch.ones_like(ids), pad_token_id=118
        )
    assert gen_hf.tolist() == gen_ours.tolist()


def test_state_dict_mapping_rejects_unsupported_architectures():
    with pytest.raises(ValueError):
        transformers_config_dict(ModelConfig(**{**OLMO2, "alibi": True, "rope": False}))
    with pytest.raises(ValueError):
        transformers_config_dict(ModelConfig(**{**OLMO2, "norm_after": False}))
    with pytest.raises(ValueError):
        transformers_config_dict(ModelConfig(**{**OLMO1, "block_type": "llama"}))
    cfg = ModelConfig(**{**OLMO2, "n_kv_heads": 2})
    m = native({**OLMO2, "n_kv_heads": 2})
    sd = to_transformers_state_dict(m.state_dict(), cfg)
    assert sd["model.layers.0.self_attn.k_proj.weight"].shape == (32, 64)
    assert sd["model.layers.1.mlp.gate_proj.weight"].shape == (128, 64)
    assert transformers_config_dict(cfg)["num_key_value_heads"] == 2


def test_hf_olmo_layout_round_trip_and_auto_classes(tmp_path):
    model = native(OLMO2)
    folder = write_hf_olmo_checkpoint(save_unsharded(model, tmp_path / "ckpt"), tmp_path / "hf_olmo")
    cfg = transformers.AutoConfig.from_pretrained(str(folder))
    assert isinstance(cfg, OLMoConfig) and cfg.model_type == "hf_olmo" and cfg.hidden_size == 64 and cfg.num_hidden_layers == 2
    loaded = transformers.AutoModelForCausalLM.from_pretrained(str(folder), torch_dtype=torch.float32).eval()
    assert isinstance(loaded, OLMoForCausalLM)
    ids = torch.randint(0, 118, (2, 9))
    with torch.no_grad():
        torch.testing.assert_close(loaded(ids).logits, model(ids).logits)
        out = loaded(ids, labels=ids)
    want = torch.nn.functional.cross_entropy(out.logits[:, :-1].reshape(-1, 128), ids[:, 1:].reshape(-1))
    torch.testing.assert_close(out.loss, want)
    loaded.save_pretrained(str(tmp_path / "again"))
    again = OLMoForCausalLM.from_pretrained(str(tmp_path / "again"), torch_dtype=torch.float32).eval()
    with torch.no_grad():
        torch.testing.assert_close(again(ids).logits, model(ids).logits)


def test_wrapper_toggles_and_embedding_resize():
    wrapper = OLMoForCausalLM(OLMoConfig(**{**OLMO2, "weight_tying": True}), init_params=True)
    assert wrapper.get_output_embeddings() is wrapper.get_input_embeddings()
    wrapper.gradient_checkpointing = True
    assert wrapper.model.activation_checkpointing_strategy is not None
    wrapper.gradient_checkpointing = False
    assert wrapper.model.activation_checkpointing_strategy is None
    before = wrapper.get_input_embeddings().weight.detach().clone()
    emb = wrapper.resize_token_embeddings(130, pad_to_multiple_of=64)
    assert emb.weight.shape == (192, 64) and wrapper.config.embedding_size == 192 and wrapper.model.config.embedding_size == 192
    torch.testing.assert_close(emb.weight[:128], before)
    ids = torch.randint(0, 118, (1, 5))
    assert wrapper(ids).logits.shape == (1, 5, 192)
    untied = OLMoForCausalLM(OLMoConfig(**OLMO2), init_params=True)
    untied.resize_token_embeddings(256)
    assert untied.model.transformer.ff_out.out_features == 256 and untied(ids).logits.shape[-1] == 256
    with pytest.raises(ValueError):
        untied(ids, output_attentions=True)
    cfg = OLMoConfig(n_heads=8, multi_query_attention=True)
    assert cfg.effective_n_kv_heads == 1 and OLMoConfig(n_heads=8, n_kv_heads=2).effective_n_kv_heads == 2


def test_transformers_generate_uses_the_key_value_cache_and_matches_greedy_decoding():
    """``generate`` of the transformers wrapper (greedy, with its cache plumbing through ``prepare_inputs_for_generation``)
    produces the tokens a cache-free argmax loop over the native model produces."""
    wrapper = OLMoForCausalLM(OLMoConfig(**OLMO2), init_params=True).eval()
    torch.manual_seed(3)
    ids = torch.randint(0, 118, (1, 7))
    out = wrapper.generate(ids, max_new_tokens=8, do_sample=False, pad_token_id=wrapper.config.pad_token_id)
    want = ids[0].tolist()
    with torch.no_grad():
        for _ in range(8):
            want.append(int(wrapper.model(torch.tensor([want])).logits[0, -1].argmax()))
            if want[-1] == wrapper.config.eos_token_id:  # generation stops after emitting the end token
                break
    assert out[0].tolist() == want and len(want) > 9


def test_text_generation_pipeline_with_converted_checkpoint_and_tokenizer(tmp_path):
    """A checkpoint converted with its tokenizer file loads through ``AutoTokenizer`` / ``AutoModelForCausalLM`` and runs
    in a transformers text-generation pipeline."""
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    from olmo_b200.hf import OLMoTokenizerFast

    vocab = {f"w{i}": i for i in range(118)}
    vocab["<pad>"], vocab["<eos>"] = 118, 119
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="<pad>"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.add_special_tokens(["<pad>", "<eos>"])
    tok.save(str(tmp_path / "tokenizer.json"))

    model = native(OLMO2)
    folder = write_hf_olmo_checkpoint(save_unsharded(model, tmp_path / "ckpt"), tmp_path / "hf_olmo", tokenizer_path=tmp_path / "tokenizer.json")
    tokenizer = transformers.AutoTokenizer.from_pretrained(str(folder))
    assert isinstance(tokenizer, OLMoTokenizerFast)
    assert tokenizer("w1 w2 w3")["input_ids"][:3] == [1, 2, 3]
    loaded = transformers.AutoModelForCausalLM.from_pretrained(str(folder), torch_dtype=torch.float32).eval()
    pipe = transformers.pipeline("text-generation", model=loaded, tokenizer=tokenizer)
    text = pipe("w5 w6 w7", max_new_tokens=4, do_sample=False)[0]["generated_text"]
    words = text.split()
    assert words[:3] == ["w5", "w6", "w7"] and 3 < len(words) <= 7
    ids = [vocab[w] for w in words[:3]]
    with torch.no_grad():
        first = int(model(torch.tensor([ids])).logits[0, -1].argmax())
    assert words[3] == {v: k for k, v in vocab.items()}[first]


def test_hf_olmo_converter_steps_local_and_remote(tmp_path):
    """The converter command: into another folder (source untouched), in place, from and to a remote store; and the
    reference's module paths resolve."""
    import importlib

    from hf_olmo import convert_olmo_to_hf as conv
    from olmo_b200 import util

    for mod, name in (("configuration_olmo", "OLMoConfig"), ("modeling_olmo", "OLMoForCausalLM"), ("tokenization_olmo_fast", "OLMoTokenizerFast")):
        assert getattr(importlib.import_module(f"hf_olmo.{mod}"), name) is getattr(hf_olmo, name)
    assert conv.longest_common_prefix(["s3://b/run/step1/model.pt", "s3://b/run/step1/config.yaml"]) == "s3://b/run/step1/"
    assert conv.longest_common_prefix([]) == "" and conv.longest_common_prefix(["abc"]) == "abc"

    model = native(OLMO2)
    src = save_unsharded(model, tmp_path / "ckpt")
    (src / "optim.pt").write_bytes(b"x")
    ids = torch.randint(0, 118, (2, 9))

    out = tmp_path / "converted"
    conv.main(["--checkpoint-dir", str(src), "--destination-dir", str(out)])
    assert sorted(p.name for p in out.iterdir()) == ["config.json", "pytorch_model.bin"]  # no tokenizer: the configured file is missing
    assert (src / "model.pt").is_file() and (src / "optim.pt").is_file() and not (src / "config.json").exists()
    loaded = transformers.AutoModelForCausalLM.from_pretrained(str(out), torch_dtype=torch.float32).eval()
    with torch.no_grad():
        torch.testing.assert_close(loaded(ids).logits, model(ids).logits)

    inplace = save_unsharded(model, tmp_path / "inplace")
    conv.main(["--checkpoint-dir", str(inplace), "--keep-olmo-artifacts", "--safetensors"])
    assert {"config.json", "model.safetensors", "config.yaml", "model.pt"} <= {p.name for p in inplace.iterdir()}

    class Store(util.StorageBackend):
        def __init__(self):
            self.blobs = {}

        def file_size(self, url):
            return len(self.blobs[url])

        def get_bytes_range(self, url, start, num):
            return self.blobs[url][start : start + num]

        def upload(self, source, url, save_overwrite=False):
            self.blobs[url] = Path(source).read_bytes()

        def list_files(self, url):
            return sorted(k for k in self.blobs if k.startswith(url.rstrip("/") + "/"))

    store = Store()
    util.register_storage_backend("mem", store)
    try:
        for p in src.iterdir():
            store.blobs[f"mem://bucket/run/step5-unsharded/{p.name}"] = p.read_bytes()
        conv.main(["--checkpoint-dir", "mem://bucket/run/step5-unsharded", "--destination-dir", "mem://bucket/hf/step5"])
        names = sorted(k.rsplit("/", 1)[1] for k in store.blobs if k.startswith("mem://bucket/hf/step5/"))
        assert names == ["config.json", "pytorch_model.bin"]
        assert "mem://bucket/run/step5-unsharded/model.pt" in store.blobs  # the source is left alone
    finally:
        util._BACKENDS.pop("mem", None)


def test_transformers_export_options(tmp_path):
    model = native({**OLMO1, "eos_token_id": 0})
    src = save_unsharded(model, tmp_path / "ckpt")
    fixed, _ = write_transformers_checkpoint(src, tmp_path / "fixed", include_tokenizer=False, safe_serialization=False)
    assert json.loads((fixed / "config.json").read_text())["eos_token_id"] == 50279
    assert json.loads((fixed / "generation_config.json").read_text())["eos_token_id"] == 50279
    assert (fixed / "pytorch_model.bin").is_file() and not (fixed / "model.safetensors").exists() and not (fixed / "tokenizer.json").exists()
    kept, _ = write_transformers_checkpoint(src, tmp_path / "kept", fix_eos_token_id=False)
    assert json.loads((kept / "config.json").read_text())["eos_token_id"] == 0 and (kept / "model.safetensors").is_file()
