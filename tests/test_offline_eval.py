"""Offline evaluation pipeline: task construction, perplexity arithmetic, caching in the workspace, rows."""
import gzip
import json
import math

import numpy as np
import pytest
import torch
import yaml

from olmo_b200.config import ActivationType, LayerNormType, ModelConfig
from olmo_b200.eval import offline
from olmo_b200.models.olmo import OLMo

datasets = pytest.importorskip("datasets")
EOS = 1


class CharTokenizer:
    pad_token_id = 0
    eos_token_id = EOS

    def encode(self, s, add_special_tokens=True):
        return [min(ord(c), 127) for c in s] + ([EOS] if add_special_tokens else [])

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(i) for i in ids if i > 1)


@pytest.fixture()
def eval_model():
    torch.manual_seed(0)
    cfg = ModelConfig(
        d_model=32, n_heads=2, n_layers=2, mlp_hidden_size=64, activation_type=ActivationType.swiglu, rope=True,
        layer_norm_type=LayerNormType.rms, include_bias=False, vocab_size=128, embedding_size=128, max_sequence_length=32,
        eos_token_id=EOS, pad_token_id=0, weight_tying=False, init_device="cpu",
    )
    return offline.EvalModel("tiny", OLMo(cfg).eval(), CharTokenizer(), torch.device("cpu"))


def test_perplexity_metrics_match_a_direct_computation(tmp_path, eval_model):
    docs = ["the cat sat on the mat", "a much longer document that needs more than one window of thirty-two tokens to score"]
    text_file = tmp_path / "val.jsonl.gz"
    with gzip.open(text_file, "wt") as f:
        for d in docs:
            f.write(json.dumps({"text": d}) + "\n")
    task = offline.construct_task("ppl", eval_model.tokenizer, {"files": [str(text_file)]})
    out = offline.predict_and_calculate_metrics(eval_model, task, {"batch_size": 2, "model_max_length": 16})

    nll = 0.0
    with torch.no_grad():
        for d in docs:
            ids = eval_model.tokenizer.encode(d, add_special_tokens=False)
            for start in range(0, len(ids), 15):
                window = torch.tensor([[EOS] + ids[start : start + 15]])
                logp = torch.log_softmax(eval_model.model(window).logits[0].float(), dim=-1)
                nll -= float(logp[:-1].gather(1, window[0, 1:, None]).sum())
    chars = sum(map(len, docs))
    words = sum(len(d.split()) for d in docs)
    assert out["num_instances"] == 2 and out["num_tokens"] == chars
    assert out["metrics"]["ppl_token"] == pytest.approx(math.exp(nll / chars), rel=1e-5)
    assert out["metrics"]["ppl_word"] == pytest.approx(math.exp(nll / words), rel=1e-5)
    assert out["metrics"]["bits_per_byte"] == pytest.approx(nll / chars / math.log(2), rel=1e-5)

    # the same documents as a token memmap (separated by the end token) give the same numbers
    tokens = []
    for d in docs:
        tokens += eval_model.tokenizer.encode(d, add_special_tokens=True)
    np.array(tokens, dtype=np.uint16).tofile(tmp_path / "val.npy")
    mm = offline.construct_task("ppl", eval_model.tokenizer, {"files": [str(tmp_path / "val.npy")]})
    again = offline.predict_and_calculate_metrics(eval_model, mm, {"model_max_length": 16})
    assert again["metrics"]["ppl_token"] == pytest.approx(out["metrics"]["ppl_token"], rel=1e-6)
    limited = offline.predict_and_calculate_metrics(eval_model, mm, {"model_max_length": 16, "limit": 1})
    assert limited["num_instances"] == 1


def test_experiment_runs_the_cross_product_and_reuses_cached_steps(tmp_path, monkeypatch, eval_model):
    rows = [{"goal": f"goal {i}", "sol1": "ab" * (1 + i % 3), "sol2": "cd", "label": i % 2} for i in range(8)]
    datasets.Dataset.from_list(rows).save_to_disk(str(tmp_path / "hf_datasets" / "piqa" / "plain_text" / "validation"))
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))
    text_file = tmp_path / "val.jsonl"
    text_file.write_text(json.dumps({"text": "hello evaluation"}) + "\n")
    (tmp_path / "task_sets").mkdir()
    (tmp_path / "task_sets" / "my_rc.yaml").write_text(yaml.safe_dump(
        {"name": "my_rc", "task_names": ["piqa"], "prediction_kwargs": {"limit": 6, "num_recorded_inputs": 2}}))
    experiment = {
        "workspace": str(tmp_path / "ws"), "output": str(tmp_path / "out" / "rows.jsonl"),
        "models": [{"model_path": "tiny-a"}, {"model_path": "tiny-b", "prediction_kwargs": {"limit": 4}}],
        "task_sets": ["my_rc", {"name": "ppl_set", "tasks": [{"task_name": "ppl", "task_rename": "ppl_hello", "task_kwargs": {"files": [str(text_file)]}}]}],
    }
    (tmp_path / "exp.yaml").write_text(yaml.safe_dump(experiment))
    spec = offline.load_experiment(str(tmp_path / "exp.yaml"))
    assert spec["task_sets"][0]["tasks"][0] == {"task_name": "piqa", "task_kwargs": {}, "prediction_kwargs": {"limit": 6, "num_recorded_inputs": 2}}

    loads = []

    def loader(model_path, **kwargs):
        loads.append(model_path)
        return offline.EvalModel(model_path, eval_model.model, eval_model.tokenizer, eval_model.device)

    out = offline.run_experiment(spec, loader=loader)
    assert [(r["model_path"], r["task_set"], r["task"]) for r in out] == [
        ("tiny-a", "my_rc", "piqa"), ("tiny-a", "ppl_set", "ppl_hello"), ("tiny-b", "my_rc", "piqa"), ("tiny-b", "ppl_set", "ppl_hello")]
    assert out[0]["num_instances"] == 6 and out[2]["num_instances"] == 4 and out[2]["limit"] == 4
    assert 0.0 <= out[0]["metric_len_norm"] <= 1.0 and out[1]["metric_ppl_token"] > 1.0
    assert loads == ["tiny-a", "tiny-b"]
    assert len(list((tmp_path / "ws").glob("*.json"))) == 4

    lines = [json.loads(l) for l in (tmp_path / "out" / "rows.jsonl").read_text().splitlines()]
    assert lines == json.loads(json.dumps(out))
    table = (tmp_path / "out" / "rows.tsv").read_text().splitlines()
    assert table[0].split("\t")[:4] == ["model_path", "revision", "task_set", "task"] and len(table) == 5
    assert "metric_len_norm" in table[0] and "metric_bits_per_byte" in table[0]

    # a second run finds every step in the workspace: no model is loaded, numbers are identical
    loads.clear()
    second = offline.run_experiment(spec, loader=loader)
    assert loads == [] and [r["metric_len_norm"] for r in second[::2]] == [r["metric_len_norm"] for r in out[::2]]
    # a new task set only computes what is new
    spec["task_sets"].append({"name": "more", "tasks": [{"task_name": "ppl", "task_kwargs": {"files": [str(text_file)]}, "prediction_kwargs": {"model_max_length": 8}}]})
    third = offline.run_experiment(spec, loader=loader)
    assert loads == ["tiny-a", "tiny-b"] and len(third) == 6

    with pytest.raises(KeyError):
        offline.construct_task("no_such_task", eval_model.tokenizer)
    with pytest.raises(FileNotFoundError):
        offline.resolve_task_set("no_such_set")


def test_shipped_task_sets_name_known_tasks():
    from olmo_b200.eval.downstream import label_to_task_map

    files = sorted(offline.TASK_SET_DIR.glob("*.yaml"))
    assert {f.stem for f in files} >= {"rc_tasks", "mmlu_tasks", "bpb_tasks", "ppl_val_example"}
    for file in files:
        task_set = offline.resolve_task_set(file.stem)
        assert task_set["name"] == file.stem and task_set["tasks"]
        for task in task_set["tasks"]:
            assert task["task_name"] in ("ppl", "gen") or task["task_name"] in label_to_task_map, (file.name, task["task_name"])


def test_run_eval_command_line_on_a_checkpoint_folder(tmp_path, monkeypatch):
    """``evaluation/run_eval.py`` end to end: checkpoint folder -> model + tokenizer -> rows on disk."""
    import importlib.util
    from pathlib import Path

    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    from olmo_b200.config import TokenizerConfig, TrainConfig

    words = ["hello", "evaluation", "the", "cat", "sat", "on", "mat"]
    vocab = {"<pad>": 0, **{w: i + 1 for i, w in enumerate(words)}, "<eos>": len(words) + 1}
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="<pad>"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.save(str(tmp_path / "tokenizer.json"))
    torch.manual_seed(0)
    cfg = ModelConfig(
        d_model=32, n_heads=2, n_layers=1, mlp_hidden_size=64, activation_type=ActivationType.swiglu, rope=True,
        layer_norm_type=LayerNormType.rms, include_bias=False, vocab_size=len(vocab), embedding_size=16, max_sequence_length=16,
        eos_token_id=len(words) + 1, pad_token_id=0, weight_tying=False, init_device="cpu",
    )
    ckpt = tmp_path / "step0-unsharded"
    ckpt.mkdir()
    torch.save(OLMo(cfg).state_dict(), ckpt / "model.pt")
    TrainConfig(model=cfg, tokenizer=TokenizerConfig(identifier=str(tmp_path / "tokenizer.json"))).save(ckpt / "config.yaml")
    (tmp_path / "val.jsonl").write_text(json.dumps({"text": "the cat sat on the mat"}) + "\n" + json.dumps({"text": "hello evaluation"}) + "\n")
    experiment = {
        "models": [str(ckpt)],
        "task_sets": [{"name": "ppl", "tasks": [{"task_name": "ppl", "task_kwargs": {"files": [str(tmp_path / "val.jsonl")]}}]}],
    }
    (tmp_path / "exp.yaml").write_text(yaml.safe_dump(experiment))
    script = Path(__file__).resolve().parent.parent / "evaluation" / "run_eval.py"
    spec = importlib.util.spec_from_file_location("run_eval_script", script)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.main([str(tmp_path / "exp.yaml"), "--workspace", str(tmp_path / "ws"), "--output", str(tmp_path / "rows.jsonl"), "--device", "cpu"]) == 0
    rows = [json.loads(l) for l in (tmp_path / "rows.jsonl").read_text().splitlines()]
    assert len(rows) == 1 and rows[0]["num_instances"] == 2 and rows[0]["metric_ppl_token"] > 1.0
    assert (tmp_path / "rows.tsv").is_file()


def test_fixture_experiment_runs_from_the_repository_root(tmp_path, monkeypatch):
    """The committed example experiment (tiny checkpoint + synthetic corpus under ``test_fixtures/``)."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    proc = subprocess.run(
        [sys.executable, "evaluation/run_eval.py", "evaluation/experiments/fixture_config.yaml", "--workspace", str(tmp_path / "ws"),
         "--output", str(tmp_path / "rows.jsonl")], cwd=root, capture_output=True, text=True, timeout=600,
    )
    assert proc.returncode == 0, proc.stderr[-2000:]
    row = json.loads((tmp_path / "rows.jsonl").read_text().splitlines()[0])
    assert row["task"] == "ppl_sample_docs" and row["num_instances"] == 48
    assert 30 < row["metric_ppl_token"] < 200  # an untrained model over a 68-word vocabulary: near-uniform


def test_rows_are_appended_to_a_sheet_through_a_fake_client():
    from olmo_b200.eval.offline import append_rows_to_gsheet, merge_sheet_rows

    class Sheet:
        def __init__(self, title):
            self.title, self.cells = title, []

        def get_all_values(self):
            return [list(r) for r in self.cells] + [["", ""]]  # a real sheet pads with empty rows

        def update_values(self, where, table):
            assert where == "A1"
            self.cells = [list(r) for r in table]

    class Book:
        def __init__(self):
            self.sheets = [Sheet("Sheet1")]

        def worksheets(self):
            return self.sheets

        def add_worksheet(self, title, rows, cols):
            self.sheets.append(Sheet(title))

        def worksheet_by_title(self, title):
            return next(s for s in self.sheets if s.title == title)

    class Client:
        def __init__(self):
            self.books = {}

        def open(self, name):
            return self.books.setdefault(name, Book())

    client = Client()
    assert append_rows_to_gsheet("results", [{"task": "piqa", "metric_acc": 0.5}], client=client) == 1
    assert append_rows_to_gsheet("results", [{"task": "arc", "metric_f1": 0.25, "limit": None}], client=client) == 2
    cells = client.books["results"].worksheet_by_title("Sheet1").cells
    assert cells[0] == ["date", "task", "metric_acc", "metric_f1", "limit"]
    assert cells[1][1:] == ["piqa", 0.5, "", ""] and cells[2][1:] == ["arc", "", 0.25, ""]
    assert append_rows_to_gsheet("results", [{"task": "x"}], sheet_title="ppl", client=client) == 1
    assert [s.title for s in client.books["results"].worksheets()] == ["Sheet1", "ppl"]
    assert merge_sheet_rows([], [{"a": 1}]) == [["a"], [1]]


def test_generation_metrics_and_task(tmp_path, eval_model, monkeypatch):
    assert offline.exact_match("The Eiffel Tower.", ["eiffel tower"]) == 1.0 and offline.exact_match("a tower", ["eiffel tower"]) == 0.0
    assert offline.token_f1("the big red dog", ["red dog", "cat"]) == pytest.approx(2 * (2 / 3) * 1.0 / (2 / 3 + 1.0))
    assert offline.token_f1("", ["x"]) == 0.0 and offline.token_f1("", [""]) == 1.0
    # longest common subsequence "quick fox jumps" (3 words) of 4 predicted and 5 reference words
    assert offline.rouge_l("quick brown fox jumps", ["the quick lazy fox often jumps"]) == pytest.approx(2 * (3 / 4) * (3 / 5) / (3 / 4 + 3 / 5))

    data = tmp_path / "gen" / "toy"
    data.mkdir(parents=True)
    rows = [{"input": f"what follows {w}", "answers": [w[::-1], "other"]} for w in ("abc", "def", "ghi", "jkl")]
    with gzip.open(data / "validation.jsonl.gz", "wt") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
    monkeypatch.setenv("EVAL_DATA_PATH", str(tmp_path))
    task = offline.construct_task("gen", eval_model.tokenizer, {"files": ["gen/toy"], "max_new_tokens": 4, "template": "{input} ->"})
    assert isinstance(task, offline.GenerationTask) and len(task.examples()) == 4

    prompts = []

    def oracle(prompt_ids, max_new_tokens):  # answers every question correctly except the last, and keeps talking after a newline
        prompt = eval_model.tokenizer.decode(list(prompt_ids))
        prompts.append(prompt)
        word = prompt.rsplit("what follows ", 1)[1].split(" ->")[0]
        return (" " + word[::-1] if word != "jkl" else " nope") + "\nextra text"

    monkeypatch.setattr(eval_model, "generate_text", oracle)
    out = offline.predict_and_calculate_metrics(eval_model, task, {"num_shots": 2, "fewshot_seed": 5, "num_recorded_inputs": 1})
    assert out["num_instances"] == 4 and out["metrics"]["exact_match"] == 0.75 and out["metrics"]["f1"] == 0.75 and out["metrics"]["rouge_l"] == 0.75
    full = out["recorded_inputs"][0]["prompt"]  # what the model is shown is the tail of this that fits its context
    assert full.count("->") == 3 and full.endswith("what follows abc ->") and prompts[0] == full[-len(prompts[0]):]
    assert "what follows abc" not in full.rsplit("\n\n", 1)[0]  # the question itself is never one of its own examples
    assert out["recorded_inputs"][0]["prediction"] == "cba"
    limited = offline.predict_and_calculate_metrics(eval_model, task, {"limit": 2})
    assert limited["num_instances"] == 2 and limited["metrics"]["exact_match"] == 1.0

    # the real generation path of a model wrapper: greedy continuation, decoded, bounded
    monkeypatch.undo()
    text = eval_model.generate_text(eval_model.tokenizer.encode("abc", add_special_tokens=False), 5)
    assert isinstance(text, str) and len(eval_model.tokenizer.encode(text, add_special_tokens=False)) <= 5


def test_reference_named_task_sets_resolve():
    for name in ("rc20_tasks", "gen_tasks", "summary_tasks", "eval_suite_ppl_val_v3", "eval_suite_ppl_val_v3_small", "eval_suite_ppl_val_v2_small"):
        resolved = offline.resolve_task_set(name)
        assert resolved["tasks"] and all("task_name" in t for t in resolved["tasks"]), name
    assert len(offline.resolve_task_set("eval_suite_ppl_val_v3")["tasks"]) == 17
    from olmo_b200.eval.downstream import label_to_task_map

    assert all(t["task_name"] in label_to_task_map for t in offline.resolve_task_set("rc20_tasks")["tasks"])
    spec = offline.load_experiment(str(offline.TASK_SET_DIR.parent / "experiments" / "evaluation_2023_07_26.yaml"))
    assert [ts["name"] for ts in spec["task_sets"]] == ["rc20_tasks", "gen_tasks", "summary_tasks", "eval_suite_ppl_val_v2_small"]


def test_generation_metrics_against_brute_force():
    """Property test: ROUGE-L's longest common subsequence equals an exhaustive search over subsequences, word F1 equals
    the multiset-overlap definition, both are symmetric in their F-measure, 1 on identical texts and 0 on disjoint ones."""
    from itertools import combinations

    from hypothesis import given, settings
    from hypothesis import strategies as st

    from olmo_b200.eval.offline import exact_match, rouge_l, token_f1

    words = st.lists(st.sampled_from(["red", "green", "blue", "cat", "dog"]), min_size=0, max_size=7)

    def lcs_brute(a, b):
        for n in range(min(len(a), len(b)), 0, -1):
            subs = {tuple(a[i] for i in idx) for idx in combinations(range(len(a)), n)}
            if any(tuple(b[i] for i in idx) in subs for idx in combinations(range(len(b)), n)):
                return n
        return 0

    def f(p, r):
        return 0.0 if p == 0 or r == 0 else 2 * p * r / (p + r)

    @settings(max_examples=120, deadline=None)
    @given(a=words, b=words)
    def check(a, b):
        ta, tb = " ".join(a), " ".join(b)
        got = rouge_l(ta, [tb])
        want = f(lcs_brute(a, b) / len(a), lcs_brute(a, b) / len(b)) if a and b else 0.0
        assert got == pytest.approx(want)
        assert rouge_l(tb, [ta]) == pytest.approx(got)
        overlap = sum(min(a.count(w), b.count(w)) for w in set(a))
        want_f1 = float(a == b) if not a or not b else f(overlap / len(a), overlap / len(b))
        assert token_f1(ta, [tb]) == pytest.approx(want_f1) and token_f1(tb, [ta]) == pytest.approx(want_f1)
        assert token_f1(ta, [tb]) >= rouge_l(ta, [tb]) - 1e-12  # a subsequence is also a multiset overlap
        if a:
            assert rouge_l(ta, [ta]) == 1.0 and token_f1(ta, ["The " + ta + "."]) == 1.0 and exact_match(ta.upper() + "!", [ta]) == 1.0
        assert rouge_l(ta, [tb, ta]) >= got  # the best reference counts

    check()
