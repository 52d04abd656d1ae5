"""Downstream (in-context) evaluation: request construction, padding, task table and metrics."""
import gzip
import json
import math

import pytest
import torch

from olmo_b200.eval.downstream import (
    MMLU,
    PIQA,
    ArcEasy,
    ArcEasyCELoss,
    COPA,
    HellaSwag,
    OEEvalTask,
    WinoGrande,
    label_to_task_map,
    list_tasks,
)
from olmo_b200.eval.metrics import ICLMetric

datasets = pytest.importorskip("datasets")


class CharTokenizer:
    """One token per character; id = code point.  Enough to make request arithmetic checkable."""

    pad_token_id = 0
    eos_token_id = 1

    def encode(self, s, add_special_tokens=True):
        return [ord(c) for c in s] + ([self.eos_token_id] if add_special_tokens else [])

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(i) for i in ids if i > 1)


def store(root, path, name, split, rows):
    datasets.Dataset.from_list(rows).save_to_disk(str(root / "hf_datasets" / path / (name or "none") / split))


@pytest.fixture()
def data_root(tmp_path, monkeypatch):
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))
    return tmp_path


def test_piqa_requests_and_collation(data_root):
    rows = [
        {"goal": "open a jar", "sol1": "twist the lid", "sol2": "hit it", "label": 0},
        {"goal": "boil water", "sol1": "freeze it", "sol2": "heat the pot until it bubbles", "label": 1},
    ]
    store(data_root, "piqa", "plain_text", "validation", rows)
    task = PIQA(CharTokenizer())
    assert len(task) == 4 and task.metric_type == "len_norm"
    s = task[1]
    ctx = "Question: open a jar\nAnswer:"
    assert s["doc_id"] == 0 and s["cont_id"] == 1 and s["label_id"] == 0
    assert s["ctx"] == [ord(c) for c in ctx]
    assert s["continuation"] == [ord(c) for c in " hit it"]
    assert s["query"] == [ord(c) for c in ctx + " hit i"]  # last continuation token is never fed
    assert s["ctx_len"] == len(ctx) and s["cont_len"] == 7 and s["cont_str_len"] == 6 and s["cont_byte_len"] == 6
    assert s["dc_query"] == [ord(c) for c in "Answer: hit i"] and s["dc_len"] == 7

    batch = task.collate_fn([task[i] for i in range(4)])
    widest = max(len(task[i]["query"]) for i in range(4))
    assert batch["input_ids"].shape == (4, widest)
    assert batch["input_ids"][0, len(task[0]["query"]) :].eq(0).all()
    assert batch["label_id"].tolist() == [0, 0, 1, 1]
    assert batch["doc_id"].tolist() == [0, 0, 1, 1] and batch["cont_id"].tolist() == [0, 1, 0, 1]
    for key in ("ctx", "continuation", "dc_input_ids", "ctx_len", "dc_len", "cont_len", "cont_str_len", "cont_byte_len"):
        assert key in batch


def test_context_truncation_keeps_the_tail(data_root):
    store(data_root, "piqa", "plain_text", "validation", [{"goal": "x" * 100, "sol1": "abc", "sol2": "de", "label": 0}])
    task = PIQA(CharTokenizer(), model_ctx_len=32)
    s = task[0]
    assert len(s["query"]) == 32
    assert s["ctx_len"] == 32 - len(" abc") + 1
    assert task.pad_tokens_until_max(list(range(40)), max_len=50) == list(range(8, 40))
    assert task.pad_tokens_until_max([5, 6], max_len=40) == [5, 6] + [0] * 30  # padding is capped at the context length


def test_metric_picks_most_likely_continuation(data_root):
    rows = [{"goal": "g", "sol1": "aa", "sol2": "bb", "label": 1}, {"goal": "h", "sol1": "cc", "sol2": "dd", "label": 0}]
    store(data_root, "piqa", "plain_text", "validation", rows)
    task = PIQA(CharTokenizer(), metric_type="acc")
    batch = task.collate_fn([task[i] for i in range(4)])
    vocab = 128
    logits = torch.zeros(4, batch["input_ids"].shape[1], vocab)
    # favour the characters 'b' and 'c' everywhere: docs are then answered "bb" (right) and "cc" (right)
    logits[..., ord("b")] = 5.0
    logits[..., ord("c")] = 5.0
    metric = ICLMetric("acc")
    metric.update(batch, logits)
    assert float(metric.compute()) == pytest.approx(1.0)
    metric = ICLMetric("acc")
    logits = torch.zeros_like(logits)
    logits[..., ord("a")] = 5.0  # doc 0 answered "aa" (wrong); doc 1 is a tie resolved to index 0 (right)
    metric.update(batch, logits)
    assert float(metric.compute()) == pytest.approx(0.5)

    ce = ICLMetric("ce_loss")
    uniform = torch.zeros(4, batch["input_ids"].shape[1], vocab)
    ce_batch = {k: v for k, v in batch.items()}
    ce_batch["label_id"] = torch.zeros(4, dtype=torch.long)
    ce_batch["cont_id"] = torch.zeros(4, dtype=torch.long)
    ce_batch["doc_id"] = torch.arange(4)
    ce.update(ce_batch, uniform)
    # three continuation tokens each with probability 1/vocab, normalised by the two characters after the blank
    assert float(ce.compute()) == pytest.approx(3 * math.log(vocab) / 2, rel=1e-5)


def test_prompt_formats(data_root):
    store(
        data_root, "hellaswag", None, "validation",
        [{"activity_label": "Baking", "ctx_a": "A man [header] mixes.", "ctx_b": "he", "endings": ["stirs  more.", "leaves [step] now."], "label": "1"}],
    )
    h = HellaSwag(CharTokenizer())
    doc = h.dataset[0]
    assert h.doc_to_text(doc) == "Baking: A man mixes. He"
    assert h.doc_to_continuations(doc) == [" stirs more.", " leaves now."]
    assert h.doc_to_label(doc) == 1 and h.doc_to_domain_conditional(doc) == "He"

    store(data_root, "winogrande", "winogrande_xl", "validation", [{"sentence": "Ann told Bea that _ was late.", "option1": "Ann", "option2": "Bea", "answer": "2"}])
    w = WinoGrande(CharTokenizer())
    assert len(w) == 2
    assert [w.tokenizer.decode(s["ctx"]) for s in w.samples] == ["Ann told Bea that Ann", "Ann told Bea that Bea"]
    assert w.tokenizer.decode(w[0]["continuation"]) == " was late."
    assert w[0]["continuation"] == w[1]["continuation"] and w[0]["label_id"] == 1
    assert [w.tokenizer.decode(s["dc_query"]) for s in w.samples] == ["Ann was late", "Bea was late"]

    store(data_root, "super_glue", "copa", "validation", [{"premise": "It rained.", "choice1": "The grass is wet.", "choice2": "I slept.", "question": "effect", "label": 0}])
    c = COPA(CharTokenizer())
    doc = c.dataset[0]
    assert c.doc_to_text(doc) == "It rained therefore" and c.doc_to_continuations(doc) == [" the grass is wet.", " i slept."]

    arc_rows = [
        {"question": "2+2?", "choices": {"text": ["3", "4", "5"], "label": ["A", "B", "C"]}, "answerKey": "B"},
        {"question": "1+1?", "choices": {"text": ["2", "3", "4"], "label": ["1", "2", "3"]}, "answerKey": "1"},
    ]
    store(data_root, "ai2_arc", "ARC-Easy", "validation", arc_rows)
    a = ArcEasy(CharTokenizer())
    assert [a.doc_to_label(d) for d in a.dataset] == [1, 0]
    p = ArcEasyCELoss(CharTokenizer())
    assert len(p) == 2 and p.tokenizer.decode(p[0]["continuation"]) == " 4" and p[1]["label_id"] == 0


def test_mmlu_variants(data_root):
    q = {"question": " What is 1+1? ", "subject": "abstract_algebra", "choices": ["1", "2", "3", "4"], "answer": 1}
    dev = [{"question": f"dev {i}?", "subject": "abstract_algebra", "choices": ["a", "b", "c", "d"], "answer": i % 4} for i in range(5)]
    for subject in MMLU.subjects_for("math"):
        store(data_root, "hails/mmlu_no_train", subject, "validation", [dict(q, subject=subject)])
        store(data_root, "hails/mmlu_no_train", subject, "dev", [dict(d, subject=subject) for d in dev])
    plain = MMLU(CharTokenizer(), dataset_name="math")
    assert len(plain) == 5 * 4
    assert plain.tokenizer.decode(plain[0]["ctx"]) == "Question: What is 1+1?\nAnswer:"
    var = MMLU(CharTokenizer(), dataset_name="abstract_algebra", prompt_variations=1)
    assert len(var) == 7 * 4
    texts = [var.tokenizer.decode(var[i * 4]["ctx"]) for i in range(7)]
    assert texts[1].startswith("The following are multiple choice questions (with answers) about abstract algebra:\n\nQuestion: What")
    assert texts[3].count("Question:") == 3 and "Question: dev 0?\nAnswer: a\n\n" in texts[3]
    mc = MMLU(CharTokenizer(), dataset_name="abstract_algebra", prompt_variations=2, mc_labels=True)
    assert len(mc) == 4
    text = mc.tokenizer.decode(mc[0]["ctx"])
    assert text.endswith("What is 1+1?\nA. 1\nB. 2\nC. 3\nD. 4\nAnswer:") and "dev 4?\nA. a\nB. b\nC. c\nD. d\nAnswer: A\n\n" in text
    assert [mc.tokenizer.decode(s["continuation"]) for s in mc.samples] == [" A", " B", " C", " D"]
    bpb = MMLU(CharTokenizer(), dataset_name="abstract_algebra", metric_type="bpb")
    assert len(bpb) == 1 and bpb.tokenizer.decode(bpb[0]["continuation"]) == " 2" and bpb[0]["label_id"] == 0
    with pytest.raises(ValueError):
        MMLU(CharTokenizer(), dataset_name="abstract_algebra", prompt_variations=3)
    assert set(MMLU.subjects_for("stem")) >= set(MMLU.subjects_for("math"))
    assert sum(len(MMLU.subjects_for(g)) for g in ("stem", "humanities", "social_sciences", "other")) == 57


def test_oe_eval_request_dump(data_root):
    folder = data_root / "oe_eval_tasks" / "toy" / "rc_0shot"
    folder.mkdir(parents=True)
    (folder / "config.json").write_text(json.dumps({"task_config": {"split": "validation", "primary_metric": "acc_per_char"}}))
    reqs = []
    for doc_id in range(3):
        for idx in range(2):
            reqs.append(
                {
                    "request_type": "loglikelihood", "doc_id": doc_id, "idx": idx, "label": doc_id % 2, "doc": {},
                    "request": {"context": f"Q{doc_id}:", "continuation": f" ans{idx}"},
                }
            )
    reqs.append({"request_type": "loglikelihood", "doc_id": 1000001, "idx": 0, "label": 0, "doc": {}, "request": {"context": "", "continuation": " x"}})
    with gzip.open(folder / "requests.jsonl.gz", "wt") as f:
        f.write("\n".join(json.dumps(r) for r in reqs))
    task = OEEvalTask(CharTokenizer(), dataset_path="toy", dataset_name="rc_0shot")
    assert task.metric_type == "len_norm" and len(task) == 6
    assert task[3]["doc_id"] == 1 and task[3]["cont_id"] == 1 and task[3]["label_id"] == 1
    single = OEEvalTask(CharTokenizer(), dataset_path="toy", dataset_name="rc_0shot", metric_type="bpb")
    assert len(single) == 3 and all(s["cont_id"] == 0 and s["label_id"] == 0 for s in single.samples)
    assert [single.tokenizer.decode(s["continuation"]) for s in single.samples] == [" ans0", " ans1", " ans0"]
    # two dumps concatenated: document ids of the second are shifted past the first
    both = OEEvalTask(CharTokenizer(), dataset_path="toy", dataset_name=["rc_0shot", "rc_0shot"], metric_type="acc")
    assert len(both) == 12 and both[6]["doc_id"] == 2  # offset = highest id of the first dump


def test_task_table_is_complete():
    labels = list_tasks()
    assert len(labels) == 242
    for must in ("piqa", "mmlu_stem_var_bpb", "mmlu_other_test_mc_5shot_bpb", "arc_easy_rc_0shot", "winogrande_val_rc_5shot_bpb", "gsm8k_gold_bpb_5shot", "copycolors_xl_10way_bpb"):
        assert must in label_to_task_map
    cls, kwargs = label_to_task_map["arc_easy_rc_0shot"]
    assert cls is OEEvalTask and kwargs == {"dataset_path": "arc_easy", "dataset_name": "rc_0shot", "metric_type": "acc"}
    cls, kwargs = label_to_task_map["arc_easy_test_rc_5shot"]
    assert kwargs["metric_type"] == "len_norm"
    assert "gsm8k_gold_bpb_5shot_bpb" not in label_to_task_map
