"""
Offline evaluation pipeline: every model of an experiment is scored on every task of every task set, each
(model, task) result is cached in a workspace folder, and the results are written as rows.

This is the role of the reference's ``evaluation/`` folder, which wires third-party workflow and task libraries
together (``evaluation/steps/run_catwalk.py:25-351``: build the task, build the model, predict and compute metrics,
post-process, write rows; ``evaluation/experiments/utils.libsonnet``: the models × task-sets cross product).  Here the
steps are plain functions over this framework's own model, tokenizer and task classes, and an experiment is a YAML
file:

    workspace: runs/eval-workspace
    output: runs/eval-rows.jsonl            # also written next to it as .tsv
    wandb: {project: ..., entity: ..., name: ...}   # optional
    models:
      - model_path: /checkpoints/step1000-unsharded
        prediction_kwargs: {limit: 500}    # overrides the task sets' values for this model
    task_sets:
      - rc_tasks                            # a name under evaluation/task_sets/, or an inline mapping
      - name: my_ppl
        tasks:
          - {task_name: ppl, task_kwargs: {files: [/data/val.jsonl.gz]}, prediction_kwargs: {model_max_length: 2048}}

Three task kinds exist.  A *generation* task (``gen``) reads prompts and reference answers from ``.jsonl[.gz]`` files, continues
each prompt greedily (optionally after ``num_shots`` examples) and reports ``exact_match``, ``f1`` and ``rouge_l``.
A *ranked-classification* task is any label of
:data:`olmo_b200.eval.downstream.label_to_task_map` and reports that task's metric.  A *perplexity* task (``ppl``) reads
documents from ``.jsonl[.gz]`` files with a ``text`` field, or token ids from ``.npy`` memmaps, and reports
``ppl_token``, ``ppl_char``, ``ppl_word``, ``ppl_byte`` and ``bits_per_byte``.
"""
from __future__ import annotations

import gzip
import hashlib
import json
import logging
import math
import os
import string
import time
from collections import Counter
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, Iterator, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

log = logging.getLogger(__name__)

__all__ = [
    "EvalModel", "load_experiment", "resolve_task_set", "construct_task", "predict_and_calculate_metrics", "run_experiment",
    "write_rows", "merge_sheet_rows", "append_rows_to_gsheet", "TASK_SET_DIR", "GenerationTask", "PerplexityTask", "exact_match",
    "token_f1", "rouge_l",
]

#: task-set files shipped with the repository (``<repo>/evaluation/task_sets/*.yaml``)
TASK_SET_DIR = Path(__file__).resolve().parent.parent.parent / "evaluation" / "task_sets"


# --------------------------------------------------------------------------------------------- model
@dataclass
class EvalModel:
    """A loaded model with its tokenizer.  ``model_path`` is a native checkpoint folder (sharded or unsharded)."""

    model_path: str
    model: Any
    tokenizer: Any
    device: torch.device

    @classmethod
    def load(cls, model_path: str, device: Optional[str] = None, dtype: Optional[str] = None, tokenizer: Optional[str] = None) -> "EvalModel":
        from ..models.olmo import OLMo
        from ..tokenizer import Tokenizer

        dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
        model = OLMo.from_checkpoint(model_path, device="cpu")
        dtype = dtype or ("bf16" if dev.type == "cuda" else "fp32")
        model = model.to({"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]).to(dev).eval()
        if tokenizer is None:
            tok = Tokenizer.from_checkpoint(model_path)
        else:
            tok = Tokenizer.from_file(tokenizer) if tokenizer.endswith(".json") else Tokenizer.from_pretrained(tokenizer)
        return cls(model_path, model, tok, dev)

    @property
    def max_length(self) -> int:
        return self.model.config.max_sequence_length

    @torch.no_grad()
    def generate_text(self, prompt_ids: Sequence[int], max_new_tokens: int) -> str:
        """Greedy continuation of one prompt, decoded, cut at the end-of-text token."""
        ids = torch.tensor([list(prompt_ids)], dtype=torch.long, device=self.device)
        out = self.model.generate(ids, max_steps=max_new_tokens, beam_size=1).token_ids[0, 0].tolist()
        eos = self.tokenizer.eos_token_id
        if eos in out:
            out = out[: out.index(eos)]
        return self.tokenizer.decode(out)

    @torch.no_grad()
    def logits(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.model(input_ids.to(self.device), attention_mask=None if attention_mask is None else attention_mask.to(self.device)).logits


# ------------------------------------------------------------------------------------- configuration
def _read_yaml(path: Path) -> Any:
    import yaml

    with open(path) as f:
        return yaml.safe_load(f)


def resolve_task_set(entry: Any, search: Sequence[Path] = ()) -> Dict[str, Any]:
    """A task set is ``{name, tasks: [{task_name, task_kwargs?, prediction_kwargs?}]}``; a string names a YAML file."""
    if isinstance(entry, str):
        for folder in list(search) + [TASK_SET_DIR]:
            for candidate in (folder / entry, folder / f"{entry}.yaml"):
                if candidate.is_file():
                    entry = _read_yaml(candidate)
                    break
            if not isinstance(entry, str):
                break
        else:
            raise FileNotFoundError(f"task set '{entry}' not found under {[str(p) for p in list(search) + [TASK_SET_DIR]]}")
    if "task_names" in entry:  # short form: the same kwargs for a list of labels
        shared = {k: entry.get(k, {}) for k in ("task_kwargs", "prediction_kwargs")}
        entry = {"name": entry["name"], "tasks": [{"task_name": t, **json.loads(json.dumps(shared))} for t in entry["task_names"]]}
    for task in entry["tasks"]:
        task.setdefault("task_kwargs", {})
        task.setdefault("prediction_kwargs", {})
    return entry


def load_experiment(path: str) -> Dict[str, Any]:
    file = Path(path)
    spec = _read_yaml(file)
    if not spec.get("models") or not spec.get("task_sets"):
        raise ValueError("an experiment needs 'models' and 'task_sets'")
    spec["task_sets"] = [resolve_task_set(t, search=[file.parent, file.parent / "task_sets"]) for t in spec["task_sets"]]
    spec["models"] = [{"model_path": m} if isinstance(m, str) else dict(m) for m in spec["models"]]
    return spec


# --------------------------------------------------------------------------------------------- tasks
@dataclass
class PerplexityTask:
    """Documents from text or token files, scored in disjoint windows of ``model_max_length`` tokens, each window
    conditioned on the end-of-text token."""

    files: Sequence[str]
    text_field: str = "text"
    memmap_dtype: str = "uint16"
    name: str = "ppl"

    def documents(self, tokenizer) -> Iterator[Tuple[List[int], str]]:
        import numpy as np

        for file in _data_files(self.files):
            if str(file).endswith(".npy"):
                tokens = np.memmap(file, dtype=getattr(np, self.memmap_dtype), mode="r")
                eos = tokenizer.eos_token_id
                start = 0
                for end in list(np.nonzero(tokens == eos)[0]) + [len(tokens)]:
                    ids = tokens[start:end].astype(np.int64).tolist()
                    start = end + 1
                    if ids:
                        yield ids, tokenizer.decode(ids)
            else:
                opener = gzip.open if str(file).endswith(".gz") else open
                with opener(file, "rt", encoding="utf-8") as f:
                    for line in f:
                        if line.strip():
                            text = json.loads(line)[self.text_field]
                            yield tokenizer.encode(text, add_special_tokens=False), text


def _expand(path: str) -> str:
    """``$EVAL_DATA_PATH/...`` and ``~`` in task files; a relative path is taken below ``EVAL_DATA_PATH`` when that is set
    and the file exists there (how the reference's perplexity suites locate their data)."""
    expanded = os.path.expanduser(os.path.expandvars(str(path)))
    root = os.environ.get("EVAL_DATA_PATH")
    if root and not os.path.isabs(expanded) and not os.path.exists(expanded):
        for candidate in (os.path.join(root, expanded), os.path.join(root, expanded + ".jsonl.gz"), os.path.join(root, expanded + ".jsonl")):
            if os.path.exists(candidate):
                return candidate
    return expanded


def _data_files(paths: Sequence[str]) -> List[str]:
    """Every data file named by a task: a path may be a file or a folder of ``.jsonl[.gz]`` / ``.npy`` files."""
    out: List[str] = []
    for path in paths:
        path = _expand(path)
        if os.path.isdir(path):
            out += sorted(os.path.join(path, n) for n in os.listdir(path) if n.endswith((".jsonl", ".jsonl.gz", ".json.gz", ".npy")))
        else:
            out.append(path)
    return out


def _normalise_answer(text: str) -> str:
    """Lower case, no punctuation, no articles, single spaces (the usual normalisation of reading-comprehension scoring)."""
    text = "".join(ch for ch in text.lower() if ch not in string.punctuation)
    return " ".join(w for w in text.split() if w not in ("a", "an", "the"))


def exact_match(prediction: str, answers: Sequence[str]) -> float:
    return float(any(_normalise_answer(prediction) == _normalise_answer(a) for a in answers))


def token_f1(prediction: str, answers: Sequence[str]) -> float:
    """Best bag-of-words F1 against any reference answer."""
    best = 0.0
    pred = _normalise_answer(prediction).split()
    for answer in answers:
        gold = _normalise_answer(answer).split()
        common = sum((Counter(pred) & Counter(gold)).values())
        if not pred or not gold:
            best = max(best, float(pred == gold))
        elif common:
            precision, recall = common / len(pred), common / len(gold)
            best = max(best, 2 * precision * recall / (precision + recall))
    return best


def rouge_l(prediction: str, answers: Sequence[str]) -> float:
    """Best ROUGE-L F-measure (longest common subsequence of words) against any reference."""
    best = 0.0
    pred = _normalise_answer(prediction).split()
    for answer in answers:
        gold = _normalise_answer(answer).split()
        if not pred or not gold:
            continue
        row = [0] * (len(gold) + 1)
        for p_word in pred:
            prev = 0
            for j, g_word in enumerate(gold, start=1):
                cur = row[j]
                row[j] = prev + 1 if p_word == g_word else max(row[j], row[j - 1])
                prev = cur
        lcs = row[-1]
        if lcs:
            precision, recall = lcs / len(pred), lcs / len(gold)
            best = max(best, 2 * precision * recall / (precision + recall))
    return best


@dataclass
class GenerationTask:
    """Free-form answers: every line of ``files`` holds a prompt (``input_field``) and one or more reference answers
    (``answer_field``: a string or a list).  ``num_shots`` examples drawn with ``fewshot_seed`` from the same files are put in
    front of every prompt; the model continues greedily up to ``max_new_tokens`` or the first ``stop`` string.  Metrics:
    exact match, word F1 and ROUGE-L (question answering and summarisation suites of the reference, ``gen_tasks`` and
    ``summary_tasks``, run through generation the same way)."""

    files: Sequence[str]
    input_field: str = "input"
    answer_field: str = "answers"
    template: str = "{input}\nAnswer:"
    separator: str = "\n\n"
    max_new_tokens: int = 32
    stop: Sequence[str] = ("\n",)
    name: str = "gen"

    def examples(self) -> List[Tuple[str, List[str]]]:
        rows = []
        for file in _data_files(self.files):
            opener = gzip.open if str(file).endswith(".gz") else open
            with opener(file, "rt", encoding="utf-8") as f:
                for line in f:
                    if line.strip():
                        rec = json.loads(line)
                        answers = rec[self.answer_field]
                        rows.append((str(rec[self.input_field]), [answers] if isinstance(answers, str) else [str(a) for a in answers]))
        return rows


def construct_task(task_name: str, tokenizer, task_kwargs: Optional[Dict[str, Any]] = None, model_max_length: Optional[int] = None):
    """Build the task object: a :class:`PerplexityTask` for ``ppl``, else the labelled multiple-choice dataset."""
    task_kwargs = dict(task_kwargs or {})
    if task_name == "ppl":
        return PerplexityTask(**task_kwargs)
    if task_name == "gen":
        return GenerationTask(**task_kwargs)
    from .downstream import label_to_task_map

    if task_name not in label_to_task_map:
        raise KeyError(f"unknown task '{task_name}'; ranked-classification labels: {sorted(label_to_task_map)[:8]}… or 'ppl'")
    entry = label_to_task_map[task_name]
    cls, fixed = entry if isinstance(entry, tuple) else (entry, {})
    kwargs = {**fixed, **task_kwargs}
    if model_max_length is not None:
        kwargs.setdefault("model_ctx_len", model_max_length)
    return cls(tokenizer=tokenizer, **kwargs)


def _score_perplexity(model: EvalModel, task: PerplexityTask, limit: Optional[int], max_length: int, batch_size: int) -> Dict[str, Any]:
    eos = model.tokenizer.eos_token_id
    totals = {"logprob": 0.0, "tokens": 0, "chars": 0, "words": 0, "bytes": 0, "documents": 0}
    windows: List[List[int]] = []

    def flush() -> None:
        if not windows:
            return
        width = max(len(w) for w in windows)
        ids = torch.full((len(windows), width), model.model.config.pad_token_id, dtype=torch.long)
        mask = torch.zeros(len(windows), width)
        for i, w in enumerate(windows):  # right padding: causal attention never looks at it
            ids[i, : len(w)] = torch.tensor(w)
            mask[i, : len(w)] = 1
        logp = F.log_softmax(model.logits(ids).float(), dim=-1).cpu()
        gathered = logp[:, :-1].gather(2, ids[:, 1:].unsqueeze(-1)).squeeze(-1)
        totals["logprob"] += float((gathered * mask[:, 1:]).sum())
        windows.clear()

    for n, (ids, text) in enumerate(task.documents(model.tokenizer)):
        if limit is not None and n >= limit:
            break
        totals["documents"] += 1
        totals["tokens"] += len(ids)
        totals["chars"] += len(text)
        totals["words"] += len(text.split())
        totals["bytes"] += len(text.encode("utf-8"))
        for start in range(0, len(ids), max_length - 1):
            windows.append([eos] + ids[start : start + max_length - 1])
            if len(windows) == batch_size:
                flush()
    flush()
    nll = -totals["logprob"]
    metrics = {f"ppl_{unit[:-1]}": math.exp(nll / max(1, totals[unit])) for unit in ("tokens", "chars", "words", "bytes")}
    metrics["bits_per_byte"] = nll / max(1, totals["bytes"]) / math.log(2)
    return {"metrics": metrics, "num_instances": totals["documents"], "num_tokens": totals["tokens"]}


def _score_ranked(model: EvalModel, task, limit: Optional[int], batch_size: int, num_recorded_inputs: int) -> Dict[str, Any]:
    from .metrics import ICLMetric

    metric = ICLMetric(metric_type=task.metric_type)
    doc_limit = None
    if limit is not None:  # keep whole documents: every continuation of the first ``limit`` documents
        doc_limit = sorted({int(task[i]["doc_id"]) for i in range(len(task))})[:limit]
        doc_limit = set(doc_limit)
    items = [task[i] for i in range(len(task)) if doc_limit is None or int(task[i]["doc_id"]) in doc_limit]
    recorded = []
    for start in range(0, len(items), batch_size):
        batch = task.collate_fn(items[start : start + batch_size])
        logits = model.logits(batch["input_ids"]).cpu()
        dc_logits = model.logits(batch["dc_input_ids"]).cpu() if task.metric_type == "pmi_dc" else None
        metric.update(batch, logits, dc_logits)
    for item in items[:num_recorded_inputs]:
        recorded.append({"query": model.tokenizer.decode(item["query"]), "continuation": model.tokenizer.decode(item["continuation"]),
                         "label_id": int(item["label_id"])})
    documents = len({int(it["doc_id"]) for it in items})
    return {"metrics": {task.metric_type: float(metric.compute())}, "num_instances": documents, "recorded_inputs": recorded}


def _score_generation(model: EvalModel, task: GenerationTask, limit: Optional[int], max_length: int, num_shots: int, fewshot_seed: int,
                      num_recorded_inputs: int) -> Dict[str, Any]:
    import random

    rows = task.examples()
    rng = random.Random(fewshot_seed)
    totals = {"exact_match": 0.0, "f1": 0.0, "rouge_l": 0.0}
    recorded = []
    todo = rows if limit is None else rows[:limit]
    for n, (question, answers) in enumerate(todo):
        pool = [r for r in rows if r[0] != question]
        shots = rng.sample(pool, min(num_shots, len(pool))) if num_shots else []
        prompt = task.separator.join([task.template.format(input=q) + " " + a[0] for q, a in shots] + [task.template.format(input=question)])
        ids = model.tokenizer.encode(prompt, add_special_tokens=False)
        room = max(1, min(task.max_new_tokens, max_length - 1))
        ids = ids[-(max_length - room):]  # keep the end of an over-long prompt: the question is there
        text = model.generate_text(ids, room)
        cuts = [text.index(s) for s in task.stop if s and s in text]
        text = (text[: min(cuts)] if cuts else text).strip()
        totals["exact_match"] += exact_match(text, answers)
        totals["f1"] += token_f1(text, answers)
        totals["rouge_l"] += rouge_l(text, answers)
        if n < num_recorded_inputs:
            recorded.append({"prompt": prompt, "prediction": text, "answers": answers})
    count = max(1, len(todo))
    return {"metrics": {k: v / count for k, v in totals.items()}, "num_instances": len(todo), "recorded_inputs": recorded}


def predict_and_calculate_metrics(model: EvalModel, task, prediction_kwargs: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """Run one task.  Understood ``prediction_kwargs``: ``limit`` (documents), ``batch_size``, ``model_max_length``,
    ``num_recorded_inputs``, and for generation tasks ``num_shots`` and ``fewshot_seed``."""
    kw = dict(prediction_kwargs or {})
    limit = kw.get("limit")
    batch_size = int(kw.get("batch_size", 8))
    max_length = min(int(kw.get("model_max_length") or model.max_length), model.max_length)
    started = time.time()
    if isinstance(task, PerplexityTask):
        out = _score_perplexity(model, task, limit, max_length, batch_size)
    elif isinstance(task, GenerationTask):
        out = _score_generation(model, task, limit, max_length, int(kw.get("num_shots", 0)), int(kw.get("fewshot_seed", 1234)),
                                int(kw.get("num_recorded_inputs", 0)))
    else:
        out = _score_ranked(model, task, limit, batch_size, int(kw.get("num_recorded_inputs", 0)))
    out["processing_time"] = time.time() - started
    return out


# ------------------------------------------------------------------------------------------ pipeline
def _step_key(model_spec: Dict[str, Any], task: Dict[str, Any], prediction_kwargs: Dict[str, Any]) -> str:
    blob = json.dumps({"model": model_spec, "task": task["task_name"], "task_kwargs": task["task_kwargs"], "pred": prediction_kwargs},
                      sort_keys=True, default=str)
    return hashlib.sha256(blob.encode()).hexdigest()[:24]


def run_experiment(spec: Dict[str, Any], loader=EvalModel.load) -> List[Dict[str, Any]]:
    """The models × task-sets cross product.  A (model, task, kwargs) result found in the workspace is reused, so an
    interrupted or extended experiment only computes what is new.  Returns one row per (model, task set, task)."""
    workspace = Path(spec.get("workspace") or "eval-workspace")
    workspace.mkdir(parents=True, exist_ok=True)
    rows: List[Dict[str, Any]] = []
    for model_spec in spec["models"]:
        model: Optional[EvalModel] = None
        identity = {k: v for k, v in model_spec.items() if k not in ("prediction_kwargs", "gpus_needed")}
        for task_set in spec["task_sets"]:
            for task in task_set["tasks"]:
                pred = {**task["prediction_kwargs"], **model_spec.get("prediction_kwargs", {})}
                cache = workspace / f"{_step_key(identity, task, pred)}.json"
                if cache.is_file():
                    result = json.loads(cache.read_text())
                    log.info("reusing %s for %s / %s", cache.name, model_spec["model_path"], task["task_name"])
                else:
                    if model is None:
                        model = loader(**{k: v for k, v in identity.items() if k in ("model_path", "device", "dtype", "tokenizer")})
                    built = construct_task(task["task_name"], model.tokenizer, task["task_kwargs"], pred.get("model_max_length"))
                    result = predict_and_calculate_metrics(model, built, pred)
                    tmp = cache.with_suffix(".tmp")
                    tmp.write_text(json.dumps(result))
                    tmp.replace(cache)
                row = {
                    "model_path": model_spec["model_path"], "revision": model_spec.get("revision"), "task_set": task_set["name"],
                    "task": task.get("task_rename") or task["task_name"], "split": task["task_kwargs"].get("split"),
                    "limit": pred.get("limit"), "num_instances": result.get("num_instances"),
                    "processing_time": result.get("processing_time"), **{f"metric_{k}": v for k, v in result["metrics"].items()},
                }
                rows.append(row)
    if spec.get("output"):
        write_rows(rows, spec["output"])
    if spec.get("wandb"):
        _log_to_wandb(rows, spec["wandb"])
    if spec.get("gsheet"):
        append_rows_to_gsheet(spec["gsheet"], rows, sheet_title=spec.get("gsheet_title", "Sheet1"))
    return rows


def write_rows(rows: List[Dict[str, Any]], output: str) -> Tuple[Path, Path]:
    """JSON lines plus a tab-separated table with the union of all columns."""
    out = Path(output)
    out.parent.mkdir(parents=True, exist_ok=True)
    with open(out, "w") as f:
        for row in rows:
            f.write(json.dumps(row) + "\n")
    columns: List[str] = []
    for row in rows:
        columns += [c for c in row if c not in columns]
    table = out.with_suffix(".tsv")
    with open(table, "w") as f:
        f.write("\t".join(columns) + "\n")
        for row in rows:
            f.write("\t".join("" if row.get(c) is None else str(row[c]) for c in columns) + "\n")
    return out, table


def merge_sheet_rows(existing: List[List[Any]], rows: List[Dict[str, Any]]) -> List[List[Any]]:
    """The table (header row first) that results from appending ``rows`` to a sheet whose current cells are ``existing``.
    Columns the sheet has keep their position, new columns are added on the right, cells without a value are empty."""
    header = [str(c) for c in existing[0]] if existing and any(str(c) for c in existing[0]) else []
    body = [list(r) for r in existing[1:]] if header else []
    for row in rows:
        header += [c for c in row if c not in header]
    body = [r + [""] * (len(header) - len(r)) for r in body]
    for row in rows:
        body.append(["" if row.get(c) is None else row[c] for c in header])
    return [header] + body


def append_rows_to_gsheet(gsheet: str, rows: List[Dict[str, Any]], sheet_title: str = "Sheet1", client: Any = None) -> int:
    """Append result rows to the worksheet ``sheet_title`` of the Google spreadsheet named ``gsheet`` (created when it does not
    exist yet), stamping each row with the time of writing — the reference's ``write_to_gsheet``
    (``evaluation/steps/run_catwalk.py:354``).  ``client`` is a ``pygsheets`` client (anything with the same ``open`` /
    ``worksheets`` / ``add_worksheet`` / ``worksheet_by_title`` / ``get_all_values`` / ``update_values`` methods);
    by default one is authorised from the service-account file named by ``GDRIVE_SERVICE_ACCOUNT_JSON``.  Returns the number
    of data rows the worksheet holds afterwards."""
    import os
    from datetime import datetime, timezone

    if client is None:
        try:
            import pygsheets  # optional dependency: only needed when an experiment names a sheet
        except ImportError as e:
            raise RuntimeError("writing to a Google sheet needs the `pygsheets` package; results are still in the output files") from e
        if "GDRIVE_SERVICE_ACCOUNT_JSON" not in os.environ:
            raise RuntimeError("set GDRIVE_SERVICE_ACCOUNT_JSON to a service-account key file that may edit the sheet")
        client = pygsheets.authorize(service_account_json=os.environ["GDRIVE_SERVICE_ACCOUNT_JSON"])
    stamp = datetime.now(tz=timezone.utc).strftime("%Y-%m-%d %H:%M:%S UTC")
    stamped = [{"date": stamp, **row} for row in rows]
    book = client.open(gsheet)
    if sheet_title not in [w.title for w in book.worksheets()]:
        width = max((len(r) for r in stamped), default=1)
        book.add_worksheet(sheet_title, rows=len(stamped) + 1, cols=width)
    sheet = book.worksheet_by_title(sheet_title)
    existing = [r for r in sheet.get_all_values() if any(str(c) for c in r)]
    table = merge_sheet_rows(existing, stamped)
    sheet.update_values("A1", table)
    return len(table) - 1


def _log_to_wandb(rows: List[Dict[str, Any]], settings: Dict[str, Any]) -> None:
    """One summary entry per (task set, task, metric), as the reference's metrics step does (``evaluation/steps/wandb_metrics.py``)."""
    import wandb  # optional dependency: only needed when an experiment asks for it

    run = wandb.init(project=settings.get("project"), entity=settings.get("entity"), name=settings.get("name"), config={"rows": len(rows)})
    for row in rows:
        for key, value in row.items():
            if key.startswith("metric_"):
                run.summary[f"{row['task_set']}/{row['task']}/{key[7:]}"] = value
    run.finish()
