"""
In-context-learning evaluation tasks (rank-choice scoring of continuations).

Every task turns a document into one *context* string, several *continuation* strings (each with a
leading blank), the index of the gold continuation and a short *domain-conditional* prefix used by
the ``pmi_dc`` metric.  A request is ``context + continuation[:-1]`` (left-truncated to the model's
context length); the metric reads the log-probabilities of the continuation tokens from the
logits.  Prompt formats, dataset identifiers, metric choices and the ``label -> task`` table match
the reference's ``olmo/eval/downstream.py:168-2376`` so that scores are comparable.

Design: one generic dataset class builds, pads and collates requests; tasks are small subclasses
that only state their prompt format; the large family of pre-rendered request dumps (``OEEvalTask``)
and the MMLU variants are generated from compact tables instead of being listed one by one.
"""
from __future__ import annotations

import abc
import logging
import re
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple, Union

import torch

from ..util import load_hf_dataset, load_oe_eval_requests
from .metrics import ICLMetric

__all__ = [
    "ICLMetric",
    "ICLMultiChoiceTaskDataset",
    "OEEvalTask",
    "MMLU",
    "label_to_task_map",
    "list_tasks",
]

log = logging.getLogger(__name__)

# oe-eval's metric names -> the metric types ICLMetric understands
METRIC_FROM_OE_EVAL = {"acc_raw": "acc", "acc_per_char": "len_norm", "acc_uncond": "pmi_dc", "logits_per_byte": "bpb"}
_SINGLE_TARGET_METRICS = ("ce_loss", "bpb")  # scored on the gold continuation only

_INT_FIELDS = ("doc_id", "cont_id", "ctx_len", "dc_len", "cont_len", "cont_str_len", "cont_byte_len")
_SEQ_FIELDS = (("ctx", "ctx"), ("continuation", "continuation"), ("query", "input_ids"), ("dc_query", "dc_input_ids"))


def _as_name_list(name: Union[str, Sequence[Optional[str]], None]) -> List[Optional[str]]:
    return [name] if isinstance(name, str) or name is None else list(name)


class ICLMultiChoiceTaskDataset(metaclass=abc.ABCMeta):
    """
    Zero-shot multiple-choice task over a HuggingFace dataset stored in the packaged data tree.

    Subclasses set ``metric_type`` and implement ``doc_to_text`` / ``doc_to_continuations`` /
    ``doc_to_label`` (and optionally ``doc_to_domain_conditional``).  Items are dictionaries with
    token lists; :meth:`collate_fn` pads them into the batch format
    :class:`olmo_b200.eval.metrics.ICLMetric` consumes.
    """

    metric_type: str = None  # type: ignore[assignment]

    def __init__(
        self,
        tokenizer,
        dataset_path: str,
        dataset_name: Union[str, Sequence[str], None] = None,
        model_ctx_len: int = 2048,
        split: str = "validation",
        metric_type: Optional[str] = None,
        prompts: Sequence[Optional[str]] = (None,),
    ):
        self.tokenizer = tokenizer
        self.dataset_path = dataset_path
        self.dataset_name = dataset_name
        self.model_ctx_len = model_ctx_len
        self.prompts = list(prompts)
        self.current_prompt: Optional[str] = None
        if metric_type is not None:
            self.metric_type = metric_type
        self.log_instances = 0  # raise to log the first few rendered documents
        self.samples: List[Dict[str, Any]] = []
        self.dataset = self._load_documents(split)
        self.prep_examples()

    def _load_documents(self, split: str) -> Iterable[Dict[str, Any]]:
        parts = [load_hf_dataset(self.dataset_path, name, split) for name in _as_name_list(self.dataset_name)]
        if len(parts) == 1:
            return parts[0]
        import datasets

        return datasets.concatenate_datasets(parts)

    # -- dataset protocol ------------------------------------------------------------------------

    def __getitem__(self, index: int) -> Dict[str, Any]:
        return self.samples[index]

    def __len__(self) -> int:
        return len(self.samples)

    # -- request construction --------------------------------------------------------------------

    def token_encode(self, string: str) -> List[int]:
        return self.tokenizer.encode(string, add_special_tokens=False)

    def token_decode(self, tokens: List[int]) -> str:
        return self.tokenizer.decode(tokens)

    def _request(
        self, doc_id: int, cont_id: int, ctx: List[int], dc: List[int], continuation_str: str, label_id, *, ctx_len_from_query: bool = True
    ) -> Dict[str, Any]:
        """
        One scored request.  The model sees ``ctx + continuation[:-1]`` and its logits at the last
        ``len(continuation)`` positions predict the continuation tokens.
        """
        continuation = self.token_encode(continuation_str)
        query = (ctx + continuation[:-1])[-self.model_ctx_len :]
        return {
            "doc_id": doc_id,
            "cont_id": cont_id,
            "ctx": ctx,
            "continuation": continuation,
            # after left truncation fewer context tokens remain than len(ctx)
            "ctx_len": len(query) - len(continuation) + 1 if ctx_len_from_query else len(ctx),
            "dc_len": len(dc),
            "cont_len": len(continuation),
            "cont_str_len": len(continuation_str) - 1,  # without the leading blank
            "cont_byte_len": len(continuation_str[1:].encode("utf-8")),
            "query": query,
            "dc_query": dc + continuation[:-1],
            "label_id": label_id,
        }

    def _maybe_log(self, doc_text: str, continuations: Any) -> None:
        if self.log_instances > 0:
            self.log_instances -= 1
            name = self.dataset_name[0] if isinstance(self.dataset_name, list) else self.dataset_name
            log.info(
                "Sample doc from (%s, %s, %s):\ndoc_text: %s\ncontinuations: %s",
                self.dataset_path, name, self.current_prompt, doc_text, continuations,
            )

    def prep_examples(self) -> None:
        """All continuations of one (document, prompt variant) share a ``doc_id``."""
        doc_id = 0
        for doc in self.dataset:
            for prompt in self.prompts:
                self.current_prompt = prompt
                continuations = self.doc_to_continuations(doc)
                label_id = self.doc_to_label(doc)
                doc_text = self.doc_to_text(doc)
                ctx = self.token_encode(doc_text)
                dc = self.token_encode(self.doc_to_domain_conditional(doc))
                self._maybe_log(doc_text, continuations)
                for cont_id, continuation_str in enumerate(continuations):
                    self.samples.append(self._request(doc_id, cont_id, ctx, dc, continuation_str, label_id))
                doc_id += 1

    # -- batching --------------------------------------------------------------------------------

    def pad_tokens_until_max(self, tokens: List[int], max_len: int = 2048) -> List[int]:
        """Left-truncate to the context length, else right-pad to ``max_len`` (capped at the context length)."""
        if len(tokens) > self.model_ctx_len:
            return tokens[-self.model_ctx_len :]
        padded = tokens + [self.tokenizer.pad_token_id] * (max_len - len(tokens))
        return padded[: self.model_ctx_len]

    def collate_fn(self, data: List[Dict[str, Any]]) -> Dict[str, torch.Tensor]:
        batch: Dict[str, torch.Tensor] = {name: torch.tensor([s[name] for s in data], dtype=torch.long) for name in _INT_FIELDS}
        for field, out_name in _SEQ_FIELDS:
            width = max(len(s[field]) for s in data)
            batch[out_name] = torch.tensor([self.pad_tokens_until_max(s[field], max_len=width) for s in data], dtype=torch.long)
        labels = [s["label_id"] for s in data]
        if not any(isinstance(x, str) for x in labels):
            batch["label_id"] = torch.tensor(labels, dtype=torch.long)
        return batch

    # -- task format -----------------------------------------------------------------------------

    @abc.abstractmethod
    def doc_to_text(self, doc) -> str:
        raise NotImplementedError

    @abc.abstractmethod
    def doc_to_continuations(self, doc) -> List[str]:
        raise NotImplementedError

    @abc.abstractmethod
    def doc_to_label(self, doc) -> int:
        raise NotImplementedError

    def doc_to_domain_conditional(self, doc) -> str:
        return " "


class _Task(ICLMultiChoiceTaskDataset):
    """Task with fixed dataset coordinates (class attributes ``path`` / ``name``)."""

    path: str = ""
    name: Optional[str] = None

    def __init__(self, tokenizer, dataset_path: Optional[str] = None, dataset_name: Optional[str] = None, **kwargs):
        super().__init__(
            tokenizer=tokenizer,
            dataset_path=dataset_path if dataset_path is not None else self.path,
            dataset_name=dataset_name if dataset_name is not None else self.name,
            **kwargs,
        )


_ANSWER_DC = "Answer:"


def _detokenise_glue(s: str) -> str:
    """Undo PTB-style spacing in GLUE sentences."""
    for a, b in ((" n't", "n't"), (" )", ")"), ("( ", "("), ('" ', '"'), (' "', '"')):
        s = s.replace(a, b)
    return re.sub(r" (['.,])", r"\1", s)


class PIQA(_Task):
    """Physical commonsense: ``Question: GOAL\\nAnswer:`` -> two solutions."""

    metric_type, path, name = "len_norm", "piqa", "plain_text"

    def doc_to_text(self, doc):
        return f"Question: {doc['goal']}\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" " + doc["sol1"], " " + doc["sol2"]]

    def doc_to_label(self, doc):
        return doc["label"]

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class HellaSwag(_Task):
    """Sentence completion: ``ACTIVITY: CTX_A Ctx_b`` -> four endings (WikiHow brackets removed)."""

    metric_type, path, name = "len_norm", "hellaswag", None

    @classmethod
    def preprocess(cls, text: str) -> str:
        text = text.strip().replace(" [title]", ". ")
        return re.sub(r"\[.*?\]", "", text).replace("  ", " ")

    def doc_to_text(self, doc):
        return self.preprocess(f"{doc['activity_label']}: {doc['ctx_a']} {doc['ctx_b'].capitalize()}")

    def doc_to_continuations(self, doc):
        return [" " + self.preprocess(e) for e in doc["endings"]]

    def doc_to_label(self, doc):
        return int(doc["label"])

    def doc_to_domain_conditional(self, doc):
        dc = self.preprocess(doc["ctx_b"].capitalize())
        return dc if dc else self.preprocess(doc["ctx_a"]).split(" ")[-1]


class WinoGrande(_Task):
    """
    Pronoun resolution, scored "partially": two contexts (the sentence up to the blank, filled
    with either option) share one continuation (the rest of the sentence).
    """

    metric_type, path, name = "acc", "winogrande", "winogrande_xl"

    def prep_examples(self) -> None:
        for doc_id, doc in enumerate(self.dataset):
            continuation_str = self.doc_to_continuations(doc)
            label_id = self.doc_to_label(doc)
            for cont_id, (ctx_str, dc_str) in enumerate(zip(self.doc_to_text(doc), self.doc_to_domain_conditional(doc))):
                self.samples.append(
                    self._request(
                        doc_id, cont_id, self.token_encode(ctx_str), self.token_encode(dc_str), continuation_str, label_id,
                        ctx_len_from_query=False,
                    )
                )

    def doc_to_text(self, doc):
        stem = doc["sentence"][: doc["sentence"].index("_")]
        return [stem + doc["option1"], stem + doc["option2"]]

    def doc_to_continuations(self, doc):
        return " " + doc["sentence"][doc["sentence"].index("_") + 1 :].strip()

    def doc_to_label(self, doc):
        return int(doc["answer"]) - 1

    def doc_to_domain_conditional(self, doc):
        return [doc["option1"], doc["option2"]]


class OpenBookQA(_Task):
    """Bare question stem -> four choices."""

    metric_type, path, name = "len_norm", "openbookqa", "main"

    def doc_to_text(self, doc):
        return doc["question_stem"]

    def doc_to_continuations(self, doc):
        return [" " + c for c in doc["choices"]["text"]]

    def doc_to_label(self, doc):
        return "ABCD".index(doc["answerKey"].strip())

    def doc_to_domain_conditional(self, doc):
        return doc["question_stem"].strip().split(" ")[-1]


class BoolQ(_Task):
    """``PASSAGE\\nQuestion: Q?\\nAnswer:`` -> yes / no."""

    metric_type, path, name = "acc", "boolq", None

    def doc_to_text(self, doc):
        return f"{doc['passage']}\nQuestion: {doc['question']}?\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" yes", " no"]

    def doc_to_label(self, doc):
        return 0 if doc["answer"] else 1

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class SciQ(_Task):
    """``SUPPORT\\nQuestion: Q\\nAnswer:`` -> three distractors, then the correct answer."""

    metric_type, path, name = "acc", "sciq", None

    def doc_to_text(self, doc):
        return f"{doc['support'].strip()}\nQuestion: {doc['question']}\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" " + doc[k] for k in ("distractor1", "distractor2", "distractor3", "correct_answer")]

    def doc_to_label(self, doc):
        return 3

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class ArcEasy(_Task):
    """``Question: Q\\nAnswer:`` -> the listed choices; answer keys may be letters or digits."""

    metric_type, path, name = "acc", "ai2_arc", "ARC-Easy"

    def doc_to_text(self, doc):
        return f"Question: {doc['question']}\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" " + c for c in doc["choices"]["text"]]

    def doc_to_label(self, doc):
        key = doc["answerKey"]
        if key in "12345" and len(key) == 1:
            return int(key) - 1
        return "ABCDE".index(key)

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class ArcChallenge(ArcEasy):
    metric_type, name = "len_norm", "ARC-Challenge"


class ArcEasyCELoss(ArcEasy):
    """ARC-Easy scored by the cross-entropy of the gold answer only."""

    metric_type = "ce_loss"

    def doc_to_continuations(self, doc):
        return [" " + doc["choices"]["text"][ArcEasy.doc_to_label(self, doc)]]

    def doc_to_label(self, doc):
        return 0


class BasicArithmetic(ArcEasy):
    metric_type, path, name = "acc", "allenai/basic_arithmetic", None


class CommonsenseQA(ArcEasy):
    metric_type, path, name = "len_norm", "tau/commonsense_qa", None


class SocialIQa(_Task):
    """``Question: CONTEXT QUESTION\\nAnswer:`` -> three answers (1-based label)."""

    metric_type, path, name = "len_norm", "social_i_qa", None

    def doc_to_text(self, doc):
        return f"Question: {doc['context']} {doc['question']}\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" " + doc[k] for k in ("answerA", "answerB", "answerC")]

    def doc_to_label(self, doc):
        return int(doc["label"]) - 1

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class COPA(_Task):
    """``PREMISE-without-period because|therefore`` -> two lower-cased alternatives."""

    metric_type, path, name = "acc", "super_glue", "copa"

    @staticmethod
    def _connector(doc) -> str:
        return "because" if doc["question"] == "cause" else "therefore"

    def doc_to_text(self, doc):
        return doc["premise"].strip()[:-1] + " " + self._connector(doc)

    def doc_to_continuations(self, doc):
        return [" " + c[0].lower() + c[1:] for c in (doc["choice1"], doc["choice2"])]

    def doc_to_label(self, doc):
        return doc["label"]

    def doc_to_domain_conditional(self, doc):
        return self._connector(doc)


class RTE(_Task):
    """``S1\\nQuestion: S2 True or False?\\nAnswer:`` -> True / False."""

    metric_type, path, name = "len_norm", "glue", "rte"

    def doc_to_text(self, doc):
        return f"{doc['sentence1']}\nQuestion: {doc['sentence2']} True or False?\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" True", " False"]

    def doc_to_label(self, doc):
        return doc["label"]

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class CommitmentBank(_Task):
    """``PREMISE\\nQuestion: HYPOTHESIS. True, False or Neither?\\nAnswer:`` -> True / False / Neither."""

    metric_type, path, name = "acc", "super_glue", "cb"

    def doc_to_text(self, doc):
        return f"{doc['premise']}\nQuestion: {doc['hypothesis']}. True, False or Neither?\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" True", " False", " Neither"]

    def doc_to_label(self, doc):
        return doc["label"]

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class MRPC(_Task):
    """Paraphrase detection, F1-scored: yes / no."""

    metric_type, path, name = "f1", "glue", "mrpc"
    preprocess = staticmethod(_detokenise_glue)

    def doc_to_text(self, doc):
        return (
            f"Sentence 1: {self.preprocess(doc['sentence1'])}\nSentence 2: {self.preprocess(doc['sentence2'])}"
            "\nQuestion: Do both sentences mean the same thing?\nAnswer:"
        )

    def doc_to_continuations(self, doc):
        return [" yes", " no"]

    def doc_to_label(self, doc):
        return 0 if doc["label"] else 1

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class SST2(_Task):
    """Sentiment: negative (label 0) / positive (label 1)."""

    metric_type, path, name = "acc", "glue", "sst2"
    preprocess = staticmethod(_detokenise_glue)

    def doc_to_text(self, doc):
        return f"{self.preprocess(doc['sentence'])}\nQuestion: Is this sentence positive or negative?\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" negative", " positive"]

    def doc_to_label(self, doc):
        return doc["label"]

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class TriviaQACELoss(_Task):
    """Cross-entropy of the canonical answer string."""

    metric_type, path, name = "ce_loss", "trivia_qa", "rc.wikipedia.nocontext"

    def doc_to_text(self, doc):
        return f"\nQuestion: {doc['question']}\nAnswer:"

    def doc_to_continuations(self, doc):
        return [" " + doc["answer"]["value"]]

    def doc_to_label(self, doc):
        return 0

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


class NaturalQuestionsCELoss(TriviaQACELoss):
    """Cross-entropy of the first listed answer."""

    path, name = "nq_open", None

    def doc_to_continuations(self, doc):
        return [" " + doc["answer"][0]]


# ---------------------------------------------------------------------------------------------- MMLU

# field of study of every MMLU subject
_MMLU_FIELD = {
    "math": ["abstract_algebra", "college_mathematics", "elementary_mathematics", "high_school_mathematics", "high_school_statistics"],
    "health": [
        "anatomy", "clinical_knowledge", "college_medicine", "human_aging", "medical_genetics", "nutrition",
        "professional_medicine", "virology",
    ],
    "physics": ["astronomy", "college_physics", "conceptual_physics", "high_school_physics"],
    "business": ["business_ethics", "management", "marketing"],
    "biology": ["college_biology", "high_school_biology"],
    "chemistry": ["college_chemistry", "high_school_chemistry"],
    "computer science": ["college_computer_science", "computer_security", "high_school_computer_science", "machine_learning"],
    "economics": ["econometrics", "high_school_macroeconomics", "high_school_microeconomics"],
    "engineering": ["electrical_engineering"],
    "philosophy": ["formal_logic", "logical_fallacies", "moral_disputes", "moral_scenarios", "philosophy", "world_religions"],
    "other": ["global_facts", "miscellaneous", "professional_accounting"],
    "history": ["high_school_european_history", "high_school_us_history", "high_school_world_history", "prehistory"],
    "geography": ["high_school_geography"],
    "politics": ["high_school_government_and_politics", "public_relations", "security_studies", "us_foreign_policy"],
    "psychology": ["high_school_psychology", "professional_psychology"],
    "culture": ["human_sexuality", "sociology"],
    "law": ["international_law", "jurisprudence", "professional_law"],
}
_MMLU_GROUP = {
    "stem": ["physics", "chemistry", "biology", "computer science", "math", "engineering"],
    "humanities": ["history", "philosophy", "law"],
    "social_sciences": ["politics", "culture", "economics", "geography", "psychology"],
    "other": ["other", "business", "health"],
}
_MMLU_SUBJECT_ORDER = sorted(s for subjects in _MMLU_FIELD.values() for s in subjects)


class MMLU(ICLMultiChoiceTaskDataset):
    """
    MMLU by group (``stem`` ...), field (``math`` ...) or single subject.  ``prompt_variations=1``
    evaluates seven prompt variants per question (plain, instruction, instruction + 1..5 shots),
    ``=2`` only instruction + 5 shots; shots come from the ``dev`` split.  ``mc_labels`` lists the
    choices as ``A. ... D.`` and scores the letters instead of the answer texts.
    """

    metric_type = "len_norm"
    _subcategories = {s: [f] for f, subjects in _MMLU_FIELD.items() for s in subjects}
    _categories = _MMLU_GROUP

    @staticmethod
    def subjects_for(selector: Optional[str]) -> List[str]:
        if selector in _MMLU_GROUP:
            # field order within the group, alphabetical subject order within the field
            return [s for f in _MMLU_GROUP[selector] for s in _MMLU_SUBJECT_ORDER if s in _MMLU_FIELD[f]]
        if selector in _MMLU_SUBJECT_ORDER:
            return [selector]  # type: ignore[list-item]
        return [s for s in _MMLU_SUBJECT_ORDER if s in _MMLU_FIELD.get(selector or "", [])]

    def __init__(
        self,
        tokenizer,
        dataset_path: str = "hails/mmlu_no_train",
        dataset_name: Optional[str] = None,
        split: str = "validation",
        prompt_variations: Optional[int] = None,
        mc_labels: bool = False,
        metric_type: Optional[str] = None,
    ):
        subjects = self.subjects_for(dataset_name)
        self.mc_labels = mc_labels
        self.dev_set: Dict[str, Any] = {}
        if prompt_variations is None:
            prompts: List[Optional[str]] = [None]
        elif prompt_variations == 1:
            prompts = [None, "inst"] + [f"inst+{k}" for k in range(1, 6)]
        elif prompt_variations == 2:
            prompts = ["inst+5"]
        else:
            raise ValueError(f"Unknown prompt variations: {prompt_variations}")
        if prompt_variations is not None:
            for subject in subjects:
                self.dev_set[subject] = load_hf_dataset(dataset_path, subject, "dev")
        super().__init__(
            tokenizer=tokenizer, dataset_path=dataset_path, dataset_name=subjects, split=split, prompts=prompts, metric_type=metric_type,
        )

    def _render(self, doc) -> str:
        if self.mc_labels:
            listing = "".join(f"{key}. {choice}\n" for key, choice in zip("ABCD", doc["choices"]))
            return f"{doc['question'].strip()}\n{listing}Answer:"
        return f"Question: {doc['question'].strip()}\nAnswer:"

    def doc_to_text(self, doc):
        text = self._render(doc)
        variant = self.current_prompt
        if variant is None:
            return text
        head = ""
        if "inst" in variant:
            head = f"The following are multiple choice questions (with answers) about {doc.get('subject').replace('_', ' ')}:\n\n"
        shots = re.findall(r"\+(\d+)", variant)
        if shots:
            for i, shot in enumerate(self.dev_set.get(doc.get("subject"), [])):
                if i >= int(shots[0]):
                    break
                gold = "ABCD"[shot["answer"]] if self.mc_labels else shot["choices"][shot["answer"]]
                head += f"{self._render(shot)} {gold}\n\n"
        return head + text

    def doc_to_continuations(self, doc):
        choices = [" A", " B", " C", " D"] if self.mc_labels else [" " + c for c in doc["choices"]]
        return [choices[doc["answer"]]] if self.metric_type in _SINGLE_TARGET_METRICS else choices

    def doc_to_label(self, doc):
        return 0 if self.metric_type in _SINGLE_TARGET_METRICS else doc["answer"]

    def doc_to_domain_conditional(self, doc):
        return _ANSWER_DC


# ------------------------------------------------------------------------------------- request dumps


class OEEvalTask(ICLMultiChoiceTaskDataset):
    """
    Task whose prompts were rendered ahead of time by the oe-eval toolkit: a ``config.json`` plus
    a gzip'd JSON-lines file of ``loglikelihood`` requests (context, continuation, label, idx).
    With a single-target metric only the gold continuation of each document is kept.
    """

    def __init__(
        self,
        tokenizer,
        dataset_path: str,
        dataset_name: Union[str, Sequence[str], None] = None,
        model_ctx_len: int = 2048,
        split: Optional[str] = None,
        metric_type: Optional[str] = None,
        prompts: Sequence[Optional[str]] = (None,),
    ):
        self.tokenizer = tokenizer
        self.dataset_path = dataset_path
        self.dataset_name = dataset_name
        self.model_ctx_len = model_ctx_len
        self.prompts = list(prompts)
        self.current_prompt = None
        self.log_instances = 0
        self.samples = []
        loaded = [load_oe_eval_requests(dataset_path, name, split) for name in _as_name_list(dataset_name)]
        if metric_type is not None:
            self.metric_type = metric_type
        else:
            for config, _ in loaded:
                raw = (config or {}).get("task_config", {}).get("primary_metric")
                if raw is None:
                    continue
                resolved = METRIC_FROM_OE_EVAL[raw]
                if self.metric_type is not None and self.metric_type != resolved:
                    raise ValueError(f"Conflicting metric types: {self.metric_type} and {resolved}")
                self.metric_type = resolved
        self.dataset = [requests for _, requests in loaded]
        self.prep_examples()

    def prep_examples(self) -> None:
        offset = 0
        for requests in self.dataset:
            highest = 0
            for request in requests:
                doc_id = request["doc_id"]
                if doc_id >= 1000000:
                    continue  # oe-eval encodes unconditional requests this way; they are not scored here
                highest = max(highest, doc_id)
                if request["request_type"] != "loglikelihood":
                    raise AssertionError(f"Unsupported request type: {request['request_type']}")
                label_id, cont_id = request["label"], request["idx"]
                if self.metric_type in _SINGLE_TARGET_METRICS:
                    if label_id != cont_id and not isinstance(label_id, str):
                        continue
                    label_id = cont_id = 0
                body = request["request"]
                ctx = self.token_encode(body["context"])
                dc = self.token_encode(self.doc_to_domain_conditional(request["doc"]))
                self._maybe_log(body["context"], body["continuation"])
                self.samples.append(self._request(doc_id + offset, cont_id, ctx, dc, body["continuation"], label_id))
            offset += highest

    def doc_to_text(self, doc) -> str:
        raise NotImplementedError

    def doc_to_continuations(self, doc) -> List[str]:
        raise NotImplementedError

    def doc_to_label(self, doc) -> int:
        raise NotImplementedError


# --------------------------------------------------------------------------------------- task table

TaskEntry = Union[type, Tuple[type, Dict[str, Any]]]


def _oe(path: str, name: str, metric: str) -> Dict[str, TaskEntry]:
    """A rendered-request task under its metric and, unless that already is bpb, also as ``_bpb``."""
    out: Dict[str, TaskEntry] = {f"{path}_{name}": (OEEvalTask, {"dataset_path": path, "dataset_name": name, "metric_type": metric})}
    if metric != "bpb":
        out[f"{path}_{name}_bpb"] = (OEEvalTask, {"dataset_path": path, "dataset_name": name, "metric_type": "bpb"})
    return out


def _oe_family(path: str, splits: Sequence[str], rc_metric: str, rc_base_metric: Optional[str] = None) -> Dict[str, TaskEntry]:
    """
    ``mc_5shot`` / ``rc_0shot`` / ``rc_5shot`` on the default split plus ``{split}_{mc,rc}_5shot``.
    Multiple-choice variants are scored by accuracy, rank-choice variants by ``rc_metric``
    (``rc_base_metric`` for the default-split ones when it differs).
    """
    out: Dict[str, TaskEntry] = {}
    out.update(_oe(path, "mc_5shot", "acc"))
    for name in ("rc_0shot", "rc_5shot"):
        out.update(_oe(path, name, rc_base_metric or rc_metric))
    for split in splits:
        out.update(_oe(path, f"{split}_mc_5shot", "acc"))
        out.update(_oe(path, f"{split}_rc_5shot", rc_metric))
    return out


def _mmlu_entries() -> Dict[str, TaskEntry]:
    out: Dict[str, TaskEntry] = {}

    def add(label: str, **kwargs: Any) -> None:
        out[label] = (MMLU, kwargs)

    for group in _MMLU_GROUP:
        base = f"mmlu_{group}"
        add(base, dataset_name=group)
        add(f"{base}_test", dataset_name=group, split="test")
        add(f"{base}_bpb", dataset_name=group, metric_type="bpb")
        add(f"{base}_var", dataset_name=group, prompt_variations=1)
        add(f"{base}_var_bpb", dataset_name=group, prompt_variations=1, metric_type="bpb")
        add(f"{base}_mc_5shot", dataset_name=group, prompt_variations=2, mc_labels=True)
        add(f"{base}_mc_5shot_test", dataset_name=group, split="test", prompt_variations=2, mc_labels=True)
        for split_tag, split_kw in (("val", {}), ("test", {"split": "test"})):
            for style, style_kw in (
                ("rc_var", {"prompt_variations": 1}),
                ("rc_5shot", {"prompt_variations": 2}),
                ("mc_5shot", {"prompt_variations": 2, "mc_labels": True}),
            ):
                add(f"{base}_{split_tag}_{style}", dataset_name=group, **split_kw, **style_kw)
                add(f"{base}_{split_tag}_{style}_bpb", dataset_name=group, **split_kw, **style_kw, metric_type="bpb")
    return out


def _build_task_table() -> Dict[str, TaskEntry]:
    table: Dict[str, TaskEntry] = {
        "piqa": PIQA,
        "hellaswag": HellaSwag,
        "winogrande": WinoGrande,
        "openbook_qa": OpenBookQA,
        "boolq": BoolQ,
        "sciq": SciQ,
        "arc_easy": ArcEasy,
        "arc_easy_ppl": ArcEasyCELoss,
        "arc_challenge": ArcChallenge,
        "basic_arithmetic": BasicArithmetic,
        "copa": COPA,
        "rte": RTE,
        "commitment_bank": CommitmentBank,
        "mrpc": MRPC,
        "sst2": SST2,
        "commonsense_qa": CommonsenseQA,
        "social_iqa": SocialIQa,
        "trivia_qa_wiki_ppl": TriviaQACELoss,
        "natural_qs_open_ppl": NaturalQuestionsCELoss,
    }
    table.update(_mmlu_entries())
    three, two = ("train", "val", "test"), ("train", "val")
    table.update(_oe_family("arc_challenge", three, "len_norm"))
    table.update(_oe_family("arc_easy", three, "len_norm", rc_base_metric="acc"))
    table.update(_oe_family("boolq", two, "acc"))
    table.update(_oe_family("csqa", two, "len_norm"))
    table.update(_oe_family("hellaswag", two, "len_norm"))
    table.update(_oe_family("openbookqa", three, "len_norm"))
    table.update(_oe_family("piqa", two, "len_norm"))
    table.update(_oe_family("socialiqa", two, "len_norm"))
    table.update(_oe_family("winogrande", two, "len_norm", rc_base_metric="acc"))
    table.update(_oe("copa", "rc_0shot", "acc"))
    table.update(_oe("sciq", "rc_0shot", "acc"))
    table.update(_oe("copycolors", "10way", "acc"))
    table.update(_oe("copycolors", "xl_10way", "acc"))
    table.update(_oe("gsm8k", "gold_bpb_5shot", "bpb"))
    return table


label_to_task_map: Dict[str, TaskEntry] = _build_task_table()


def list_tasks() -> List[str]:
    """All evaluator labels accepted in ``evaluators[*].label``."""
    return sorted(label_to_task_map)
