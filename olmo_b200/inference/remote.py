"""
Evaluation against an OpenAI-compatible HTTP endpoint (this framework's own server, ``scripts/serve_openai.py``, or any
other): many requests in flight at once, retries with back-off, results in request order, and an optional JSONL cache so
that an interrupted run resumes where it stopped.

This is the counterpart of the reference's ``inference/eval/dispatch_openai_requests.py`` (concurrent chat / completion
calls) and of ``query_openai_chat_model`` / ``query_openai_model`` in ``inference/eval/utils.py:200-349`` (batched
queries with retries whose results are appended to an output file).  It talks plain HTTP through ``aiohttp`` instead of
the ``openai`` client package, so it has no dependency beyond what the server itself needs.

    python -m olmo_b200.inference.remote --base-url http://127.0.0.1:8000/v1 --model olmo --mmlu-group stem --limit 50
"""
from __future__ import annotations

import argparse
import asyncio
import json
import logging
import os
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence

__all__ = ["dispatch_chat_requests", "dispatch_prompt_requests", "query_chat_model", "query_completion_model", "score_mmlu_remote"]

log = logging.getLogger(__name__)


async def _post_all(base_url: str, route: str, payloads: Sequence[Dict[str, Any]], api_key: Optional[str], concurrency: int,
                    retries: int, timeout_s: float, backoff_s: float) -> List[Dict[str, Any]]:
    import aiohttp

    headers = {"Content-Type": "application/json"}
    if api_key:
        headers["Authorization"] = f"Bearer {api_key}"
    gate = asyncio.Semaphore(max(1, concurrency))
    url = base_url.rstrip("/") + route

    async def one(session, payload):
        last: Optional[BaseException] = None
        for attempt in range(retries + 1):
            try:
                async with gate:
                    async with session.post(url, json=payload, headers=headers) as resp:
                        body = await resp.text()
                        if resp.status == 200:
                            return json.loads(body)
                        if resp.status < 500 and resp.status != 429:  # a request the server will never accept
                            raise ValueError(f"{url} answered {resp.status}: {body[:500]}")
                        last = RuntimeError(f"{url} answered {resp.status}: {body[:200]}")
            except (aiohttp.ClientError, asyncio.TimeoutError) as e:
                last = e
            await asyncio.sleep(backoff_s * (2**attempt))
        raise RuntimeError(f"request failed after {retries + 1} attempts") from last

    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=timeout_s)) as session:
        return list(await asyncio.gather(*(one(session, p) for p in payloads)))


async def dispatch_chat_requests(base_url: str, messages_list: Sequence[List[Dict[str, str]]], model: str, api_key: Optional[str] = None,
                                 concurrency: int = 16, retries: int = 3, timeout_s: float = 600.0, backoff_s: float = 1.0,
                                 **completion_kwargs) -> List[Dict[str, Any]]:
    """One ``/chat/completions`` call per conversation, all in flight together (at most ``concurrency`` at a time);
    responses come back in the order of ``messages_list``."""
    payloads = [{"model": model, "messages": m, **completion_kwargs} for m in messages_list]
    return await _post_all(base_url, "/chat/completions", payloads, api_key, concurrency, retries, timeout_s, backoff_s)


async def dispatch_prompt_requests(base_url: str, prompts: Sequence[str], model: str, api_key: Optional[str] = None, concurrency: int = 16,
                                   retries: int = 3, timeout_s: float = 600.0, backoff_s: float = 1.0, **completion_kwargs) -> List[Dict[str, Any]]:
    """One ``/completions`` call per prompt; same contract as :func:`dispatch_chat_requests`."""
    payloads = [{"model": model, "prompt": p, **completion_kwargs} for p in prompts]
    return await _post_all(base_url, "/completions", payloads, api_key, concurrency, retries, timeout_s, backoff_s)


def _read_cache(path: Optional[Path]) -> Dict[str, Dict[str, Any]]:
    done: Dict[str, Dict[str, Any]] = {}
    if path is not None and path.is_file():
        for line in path.read_text().splitlines():
            if line.strip():
                row = json.loads(line)
                done[str(row["id"])] = row
    return done


def _query(kind: str, base_url: str, model: str, instances: Sequence[Dict[str, Any]], batch_size: int, output_path: Optional[str],
           api_key: Optional[str], reuse_existing: bool, **kwargs) -> List[Dict[str, Any]]:
    """Shared driver: instances are ``{"id": ..., "prompt": ...}``; results ``{"id", "prompt", "output", "response"}`` in
    instance order, appended batch by batch to ``output_path`` when one is given."""
    path = Path(output_path) if output_path else None
    done = _read_cache(path) if reuse_existing else {}
    if path is not None:
        path.parent.mkdir(parents=True, exist_ok=True)
        if not reuse_existing and path.exists():
            path.unlink()
    todo = [x for x in instances if str(x["id"]) not in done]
    for start in range(0, len(todo), batch_size):
        chunk = todo[start : start + batch_size]
        if kind == "chat":
            responses = asyncio.run(dispatch_chat_requests(base_url, [[{"role": "user", "content": x["prompt"]}] for x in chunk], model,
                                                           api_key=api_key, **kwargs))
            texts = [r["choices"][0]["message"]["content"] for r in responses]
        else:
            responses = asyncio.run(dispatch_prompt_requests(base_url, [x["prompt"] for x in chunk], model, api_key=api_key, **kwargs))
            texts = [r["choices"][0]["text"] for r in responses]
        rows = [{"id": x["id"], "prompt": x["prompt"], "output": t, "response": r} for x, t, r in zip(chunk, texts, responses)]
        for row in rows:
            done[str(row["id"])] = row
        if path is not None:
            with open(path, "a") as f:
                for row in rows:
                    f.write(json.dumps(row) + "\n")
        log.info("%d / %d instances answered", min(start + batch_size, len(todo)), len(todo))
    return [done[str(x["id"])] for x in instances]


def query_chat_model(base_url: str, model: str, instances: Sequence[Dict[str, Any]], batch_size: int = 16, output_path: Optional[str] = None,
                     api_key: Optional[str] = None, reuse_existing: bool = True, **completion_kwargs) -> List[Dict[str, Any]]:
    """Ask a chat model every instance's ``prompt`` (as one user turn).  With ``output_path``, answered instances are
    kept in that JSONL file and skipped on the next call."""
    return _query("chat", base_url, model, instances, batch_size, output_path, api_key, reuse_existing, **completion_kwargs)


def query_completion_model(base_url: str, model: str, instances: Sequence[Dict[str, Any]], batch_size: int = 16,
                           output_path: Optional[str] = None, api_key: Optional[str] = None, reuse_existing: bool = True,
                           **completion_kwargs) -> List[Dict[str, Any]]:
    """Same as :func:`query_chat_model` through the plain completions route."""
    return _query("completion", base_url, model, instances, batch_size, output_path, api_key, reuse_existing, **completion_kwargs)


def _first_choice_letter(text: str) -> Optional[str]:
    for ch in text.strip():
        if ch in "ABCD":
            return ch
        if not (ch.isspace() or ch in "(:."):
            break
    return None


def score_mmlu_remote(base_url: str, model: str, tokenizer, group: str = "stem", split: str = "test", shots: int = 5,
                      limit: Optional[int] = None, chat: bool = False, output_path: Optional[str] = None, api_key: Optional[str] = None,
                      batch_size: int = 16) -> Dict[str, float]:
    """MMLU accuracy of a served model: the k-shot prompt of :class:`olmo_b200.eval.downstream.MMLU` is sent as text, one
    token is generated greedily, and its first letter is the prediction (``inference/eval/mmlu/run_eval.py:119-170`` does
    the same for API models).  ``tokenizer`` only turns the task's token ids back into prompt text."""
    from ..eval.downstream import MMLU

    task = MMLU(tokenizer, dataset_name=group, split=split, prompt_variations=2 if shots > 0 else None, mc_labels=True)
    docs: Dict[int, Dict] = {}
    for s in task.samples:
        docs.setdefault(s["doc_id"], s)
    rows = list(docs.values())[:limit]
    instances = [{"id": i, "prompt": tokenizer.decode(r["ctx"])} for i, r in enumerate(rows)]
    ask = query_chat_model if chat else query_completion_model
    answers = ask(base_url, model, instances, batch_size=batch_size, output_path=output_path, api_key=api_key, max_tokens=1 if not chat else 4,
                  temperature=0.0)
    hits = [int(_first_choice_letter(a["output"]) == "ABCD"[r["label_id"]]) for a, r in zip(answers, rows)]
    return {"acc": sum(hits) / max(1, len(hits)), "n": float(len(hits))}


def main(argv=None) -> Dict[str, float]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--base-url", required=True, help="e.g. http://127.0.0.1:8000/v1")
    ap.add_argument("--model", required=True, help="model name the endpoint expects")
    ap.add_argument("--tokenizer", default="allenai_dolma2.json", help="tokenizer file or packaged tokenizer name used to build the prompts")
    ap.add_argument("--mmlu-group", default="stem")
    ap.add_argument("--split", default="test")
    ap.add_argument("--ntrain", type=int, default=5)
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--chat", action="store_true", help="use the chat route instead of plain completions")
    ap.add_argument("--output", default=None, help="JSONL file of answered instances (resumable)")
    ap.add_argument("--batch-size", type=int, default=16)
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    from ..tokenizer import Tokenizer

    tokenizer = Tokenizer.from_file(args.tokenizer) if os.path.exists(args.tokenizer) else Tokenizer.from_pretrained(args.tokenizer)
    result = score_mmlu_remote(args.base_url, args.model, tokenizer, group=args.mmlu_group, split=args.split, shots=args.ntrain,
                               limit=args.limit, chat=args.chat, output_path=args.output, api_key=os.environ.get("OPENAI_API_KEY"),
                               batch_size=args.batch_size)
    print(json.dumps(result))
    return result


if __name__ == "__main__":
    main()
