"""
OpenAI-compatible HTTP front end for :class:`olmo_b200.serve.engine.Engine`.

Endpoints: ``GET /health``, ``GET /metrics`` (Prometheus text), ``GET /v1/models``, ``POST /v1/completions``, ``POST /v1/chat/completions`` (both with
``stream: true`` as server-sent events).  This is the surface the reference reaches by deploying a third-party server
for an OLMo-2 instruct checkpoint (``scripts/olmo2_modal_openai.py``: ``MODEL_NAME``, ``serve()``); here it runs on the
framework's own model and scheduler.  An optional bearer token guards the ``/v1`` routes, as that deployment does.
"""
import asyncio
import json
import time
import uuid
from typing import Any, AsyncIterator, Callable, Dict, List, Optional, Sequence, Tuple

from .engine import ContextLengthError, Engine, GenerationRequest, QueueFullError, SamplingParams

__all__ = ["create_app", "default_chat_template", "load_chat_template"]


def default_chat_template(messages: Sequence[Dict[str, Any]], bos: str = "<|endoftext|>") -> str:
    """The OLMo-2 instruct layout: ``<|endoftext|><|system|>\\n…\\n<|user|>\\n…\\n<|assistant|>\\n``; an assistant turn
    that is followed by more turns is closed with the end-of-text token."""
    parts = [bos]
    for i, message in enumerate(messages):
        role, content = message.get("role"), message.get("content", "")
        if isinstance(content, list):  # content parts: keep the text ones
            content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
        if role not in ("system", "user", "assistant"):
            raise ValueError(f"unsupported role {role!r}")
        parts.append(f"<|{role}|>\n{content}")
        parts.append(bos + "\n" if role == "assistant" and i + 1 < len(messages) else "\n")
    parts.append("<|assistant|>\n")
    return "".join(parts)


def load_chat_template(path: str, bos_token: str = "<|endoftext|>", eos_token: str = "<|endoftext|>") -> Callable[[Sequence[Dict[str, Any]]], str]:
    """A chat template from a file: either a Jinja template as text, or a ``tokenizer_config.json`` whose ``chat_template``
    entry holds one (the form instruct checkpoints on the HuggingFace Hub ship).  The template sees ``messages``,
    ``add_generation_prompt=True``, ``bos_token`` and ``eos_token``, like ``apply_chat_template`` in transformers."""
    import jinja2
    from jinja2.sandbox import ImmutableSandboxedEnvironment

    text = open(path, encoding="utf-8").read()
    if path.endswith(".json"):
        config = json.loads(text)
        text = config["chat_template"]
        bos_token = config.get("bos_token") or bos_token
        eos_token = config.get("eos_token") or eos_token
        if isinstance(bos_token, dict):
            bos_token = bos_token.get("content", "")
        if isinstance(eos_token, dict):
            eos_token = eos_token.get("content", "")

    def raise_exception(message: str):
        raise ValueError(message)

    env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True, undefined=jinja2.StrictUndefined)
    env.globals["raise_exception"] = raise_exception
    template = env.from_string(text)

    def render(messages: Sequence[Dict[str, Any]]) -> str:
        try:
            return template.render(messages=list(messages), add_generation_prompt=True, bos_token=bos_token, eos_token=eos_token)
        except jinja2.TemplateError as exc:
            raise ValueError(f"chat template failed: {exc}") from exc

    return render


class _BadRequest(Exception):
    def __init__(self, message: str, code: Optional[str] = None, status: int = 400):
        super().__init__(message)
        self.message, self.code, self.status = message, code, status


def _sampling(body: Dict[str, Any], default_max_tokens: int) -> SamplingParams:
    stop = body.get("stop") or ()
    if isinstance(stop, str):
        stop = (stop,)
    max_tokens = body.get("max_completion_tokens", body.get("max_tokens"))
    try:
        params = SamplingParams(
            max_tokens=int(default_max_tokens if max_tokens is None else max_tokens),
            temperature=float(1.0 if body.get("temperature") is None else body["temperature"]),
            top_p=float(1.0 if body.get("top_p") is None else body["top_p"]),
            top_k=int(body.get("top_k") or 0),
            stop=tuple(stop),
            stop_token_ids=tuple(body.get("stop_token_ids") or ()),
            seed=body.get("seed"),
            logprobs=bool(body.get("logprobs")),
            ignore_eos=bool(body.get("ignore_eos", False)),
        )
        params.validate()
    except (TypeError, ValueError) as exc:
        raise _BadRequest(str(exc)) from exc
    return params


def _prompts(engine: Engine, prompt: Any) -> List[List[int]]:
    """``prompt`` may be a string, a list of strings, a list of token ids or a list of such lists."""
    if isinstance(prompt, str):
        return [engine.tokenizer.encode(prompt, add_special_tokens=False)]
    if isinstance(prompt, list) and prompt:
        if all(isinstance(p, str) for p in prompt):
            return [engine.tokenizer.encode(p, add_special_tokens=False) for p in prompt]
        if all(isinstance(p, int) for p in prompt):
            return [list(prompt)]
        if all(isinstance(p, list) and all(isinstance(t, int) for t in p) for p in prompt):
            return [list(p) for p in prompt]
    raise _BadRequest("'prompt' must be a string, a list of strings, or token ids")


def create_app(
    engine: Engine,
    model_name: str = "olmo",
    api_key: Optional[str] = None,
    chat_template: Callable[[Sequence[Dict[str, Any]]], str] = default_chat_template,
    default_max_tokens: int = 16,
    default_chat_max_tokens: int = 512,
):
    """Build the FastAPI application.  The engine's background thread is started with the app and stopped with it."""
    from contextlib import asynccontextmanager

    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, StreamingResponse

    @asynccontextmanager
    async def lifespan(app):
        engine.start()
        yield
        engine.stop()

    app = FastAPI(title="olmo_b200 OpenAI-compatible server", lifespan=lifespan)
    created = int(time.time())

    def error(message: str, status: int = 400, code: Optional[str] = None, kind: str = "invalid_request_error"):
        return JSONResponse({"error": {"message": message, "type": kind, "param": None, "code": code}}, status_code=status)

    async def body_of(request: Request) -> Dict[str, Any]:
        if api_key is not None and request.headers.get("authorization") != f"Bearer {api_key}":
            raise _BadRequest("invalid or missing bearer token", code="invalid_api_key", status=401)
        try:
            body = await request.json()
        except Exception as exc:
            raise _BadRequest(f"request body is not JSON: {exc}") from exc
        if not isinstance(body, dict):
            raise _BadRequest("request body must be a JSON object")
        if body.get("model") not in (None, model_name):
            raise _BadRequest(f"The model `{body.get('model')}` does not exist.", code="model_not_found", status=404)
        n = body.get("n", 1)
        if not isinstance(n, int) or not 1 <= n <= 16:
            raise _BadRequest("'n' must be an integer between 1 and 16")
        return body

    def submit_all(prompts: List[List[int]], params: SamplingParams, n: int, sink=None, on_done=None) -> List[GenerationRequest]:
        requests = []
        try:
            for prompt in prompts:
                for k in range(n):
                    # choices of one prompt must differ: derive a stream per choice from the request's seed
                    p = params if params.seed is None or n == 1 else SamplingParams(**{**params.__dict__, "seed": params.seed + k})
                    callback = None if sink is None else sink(len(requests))
                    requests.append(engine.submit(prompt, p, callback, on_done))
        except ContextLengthError as exc:
            for r in requests:
                engine.cancel(r)
            raise _BadRequest(str(exc), code="context_length_exceeded") from exc
        except QueueFullError as exc:
            for r in requests:
                engine.cancel(r)
            raise _BadRequest(f"the server is busy: {exc}", code="queue_full", status=429) from exc
        return requests

    async def submit_and_wait(prompts: List[List[int]], params: SamplingParams, n: int) -> List[GenerationRequest]:
        """Submit, then sleep on an event the engine's thread sets through the loop: a waiting request holds no thread."""
        loop = asyncio.get_running_loop()
        finished = asyncio.Event()
        total = len(prompts) * n
        count = {"done": 0}

        def one_done() -> None:  # runs in the event loop
            count["done"] += 1
            if count["done"] >= total:
                finished.set()

        requests = submit_all(prompts, params, n, on_done=lambda _r: loop.call_soon_threadsafe(one_done))
        try:
            await finished.wait()
        except asyncio.CancelledError:  # the client went away
            for r in requests:
                if not r.finished:
                    engine.cancel(r)
            raise
        for r in requests:
            if r.error is not None:
                raise r.error
        return requests

    def usage(requests: List[GenerationRequest], n: int) -> Dict[str, int]:
        prompt_tokens = sum(len(r.prompt_ids) for r in requests[::n])
        completion_tokens = sum(len(r.token_ids) for r in requests)
        return {"prompt_tokens": prompt_tokens, "completion_tokens": completion_tokens, "total_tokens": prompt_tokens + completion_tokens}

    def token_logprobs(r: GenerationRequest) -> Optional[Dict[str, Any]]:
        if not r.params.logprobs:
            return None
        tokens = [engine.tokenizer.decode([t]) for t in r.token_ids]
        return {"tokens": tokens, "token_logprobs": r.token_logprobs, "top_logprobs": None, "text_offset": None}

    async def stream(requests: List[GenerationRequest], queue: "asyncio.Queue", frame: Callable[[int, str, Optional[str]], Dict[str, Any]], first: Sequence[Dict[str, Any]] = ()) -> AsyncIterator[bytes]:
        for chunk in first:
            yield f"data: {json.dumps(chunk)}\n\n".encode()
        open_choices = len(requests)
        try:
            while open_choices:
                index, delta, reason = await queue.get()
                if reason is not None:
                    open_choices -= 1
                if delta or reason is not None:
                    yield f"data: {json.dumps(frame(index, delta, reason))}\n\n".encode()
            yield b"data: [DONE]\n\n"
        finally:  # the client went away (the response generator was closed): free the rows
            for r in requests:
                if not r.finished:
                    engine.cancel(r)

    def make_sink(queue: "asyncio.Queue", loop):
        def sink(index: int):
            def on_token(request: GenerationRequest, token: int, delta: str) -> None:
                loop.call_soon_threadsafe(queue.put_nowait, (index, delta, request.finish_reason))
            return on_token
        return sink

    @app.get("/health")
    async def health():
        return {"status": "ok", **{k: (round(v, 3) if isinstance(v, float) else int(v)) for k, v in engine.stats.items()}}

    @app.get("/metrics")
    async def metrics():
        """Prometheus text exposition of the engine's counters."""
        from fastapi.responses import PlainTextResponse

        with engine._lock:
            waiting, running = len(engine._queue), len(engine._rows)
        lines = []
        for name, value, kind, text in [
            ("olmo_requests_total", engine.stats["requests"], "counter", "requests admitted to the decode batch"),
            ("olmo_prompt_tokens_total", engine.stats["prefill_tokens"], "counter", "prompt tokens processed"),
            ("olmo_generated_tokens_total", engine.stats["decode_tokens"] + engine.stats["requests"], "counter", "tokens generated"),
            ("olmo_decode_steps_total", engine.stats["decode_steps"], "counter", "decode steps run"),
            ("olmo_requests_waiting", waiting, "gauge", "requests in the queue"),
            ("olmo_requests_running", running, "gauge", "rows of the decode batch in use"),
        ]:
            lines += [f"# HELP {name} {text}", f"# TYPE {name} {kind}", f"{name} {int(value)}"]
        return PlainTextResponse("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "created": created, "owned_by": "olmo_b200",
                                            "max_model_len": engine.config.max_sequence_length}]}

    @app.post("/v1/completions")
    async def completions(request: Request):
        try:
            body = await body_of(request)
            if "prompt" not in body:
                raise _BadRequest("'prompt' is required")
            prompts, params, n = _prompts(engine, body["prompt"]), _sampling(body, default_max_tokens), body.get("n", 1)
            rid, echo = f"cmpl-{uuid.uuid4().hex}", bool(body.get("echo"))
            if body.get("stream"):
                queue: asyncio.Queue = asyncio.Queue()
                requests = submit_all(prompts, params, n, make_sink(queue, asyncio.get_running_loop()))

                def frame(index: int, delta: str, reason: Optional[str]) -> Dict[str, Any]:
                    return {"id": rid, "object": "text_completion", "created": int(time.time()), "model": model_name,
                            "choices": [{"index": index, "text": delta, "logprobs": None, "finish_reason": reason}]}

                return StreamingResponse(stream(requests, queue, frame), media_type="text/event-stream")
            requests = await submit_and_wait(prompts, params, n)
        except _BadRequest as exc:
            return error(exc.message, exc.status, exc.code)
        except Exception as exc:  # the engine failed the request
            return error(f"{type(exc).__name__}: {exc}", 500, kind="server_error")
        choices = []
        for i, r in enumerate(requests):
            text = (engine.tokenizer.decode(r.prompt_ids) if echo else "") + r.text
            choices.append({"index": i, "text": text, "logprobs": token_logprobs(r), "finish_reason": r.finish_reason})
        return {"id": rid, "object": "text_completion", "created": int(time.time()), "model": model_name, "choices": choices,
                "usage": usage(requests, n)}

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        try:
            body = await body_of(request)
            messages = body.get("messages")
            if not isinstance(messages, list) or not messages:
                raise _BadRequest("'messages' must be a non-empty list")
            try:
                prompt = chat_template(messages)
            except (ValueError, AttributeError) as exc:
                raise _BadRequest(str(exc)) from exc
            prompts = [engine.tokenizer.encode(prompt, add_special_tokens=False)]
            params, n = _sampling(body, default_chat_max_tokens), body.get("n", 1)
            rid = f"chatcmpl-{uuid.uuid4().hex}"
            if body.get("stream"):
                queue: asyncio.Queue = asyncio.Queue()
                requests = submit_all(prompts, params, n, make_sink(queue, asyncio.get_running_loop()))

                def frame(index: int, delta: str, reason: Optional[str], role: Optional[str] = None) -> Dict[str, Any]:
                    d: Dict[str, Any] = {"content": delta} if delta else {}
                    if role:
                        d["role"] = role
                    return {"id": rid, "object": "chat.completion.chunk", "created": int(time.time()), "model": model_name,
                            "choices": [{"index": index, "delta": d, "finish_reason": reason}]}

                first = [frame(i, "", None, role="assistant") for i in range(len(requests))]
                return StreamingResponse(stream(requests, queue, frame, first), media_type="text/event-stream")
            requests = await submit_and_wait(prompts, params, n)
        except _BadRequest as exc:
            return error(exc.message, exc.status, exc.code)
        except Exception as exc:  # the engine failed the request
            return error(f"{type(exc).__name__}: {exc}", 500, kind="server_error")
        choices = [
            {"index": i, "message": {"role": "assistant", "content": r.text}, "logprobs": None, "finish_reason": r.finish_reason}
            for i, r in enumerate(requests)
        ]
        return {"id": rid, "object": "chat.completion", "created": int(time.time()), "model": model_name, "choices": choices,
                "usage": usage(requests, n)}

    return app
