"""
Continuous-batching text generation over an :class:`olmo_b200.model.OLMo`.

The reference ships no serving engine of its own: its serving script deploys a third-party OpenAI-compatible server
for an OLMo-2 checkpoint (``scripts/olmo2_modal_openai.py``) and its efficiency runner batches prompts through
``generate`` (``inference/efficiency/run_efficiency_benchmark.py:16-114``).  This module is the first-party equivalent:
requests join and leave a running decode batch between steps.

Two decode back ends.  The *static* one (``olmo_b200/serve/static_cache.py``: preallocated windows, fixed shapes, one
CUDA graph per length bucket) is the default on a GPU for rotary models; the *dynamic* one below works for every
architecture and on every device.

Layout of the dynamic running batch.  All rows share one key/value window of length ``L`` per block (``[rows, kv_heads, L,
head_dim]``, keys stored before the rotary embedding, as ``OLMo.forward`` returns them).  A row's tokens are
right-aligned in the window and the columns to their left are masked out, so rows of different lengths decode
together; rotary and ALiBi terms depend only on distances inside the window and are unaffected by the shift.  New
requests are prefilled together (left-padded), then merged into the window by left-padding whichever side is shorter.
Finished rows are dropped with one ``index_select`` and the common left padding is trimmed, so ``L`` never exceeds the
longest live sequence.
"""
from __future__ import annotations

import itertools
import threading
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

__all__ = ["SamplingParams", "GenerationRequest", "Engine", "ContextLengthError", "QueueFullError"]


class ContextLengthError(ValueError):
    """The prompt does not leave room for a single new token."""


class QueueFullError(RuntimeError):
    """More requests are waiting than the engine was told to hold."""


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 1.0  # 0 selects the most likely token
    top_p: float = 1.0
    top_k: int = 0  # 0 = no limit
    stop: Sequence[str] = ()
    stop_token_ids: Sequence[int] = ()
    seed: Optional[int] = None
    logprobs: bool = False
    ignore_eos: bool = False

    def validate(self) -> None:
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be at least 1")
        if self.temperature < 0:
            raise ValueError("temperature must be non-negative")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k < 0:
            raise ValueError("top_k must be non-negative")


@dataclass(eq=False)  # requests are compared and looked up by identity
class GenerationRequest:
    id: int
    prompt_ids: List[int]
    params: SamplingParams
    on_token: Optional[Callable[["GenerationRequest", int, str], None]] = None
    on_done: Optional[Callable[["GenerationRequest"], None]] = None  # called from the engine's thread when the request ends
    token_ids: List[int] = field(default_factory=list)
    token_logprobs: List[float] = field(default_factory=list)
    text: str = ""
    finish_reason: Optional[str] = None  # "stop" | "length" | "error"
    error: Optional[BaseException] = None
    submitted_at: float = field(default_factory=time.monotonic)
    first_token_at: Optional[float] = None
    finished_at: Optional[float] = None
    _done: threading.Event = field(default_factory=threading.Event, repr=False)
    _generator: Optional[torch.Generator] = field(default=None, repr=False)
    _emitted: int = field(default=0, repr=False)  # characters of ``text`` already passed to ``on_token``
    _row: int = field(default=-1, repr=False)  # row of the static key/value window, when that mode is on
    _cancelled: bool = field(default=False, repr=False)

    @property
    def finished(self) -> bool:
        return self.finish_reason is not None

    def _complete(self) -> None:
        """Mark the request finished: wake blocking waiters and run the completion callback (once)."""
        self._done.set()
        callback, self.on_done = self.on_done, None
        if callback is not None:
            callback(self)

    def wait(self, timeout: Optional[float] = None) -> "GenerationRequest":
        if not self._done.wait(timeout):
            raise TimeoutError(f"request {self.id} did not finish within {timeout} s")
        if self.error is not None:
            raise self.error
        return self


def _left_pad(t: torch.Tensor, n: int, dim: int) -> torch.Tensor:
    if n == 0:
        return t
    shape = list(t.shape)
    shape[dim] = n
    return torch.cat((t.new_zeros(shape), t), dim=dim)


class Engine:
    """Owns the model and the running batch.  Thread-safe ``submit``; the batch itself is advanced either by the
    background thread (``start``) or by calling ``step`` / ``run_until_idle`` from one thread."""

    def __init__(
        self, model, tokenizer, max_batch: int = 32, device: Optional[torch.device] = None, kv_cache: str = "auto",
        window: Optional[int] = None, bucket: int = 128, cuda_graphs: Optional[bool] = None, max_queue: int = 0,
        decode_kernels: Optional[bool] = None,
    ):
        """``kv_cache``: ``"static"`` decodes against preallocated windows with fixed shapes (CUDA graphs on a GPU;
        :mod:`olmo_b200.serve.static_cache`), ``"dynamic"`` concatenates caches through ``OLMo.forward``; ``"auto"``
        picks static on a GPU when the architecture allows it.  ``window`` bounds prompt + completion per request in
        static mode (default: the model's context length).  ``decode_kernels``: use this library's decode kernels in
        static mode (default: whenever they cover the model; ``False`` keeps the module-level step)."""
        from .static_cache import StaticWindow, supports_static_window

        self.model = model.eval()
        self.tokenizer = tokenizer
        self.config = model.config
        self.device = device or next(model.parameters()).device
        # learned absolute positions do not survive the shift of a left-padded window: one row at a time then
        self.max_batch = max_batch if (self.config.rope or self.config.alibi) else 1
        if kv_cache not in ("auto", "static", "dynamic"):
            raise ValueError(f"kv_cache must be auto, static or dynamic, not {kv_cache!r}")
        if kv_cache == "static" and not supports_static_window(self.config):
            raise ValueError("the static key/value window needs rotary position embeddings and ungrouped blocks")
        use_static = kv_cache == "static" or (kv_cache == "auto" and self.device.type == "cuda" and supports_static_window(self.config))
        self._static: Optional[StaticWindow] = (
            StaticWindow(self.model, self.max_batch, window=window, bucket=bucket, cuda_graphs=cuda_graphs, fused=decode_kernels)
            if use_static else None
        )
        self._active: Optional[torch.Tensor] = None  # rows of the static window in the order of ``_rows``
        self.max_queue = max_queue  # 0 = unbounded; otherwise ``submit`` refuses when that many requests wait
        self.eos_token_id = getattr(tokenizer, "eos_token_id", None)
        if self.eos_token_id is None:
            self.eos_token_id = self.config.eos_token_id
        self._ids = itertools.count()
        self._queue: Deque[GenerationRequest] = deque()
        self._lock = threading.Lock()
        self._wake = threading.Condition(self._lock)
        self._thread: Optional[threading.Thread] = None
        self._stopping = False
        # running batch
        self._rows: List[GenerationRequest] = []
        self._kv: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None
        self._mask: Optional[torch.Tensor] = None  # [rows, L] 1 = real token
        self._last: Optional[torch.Tensor] = None  # [rows] token to feed next
        # seconds are host wall clock around a whole step; every step ends with a device-to-host read of the sampled tokens
        self.stats: Dict[str, float] = {"prefill_tokens": 0, "decode_tokens": 0, "decode_steps": 0, "requests": 0,
                                        "prefill_seconds": 0.0, "decode_seconds": 0.0}

    # ------------------------------------------------------------------------------- submission
    def submit(
        self,
        prompt_ids: Sequence[int],
        params: Optional[SamplingParams] = None,
        on_token: Optional[Callable[[GenerationRequest, int, str], None]] = None,
        on_done: Optional[Callable[[GenerationRequest], None]] = None,
    ) -> GenerationRequest:
        params = params or SamplingParams()
        params.validate()
        prompt = list(prompt_ids) or [self.eos_token_id]
        limit = self.config.max_sequence_length if self._static is None else self._static.window
        if len(prompt) + 1 > limit:
            raise ContextLengthError(f"prompt of {len(prompt)} tokens leaves no room in a context of {limit}")
        request = GenerationRequest(next(self._ids), prompt, params, on_token, on_done)
        if params.seed is not None:
            request._generator = torch.Generator(device="cpu").manual_seed(int(params.seed))
        with self._wake:
            if self.max_queue and len(self._queue) >= self.max_queue:
                raise QueueFullError(f"{len(self._queue)} requests are already waiting")
            self._queue.append(request)
            self._wake.notify()
        return request

    def cancel(self, request: GenerationRequest) -> None:
        """Stop generating for ``request`` (a client went away).  A waiting request leaves the queue at once; a
        running one is marked and gives its row back at the next step boundary."""
        with self._wake:
            if request in self._queue:
                self._queue.remove(request)
                request.finish_reason = "cancelled"
                request.finished_at = time.monotonic()
                request._complete()
                return
        request._cancelled = True

    def generate(self, prompts: Sequence[Sequence[int]], params=None) -> List[GenerationRequest]:
        """Synchronous convenience: submit, then advance the batch (or wait for the background thread)."""
        if isinstance(params, SamplingParams) or params is None:
            params = [params] * len(prompts)
        requests = [self.submit(p, sp) for p, sp in zip(prompts, params)]
        if self._thread is None:
            self.run_until_idle()
        return [r.wait() for r in requests]

    # ------------------------------------------------------------------------------- scheduling
    @property
    def idle(self) -> bool:
        with self._lock:
            return not self._queue and not self._rows

    def run_until_idle(self) -> None:
        while self.step():
            pass

    def start(self) -> None:
        if self._thread is not None:
            return
        self._stopping = False
        self._thread = threading.Thread(target=self._loop, name="olmo-serve-engine", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        with self._wake:
            self._stopping = True
            self._wake.notify_all()
        if self._thread is not None:
            self._thread.join()
            self._thread = None

    def _loop(self) -> None:
        while True:
            with self._wake:
                while not self._stopping and not self._queue and not self._rows:
                    self._wake.wait()
                if self._stopping:
                    break
            try:
                self.step()
            except BaseException as exc:  # a failed step fails the requests in flight, not the server
                self._fail_all(exc)
        self._fail_all(RuntimeError("engine stopped"))

    def _fail_all(self, exc: BaseException) -> None:
        with self._lock:
            pending = list(self._queue)
            self._queue.clear()
        for request in self._rows + pending:
            request.error, request.finish_reason = exc, "error"
            request.finished_at = time.monotonic()
            request._complete()
        if self._static is not None:
            for request in self._rows:
                self._static.release(request._row)
            self._active = None
        self._rows, self._kv, self._mask, self._last = [], None, None, None

    @torch.no_grad()
    def step(self) -> bool:
        """Admit waiting requests into free rows (one batched prefill), then decode one token for every row.
        Returns False when there was nothing to do."""
        with self._lock:
            room = self.max_batch - len(self._rows)
            admitted = [self._queue.popleft() for _ in range(min(room, len(self._queue)))]
        started = time.perf_counter()
        if admitted:
            self._prefill(admitted)
            self.stats["prefill_seconds"] += time.perf_counter() - started
        elif self._rows:
            self._decode()
            self.stats["decode_seconds"] += time.perf_counter() - started
        else:
            return False
        return True

    # ---------------------------------------------------------------------------------- prefill
    def _prefill(self, requests: List[GenerationRequest]) -> None:
        width = max(len(r.prompt_ids) for r in requests)
        pad = getattr(self.tokenizer, "pad_token_id", None)
        pad = self.config.pad_token_id if pad is None else pad
        ids = torch.full((len(requests), width), pad, dtype=torch.long)
        mask = torch.zeros(len(requests), width)
        for i, r in enumerate(requests):
            ids[i, width - len(r.prompt_ids) :] = torch.tensor(r.prompt_ids, dtype=torch.long)
            mask[i, width - len(r.prompt_ids) :] = 1
        ids, mask = ids.to(self.device), mask.to(self.device)
        ragged = bool((mask == 0).any())
        out = self.model(ids, attention_mask=mask if ragged else None, use_cache=True, last_logits_only=True)
        self.stats["prefill_tokens"] += int(mask.sum())
        self.stats["requests"] += len(requests)
        kv = [(k, v) for k, v in out.attn_key_values]
        tokens = self._sample(requests, out.logits[:, -1, :])
        if self._static is not None:
            for request, row in zip(requests, self._static.admit(kv, mask, tokens)):
                request._row = row
            self._rows = self._rows + requests
            self._active = None
            self._retire()
            return
        # merge into the running window
        if self._rows:
            assert self._kv is not None and self._mask is not None and self._last is not None
            old_len, new_len = self._mask.shape[1], width
            grow_old, grow_new = max(0, new_len - old_len), max(0, old_len - new_len)
            self._kv = [
                (torch.cat((_left_pad(ok, grow_old, -2), _left_pad(nk, grow_new, -2)), dim=0),
                 torch.cat((_left_pad(ov, grow_old, -2), _left_pad(nv, grow_new, -2)), dim=0))
                for (ok, ov), (nk, nv) in zip(self._kv, kv)
            ]
            self._mask = torch.cat((_left_pad(self._mask, grow_old, 1), _left_pad(mask, grow_new, 1)), dim=0)
            self._last = torch.cat((self._last, tokens), dim=0)
        else:
            self._kv, self._mask, self._last = kv, mask, tokens
        self._rows = self._rows + requests
        self._retire()

    # ----------------------------------------------------------------------------------- decode
    def _decode(self) -> None:
        if self._static is not None:
            if self._active is None:
                self._active = torch.tensor([r._row for r in self._rows], device=self.device)
            logits = self._static.decode(self._active)
            tokens = self._sample(self._rows, logits.index_select(0, self._active))
            self._static.advance(self._active, tokens)
            self.stats["decode_tokens"] += len(self._rows)
            self.stats["decode_steps"] += 1
            self._retire()
            return
        assert self._kv is not None and self._mask is not None and self._last is not None
        mask = torch.cat((self._mask, self._mask.new_ones(self._mask.shape[0], 1)), dim=1)
        out = self.model(
            self._last.unsqueeze(1), attention_mask=mask, past_key_values=self._kv, use_cache=True, last_logits_only=True
        )
        self._kv = [(k, v) for k, v in out.attn_key_values]
        self._mask = mask
        self._last = self._sample(self._rows, out.logits[:, -1, :])
        self.stats["decode_tokens"] += len(self._rows)
        self.stats["decode_steps"] += 1
        self._retire()

    # ---------------------------------------------------------------------------------- sampling
    def _sample(self, requests: List[GenerationRequest], logits: torch.Tensor) -> torch.Tensor:
        """One token per row under that row's own parameters; records it on the request."""
        logits = logits.float()
        n, vocab = logits.shape
        temperature = torch.tensor([r.params.temperature for r in requests], device=logits.device)
        greedy = temperature == 0
        tokens = logits.argmax(dim=-1)
        if not bool(greedy.all()):
            scaled = logits / temperature.clamp_min(1e-6).unsqueeze(1)
            top_k = torch.tensor([r.params.top_k or vocab for r in requests], device=logits.device).clamp_max(vocab)
            top_p = torch.tensor([r.params.top_p for r in requests], device=logits.device)
            if bool((top_k < vocab).any()) or bool((top_p < 1).any()):
                ordered, order = scaled.sort(dim=-1, descending=True)
                probs = ordered.softmax(dim=-1)
                before = probs.cumsum(dim=-1) - probs  # mass strictly ahead of each candidate
                rank = torch.arange(vocab, device=logits.device).unsqueeze(0)
                drop = (rank >= top_k.unsqueeze(1)) | (before >= top_p.unsqueeze(1))
                drop[:, 0] = False
                ordered = ordered.masked_fill(drop, float("-inf"))
                scaled = torch.full_like(scaled, float("-inf")).scatter(1, order, ordered)
            probs = scaled.softmax(dim=-1)
            seeded = [i for i, r in enumerate(requests) if r._generator is not None and r.params.temperature > 0]
            drawn = torch.multinomial(probs, 1).squeeze(1)
            for i in seeded:  # a seeded request draws from its own CPU stream, whatever else is in the batch
                drawn[i] = torch.multinomial(probs[i].cpu(), 1, generator=requests[i]._generator).item()
            tokens = torch.where(greedy, tokens, drawn)
        chosen = tokens.tolist()
        logprobs: Optional[List[float]] = None
        if any(r.params.logprobs for r in requests):
            logprobs = F.log_softmax(logits, dim=-1).gather(1, tokens.unsqueeze(1)).squeeze(1).tolist()
        now = time.monotonic()
        for i, (request, token) in enumerate(zip(requests, chosen)):
            if request.first_token_at is None:
                request.first_token_at = now
            self._record(request, token, None if logprobs is None else logprobs[i])
        return tokens

    def _record(self, request: GenerationRequest, token: int, logprob: Optional[float]) -> None:
        params = request.params
        if request._cancelled:
            request.finish_reason = "cancelled"
        elif (token == self.eos_token_id and not params.ignore_eos) or token in params.stop_token_ids:
            request.finish_reason = "stop"
        else:
            request.token_ids.append(token)
            if logprob is not None and params.logprobs:
                request.token_logprobs.append(logprob)
            text = self.tokenizer.decode(request.token_ids)
            cut = min((p for p in (text.find(s) for s in params.stop if s) if p >= 0), default=-1)
            if cut >= 0:
                text, request.finish_reason = text[:cut], "stop"
            request.text = text
            context = self.config.max_sequence_length if self._static is None else self._static.window
            budget = min(params.max_tokens, context - len(request.prompt_ids))
            if request.finish_reason is None and len(request.token_ids) >= budget:
                request.finish_reason = "length"
        if request.on_token is not None:
            # hold back a trailing partial character (an incomplete byte sequence decodes to U+FFFD) and anything
            # that could still turn into a stop string
            upto = len(request.text)
            if request.finish_reason is None:
                if request.text.endswith("\ufffd"):
                    upto = len(request.text.rstrip("\ufffd"))
                hold = max((len(s) - 1 for s in params.stop if s), default=0)
                upto = max(request._emitted, upto - hold)
            delta = request.text[request._emitted : upto]
            request._emitted = max(request._emitted, upto)
            if delta or request.finish_reason is not None:
                request.on_token(request, token, delta)

    def _retire(self) -> None:
        """Drop finished rows and trim the padding every remaining row shares."""
        keep = [i for i, r in enumerate(self._rows) if not r.finished]
        done = [r for r in self._rows if r.finished]
        if self._static is not None:
            if done:
                now = time.monotonic()
                for r in done:
                    self._static.release(r._row)
                    r.finished_at = now
                    r._complete()
                self._rows = [self._rows[i] for i in keep]
                self._active = None
                self._static.compact()
            return
        if done:
            now = time.monotonic()
            if keep:
                index = torch.tensor(keep, device=self.device)
                assert self._kv is not None and self._mask is not None and self._last is not None
                self._kv = [(k.index_select(0, index), v.index_select(0, index)) for k, v in self._kv]
                self._mask = self._mask.index_select(0, index)
                self._last = self._last.index_select(0, index)
            else:
                self._kv, self._mask, self._last = None, None, None
            self._rows = [self._rows[i] for i in keep]
            for r in done:
                r.finished_at = now
                r._complete()
        if self._rows and self._mask is not None and self._kv is not None:
            slack = int(self._mask.shape[1] - int(self._mask.sum(dim=1).max()))
            if slack > 0:
                self._kv = [(k[..., slack:, :], v[..., slack:, :]) for k, v in self._kv]
                self._mask = self._mask[:, slack:]
