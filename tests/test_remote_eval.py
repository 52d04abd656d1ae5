"""Remote (OpenAI-compatible endpoint) evaluation helpers against an in-process fake server."""
import asyncio
import json
import socket
import threading

import pytest

from olmo_b200.inference import remote


class FakeEndpoint:
    """Completions and chat routes that echo; the first ``fail_first`` requests get a 500."""

    def __init__(self, fail_first: int = 0):
        from aiohttp import web

        self.calls, self.fail_first, self.in_flight, self.max_in_flight = [], fail_first, 0, 0
        self.app = web.Application()
        self.app.router.add_post("/v1/completions", self.completions)
        self.app.router.add_post("/v1/chat/completions", self.chat)
        self.web = web
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            self.port = s.getsockname()[1]
        self.loop = asyncio.new_event_loop()
        self.ready = threading.Event()
        self.thread = threading.Thread(target=self._serve, daemon=True)
        self.thread.start()
        assert self.ready.wait(20)

    def _serve(self):
        asyncio.set_event_loop(self.loop)
        self.runner = self.web.AppRunner(self.app)
        self.loop.run_until_complete(self.runner.setup())
        self.loop.run_until_complete(self.web.TCPSite(self.runner, "127.0.0.1", self.port).start())
        self.ready.set()
        self.loop.run_forever()

    async def _handle(self, request, make):
        body = await request.json()
        self.calls.append(body)
        if len(self.calls) <= self.fail_first:
            return self.web.Response(status=500, text="try again")
        if body.get("model") == "missing":
            return self.web.Response(status=404, text="no such model")
        self.in_flight += 1
        self.max_in_flight = max(self.max_in_flight, self.in_flight)
        await asyncio.sleep(0.02)
        self.in_flight -= 1
        return self.web.json_response({"choices": [make(body)], "auth": request.headers.get("Authorization")})

    async def completions(self, request):
        return await self._handle(request, lambda b: {"text": " " + b["prompt"].split()[-1].upper()})

    async def chat(self, request):
        return await self._handle(request, lambda b: {"message": {"role": "assistant", "content": b["messages"][-1]["content"][::-1]}})

    def close(self):
        self.loop.call_soon_threadsafe(self.loop.stop)
        self.thread.join(10)

    @property
    def url(self):
        return f"http://127.0.0.1:{self.port}/v1"


@pytest.fixture
def endpoint():
    ep = FakeEndpoint(fail_first=2)
    yield ep
    ep.close()


def test_requests_are_concurrent_ordered_and_retried(endpoint):
    prompts = [f"say w{i}" for i in range(12)]
    out = asyncio.run(remote.dispatch_prompt_requests(endpoint.url, prompts, "m", api_key="k", concurrency=4, backoff_s=0.01, max_tokens=1))
    assert [r["choices"][0]["text"] for r in out] == [f" W{i}" for i in range(12)]
    assert out[0]["auth"] == "Bearer k" and 1 < endpoint.max_in_flight <= 4
    assert len(endpoint.calls) == 14 and endpoint.calls[-1]["max_tokens"] == 1  # two rejected attempts were repeated
    chats = asyncio.run(remote.dispatch_chat_requests(endpoint.url, [[{"role": "user", "content": "abc"}]], "m"))
    assert chats[0]["choices"][0]["message"]["content"] == "cba"
    with pytest.raises(ValueError, match="404"):  # a request the server will never accept is not retried
        asyncio.run(remote.dispatch_prompt_requests(endpoint.url, ["x y"], "missing", retries=5, backoff_s=0.01))


def test_answers_are_cached_so_that_a_rerun_only_asks_what_is_missing(tmp_path, endpoint):
    instances = [{"id": i, "prompt": f"q a{i}"} for i in range(5)]
    cache = tmp_path / "out" / "answers.jsonl"
    first = remote.query_completion_model(endpoint.url, "m", instances[:3], batch_size=2, output_path=str(cache), backoff_s=0.01)
    assert [r["output"] for r in first] == [" A0", " A1", " A2"] and len(cache.read_text().splitlines()) == 3
    before = len(endpoint.calls)
    again = remote.query_completion_model(endpoint.url, "m", instances, batch_size=8, output_path=str(cache))
    assert [r["output"] for r in again] == [f" A{i}" for i in range(5)] and len(endpoint.calls) - before == 2
    assert [json.loads(line)["id"] for line in cache.read_text().splitlines()] == [0, 1, 2, 3, 4]
    chat = remote.query_chat_model(endpoint.url, "m", [{"id": "a", "prompt": "xyz"}], reuse_existing=False)
    assert chat[0]["output"] == "zyx"
    assert remote._first_choice_letter(" (B) because") == "B" and remote._first_choice_letter("The answer") is None
