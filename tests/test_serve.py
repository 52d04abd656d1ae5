"""Serving: the continuous-batching engine against single-sequence decoding, and the OpenAI-compatible routes."""
import json

import pytest
import torch

from olmo_b200.config import ActivationType, LayerNormType, ModelConfig
from olmo_b200.models.olmo import OLMo
from olmo_b200.serve import ContextLengthError, Engine, SamplingParams, create_app, default_chat_template

VOCAB = 128
EOS = 1


class CharTokenizer:
    """One token per character (id = code point below 128); id 1 ends a text."""

    pad_token_id = 0
    eos_token_id = EOS

    def encode(self, s, add_special_tokens=True):
        return [min(ord(c), VOCAB - 1) for c in s] + ([EOS] if add_special_tokens else [])

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(i) for i in ids if i > 1)


def tiny_model(**overrides) -> OLMo:
    torch.manual_seed(0)
    cfg = ModelConfig(
        d_model=64, n_heads=4, n_layers=2, mlp_hidden_size=128, activation_type=ActivationType.swiglu, rope=True,
        layer_norm_type=LayerNormType.rms, layer_norm_with_affine=True, include_bias=False, vocab_size=VOCAB,
        embedding_size=VOCAB, max_sequence_length=48, eos_token_id=EOS, pad_token_id=0, weight_tying=False, init_device="cpu",
    )
    for k, v in overrides.items():
        setattr(cfg, k, v)
    model = OLMo(cfg).eval()
    with torch.no_grad():  # make the end token rare but possible, so that runs have some length
        model.transformer.ff_out.weight[EOS] *= 0.5
    return model


def greedy_reference(model: OLMo, prompt, steps):
    """Most likely continuation by full re-evaluation of the growing sequence (no cache, no batch, no padding)."""
    ids, out = list(prompt), []
    with torch.no_grad():
        for _ in range(steps):
            token = int(model(torch.tensor([ids])).logits[0, -1].argmax())
            if token == EOS:
                break
            ids.append(token)
            out.append(token)
    return out


PROMPTS = [[ord(c) for c in p] for p in ("hello world", "a", "the quick brown fox", "olmo!", "zz top", "serve me tokens")]


@pytest.mark.parametrize("variant", [dict(), dict(alibi=True, rope=False), dict(n_kv_heads=2, attention_layer_norm=True, norm_after=True)])
def test_continuous_batching_matches_single_sequence_greedy(variant):
    model = tiny_model(**variant)
    engine = Engine(model, CharTokenizer(), max_batch=4)
    greedy = SamplingParams(max_tokens=12, temperature=0.0)
    requests = [engine.submit(p, greedy) for p in PROMPTS[:3]]
    for _ in range(4):  # let the first group run ahead, then more requests join a batch that is mid-flight
        engine.step()
    requests += [engine.submit(p, greedy) for p in PROMPTS[3:]]
    engine.run_until_idle()
    assert engine.idle
    for prompt, request in zip(PROMPTS, requests):
        assert request.finished
        assert request.token_ids == greedy_reference(model, prompt, 12), prompt
        assert request.finish_reason == ("length" if len(request.token_ids) == 12 else "stop")
    assert engine.stats["requests"] == len(PROMPTS) and engine.stats["prefill_tokens"] == sum(map(len, PROMPTS))
    # six requests with at most four rows: the later ones waited for rows to free up
    assert engine.stats["decode_steps"] < sum(len(r.token_ids) for r in requests)


def test_learned_positions_decode_one_row_at_a_time():
    model = tiny_model(rope=False)
    engine = Engine(model, CharTokenizer(), max_batch=8)
    assert engine.max_batch == 1
    done = engine.generate(PROMPTS[:3], SamplingParams(max_tokens=5, temperature=0.0))
    for prompt, request in zip(PROMPTS, done):
        assert request.token_ids == greedy_reference(model, prompt, 5)


def test_stop_conditions_and_limits():
    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=4)
    base = engine.generate([PROMPTS[0]], SamplingParams(max_tokens=16, temperature=0.0, ignore_eos=True))[0]
    assert len(base.token_ids) == 16 and base.finish_reason == "length"
    needle = base.text[5:7]
    cut = base.text.find(needle)
    stopped = engine.generate([PROMPTS[0]], SamplingParams(max_tokens=16, temperature=0.0, ignore_eos=True, stop=[needle]))[0]
    assert stopped.finish_reason == "stop" and stopped.text == base.text[:cut]
    by_id = engine.generate([PROMPTS[0]], SamplingParams(max_tokens=16, temperature=0.0, ignore_eos=True, stop_token_ids=[base.token_ids[3]]))[0]
    assert by_id.finish_reason == "stop" and by_id.token_ids == base.token_ids[: base.token_ids.index(base.token_ids[3])]
    # the context bounds the completion, and a prompt that fills it is refused
    long_prompt = [65] * 44
    capped = engine.generate([long_prompt], SamplingParams(max_tokens=100, temperature=0.0, ignore_eos=True))[0]
    assert len(capped.token_ids) == 4 and capped.finish_reason == "length"
    with pytest.raises(ContextLengthError):
        engine.submit([65] * 48)
    with pytest.raises(ValueError):
        engine.submit([65], SamplingParams(top_p=0.0))


def test_sampling_is_reproducible_per_request_and_respects_truncation():
    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=8)
    seeded = SamplingParams(max_tokens=10, temperature=1.5, seed=7, ignore_eos=True)
    alone = engine.generate([PROMPTS[0]], seeded)[0].token_ids
    # the same seeded request inside a batch of unrelated sampled and greedy rows draws the same tokens
    mixed = engine.generate(
        [PROMPTS[1], PROMPTS[0], PROMPTS[2]],
        [SamplingParams(max_tokens=10, temperature=0.9), seeded, SamplingParams(max_tokens=10, temperature=0.0)],
    )
    assert mixed[1].token_ids == alone
    assert mixed[2].token_ids == greedy_reference(model, PROMPTS[2], 10)
    other = engine.generate([PROMPTS[0]], SamplingParams(max_tokens=10, temperature=1.5, seed=8, ignore_eos=True))[0].token_ids
    assert other != alone
    # top_k = 1 and a vanishing nucleus both reduce to the most likely token
    greedy = greedy_reference(model, PROMPTS[3], 8)
    for params in (SamplingParams(max_tokens=8, temperature=2.0, top_k=1), SamplingParams(max_tokens=8, temperature=2.0, top_p=1e-6)):
        assert engine.generate([PROMPTS[3]], params)[0].token_ids == greedy
    # log-probabilities of the chosen tokens
    lp = engine.generate([PROMPTS[3]], SamplingParams(max_tokens=8, temperature=0.0, logprobs=True))[0]
    ids = torch.tensor([PROMPTS[3] + lp.token_ids])
    with torch.no_grad():
        ref = torch.log_softmax(model(ids).logits[0].float(), dim=-1)
    start = len(PROMPTS[3]) - 1
    expect = [float(ref[start + i, t]) for i, t in enumerate(lp.token_ids)]
    assert lp.token_logprobs == pytest.approx(expect, abs=1e-4)


def test_streaming_callbacks_reassemble_the_text():
    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=4)
    pieces, reasons = [], []

    def on_token(request, token, delta):
        pieces.append(delta)
        reasons.append(request.finish_reason)

    base = engine.generate([PROMPTS[2]], SamplingParams(max_tokens=14, temperature=0.0, ignore_eos=True))[0]
    needle = base.text[8:10]
    request = engine.submit(PROMPTS[2], SamplingParams(max_tokens=14, temperature=0.0, ignore_eos=True, stop=[needle]), on_token)
    engine.run_until_idle()
    assert "".join(pieces) == request.text == base.text[: base.text.find(needle)]
    assert reasons[-1] == "stop" and all(r is None for r in reasons[:-1])


def test_chat_template_layout():
    text = default_chat_template([
        {"role": "system", "content": "Be brief."}, {"role": "user", "content": "Hi"},
        {"role": "assistant", "content": "Hello."}, {"role": "user", "content": [{"type": "text", "text": "Bye"}]},
    ])
    assert text == "<|endoftext|><|system|>\nBe brief.\n<|user|>\nHi\n<|assistant|>\nHello.<|endoftext|>\n<|user|>\nBye\n<|assistant|>\n"
    with pytest.raises(ValueError):
        default_chat_template([{"role": "tool", "content": "x"}])


def test_openai_routes():
    pytest.importorskip("fastapi")
    pytest.importorskip("httpx")
    from fastapi.testclient import TestClient

    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=4)
    app = create_app(engine, model_name="tiny-olmo", api_key="secret")
    auth = {"Authorization": "Bearer secret"}
    with TestClient(app) as client:
        assert client.get("/health").json()["status"] == "ok"
        listing = client.get("/v1/models").json()
        assert listing["data"][0]["id"] == "tiny-olmo" and listing["data"][0]["max_model_len"] == 48

        assert client.post("/v1/completions", json={"prompt": "hi"}).status_code == 401
        body = {"model": "tiny-olmo", "prompt": ["hello world", "a"], "max_tokens": 6, "temperature": 0, "logprobs": 1, "echo": True}
        reply = client.post("/v1/completions", json=body, headers=auth).json()
        assert reply["object"] == "text_completion" and len(reply["choices"]) == 2
        for choice, prompt in zip(reply["choices"], ("hello world", "a")):
            expect = greedy_reference(model, [ord(c) for c in prompt], 6)
            assert choice["text"] == prompt + CharTokenizer().decode(expect)
            assert len(choice["logprobs"]["token_logprobs"]) == len(expect)
        assert reply["usage"]["prompt_tokens"] == 12
        assert reply["usage"]["total_tokens"] == 12 + reply["usage"]["completion_tokens"]

        by_ids = client.post("/v1/completions", json={"prompt": [104, 105], "max_tokens": 4, "temperature": 0}, headers=auth).json()
        assert by_ids["choices"][0]["text"] == CharTokenizer().decode(greedy_reference(model, [104, 105], 4))

        several = client.post("/v1/completions", json={"prompt": "x", "max_tokens": 8, "temperature": 1.3, "n": 3, "seed": 5, "ignore_eos": True}, headers=auth).json()
        texts = [c["text"] for c in several["choices"]]
        assert len(texts) == 3 and len(set(texts)) > 1
        again = client.post("/v1/completions", json={"prompt": "x", "max_tokens": 8, "temperature": 1.3, "n": 3, "seed": 5, "ignore_eos": True}, headers=auth).json()
        assert [c["text"] for c in again["choices"]] == texts

        chat = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "Hi"}], "max_tokens": 5, "temperature": 0}, headers=auth).json()
        prompt_ids = CharTokenizer().encode(default_chat_template([{"role": "user", "content": "Hi"}]), add_special_tokens=False)
        assert chat["object"] == "chat.completion"
        assert chat["choices"][0]["message"] == {"role": "assistant", "content": CharTokenizer().decode(greedy_reference(model, prompt_ids, 5))}
        assert chat["usage"]["prompt_tokens"] == len(prompt_ids)

        with client.stream("POST", "/v1/chat/completions", json={"messages": [{"role": "user", "content": "Hi"}], "max_tokens": 5, "temperature": 0, "stream": True}, headers=auth) as response:
            assert response.headers["content-type"].startswith("text/event-stream")
            events = [line[6:] for line in response.iter_lines() if line.startswith("data: ")]
        assert events[-1] == "[DONE]"
        chunks = [json.loads(e) for e in events[:-1]]
        assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
        assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == chat["choices"][0]["message"]["content"]
        assert chunks[-1]["choices"][0]["finish_reason"] in ("stop", "length")

        with client.stream("POST", "/v1/completions", json={"prompt": "hello world", "max_tokens": 6, "temperature": 0, "stream": True}, headers=auth) as response:
            events = [line[6:] for line in response.iter_lines() if line.startswith("data: ")]
        streamed = "".join(json.loads(e)["choices"][0]["text"] for e in events[:-1])
        assert streamed == CharTokenizer().decode(greedy_reference(model, [ord(c) for c in "hello world"], 6))

        exposition = client.get("/metrics").text
        assert "# TYPE olmo_generated_tokens_total counter" in exposition
        counters = dict(line.split() for line in exposition.splitlines() if line and not line.startswith("#"))
        assert int(counters["olmo_requests_total"]) == engine.stats["requests"] > 0 and counters["olmo_requests_running"] == "0"

        for bad, status, code in [
            ({"prompt": "x" * 60}, 400, "context_length_exceeded"),
            ({"prompt": "x", "model": "other"}, 404, "model_not_found"),
            ({"prompt": "x", "temperature": -1}, 400, None),
            ({"prompt": {"a": 1}}, 400, None),
            ({"prompt": "x", "n": 0}, 400, None),
        ]:
            r = client.post("/v1/completions", json=bad, headers=auth)
            assert r.status_code == status and r.json()["error"]["code"] == code, bad
        assert client.post("/v1/chat/completions", json={"messages": []}, headers=auth).status_code == 400
    assert engine._thread is None  # stopped with the application


@pytest.mark.gpu
def test_engine_on_gpu_with_native_attention_shapes():
    """The engine on the device: batched decoding with padding agrees with cache-free greedy decoding of each prompt,
    for both decode back ends (the static one replays CUDA graphs), with full-precision weights and with 4-bit weights
    (whose matrix-vector kernel serves the decode steps)."""
    from olmo_b200.inference.quantize import quantize_model

    model = tiny_model(d_model=256, n_heads=2, mlp_hidden_size=512).cuda()

    def reference(prompt):
        ids, out = list(prompt), []
        with torch.no_grad():
            for _ in range(10):
                token = int(model(torch.tensor([ids], device="cuda")).logits[0, -1].argmax())
                if token == EOS:
                    break
                ids.append(token)
                out.append(token)
        return out

    for quantized in (False, True):
        if quantized:
            quantize_model(model, [torch.full((1, 8), 5, device="cuda")], method="rtn", group=128)
        expected = [reference(p) for p in PROMPTS]
        for kv_cache in ("dynamic", "static"):
            engine = Engine(model, CharTokenizer(), max_batch=4, kv_cache=kv_cache, bucket=16)
            done = engine.generate(PROMPTS, SamplingParams(max_tokens=10, temperature=0.0))
            if kv_cache == "static":
                assert engine._static.cuda_graphs and engine._static.graph_replays == engine.stats["decode_steps"] > 0
            agree = total = 0
            for out, request in zip(expected, done):
                got = request.token_ids
                if quantized:  # bf16 rounding differs between the row counts: compare the first choice only
                    out, got = out[:1], got[:1]
                n = min(len(out), len(got))
                agree += sum(a == b for a, b in zip(out[:n], got[:n]))
                total += max(len(out), len(got))
            # a near-tie may flip one argmax between the batched and the single-row kernels
            assert agree >= 0.8 * total, (quantized, kv_cache, agree, total)


@pytest.mark.parametrize("variant", [dict(), dict(n_kv_heads=2, attention_layer_norm=True, norm_after=True, rope_full_precision=False)])
def test_static_window_matches_single_sequence_greedy(variant):
    """Fixed-shape decoding: rows join mid-flight, long prompts push the window right, retired rows let it slide
    back, and every request still equals cache-free greedy decoding of its own prompt."""
    model = tiny_model(**variant)
    engine = Engine(model, CharTokenizer(), max_batch=3, kv_cache="static", bucket=8)
    window = engine._static
    assert window is not None and window.window == 48 and window.kv_bytes() > 0
    greedy = SamplingParams(max_tokens=12, temperature=0.0)
    requests = [engine.submit(p, greedy) for p in PROMPTS[:2]]  # lengths 11 and 1
    for _ in range(5):
        engine.step()
    requests.append(engine.submit(PROMPTS[2], greedy))  # 19 tokens: longer than the window's write column
    engine.step()
    assert window.cur >= len(PROMPTS[2])
    requests += [engine.submit(p, greedy) for p in PROMPTS[3:]]
    engine.run_until_idle()
    for prompt, request in zip(PROMPTS, requests):
        assert request.token_ids == greedy_reference(model, prompt, 12), prompt
    assert window.free_rows == 3 and window.cur == 0

    # a request that runs to the end of the window finishes by length; with neighbours retiring the window compacts
    long_prompt = [66] * 30
    capped = engine.submit(long_prompt, SamplingParams(max_tokens=100, temperature=0.0, ignore_eos=True))
    short = engine.submit(PROMPTS[1], SamplingParams(max_tokens=30, temperature=0.0, ignore_eos=True))
    engine.run_until_idle()
    assert len(capped.token_ids) == 18 and capped.finish_reason == "length"
    assert short.token_ids == greedy_reference_no_eos(model, PROMPTS[1], 30)
    with pytest.raises(ContextLengthError):
        engine.submit([65] * 48)


def greedy_reference_no_eos(model, prompt, steps):
    ids, out = list(prompt), []
    with torch.no_grad():
        for _ in range(steps):
            token = int(model(torch.tensor([ids])).logits[0, -1].argmax())
            ids.append(token)
            out.append(token)
    return out


def test_static_window_slides_left_when_it_fills():
    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=2, kv_cache="static", window=24, bucket=4)
    window = engine._static
    # a stream of short requests keeps the window busy far longer than its width
    params = SamplingParams(max_tokens=9, temperature=0.0, ignore_eos=True)
    requests = []
    for i in range(8):
        requests.append(engine.submit(PROMPTS[i % len(PROMPTS)][:6], params))
        engine.step()
        engine.step()
    engine.run_until_idle()
    for i, request in enumerate(requests):
        assert request.token_ids == greedy_reference_no_eos(model, PROMPTS[i % len(PROMPTS)][:6], 9), i
    assert engine.stats["decode_steps"] + 8 > window.window  # more columns were written than the window holds


def test_static_window_is_refused_where_it_cannot_work():
    with pytest.raises(ValueError):
        Engine(tiny_model(alibi=True, rope=False), CharTokenizer(), kv_cache="static")
    assert Engine(tiny_model(alibi=True, rope=False), CharTokenizer(), kv_cache="auto")._static is None


def test_load_engine_from_a_checkpoint_folder(tmp_path):
    """``load_engine`` (what ``scripts/serve_openai.py`` calls): model, tokenizer and engine from an unsharded checkpoint."""
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    from olmo_b200.config import TokenizerConfig, TrainConfig
    from olmo_b200.serve import load_engine

    words = [f"w{i}" for i in range(60)]
    vocab = {w: i + 2 for i, w in enumerate(words)}
    vocab["<pad>"], vocab["<eos>"] = 0, 1
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="<pad>"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.add_special_tokens(["<eos>", "<pad>"])
    tok.save(str(tmp_path / "tokenizer.json"))

    model = tiny_model(vocab_size=62, embedding_size=64)
    ckpt = tmp_path / "step0-unsharded"
    ckpt.mkdir()
    torch.save(model.state_dict(), ckpt / "model.pt")
    cfg = TrainConfig(model=model.config, tokenizer=TokenizerConfig(identifier=str(tmp_path / "tokenizer.json")))
    cfg.save(ckpt / "config.yaml")

    engine = load_engine(str(ckpt), device="cpu", dtype="fp32", max_batch=2, kv_cache="static", window=32)
    prompt = engine.tokenizer.encode("w1 w2 w3 w4", add_special_tokens=False)
    assert prompt == [3, 4, 5, 6]
    done = engine.generate([prompt], SamplingParams(max_tokens=6, temperature=0.0))[0]
    assert done.token_ids == greedy_reference(model, prompt, 6)
    assert done.text == engine.tokenizer.decode(done.token_ids)


def test_cancellation_and_queue_limit():
    from olmo_b200.serve import QueueFullError

    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=1, max_queue=2)
    long_run = SamplingParams(max_tokens=30, temperature=0.0, ignore_eos=True)
    running = engine.submit(PROMPTS[0], long_run)
    engine.step()  # prefill: the only row is taken
    waiting = [engine.submit(PROMPTS[1], long_run), engine.submit(PROMPTS[2], long_run)]
    with pytest.raises(QueueFullError):
        engine.submit(PROMPTS[3], long_run)
    engine.cancel(waiting[0])  # leaves the queue at once
    assert waiting[0].finish_reason == "cancelled" and waiting[0]._done.is_set()
    for _ in range(3):
        engine.step()
    engine.cancel(running)  # gives its row back at the next step
    engine.step()
    assert running.finish_reason == "cancelled" and 0 < len(running.token_ids) < 30
    engine.run_until_idle()
    assert waiting[1].finish_reason == "length" and waiting[1].token_ids == greedy_reference_no_eos(model, PROMPTS[2], 29)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [dict(attention_layer_norm=True, norm_after=True), dict(layer_norm_type=LayerNormType.default, layer_norm_with_affine=False, clip_qkv=4.0), dict(n_kv_heads=1, attention_layer_norm=True, norm_after=True)])
def test_decode_kernels_match_the_module_level_step(variant):
    """One decode step on identical window state: this library's decode kernels against the module-level step (bf16)."""
    model = tiny_model(d_model=256, n_heads=2, mlp_hidden_size=512, attention_dropout=0.0, residual_dropout=0.0, embedding_dropout=0.0,
                       **variant).to(torch.bfloat16).cuda()
    engine = Engine(model, CharTokenizer(), max_batch=4, kv_cache="static", bucket=16, cuda_graphs=False)
    window = engine._static
    assert window.fused
    for p in PROMPTS[:3]:
        engine.submit(p, SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True))
    engine.step()  # prefill: three rows live, one idle
    engine.step()  # one decode step, so the window holds keys written by the decode kernels too
    active = torch.tensor([r._row for r in engine._rows], device="cuda")
    fused = window.decode(active).index_select(0, active).clone()
    window.fused = False
    plain = window.decode(active).index_select(0, active).clone()  # same column, same tokens: the step is idempotent
    window.fused = True
    assert torch.isfinite(fused).all()
    torch.testing.assert_close(fused, plain, rtol=5e-2, atol=5e-2)
    assert (fused.argmax(-1) == plain.argmax(-1)).float().mean() >= 0.66
    engine.run_until_idle()


@pytest.mark.gpu
def test_decode_kernels_under_cuda_graphs_generate_the_same_tokens():
    model = tiny_model(d_model=256, n_heads=2, mlp_hidden_size=512, attention_layer_norm=True, norm_after=True, attention_dropout=0.0,
                       residual_dropout=0.0, embedding_dropout=0.0).to(torch.bfloat16).cuda()
    params = SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True)
    eager = Engine(model, CharTokenizer(), max_batch=4, kv_cache="static", bucket=16, cuda_graphs=False).generate(PROMPTS, params)
    engine = Engine(model, CharTokenizer(), max_batch=4, kv_cache="static", bucket=16, cuda_graphs=True)
    graphed = engine.generate(PROMPTS, params)
    assert engine._static.fused and engine._static.graph_replays == engine.stats["decode_steps"] > 0
    assert [r.token_ids for r in graphed] == [r.token_ids for r in eager]  # same kernels, same inputs, replayed


def test_many_concurrent_http_requests_share_the_batch():
    pytest.importorskip("fastapi")
    httpx = pytest.importorskip("httpx")
    import asyncio

    model = tiny_model()
    engine = Engine(model, CharTokenizer(), max_batch=4)
    app = create_app(engine, model_name="tiny-olmo")
    prompts = ["hello world", "a", "the quick brown fox", "olmo!", "zz top", "serve me tokens"] * 2

    async def run():
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app), base_url="http://test") as client:
            calls = [client.post("/v1/completions", json={"prompt": p, "max_tokens": 6, "temperature": 0}) for p in prompts]
            return await asyncio.gather(*calls)

    engine.start()  # the ASGI transport does not run the application's lifespan
    try:
        replies = asyncio.run(run())
    finally:
        engine.stop()
    for prompt, reply in zip(prompts, replies):
        assert reply.status_code == 200
        assert reply.json()["choices"][0]["text"] == CharTokenizer().decode(greedy_reference(model, [ord(c) for c in prompt], 6))
    assert engine.stats["requests"] == len(prompts) and engine.stats["decode_steps"] < 6 * len(prompts)


def test_chat_template_from_file(tmp_path):
    pytest.importorskip("jinja2")
    from olmo_b200.serve import load_chat_template

    jinja = "{{ bos_token }}{% for m in messages %}{{ '<|' + m['role'] + '|>\\n' + m['content'] + '\\n' }}{% endfor %}{% if add_generation_prompt %}{{ '<|assistant|>\\n' }}{% endif %}"
    (tmp_path / "template.jinja").write_text(jinja)
    render = load_chat_template(str(tmp_path / "template.jinja"))
    messages = [{"role": "user", "content": "Hi"}]
    assert render(messages) == default_chat_template(messages)
    (tmp_path / "tokenizer_config.json").write_text(json.dumps({"chat_template": jinja, "bos_token": {"content": "<s>"}, "eos_token": "</s>"}))
    assert load_chat_template(str(tmp_path / "tokenizer_config.json"))(messages).startswith("<s><|user|>")
    (tmp_path / "strict.jinja").write_text("{% if messages[0]['role'] != 'user' %}{{ raise_exception('first message must come from the user') }}{% endif %}ok")
    with pytest.raises(ValueError, match="first message"):
        load_chat_template(str(tmp_path / "strict.jinja"))([{"role": "system", "content": "x"}])


def test_environment_driven_endpoint_script(tmp_path, monkeypatch):
    """``scripts/olmo2_modal_openai.py`` without Modal: the app is assembled from environment variables, reports the
    configured model name and asks for the bearer token."""
    tokenizers = pytest.importorskip("tokenizers")
    pytest.importorskip("fastapi")
    import importlib.util
    from pathlib import Path

    from fastapi.testclient import TestClient
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    from olmo_b200.config import TokenizerConfig, TrainConfig

    vocab = {f"w{i}": i + 2 for i in range(60)}
    vocab["<pad>"], vocab["<eos>"] = 0, 1
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="<pad>"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.add_special_tokens(["<eos>", "<pad>"])
    tok.save(str(tmp_path / "tokenizer.json"))
    model = tiny_model(vocab_size=62, embedding_size=64)
    ckpt = tmp_path / "step0-unsharded"
    ckpt.mkdir()
    torch.save(model.state_dict(), ckpt / "model.pt")
    TrainConfig(model=model.config, tokenizer=TokenizerConfig(identifier=str(tmp_path / "tokenizer.json"))).save(ckpt / "config.yaml")

    spec = importlib.util.spec_from_file_location("olmo2_modal_openai", str(Path(__file__).resolve().parent.parent / "scripts" / "olmo2_modal_openai.py"))
    script = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(script)
    monkeypatch.delenv("OLMO_SERVE_CHECKPOINT", raising=False)
    with pytest.raises(SystemExit):
        script.build_asgi_app()
    monkeypatch.setenv("OLMO_SERVE_CHECKPOINT", str(ckpt))
    monkeypatch.setenv("OLMO_SERVE_MODEL_NAME", "olmo-test")
    monkeypatch.setenv("MODAL_TOKEN", "secret")
    monkeypatch.setenv("OLMO_SERVE_MAX_BATCH", "2")
    with TestClient(script.build_asgi_app()) as client:
        assert client.post("/v1/completions", json={"model": "olmo-test", "prompt": "w1", "max_tokens": 1}).status_code == 401
        listed = client.get("/v1/models", headers={"Authorization": "Bearer secret"}).json()
        assert [m["id"] for m in listed["data"]] == ["olmo-test"]
        out = client.post("/v1/completions", headers={"Authorization": "Bearer secret"},
                          json={"model": "olmo-test", "prompt": "w1 w2 w3", "max_tokens": 3, "temperature": 0}).json()
        assert out["choices"][0]["finish_reason"] in ("length", "stop") and out["usage"]["prompt_tokens"] == 3
