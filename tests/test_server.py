"""The OpenAI-compatible front end on CPU, over a stand-in engine: routes,
response schemas, server-sent-event streams and the chat template.  The
engine itself is exercised on the GPU by the model tests."""

import asyncio
import json

import pytest

pytest.importorskip("fastapi")

from mu_b200.serving.engine import GenerationOutput, StreamOutput  # noqa: E402
from mu_b200.serving.server import (ChatCompletionRequest, ChatMessage,  # noqa: E402
                                    CompletionRequest, MuServer)


class FakeEngine:
    def __init__(self):
        self.calls = []

    async def generate(self, prompt, sampling_params=None, request_id=None):
        self.calls.append((prompt, sampling_params, request_id))
        n = len(prompt) if isinstance(prompt, (list, str)) else 1
        return GenerationOutput(request_id, "abc", [7, 8, 9], True, "length",
                                {"prompt_tokens": n, "completion_tokens": 3, "total_tokens": n + 3})

    async def generate_stream(self, prompt, sampling_params=None, request_id=None):
        for i, t in enumerate([5, 6]):
            yield StreamOutput(request_id, f"t{t}", t, False)
        yield StreamOutput(request_id, "", -1, True, "stop")

    def get_stats(self):
        return {"total_requests": len(self.calls)}


def _collect(agen):
    async def run():
        return [x async for x in agen]
    return asyncio.run(run())


def test_routes_and_completion():
    eng = FakeEngine()
    srv = MuServer(eng, "tiny")
    paths = {r.path for r in srv.app.routes}
    for p in ("/health", "/v1/models", "/v1/models/{model_id}", "/v1/completions",
              "/v1/chat/completions", "/stats"):
        assert p in paths
    req = CompletionRequest(model="tiny", prompt=[1, 2, 3, 4], max_tokens=3, temperature=0.0)
    out = asyncio.run(srv.completion(req))
    assert out.object == "text_completion" and out.model == "tiny"
    assert out.choices[0].token_ids == [7, 8, 9] and out.choices[0].finish_reason == "length"
    assert out.usage.total_tokens == 7
    prompt, sp, rid = eng.calls[-1]
    assert prompt == [1, 2, 3, 4] and sp.max_tokens == 3 and sp.temperature == 0.0
    assert rid.startswith("cmpl-")


def test_streams_end_with_done():
    srv = MuServer(FakeEngine(), "tiny")
    req = CompletionRequest(model="tiny", prompt="hi", stream=True)
    events = _collect(srv.stream_completion(req, "cmpl-x"))
    assert events[-1] == "data: [DONE]\n\n"
    first = json.loads(events[0][len("data: "):])
    assert first["choices"][0]["text"] == "t5" and first["choices"][0]["token_id"] == 5
    last = json.loads(events[-2][len("data: "):])
    assert last["choices"][0]["finish_reason"] == "stop"
    chat = ChatCompletionRequest(model="tiny", messages=[ChatMessage(role="user", content="x")],
                                 stream=True)
    ev = _collect(srv.stream_chat(chat, "chatcmpl-x", "User: x\nAssistant:"))
    body = [json.loads(e[len("data: "):]) for e in ev[:-1]]
    assert body[0]["object"] == "chat.completion.chunk"
    assert body[0]["choices"][0]["delta"] == {"content": "t5"} and body[-1]["choices"][0]["delta"] == {}


def test_chat_template_and_response():
    eng = FakeEngine()
    srv = MuServer(eng, "tiny")
    msgs = [ChatMessage(role="system", content="be brief"), ChatMessage(role="user", content="hi"),
            ChatMessage(role="assistant", content="hello"), ChatMessage(role="user", content="?")]
    assert srv.format_chat_prompt(msgs) == ("System: be brief\nUser: hi\nAssistant: hello\n"
                                            "User: ?\nAssistant:")
    out = asyncio.run(srv.chat_completion(ChatCompletionRequest(model="tiny", messages=msgs)))
    assert out.object == "chat.completion" and out.choices[0].message.role == "assistant"
    assert out.choices[0].message.content == "abc"


def test_http_round_trip():
    """The same routes over HTTP (FastAPI's test client): JSON bodies in and
    out, validation errors, 404 for an unknown model, an SSE stream."""
    pytest.importorskip("httpx")
    from fastapi.testclient import TestClient

    srv = MuServer(FakeEngine(), "tiny")
    with TestClient(srv.app) as client:
        assert client.get("/health").json() == {"status": "healthy", "model": "tiny"}
        assert client.get("/v1/models/tiny").json()["id"] == "tiny"
        assert client.get("/v1/models/other").status_code == 404
        r = client.post("/v1/completions", json={"model": "tiny", "prompt": [1, 2], "max_tokens": 3})
        assert r.status_code == 200 and r.json()["choices"][0]["token_ids"] == [7, 8, 9]
        assert client.post("/v1/completions",
                           json={"model": "tiny", "prompt": "x", "max_tokens": 0}).status_code == 422
        r = client.post("/v1/chat/completions",
                        json={"model": "tiny", "messages": [{"role": "user", "content": "hi"}]})
        assert r.json()["choices"][0]["message"] == {"role": "assistant", "content": "abc"}
        with client.stream("POST", "/v1/completions",
                           json={"model": "tiny", "prompt": [1], "stream": True}) as s:
            lines = [ln for ln in s.iter_lines() if ln]
        assert lines[-1] == "data: [DONE]" and len(lines) == 4
        assert client.get("/stats").json()["total_requests"] == 2
