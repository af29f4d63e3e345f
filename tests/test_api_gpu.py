"""The reference's public API on the GPU, end to end from a model directory:
``MuEngine`` (one request at a time), ``MuBatchEngine`` (continuous batching
behind async ``generate`` / ``generate_stream``) and the OpenAI-compatible
HTTP server over it.  Greedy tokens are checked against the golden tokens the
reference produced for the same seeded weights and prompts (the same rule as
the model tests: a token may differ only where the reference's top-2 logit
gap is within the bf16 tolerance, and the comparison stops there)."""

import asyncio
import json

import numpy as np
import pytest

from golden_models import G, load_tiny

pytestmark = pytest.mark.gpu

GAP_TOL = 0.05


def _model_dir(tmp_path, name):
    from mu_b200.models.weights import write_model_dir

    shape, cfg, sd, d, prompts = load_tiny(name)
    path = write_model_dir(tmp_path / name, cfg, shape.arch, sd)
    toks = np.load(G / f"{name}.npz")["tokens"]
    return str(path), d, prompts, toks


def _config(max_batch):
    from mu_b200.core.config import CacheConfig, EngineConfig, MuConfig, SchedulerConfig

    return EngineConfig(mu=MuConfig(enabled=True),
                        cache=CacheConfig(max_seq_len=256, max_num_blocks=512, max_num_seqs=16),
                        scheduler=SchedulerConfig(max_batch_size=max_batch,
                                                  max_num_batched_tokens=2048))


def _greedy(n):
    from mu_b200.core.config import SamplingParams

    return SamplingParams(temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0,
                          max_tokens=n)


def _check(got, want, gaps, where):
    assert len(got) == len(want), where
    for i, t in enumerate(got):
        if t != int(want[i]):
            assert gaps[i] <= GAP_TOL, (where, i, t, int(want[i]))
            break


@pytest.mark.parametrize("name", ["llama_tiny", "deep_tiny"])
def test_mu_engine_generate_and_stream(cuda, tmp_path, name):
    from mu_b200 import MuEngine

    path, d, prompts, toks = _model_dir(tmp_path, name)
    R, n = toks.shape

    async def main():
        eng = MuEngine(_config(4), path)
        await eng.initialize(path)
        outs = []
        for r in range(2):
            outs.append(await eng.generate(prompts[r], _greedy(n), f"g{r}"))
        streamed = [o async for o in eng.generate_stream(prompts[2], _greedy(n), "s2")]
        stats = eng.get_stats()
        await eng.shutdown()
        return outs, streamed, stats

    outs, streamed, stats = asyncio.run(main())
    for r, o in enumerate(outs):
        assert o.request_id == f"g{r}" and o.finished and o.finish_reason == "length"
        assert o.usage == {"prompt_tokens": len(prompts[r]), "completion_tokens": n,
                           "total_tokens": len(prompts[r]) + n}
        _check(o.token_ids, toks[r], d["top2_gap"][r], (name, r))
    assert streamed[-1].finished and streamed[-1].finish_reason == "length"
    _check([s.token_id for s in streamed], toks[2], d["top2_gap"][2], (name, "stream"))
    assert stats["total_requests"] == 3 and stats["total_tokens_generated"] == 3 * n


@pytest.mark.parametrize("name", ["llama_tiny", "deep_tiny"])
def test_mu_batch_engine_concurrent_requests(cuda, tmp_path, name):
    """All prompts submitted at once through async generate (more requests
    than batch slots, so some join while others decode) plus one stream."""
    from mu_b200 import MuBatchEngine

    path, d, prompts, toks = _model_dir(tmp_path, name)
    R, n = toks.shape

    async def main():
        eng = MuBatchEngine(_config(max(2, R - 1)), path)
        await eng.initialize(path)

        async def stream(r):
            return [o async for o in eng.generate_stream(prompts[r], _greedy(n), f"s{r}")]

        outs = await asyncio.gather(*[eng.generate(prompts[r], _greedy(n), f"b{r}")
                                      for r in range(R - 1)], stream(R - 1))
        stats = eng.get_stats()
        await eng.shutdown()
        return outs, stats

    outs, stats = asyncio.run(main())
    for r in range(R - 1):
        o = outs[r]
        assert o.request_id == f"b{r}" and o.finish_reason == "length"
        _check(o.token_ids, toks[r], d["top2_gap"][r], (name, r))
    streamed = outs[R - 1]
    assert streamed[-1].finished and streamed[-1].token_id == -1
    _check([s.token_id for s in streamed[:-1]], toks[R - 1], d["top2_gap"][R - 1], (name, "s"))
    assert stats["engine_type"] == "continuous_batching" and stats["total_requests"] == R
    assert stats["batches_processed"] < R * n  # requests shared steps


def test_openai_server_end_to_end(cuda, tmp_path):
    """HTTP routes of the server over MuBatchEngine: a token-id completion, a
    streamed completion (server-sent events ending in [DONE]), models and stats."""
    pytest.importorskip("httpx")
    from fastapi.testclient import TestClient

    from mu_b200.serving.server import create_app

    path, d, prompts, toks = _model_dir(tmp_path, "llama_tiny")
    R, n = toks.shape
    app = create_app(path, _config(4), model_name="tiny")
    with TestClient(app) as client:
        assert client.get("/health").json()["status"] == "healthy"
        assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
        body = {"model": "tiny", "prompt": prompts[0], "max_tokens": n, "temperature": 0.0,
                "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0}
        r = client.post("/v1/completions", json=body)
        assert r.status_code == 200, r.text
        out = r.json()
        assert out["object"] == "text_completion" and out["choices"][0]["finish_reason"] == "length"
        assert out["usage"]["completion_tokens"] == n
        _check(out["choices"][0]["token_ids"], toks[0], d["top2_gap"][0], "http")
        body.update(prompt=prompts[1], stream=True)
        with client.stream("POST", "/v1/completions", json=body) as s:
            lines = [ln for ln in s.iter_lines() if ln.startswith("data: ")]
        assert lines[-1] == "data: [DONE]"
        events = [json.loads(ln[6:]) for ln in lines[:-1]]
        ids = [e["choices"][0]["token_id"] for e in events if "token_id" in e["choices"][0]]
        _check(ids, toks[1], d["top2_gap"][1], "sse")
        assert events[-1]["choices"][0]["finish_reason"] == "length"
        assert client.get("/stats").json()["total_requests"] == 2
