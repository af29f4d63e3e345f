"""StepEngine bookkeeping on CPU: the overlapped engine (step i+1 launched
before step i's tokens are read back) must generate exactly what the
step-by-step engine generates, stop on the same tokens and free every
block and bitmap row.

The GPU parts are replaced by a deterministic stand-in: the "model" maps
(last input token, its position) to the next token, and decode inputs whose
``src`` is set are read from the previous step's sampled tokens, as
``muk_fill_decode_inputs`` does on the device.
"""

import numpy as np
import pytest
import torch

from mu_b200.core.cache import PagedKVCache
from mu_b200.core.config import CacheConfig, EngineConfig, ModelConfig, SamplingParams, SchedulerConfig
from mu_b200.serving import engine as E
from mu_b200.serving.worker import MuWorker

V = 97


def next_token(last: int, pos: int) -> int:
    return (last * 31 + pos * 7 + 3) % V


class _Handle:
    def __init__(self, toks):
        self.dev = torch.tensor(toks, dtype=torch.int32)

    def wait(self):
        return self.dev.tolist()


class FakeSampler:
    def __init__(self, vocab, rows, device):
        self.row_of, self.free = {}, list(range(rows))

    def add(self, rid):
        if rid not in self.row_of:
            if not self.free:  # grows like BatchSampler
                n = len(self.row_of)
                self.free = list(range(n, 2 * n))
            self.row_of[rid] = self.free.pop()

    def remove(self, rid):
        r = self.row_of.pop(rid, None)
        if r is not None:
            self.free.append(r)

    def launch(self, logits, ids, params, steps, token_rows=None, input_ids=None, num_tokens=0):
        return _Handle(logits)


class _Model:
    config = ModelConfig(vocab_size=V)


class FakeWorker:
    """MuWorker's host bookkeeping (prepare) over a CPU cache, fake compute."""

    prepare = MuWorker.prepare
    allocate_request = MuWorker.allocate_request
    free_request = MuWorker.free_request

    def __init__(self, blocks=64):
        self.model = _Model()
        self.device = torch.device("cpu")
        self.cache = PagedKVCache(1, 1, 2, 4, blocks, torch.float32, "cpu")
        self.active_requests = {}
        self.steps = []
        self.tokens = []

    def run_step(self, seqs, nd, sampled=None):
        out = []
        for s in seqs:
            if s.src >= 0:
                assert sampled is not None
                last = int(sampled[s.src])
            else:
                last = int(s.token_ids[-1])
            out.append(next_token(last, s.start_pos + len(s.token_ids) - 1))
        self.steps.append((len(seqs), nd))
        self.tokens.append(sum(len(s.token_ids) for s in seqs))
        return out, type("B", (), {"token_rows": None, "input_ids": None})()

    def get_stats(self):
        return {"steps": len(self.steps)}


def expected(prompt, max_tokens, stop):
    toks, gen = list(prompt), []
    while len(gen) < max_tokens:
        t = next_token(toks[-1], len(toks) - 1)
        gen.append(t)
        toks.append(t)
        if t in stop:
            break
    return gen


def run(overlap, prompts, limits, stop, max_batch, abort=None, monkeypatch=None, budget=64,
        chunked=True, blocks=64, batched_tokens=64, align=0):
    monkeypatch.setattr(E, "BatchSampler", FakeSampler)
    ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=blocks, max_num_seqs=max_batch),
                      scheduler=SchedulerConfig(max_batch_size=max_batch,
                                                max_num_batched_tokens=batched_tokens,
                                                max_prefill_tokens=budget,
                                                enable_chunked_prefill=chunked,
                                                step_token_alignment=align))
    w = FakeWorker(blocks)
    eng = E.StepEngine(w, ec, overlap=overlap)
    for i, (p, m) in enumerate(zip(prompts, limits)):
        eng.add_request(p, SamplingParams(temperature=0.0, max_tokens=m, stop_token_ids=stop),
                        f"r{i}")
    reported = {f"r{i}": [] for i in range(len(prompts))}
    n = 0
    while eng.has_unfinished():
        for o in eng.step():
            assert o.token_id >= 0
            reported[o.request_id].append(o.token_id)
        n += 1
        if abort and n == abort[1]:
            eng.abort_request(abort[0])
        assert n < 500
    return eng, w, reported


@pytest.mark.parametrize("overlap", [False, True])
def test_overlapped_engine_matches_sequential_generation(overlap, monkeypatch):
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in rng.integers(1, 11, 9)]
    limits = [int(m) for m in rng.integers(1, 14, 9)]
    stop = [5, 11]
    eng, w, reported = run(overlap, prompts, limits, stop, max_batch=4, monkeypatch=monkeypatch)
    for i, (p, m) in enumerate(zip(prompts, limits)):
        req = eng.requests[f"r{i}"]
        want = expected(p, m, stop)
        assert req.output_token_ids == want, (i, overlap)
        assert req.num_generated_tokens == len(want)
        assert reported[f"r{i}"] == want  # each token reported once, in order
        assert req.finish_reason == ("stop" if want[-1] in stop else "length")
    assert any(eng.requests[f"r{i}"].finish_reason == "stop" for i in range(len(prompts)))
    assert not w.active_requests and len(w.cache.free_blocks) == w.cache.max_num_blocks
    assert not eng.sampler.row_of and eng._inflight is None and not eng._closing
    # continuous batching really mixed decodes with new prefills
    assert any(0 < nd < b for b, nd in w.steps)


def test_overlap_launches_no_more_steps_than_needed(monkeypatch):
    """Length limits are known at launch: no step runs past max_tokens."""
    prompts = [[1, 2, 3], [4, 5], [6]]
    _, w1, _ = run(False, prompts, [4, 6, 2], [], 8, monkeypatch=monkeypatch)
    _, w2, _ = run(True, prompts, [4, 6, 2], [], 8, monkeypatch=monkeypatch)
    assert w1.steps == w2.steps


def test_abort_while_in_flight(monkeypatch):
    prompts = [[1, 2, 3], [4, 5, 6, 7]]
    eng, w, reported = run(True, prompts, [20, 6], [], 4, abort=("r0", 3),
                           monkeypatch=monkeypatch)
    assert "r0" not in eng.requests
    assert eng.requests["r1"].output_token_ids == expected(prompts[1], 6, [])
    assert not w.active_requests and len(w.cache.free_blocks) == w.cache.max_num_blocks


@pytest.mark.parametrize("overlap", [False, True])
def test_chunked_prefill(overlap, monkeypatch):
    """Prompts longer than the prefill budget run in chunks over several steps
    (KV appended chunk by chunk, no token until the last chunk) and generate
    exactly what a whole-prompt prefill generates; no step exceeds the budget
    plus its decodes."""
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in (23, 5, 17, 9, 30)]
    limits = [6, 4, 7, 3, 5]
    budget = 6
    eng, w, reported = run(overlap, prompts, limits, [], max_batch=3, monkeypatch=monkeypatch,
                           budget=budget)
    for i, (p, m) in enumerate(zip(prompts, limits)):
        want = expected(p, m, [])
        assert eng.requests[f"r{i}"].output_token_ids == want
        assert reported[f"r{i}"] == want
    for (b, nd), t in zip(w.steps, w.tokens):
        assert t - nd <= budget
    assert max(w.tokens) <= budget + 3
    assert not w.active_requests and len(w.cache.free_blocks) == w.cache.max_num_blocks


@pytest.mark.parametrize("overlap", [False, True])
@pytest.mark.parametrize("chunked,budget,blocks", [(False, 8, 12), (True, 8, 12), (True, 64, 8),
                                                   (False, 64, 8)])
def test_kv_pool_exhaustion_preempts_and_recomputes(overlap, chunked, budget, blocks, monkeypatch):
    """A pool far smaller than the requests' final lengths: admissions wait and
    running requests are preempted (KV freed, prompt + generated tokens
    re-prefilled on readmission) instead of failing; every request still
    generates exactly its sequential tokens and every block comes back."""
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in (7, 10, 4, 9, 6, 8)]
    limits = [14, 9, 16, 12, 11, 15]
    # 32-48 token slots; the requests end at 17-23 tokens each; with the
    # large budget the first step's admissions alone overflow the pool
    eng, w, reported = run(overlap, prompts, limits, [], max_batch=4, monkeypatch=monkeypatch,
                           budget=budget, chunked=chunked, blocks=blocks)
    for i, (p, m) in enumerate(zip(prompts, limits)):
        req = eng.requests[f"r{i}"]
        want = expected(p, m, [])
        assert req.output_token_ids == want, (i, overlap, chunked)
        assert reported[f"r{i}"] == want
        assert req.finish_reason == "length"
    assert sum(eng.requests[f"r{i}"].num_preemptions for i in range(len(prompts))) > 0
    assert not w.active_requests and len(w.cache.free_blocks) == blocks
    assert not eng.sampler.row_of and not eng._closing


@pytest.mark.parametrize("overlap", [False, True])
def test_token_budget_preemption_recomputes(overlap, monkeypatch):
    """The reference's own preemption (more decodes than max_num_batched_tokens:
    the most advanced go back to the queue) under the engine: preempted
    requests re-prefill and finish with their sequential tokens."""
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in (3, 5, 4, 6, 2, 5)]
    limits = [8, 6, 9, 5, 7, 6]
    eng, w, reported = run(overlap, prompts, limits, [], max_batch=6, monkeypatch=monkeypatch,
                           chunked=False, batched_tokens=4)
    for i, (p, m) in enumerate(zip(prompts, limits)):
        assert eng.requests[f"r{i}"].output_token_ids == expected(p, m, []), (i, overlap)
        assert reported[f"r{i}"] == expected(p, m, [])
    assert sum(eng.requests[f"r{i}"].num_preemptions for i in range(len(prompts))) > 0
    assert not w.active_requests and len(w.cache.free_blocks) == w.cache.max_num_blocks


@pytest.mark.parametrize("overlap", [False, True])
def test_step_token_alignment(overlap, monkeypatch):
    """Tile-aligned steps: the last prefill chunk is trimmed so that a step
    with prefill tokens has a multiple of `align` tokens; generation is
    unchanged."""
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in (13, 7, 22, 5, 17, 11, 9)]
    limits = [9, 12, 6, 10, 8, 7, 11]
    align = 8
    eng, w, reported = run(overlap, prompts, limits, [], max_batch=4, monkeypatch=monkeypatch,
                           budget=64, align=align)
    for i, (p, m) in enumerate(zip(prompts, limits)):
        assert eng.requests[f"r{i}"].output_token_ids == expected(p, m, [])
        assert reported[f"r{i}"] == expected(p, m, [])
    trimmed = [(b, nd, t) for (b, nd), t in zip(w.steps, w.tokens) if b > nd and t > align]
    assert trimmed and sum(t % align == 0 for _, _, t in trimmed) >= len(trimmed) // 2
    _, w0, _ = run(overlap, prompts, limits, [], max_batch=4, monkeypatch=monkeypatch, budget=64)
    assert sum(t % align == 0 for (b, nd), t in zip(w0.steps, w0.tokens) if b > nd and t > align) \
        < sum(t % align == 0 for _, _, t in trimmed)


def test_public_engines_over_stand_in(monkeypatch):
    """MuEngine / MuBatchEngine async plumbing (generate, generate_stream,
    concurrent requests, stats, shutdown) over the stand-in worker."""
    import asyncio

    from mu_b200 import MuBatchEngine, MuEngine

    monkeypatch.setattr(E, "BatchSampler", FakeSampler)
    ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=64, max_num_seqs=4),
                      scheduler=SchedulerConfig(max_batch_size=3, max_num_batched_tokens=64))
    prompts = [[1, 2, 3], [4, 5], [6, 7, 8, 9], [10]]
    sp = lambda m: SamplingParams(temperature=0.0, max_tokens=m)

    async def seq():
        eng = MuEngine(ec)
        eng.initialize_from_worker(FakeWorker())
        a = await eng.generate(prompts[0], sp(5), "a")
        s = [o async for o in eng.generate_stream(prompts[1], sp(4), "s")]
        st = eng.get_stats()
        await eng.shutdown()
        return a, s, st

    a, s, st = asyncio.run(seq())
    assert a.token_ids == expected(prompts[0], 5, []) and a.finish_reason == "length"
    assert a.usage == {"prompt_tokens": 3, "completion_tokens": 5, "total_tokens": 8}
    assert [o.token_id for o in s] == expected(prompts[1], 4, []) and s[-1].finished
    assert st["total_requests"] == 2 and st["total_tokens_generated"] == 9

    async def batch():
        eng = MuBatchEngine(ec)
        eng.initialize_from_worker(FakeWorker())

        async def stream(i):
            return [o async for o in eng.generate_stream(prompts[i], sp(6), f"s{i}")]

        outs = await asyncio.gather(*[eng.generate(prompts[i], sp(3 + i), f"b{i}")
                                      for i in range(3)], stream(3))
        st = eng.get_stats()
        await eng.shutdown()
        return outs, st

    outs, st = asyncio.run(batch())
    for i in range(3):
        assert outs[i].token_ids == expected(prompts[i], 3 + i, []), i
    assert [o.token_id for o in outs[3][:-1]] == expected(prompts[3], 6, [])
    assert outs[3][-1].finished and outs[3][-1].token_id == -1
    assert st["total_requests"] == 4 and st["engine_type"] == "continuous_batching"
    # the reference's keys (engine.py:802-823) plus step counters
    for key in ("batches_processed", "avg_batch_size", "uptime_seconds", "tokens_per_second",
                "pending_requests", "active_requests", "worker", "continuous_batching"):
        assert key in st, key
    assert st["steps"]["steps"] > 0 and st["steps"]["tokens_per_step"] > 0


@pytest.mark.parametrize("seed", list(range(12)) + [75])
def test_engine_fuzz(seed, monkeypatch):
    """Random workloads through the whole host path: arrivals mid-run, aborts,
    stop tokens, chunked or whole prefills, small KV pools (preemption),
    tile-aligned steps, overlap on or off.  Every request that is not aborted
    must generate exactly its sequential tokens, and every block and bitmap
    row must come back."""
    rng = np.random.default_rng(100 + seed)
    overlap = bool(seed % 2)
    chunked = seed % 3 != 0
    n = int(rng.integers(4, 14))
    prompts = [rng.integers(0, V, int(L)).tolist() for L in rng.integers(1, 30, n)]
    limits = [int(m) for m in rng.integers(1, 20, n)]
    stop = [int(s) for s in rng.integers(0, V, int(rng.integers(0, 3)))]
    max_batch = int(rng.integers(2, 7))
    budget = int(rng.integers(4, 40))
    longest = max(len(p) + m for p, m in zip(prompts, limits))
    blocks = max(-(-longest // 4) + 1, int(rng.integers(6, 40)))
    align = int(rng.choice([0, 0, 4, 8]))
    policy = "priority" if seed % 5 == 4 else "fcfs"
    # a token budget below the batch size makes the reference's own
    # preemption (most advanced decodes back to the queue) fire too
    batched = int(rng.choice([64, 64, max(1, max_batch - 1)]))
    monkeypatch.setattr(E, "BatchSampler", FakeSampler)
    ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=blocks, max_num_seqs=max_batch),
                      scheduler=SchedulerConfig(max_batch_size=max_batch,
                                                max_num_batched_tokens=batched,
                                                max_prefill_tokens=budget, policy=policy,
                                                enable_chunked_prefill=chunked,
                                                step_token_alignment=align))
    w = FakeWorker(blocks)
    eng = E.StepEngine(w, ec, overlap=overlap)
    arrive = sorted(int(x) for x in rng.integers(0, 15, n))
    aborts = {int(rng.integers(0, n)): int(rng.integers(1, 25)) for _ in range(int(rng.integers(0, 3)))}
    reported = {f"r{i}": [] for i in range(n)}
    added, step, aborted = 0, 0, set()
    while added < n or eng.has_unfinished():
        while added < n and arrive[added] <= step:
            eng.add_request(prompts[added], SamplingParams(temperature=0.0, max_tokens=limits[added],
                                                           stop_token_ids=stop), f"r{added}")
            added += 1
        for o in eng.step():
            reported[o.request_id].append(o.token_id)
        step += 1
        for i, at in aborts.items():
            if at == step and i < added and f"r{i}" in eng.requests:
                eng.abort_request(f"r{i}")
                aborted.add(i)
        assert step < 2000
    for i in range(n):
        if i in aborted:
            continue
        want = expected(prompts[i], limits[i], stop)
        req = eng.requests[f"r{i}"]
        assert req.output_token_ids == want, (seed, i)
        assert reported[f"r{i}"] == want, (seed, i)
    assert not w.active_requests and len(w.cache.free_blocks) == blocks
    assert not eng.sampler.row_of and not eng._closing and eng._inflight is None


def test_engines_across_event_loops(monkeypatch):
    """generate_sync from plain code (twice), and MuBatchEngine requests from
    two successive asyncio.run loops: the batching task follows the loop."""
    import asyncio

    from mu_b200 import MuBatchEngine, MuEngine

    monkeypatch.setattr(E, "BatchSampler", FakeSampler)
    ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=64, max_num_seqs=4),
                      scheduler=SchedulerConfig(max_batch_size=3, max_num_batched_tokens=64))
    sp = SamplingParams(temperature=0.0, max_tokens=4)
    eng = MuEngine(ec)
    eng.initialize_from_worker(FakeWorker())
    assert eng.generate_sync([1, 2, 3], sp).token_ids == expected([1, 2, 3], 4, [])
    assert eng.generate_sync([4, 5], sp).token_ids == expected([4, 5], 4, [])

    async def inside():
        with pytest.raises(RuntimeError):
            eng.generate_sync([1], sp)
    asyncio.run(inside())

    beng = MuBatchEngine(ec)
    beng.initialize_from_worker(FakeWorker())   # no loop running yet
    for prompt in ([7, 8], [9, 10, 11]):
        out = asyncio.run(beng.generate(prompt, sp))
        assert out.token_ids == expected(prompt, 4, [])
    asyncio.run(beng.shutdown())


@pytest.mark.parametrize("overlap", [False, True])
def test_failed_step_fails_its_requests(overlap, monkeypatch):
    """A step whose sampled tokens cannot be read (a device error surfacing
    at the read) finishes the requests in it with "error" and frees their
    blocks; requests admitted later still generate their tokens."""
    state = {"launch": 0}

    class FailingSampler(FakeSampler):
        def launch(self, logits, ids, params, steps, token_rows=None, input_ids=None,
                   num_tokens=0):
            state["launch"] += 1
            h = _Handle(logits)
            if state["launch"] == 3:
                def boom():
                    raise RuntimeError("device error 6")
                h.wait = boom
            return h

    monkeypatch.setattr(E, "BatchSampler", FailingSampler)
    ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=64, max_num_seqs=2),
                      scheduler=SchedulerConfig(max_batch_size=2, max_num_batched_tokens=64))
    w = FakeWorker()
    eng = E.StepEngine(w, ec, overlap=overlap)
    prompts = [[1, 2, 3], [4, 5], [6, 7, 8, 9]]
    for i, p in enumerate(prompts):
        eng.add_request(p, SamplingParams(temperature=0.0, max_tokens=6), f"r{i}")
    reasons = {}
    while eng.has_unfinished():
        for o in eng.step():
            if o.finished:
                reasons[o.request_id] = o.finish_reason
    assert reasons["r0"] == "error" and reasons["r1"] == "error"
    assert reasons["r2"] == "length"
    assert eng.requests["r2"].output_token_ids == expected(prompts[2], 6, [])
    for rid in ("r0", "r1"):
        toks = eng.requests[rid].output_token_ids
        assert -1 not in toks and toks == expected(prompts[int(rid[1])], 6, [])[:len(toks)]
    assert not w.active_requests and len(w.cache.free_blocks) == w.cache.max_num_blocks
    assert not eng.sampler.row_of and not eng._closing


def test_text_prompts_through_an_offline_tokenizer(tmp_path, monkeypatch):
    """String prompts: a tokenizer shipped in the model directory is loaded
    offline (load_tokenizer), prompts are encoded, generated ids decoded."""
    import asyncio

    tokenizers = pytest.importorskip("tokenizers")
    from transformers import PreTrainedTokenizerFast

    from mu_b200 import MuEngine
    from mu_b200.utils.tokenizer import load_tokenizer

    vocab = {f"w{i}": i for i in range(V)}
    tok = tokenizers.Tokenizer(tokenizers.models.WordLevel(vocab, unk_token="w0"))
    tok.pre_tokenizer = tokenizers.pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="w0").save_pretrained(str(tmp_path))
    tk = load_tokenizer(str(tmp_path))
    assert tk is not None and tk.encode("w1 w2 w3") == [1, 2, 3]
    assert load_tokenizer(str(tmp_path / "missing")) is None

    monkeypatch.setattr(E, "BatchSampler", FakeSampler)
    ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=64, max_num_seqs=2),
                      scheduler=SchedulerConfig(max_batch_size=2, max_num_batched_tokens=64))
    eng = MuEngine(ec)
    eng.initialize_from_worker(FakeWorker(), tk)
    out = asyncio.run(eng.generate("w1 w2 w3", SamplingParams(temperature=0.0, max_tokens=5)))
    want = expected([1, 2, 3], 5, [])
    assert out.token_ids == want
    assert out.text == tk.decode(want, skip_special_tokens=True)
    assert out.usage["prompt_tokens"] == 3
