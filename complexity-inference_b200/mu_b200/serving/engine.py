"""Engines with the reference API (mu_inference/serving/engine.py).

``StepEngine`` is the synchronous continuous-batching core: each ``step()``
asks MuScheduler for a SchedulerOutput, runs it as one flat GPU step through
MuWorker, samples every sequence on the GPU (BatchSampler) and applies the
reference's stop rules (EOS of the tokenizer, stop_token_ids, max_tokens;
engine.py:231-237 / 651-660).  New requests join while others decode;
finished ones leave and free their blocks at once.

``MuEngine`` keeps the reference's sequential API (initialize / generate /
generate_stream / get_stats / shutdown, engine.py:58-426).
``MuBatchEngine`` keeps the reference's continuous-batching API
(engine.py:448-858), whose own loop cannot run (its sampling call raises
TypeError); here it drives StepEngine from a background asyncio task.

Prompts may be strings (a tokenizer is loaded from the model dir when
available) or lists of token ids.
"""

from __future__ import annotations

import asyncio
import logging
import time
import uuid
from dataclasses import dataclass
from typing import AsyncIterator, Dict, List, Optional, Sequence, Union

import numpy as np
import torch

from .. import _lib
from ..core.config import EngineConfig, SamplingParams
from ..core.scheduler import MuScheduler, Request, RequestStatus
from ..utils.sampling import BatchSampler, SampleHandle
from ..utils.tokenizer import load_tokenizer
from .worker import MuWorker

logger = logging.getLogger(__name__)

Prompt = Union[str, Sequence[int]]


@dataclass
class GenerationOutput:
    request_id: str
    text: str
    token_ids: List[int]
    finished: bool
    finish_reason: Optional[str] = None
    usage: Optional[Dict[str, int]] = None


@dataclass
class StreamOutput:
    request_id: str
    text: str
    token_id: int
    finished: bool
    finish_reason: Optional[str] = None


@dataclass
class StepOutput:
    request_id: str
    token_id: int
    finished: bool
    finish_reason: Optional[str] = None


@dataclass
class _Launched:
    """A step whose sampled tokens have not been read back yet."""

    reqs: List[Request]           # one per logits row
    idx: List[int]                # position of the pending token in output_token_ids
    row_of: Dict[str, int]        # request id -> row of its token in handle.dev
    handle: SampleHandle


_heap_frozen = False


def freeze_startup_heap() -> None:
    """Once per process: move every object alive now (imported modules, the
    loaded model's bookkeeping: typically hundreds of thousands of objects)
    out of the cyclic collector's generations.  A full collection during
    serving then walks only objects made since, instead of pausing the step
    loop for tens of milliseconds.  Frozen objects are still freed by
    reference counting; only cycles among them are never collected, which
    for a server's start-up state is no loss.  Later engines in the same
    process do not freeze again."""
    global _heap_frozen
    if _heap_frozen:
        return
    import gc

    gc.collect()
    gc.freeze()
    _heap_frozen = True


class StepEngine:
    """Scheduler + worker + sampler; one ``step()`` = one GPU forward step.

    With ``overlap`` (the default) the host never waits for the GPU between
    steps: ``step()`` packs and launches step i+1 first — decode inputs that
    are step i's samples are read on the device (``muk_fill_decode_inputs``)
    — and only then waits for step i's tokens and applies them.  So
    ``step()`` returns the outputs of the previous launch, and the
    scheduling, slot reservation and packing of a step run while the GPU
    executes the one before.  A request whose length limit is reached is
    left out of the next launch; one that stops on a stop token was already
    launched once more: that extra token is dropped (its KV slot is freed
    with the request), so the generated tokens are exactly those of the
    non-overlapped engine.  ``overlap=False`` runs each step to completion
    (the reference's order, engine.py:560-680).  ``freeze_gc`` (default)
    calls :func:`freeze_startup_heap` (a no-op after the process's first
    engine).
    """

    def __init__(self, worker: MuWorker, config: EngineConfig, eos_token_id: Optional[int] = None,
                 overlap: bool = True, freeze_gc: bool = True):
        if freeze_gc:
            freeze_startup_heap()
        self.worker = worker
        self.config = config
        self.scheduler = MuScheduler(config.scheduler)
        # requests whose last token is still in flight keep their bitmap row
        # while new ones are admitted: room for twice the batch
        self.sampler = BatchSampler(worker.model.config.vocab_size,
                                    2 * max(config.cache.max_num_seqs,
                                            config.scheduler.max_batch_size),
                                    worker.device)
        self.sampler.tp = self._sampling_tp()
        self.eos_token_id = eos_token_id
        self.overlap = overlap
        self.requests: Dict[str, Request] = {}
        self.num_steps = 0
        self.num_step_tokens = 0     # tokens run (prefill + decode) over all steps
        self.num_decode_tokens = 0
        self._t0 = time.time()
        self._inflight: Optional[_Launched] = None
        self._closing: set = set()   # last token in flight and length limit reached

    # ---- requests ------------------------------------------------------------
    def _sampling_tp(self):
        """The worker's vocabulary-parallel sampling context (None without one)."""
        f = getattr(self.worker, "sampling_tp", None)
        return f() if f is not None else None

    def add_request(self, prompt_token_ids: Sequence[int], sampling_params: SamplingParams,
                    request_id: Optional[str] = None) -> str:
        rid = request_id or uuid.uuid4().hex[:16]
        req = Request(request_id=rid, prompt_token_ids=list(prompt_token_ids),
                      sampling_params=sampling_params, num_prompt_tokens=len(prompt_token_ids),
                      max_tokens=sampling_params.max_tokens)
        self.requests[rid] = req
        self.scheduler.add_request(req)
        return rid

    def abort_request(self, request_id: str) -> None:
        self._release(request_id)
        self.scheduler.abort_request(request_id)
        self.requests.pop(request_id, None)

    def has_unfinished(self) -> bool:
        return self.scheduler.has_unfinished() or self._inflight is not None

    def get_stats(self) -> Dict:
        """Step counters: steps launched, tokens per step, and rates over the
        engine's lifetime (host wall clock)."""
        up = max(time.time() - self._t0, 1e-9)
        n = max(self.num_steps, 1)
        return {"steps": self.num_steps, "tokens_per_step": self.num_step_tokens / n,
                "decode_tokens_per_step": self.num_decode_tokens / n,
                "step_tokens_per_second": self.num_step_tokens / up,
                "steps_per_second": self.num_steps / up}

    def _release(self, rid: str) -> None:
        if rid in self.worker.active_requests:
            self.worker.free_request(rid)
        self.sampler.remove(rid)
        self._closing.discard(rid)

    def _finish(self, req: Request, reason: str, success: bool = True) -> None:
        self._release(req.request_id)
        self.scheduler.finish_request(req.request_id, success)
        req.finish_reason = reason  # type: ignore[attr-defined]

    # ---- one step ----------------------------------------------------------------
    @torch.inference_mode()
    def step(self) -> List[StepOutput]:
        results: List[StepOutput] = []
        launched = self._launch(results)
        if not self.overlap:
            if launched is not None:
                results += self._complete(launched)
            return results
        prev, self._inflight = self._inflight, launched
        if prev is not None:
            results += self._complete(prev)
        return results

    def _fail_step(self, launched: _Launched, err: Exception) -> List[StepOutput]:
        """A step whose results cannot be read: every request in it finishes
        with "error" (blocks and bitmap rows freed), as the reference maps a
        failed forward to WorkerOutput.error -> finish_reason "error"
        (worker.py:179-206, engine.py:210-212).  Requests not in the step go
        on."""
        logger.error("step failed: %s", err)
        dev = getattr(self.worker, "device", None)
        if isinstance(err, _lib.DeviceError) and getattr(dev, "type", "cuda") == "cuda":
            # read and clear the word (synchronises) so later steps start clean
            _lib.device_error()
        results: List[StepOutput] = []
        seen = set()
        for req in launched.reqs:
            rid = req.request_id
            if rid in seen or req.is_finished or self.requests.get(rid) is not req:
                continue
            seen.add(rid)
            while req.output_token_ids and req.output_token_ids[-1] == -1:  # pending tokens
                req.output_token_ids.pop()
                req.num_generated_tokens -= 1
            self._finish(req, "error", success=False)
            results.append(StepOutput(rid, -1, True, "error"))
        return results

    def flush(self) -> List[StepOutput]:
        """Wait for the step in flight, if any, and return its outputs."""
        prev, self._inflight = self._inflight, None
        return self._complete(prev) if prev is not None else []

    def _launch(self, results: List[StepOutput]) -> Optional[_Launched]:
        out = self.scheduler.schedule(self._closing)
        for req in out.preempted_requests:  # recompute preemption: drop KV, re-prefill later
            self._release(req.request_id)
        # the step's new KV blocks must fit the pool: defer admissions, then
        # preempt (recompute) until they do
        cache, active = self.worker.cache, self.worker.active_requests
        bs = cache.block_size

        def need_of(r: Request, n: int) -> int:
            if r.request_id in active:
                return cache.blocks_needed(r.request_id, n)
            return max(1, -(-n // bs))

        free = len(cache.free_blocks)
        # a decode takes at most one new block, a chunk of n tokens at most n // bs + 2
        worst = len(out.decode_requests) + sum(n // bs + 2 for _, n in out.prefill_chunks)
        if worst > free:
            for req in self.scheduler.fit_blocks(out, free, need_of,
                                                 lambda r: len(cache.block_table(r.request_id))):
                self._release(req.request_id)
        prefills: List[Request] = []
        chunks: List[tuple] = []
        for req, chunk in zip(out.prefill_requests, out.prefill_chunks):
            if req.request_id not in self.worker.active_requests:
                if not self.worker.allocate_request(req.request_id):
                    req.status = RequestStatus.PENDING
                    req.num_prefilled = 0
                    self.scheduler.running.pop(req.request_id, None)
                    self.scheduler.waiting.appendleft(req)
                    continue
            self.sampler.add(req.request_id)
            prefills.append(req)
            chunks.append(chunk)
        decodes = out.decode_requests
        if not decodes and not prefills:
            return None
        prev = self._inflight
        prev_rows = prev.row_of if prev is not None else {}
        row_of = self.sampler.row_of
        work = []
        for r in decodes:
            rid = r.request_id
            src = prev_rows.get(rid, -1)
            toks = _ZERO if src >= 0 else np.asarray(r.output_token_ids[-1:], dtype=np.int32)
            work.append((rid, toks, src, row_of[rid]))
        final = {}
        for r, (start, length) in zip(prefills, chunks):
            toks = r.prompt_token_ids + r.output_token_ids
            final[r.request_id] = start + length >= len(toks)
            work.append((r.request_id, np.asarray(toks[start:start + length], dtype=np.int32), -1,
                         row_of[r.request_id]))
        seqs, errors = self.worker.prepare(work, len(decodes))
        for rid, err in errors:
            req = self.requests[rid]
            logger.error("request %s: %s", rid, err)
            self._finish(req, "error", success=False)
            results.append(StepOutput(rid, -1, True, "error"))
        if not seqs:
            return None
        ok = {s.request_id for s in seqs}
        nd = sum(1 for r in decodes if r.request_id in ok)
        logits, batch = self.worker.run_step(seqs, nd, prev.handle.dev if prev is not None else None)
        T = sum(len(s.token_ids) for s in seqs)
        reqs = [self.requests[s.request_id] for s in seqs]
        ids = [s.request_id for s in seqs]
        self.sampler.tp = self._sampling_tp()  # follows workspace reallocations
        handle = self.sampler.launch(logits, ids, [r.sampling_params for r in reqs],
                                     [r.num_generated_tokens for r in reqs],
                                     batch.token_rows, batch.input_ids, T)
        self.num_steps += 1
        self.num_step_tokens += T
        self.num_decode_tokens += nd
        idx = []
        for s, req in zip(seqs, reqs):
            if not final.get(req.request_id, True):
                # a prefill chunk that is not the prompt's last: no token (its
                # sample is dropped), the next chunk follows in a later step
                req.num_prefilled += len(s.token_ids)
                idx.append(-1)
                continue
            # the pending token takes its place now; its value comes later
            req.num_prefilled = 0
            idx.append(len(req.output_token_ids))
            req.output_token_ids.append(-1)
            req.num_generated_tokens += 1
            req.status = RequestStatus.DECODE
            if req.num_generated_tokens >= req.sampling_params.max_tokens:
                self._closing.add(req.request_id)
        rows = {rid: i for i, (rid, j) in enumerate(zip(ids, idx)) if j >= 0}
        return _Launched(reqs, idx, rows, handle)

    def _complete(self, launched: _Launched) -> List[StepOutput]:
        err: Optional[Exception] = None
        try:
            toks = launched.handle.wait()
        except Exception as e:  # noqa: BLE001 - a failed step fails its requests, not the engine
            err = e
        agree = getattr(self.worker, "tp_agree", None)
        if agree is not None and not agree(err is None):
            # tensor parallel: some rank could not read this step, so every
            # rank fails it (the same requests: the schedulers are identical)
            # and the cross-GPU flags restart together
            res = self._fail_step(launched, err or RuntimeError(
                "step failed on another tensor-parallel rank"))
            # the step launched after it ran its collectives against the
            # failed step's flags: fail it too (same decision on every rank)
            nxt, self._inflight = self._inflight, None
            if nxt is not None and nxt is not launched:
                res += self._fail_step(nxt, RuntimeError(
                    "step launched before a failed tensor-parallel step was reset"))
            self.worker.tp_reset()
            return res
        if err is not None:
            return self._fail_step(launched, err)
        results: List[StepOutput] = []
        eos = self.eos_token_id
        for req, i, tok in zip(launched.reqs, launched.idx, toks):
            if i < 0:
                continue  # a prefill chunk before the prompt's last
            if req.is_finished or self.requests.get(req.request_id) is not req:
                continue  # stopped on the step before, or aborted
            req.output_token_ids[i] = tok
            if req.on_token:
                req.on_token(tok, "")
            sp = req.sampling_params
            reason = None
            if eos is not None and tok == eos:
                reason = "stop"
            elif sp.stop_token_ids and tok in sp.stop_token_ids:
                reason = "stop"
            elif i + 1 >= sp.max_tokens:
                reason = "length"
            if reason:
                del req.output_token_ids[i + 1:]   # a token launched after this one is dropped
                req.num_generated_tokens = i + 1
                self._finish(req, reason)
            results.append(StepOutput(req.request_id, tok, reason is not None, reason))
        return results

    def run_to_completion(self) -> Dict[str, Request]:
        while self.has_unfinished():
            self.step()
        return self.requests


_ZERO = np.zeros(1, dtype=np.int32)


def _encode(tokenizer, prompt: Prompt) -> List[int]:
    if isinstance(prompt, str):
        if tokenizer is None:
            raise ValueError("string prompts need a tokenizer in the model directory; "
                             "pass token ids instead")
        return list(tokenizer.encode(prompt))
    return [int(t) for t in prompt]


def _decode(tokenizer, ids: List[int]) -> str:
    if tokenizer is None:
        return ""
    return tokenizer.decode(ids, skip_special_tokens=True)


class MuEngine:
    """Reference-compatible engine (engine.py:58-426): one request at a time."""

    def __init__(self, config: Optional[EngineConfig] = None, model_path: Optional[str] = None):
        self.config = config or EngineConfig()
        self.model_path = model_path
        self.worker: Optional[MuWorker] = None
        self.tokenizer = None
        self.core: Optional[StepEngine] = None
        self.scheduler = None
        self._initialized = False
        self._lock = asyncio.Lock()
        self._sync_loop: Optional[asyncio.AbstractEventLoop] = None
        self.stats = {"total_requests": 0, "total_tokens_generated": 0, "start_time": None}

    async def initialize(self, model_path: Optional[str] = None) -> None:
        if self._initialized:
            return
        model_path = model_path or self.model_path
        if model_path is None:
            raise ValueError("model_path is required")
        self.tokenizer = load_tokenizer(model_path)
        self.worker = MuWorker(self.config, self.config.device)
        self.worker.load_model(model_path)
        self._make_core()

    def initialize_from_worker(self, worker: MuWorker, tokenizer=None) -> None:
        """Use an already loaded worker (random weights, tests, benchmarks)."""
        self.worker = worker
        self.tokenizer = tokenizer
        self._make_core()

    def _make_core(self) -> None:
        eos = getattr(self.tokenizer, "eos_token_id", None) if self.tokenizer else None
        self.core = StepEngine(self.worker, self.config, eos)
        self.scheduler = self.core.scheduler
        self._initialized = True
        self.stats["start_time"] = time.time()

    def _check(self) -> None:
        if not self._initialized:
            raise RuntimeError("Engine not initialized. Call initialize() first.")

    def generate_sync(self, prompt: Prompt, sampling_params: Optional[SamplingParams] = None,
                      request_id: Optional[str] = None) -> GenerationOutput:
        """Blocking generate (engine.py:131-150).  Runs on an event loop the
        engine keeps for its synchronous calls (the reference takes the
        thread's default loop, which newer Pythons no longer create)."""
        try:
            asyncio.get_running_loop()
        except RuntimeError:
            pass
        else:
            raise RuntimeError("generate_sync called inside a running event loop; await generate()")
        if self._sync_loop is None or self._sync_loop.is_closed():
            self._sync_loop = asyncio.new_event_loop()
        return self._sync_loop.run_until_complete(self.generate(prompt, sampling_params, request_id))

    async def generate(self, prompt: Prompt, sampling_params: Optional[SamplingParams] = None,
                       request_id: Optional[str] = None) -> GenerationOutput:
        out = None
        async for out in self._run(prompt, sampling_params, request_id, stream=False):
            pass
        return out

    async def generate_stream(self, prompt: Prompt, sampling_params: Optional[SamplingParams] = None,
                              request_id: Optional[str] = None) -> AsyncIterator[StreamOutput]:
        async for item in self._run(prompt, sampling_params, request_id, stream=True):
            yield item

    async def _run(self, prompt, sampling_params, request_id, stream: bool):
        self._check()
        sp = sampling_params or SamplingParams()
        ids = _encode(self.tokenizer, prompt)
        async with self._lock:
            rid = self.core.add_request(ids, sp, request_id)
            req = self.core.requests[rid]
            reason = None
            while reason is None:
                for o in self.core.step():
                    if o.request_id != rid:
                        continue
                    if o.finished:
                        reason = o.finish_reason
                    if stream and o.token_id >= 0:
                        yield StreamOutput(rid, _decode(self.tokenizer, [o.token_id]), o.token_id,
                                           o.finished, o.finish_reason)
                await asyncio.sleep(0)
            self.core.requests.pop(rid, None)
            gen = list(req.output_token_ids)
            self.stats["total_requests"] += 1
            self.stats["total_tokens_generated"] += len(gen)
            if not stream:
                yield GenerationOutput(rid, _decode(self.tokenizer, gen), gen, True, reason,
                                       {"prompt_tokens": len(ids), "completion_tokens": len(gen),
                                        "total_tokens": len(ids) + len(gen)})

    def get_stats(self) -> Dict:
        up = time.time() - self.stats["start_time"] if self.stats["start_time"] else 0
        return {
            "total_requests": self.stats["total_requests"],
            "total_tokens_generated": self.stats["total_tokens_generated"],
            "uptime_seconds": up,
            "tokens_per_second": self.stats["total_tokens_generated"] / up if up > 0 else 0,
            "worker": self.worker.get_stats() if self.worker else {},
            "mu_config": {"enabled": self.config.mu.enabled, "mu": self.config.mu.mu,
                          "clamp_min": self.config.mu.clamp_min,
                          "clamp_max": self.config.mu.clamp_max},
        }

    def clear_cache(self) -> None:
        if self.worker and self.worker.cache:
            self.worker.cache.clear()

    async def shutdown(self) -> None:
        self.clear_cache()
        self._initialized = False


class MuBatchEngine(MuEngine):
    """Continuous batching behind the reference's MuBatchEngine API (engine.py:448-858)."""

    def __init__(self, config: Optional[EngineConfig] = None, model_path: Optional[str] = None):
        super().__init__(config, model_path)
        self._futures: Dict[str, asyncio.Future] = {}
        self._queues: Dict[str, asyncio.Queue] = {}
        self._prompt_len: Dict[str, int] = {}
        self._task: Optional[asyncio.Task] = None
        self._running = False
        self.stats.update({"batches_processed": 0, "avg_batch_size": 0.0})

    def _make_core(self) -> None:
        super()._make_core()
        self._running = True
        try:
            self._task = asyncio.get_running_loop().create_task(self._loop())
        except RuntimeError:  # no loop running: started by the first request
            self._task = None

    def _ensure_task(self) -> None:
        """Run the batching loop on the caller's event loop (a task left on
        a loop that has since closed is replaced)."""
        loop = asyncio.get_running_loop()
        if self._task is None or self._task.done() or self._task.get_loop() is not loop:
            self._running = True
            self._task = loop.create_task(self._loop())

    async def _loop(self) -> None:
        while self._running:
            if not self.core.has_unfinished():
                await asyncio.sleep(self.config.scheduler.batch_wait_time_ms / 1000.0)
                continue
            try:
                outs = self.core.step()
            except Exception as e:  # keep serving other requests
                logger.error("batch step failed: %s", e)
                await asyncio.sleep(0.01)
                continue
            n = self.stats["batches_processed"] = self.stats["batches_processed"] + 1
            self.stats["avg_batch_size"] += (len(outs) - self.stats["avg_batch_size"]) / n
            for o in outs:
                q = self._queues.get(o.request_id)
                if q is not None and o.token_id >= 0:
                    await q.put(StreamOutput(o.request_id, _decode(self.tokenizer, [o.token_id]),
                                             o.token_id, False))
                if o.finished:
                    await self._complete(o.request_id, o.finish_reason)
            await asyncio.sleep(0)

    async def _complete(self, rid: str, reason: Optional[str]) -> None:
        req = self.core.requests.pop(rid, None)
        gen = list(req.output_token_ids) if req else []
        self.stats["total_requests"] += 1
        self.stats["total_tokens_generated"] += len(gen)
        fut = self._futures.pop(rid, None)
        pl = self._prompt_len.pop(rid, 0)
        if fut is not None and not fut.done():
            fut.set_result(GenerationOutput(rid, _decode(self.tokenizer, gen), gen, True, reason,
                                            {"prompt_tokens": pl, "completion_tokens": len(gen),
                                             "total_tokens": pl + len(gen)}))
        q = self._queues.pop(rid, None)
        if q is not None:
            await q.put(StreamOutput(rid, "", -1, True, reason))

    async def generate(self, prompt: Prompt, sampling_params: Optional[SamplingParams] = None,
                       request_id: Optional[str] = None) -> GenerationOutput:
        self._check()
        self._ensure_task()
        ids = _encode(self.tokenizer, prompt)
        rid = self.core.add_request(ids, sampling_params or SamplingParams(), request_id)
        fut = asyncio.get_running_loop().create_future()
        self._futures[rid] = fut
        self._prompt_len[rid] = len(ids)
        return await fut

    async def generate_stream(self, prompt: Prompt, sampling_params: Optional[SamplingParams] = None,
                              request_id: Optional[str] = None) -> AsyncIterator[StreamOutput]:
        self._check()
        self._ensure_task()
        ids = _encode(self.tokenizer, prompt)
        q: asyncio.Queue = asyncio.Queue()
        rid = self.core.add_request(ids, sampling_params or SamplingParams(), request_id)
        self._queues[rid] = q
        self._prompt_len[rid] = len(ids)
        while True:
            item = await q.get()
            yield item
            if item.finished:
                break

    def get_stats(self) -> Dict:
        s = super().get_stats()
        sched = self.core.scheduler if self.core else None
        s.update({"engine_type": "continuous_batching",
                  "batches_processed": self.stats["batches_processed"],
                  "avg_batch_size": round(self.stats["avg_batch_size"], 2),
                  "pending_requests": (len(sched.waiting) + len(sched.priority_queue)) if sched else 0,
                  "active_requests": len(sched.running) if sched else 0,
                  "continuous_batching": {
                      "enabled": self.config.scheduler.enable_continuous_batching,
                      "batch_wait_time_ms": self.config.scheduler.batch_wait_time_ms,
                      "max_batch_size": self.config.scheduler.max_batch_size},
                  "scheduler": sched.get_stats() if sched else {},
                  "steps": self.core.get_stats() if self.core else {}})
        return s

    async def shutdown(self) -> None:
        self._running = False
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except (asyncio.CancelledError, Exception):
                pass
        for rid, fut in list(self._futures.items()):
            if not fut.done():
                fut.set_exception(RuntimeError("Engine shutdown"))
        self._futures.clear()
        await super().shutdown()
