"""Request scheduler with the MuScheduler interface (mu_inference/core/scheduler.py).

Same request lifecycle, policies, token budgets and preemption bookkeeping
as the reference (scheduler.py:135-379): running DECODE requests first, then
new requests from the waiting queue (FCFS, or a heap for "priority") while
the batch and prefill token budgets allow, preemption of the most advanced
decodes when over budget.  The engine turns each SchedulerOutput into one
flat GPU step (decode requests first, then prefills) — see
``mu_b200.serving.step``.
"""

from __future__ import annotations

import heapq
import time
import uuid
from collections import deque
from dataclasses import dataclass, field
from enum import Enum
from typing import Callable, Deque, Dict, List, Optional, Set, Tuple

from .config import SamplingParams, SchedulerConfig
from .mu import MuDynamics, soft_clamp


class RequestStatus(str, Enum):
    PENDING = "pending"
    PREFILL = "prefill"
    DECODE = "decode"
    PREEMPTED = "preempted"
    FINISHED = "finished"
    FAILED = "failed"


@dataclass
class Request:
    request_id: str = field(default_factory=lambda: uuid.uuid4().hex[:16])
    prompt: str = ""
    prompt_token_ids: List[int] = field(default_factory=list)
    output_token_ids: List[int] = field(default_factory=list)
    output_text: str = ""
    sampling_params: SamplingParams = field(default_factory=SamplingParams)
    status: RequestStatus = RequestStatus.PENDING
    arrival_time: float = field(default_factory=time.time)
    start_time: Optional[float] = None
    finish_time: Optional[float] = None
    priority: float = 0.0
    num_prompt_tokens: int = 0
    num_generated_tokens: int = 0
    max_tokens: int = 512
    num_preemptions: int = 0
    # chunked prefill: tokens of (prompt + generated) already in the KV cache
    # while the request's prefill is split over several steps
    num_prefilled: int = 0
    on_token: Optional[Callable[[int, str], None]] = None
    on_finish: Optional[Callable[["Request"], None]] = None

    def __lt__(self, other: "Request") -> bool:
        return self.priority < other.priority

    @property
    def is_finished(self) -> bool:
        return self.status in (RequestStatus.FINISHED, RequestStatus.FAILED)

    @property
    def total_tokens(self) -> int:
        return self.num_prompt_tokens + self.num_generated_tokens

    @property
    def latency(self) -> Optional[float]:
        if self.finish_time and self.start_time:
            return self.finish_time - self.start_time
        return None

    @property
    def tokens_per_second(self) -> Optional[float]:
        lat = self.latency
        return self.num_generated_tokens / lat if lat and lat > 0 else None


@dataclass
class SchedulerOutput:
    prefill_requests: List[Request] = field(default_factory=list)
    decode_requests: List[Request] = field(default_factory=list)
    preempted_requests: List[Request] = field(default_factory=list)
    num_prefill_tokens: int = 0
    num_decode_tokens: int = 0
    # (start, length) of the tokens each prefill request runs this step
    prefill_chunks: List[Tuple[int, int]] = field(default_factory=list)

    @property
    def total_tokens(self) -> int:
        return self.num_prefill_tokens + self.num_decode_tokens

    @property
    def is_empty(self) -> bool:
        return not self.prefill_requests and not self.decode_requests


class MuScheduler:
    def __init__(self, config: SchedulerConfig):
        self.config = config
        self.waiting: Deque[Request] = deque()
        self.running: Dict[str, Request] = {}
        self.finished: Dict[str, Request] = {}
        self.priority_queue: List[Request] = []
        self.priority_dynamics = MuDynamics(mu=0.0, clamp_min=-10.0, clamp_max=10.0, ema_alpha=0.3)
        self.batch_dynamics = MuDynamics(mu=config.max_batch_size / 2, clamp_min=1,
                                         clamp_max=config.max_batch_size, ema_alpha=0.2)
        self._num_processed = 0
        self._total_tokens = 0

    def add_request(self, request: Request) -> str:
        request.status = RequestStatus.PENDING
        request.arrival_time = time.time()
        if self.config.policy == "priority":
            request.priority = self.priority_dynamics.update(request.priority)
            heapq.heappush(self.priority_queue, request)
        else:
            self.waiting.append(request)
        return request.request_id

    def schedule(self, hold: Optional[Set[str]] = None) -> SchedulerOutput:
        """Next step's work.  ``hold``: running requests to leave out of this
        step (an engine that has their last token in flight already knows
        they finish); they take no decode slot or budget."""
        out = SchedulerOutput()
        decode_budget = self.config.max_num_batched_tokens
        for req in list(self.running.values()):
            if req.status == RequestStatus.DECODE and not (hold and req.request_id in hold):
                out.decode_requests.append(req)
                out.num_decode_tokens += 1
                decode_budget -= 1
        prefill_budget = min(self.config.max_prefill_tokens, decode_budget)
        chunked = self.config.enable_chunked_prefill
        # Chunked prefill, for real: the reference records min(prompt, budget)
        # as the tokens needed but then runs every prompt whole.  Here a prompt
        # longer than the remaining budget runs its first `budget` tokens now
        # and the rest in the following steps (KV appended chunk by chunk;
        # only the last chunk's logits are sampled).  Requests part-way
        # through their prefill continue first, in admission order.
        continuing = [r for r in self.running.values()
                      if r.status == RequestStatus.PREFILL and r.num_prefilled > 0
                      and not (hold and r.request_id in hold)]
        for req in continuing:
            need = req.num_prompt_tokens + req.num_generated_tokens - req.num_prefilled
            take = min(need, prefill_budget)
            if take <= 0:
                continue
            out.prefill_requests.append(req)
            out.prefill_chunks.append((req.num_prefilled, take))
            out.num_prefill_tokens += take
            prefill_budget -= take
        slots = self.config.max_batch_size - len(out.decode_requests) - len(continuing)
        # Admission differs from the reference on purpose: there a popped request
        # that misses the budget is neither scheduled nor re-queued (it is lost).
        # Here a request is admitted when its prompt (plus tokens generated
        # before a preemption) fits the remaining budget, or, with chunked
        # prefill, when any budget is left (it starts with a partial chunk);
        # without chunking the first prefill of a step is always admitted
        # whole.  The rest go back to the front of the queue in their order.
        deferred: List[Request] = []
        for req in self._get_next_requests(slots):
            need = req.num_prompt_tokens + req.num_generated_tokens
            if chunked:
                take = min(need, prefill_budget)
                admit = not deferred and take > 0
            else:
                take = need
                admit = not deferred and not (out.prefill_requests and need > prefill_budget)
            if not admit:
                deferred.append(req)
                continue
            req.status = RequestStatus.PREFILL
            req.start_time = req.start_time or time.time()
            req.num_prefilled = 0
            self.running[req.request_id] = req
            out.prefill_requests.append(req)
            out.prefill_chunks.append((0, take))
            out.num_prefill_tokens += take
            prefill_budget -= take
        self._requeue_front(deferred)
        align = self.config.step_token_alignment
        if chunked and align > 0 and out.prefill_requests and out.total_tokens > align:
            # tile-aligned step: the last chunk gives up the rows past the
            # last full multiple of `align` (it continues next step)
            extra = out.total_tokens % align
            start, n = out.prefill_chunks[-1]
            if 0 < extra < n:
                out.prefill_chunks[-1] = (start, n - extra)
                out.num_prefill_tokens -= extra
        if self._should_preempt(out):
            out.preempted_requests = self._preempt_requests(out)
        return out

    def _get_next_requests(self, max_count: int) -> List[Request]:
        got: List[Request] = []
        if self.config.policy == "priority":
            while self.priority_queue and len(got) < max_count:
                got.append(heapq.heappop(self.priority_queue))
        else:  # fcfs; "fair" is FCFS in the reference too
            while self.waiting and len(got) < max_count:
                got.append(self.waiting.popleft())
        return got

    def _requeue_front(self, reqs: List[Request]) -> None:
        if self.config.policy == "priority":
            for r in reqs:
                heapq.heappush(self.priority_queue, r)
        else:
            for r in reversed(reqs):
                self.waiting.appendleft(r)

    def _should_preempt(self, out: SchedulerOutput) -> bool:
        return self.config.enable_preemption and out.total_tokens > self.config.max_num_batched_tokens

    def _preempt_requests(self, out: SchedulerOutput) -> List[Request]:
        preempted: List[Request] = []
        cands = sorted(out.decode_requests, key=lambda r: r.num_generated_tokens, reverse=True)
        to_free = out.total_tokens - self.config.max_num_batched_tokens
        for req in cands:
            if to_free <= 0:
                break
            req.status = RequestStatus.PREEMPTED
            req.num_preemptions += 1
            out.decode_requests.remove(req)
            if self.config.policy == "priority":
                req.priority = soft_clamp(req.priority - 1.0, -10.0, 10.0)
                heapq.heappush(self.priority_queue, req)
            else:
                self.waiting.appendleft(req)
            preempted.append(req)
            to_free -= 1
        return preempted

    def fit_blocks(self, out: SchedulerOutput, free: int, need_of: Callable[[Request, int], int],
                   held_of: Callable[[Request], int]) -> List[Request]:
        """Shrink a scheduled step until its new KV blocks fit the ``free`` ones.

        ``need_of(req, n)``: blocks that appending ``n`` tokens to ``req``
        takes (a request not yet in the cache counts its first block);
        ``held_of(req)``: blocks ``req`` holds now.  The reference never runs
        out of KV memory (its cache grows by ``torch.cat``), so this is an
        addition, in the reference's own terms.  In order:

        1. requests admitted by this ``schedule`` go back to the front of the
           queue (newest first); the first of them stays when no other
           request holds blocks;
        2. prefills already under way are preempted (newest first);
        3. decodes are preempted as ``_preempt_requests`` does it (most
           generated tokens first).

        Preemption is by recompute: the engine frees the request's blocks and
        it re-prefills prompt + generated tokens when readmitted.  Every
        preemption frees blocks, so the loop cannot cycle; a request that
        does not fit an otherwise empty pool is left for the cache's
        all-or-nothing reserve to reject.  Returns the requests preempted
        here (also appended to ``out.preempted_requests``)."""
        need = {id(r): need_of(r, 1) for r in out.decode_requests}
        for r, (_, n) in zip(out.prefill_requests, out.prefill_chunks):
            need[id(r)] = need_of(r, n)
        total = sum(need.values())
        if total <= free:
            return []

        def drop_prefill(req: Request) -> None:
            nonlocal total
            i = out.prefill_requests.index(req)
            out.prefill_requests.pop(i)
            _, n = out.prefill_chunks.pop(i)
            out.num_prefill_tokens -= n
            total -= need.pop(id(req))

        fresh = [r for r in out.prefill_requests if r.num_prefilled == 0 and held_of(r) == 0]
        others_hold = any(held_of(r) > 0 for r in self.running.values())
        deferred: List[Request] = []
        for req in reversed(fresh):
            # with nothing else in the pool the first admission stays (alone,
            # it either fits or is rejected by reserve)
            if total <= free or (not others_hold and req is fresh[0]):
                break
            drop_prefill(req)
            self.running.pop(req.request_id, None)
            req.status = RequestStatus.PREEMPTED if req.num_generated_tokens else RequestStatus.PENDING
            deferred.insert(0, req)
        self._requeue_front(deferred)

        victims = [r for r in reversed(out.prefill_requests) if held_of(r) > 0]
        victims += sorted(out.decode_requests, key=lambda r: r.num_generated_tokens, reverse=True)
        preempted: List[Request] = []
        for req in victims:
            if total <= free:
                break
            free += held_of(req)
            if req in out.prefill_requests:
                drop_prefill(req)
            else:
                out.decode_requests.remove(req)
                out.num_decode_tokens -= 1
                total -= need.pop(id(req))
            req.status = RequestStatus.PREEMPTED
            req.num_preemptions += 1
            req.num_prefilled = 0
            if self.config.policy == "priority":
                req.priority = soft_clamp(req.priority - 1.0, -10.0, 10.0)
                heapq.heappush(self.priority_queue, req)
            else:
                self.waiting.appendleft(req)
            preempted.append(req)
        out.preempted_requests.extend(preempted)
        return preempted

    def _unqueue(self, request_id: str) -> Optional[Request]:
        """Take a request out of the waiting queue / priority heap, if there."""
        req = next((r for r in list(self.waiting) + self.priority_queue
                    if r.request_id == request_id), None)
        if req is not None:
            self.waiting = deque(r for r in self.waiting if r is not req)
            self.priority_queue = [r for r in self.priority_queue if r is not req]
            heapq.heapify(self.priority_queue)
        return req

    def finish_request(self, request_id: str, success: bool = True) -> None:
        # A preempted request is both in `running` (status PREEMPTED, as in the
        # reference) and back in the queue: take it out of both, or it would
        # be readmitted after finishing.
        req = self.running.pop(request_id, None)
        queued = self._unqueue(request_id)
        req = req or queued
        if req:
            req.status = RequestStatus.FINISHED if success else RequestStatus.FAILED
            req.finish_time = time.time()
            self.finished[request_id] = req
            self._num_processed += 1
            self._total_tokens += req.total_tokens
            if req.on_finish:
                req.on_finish(req)

    def update_request(self, request_id: str, token_id: int, token_text: str = "") -> None:
        req = self.running.get(request_id)
        if req:
            req.output_token_ids.append(token_id)
            req.output_text += token_text
            req.num_generated_tokens += 1
            req.status = RequestStatus.DECODE
            if req.on_token:
                req.on_token(token_id, token_text)

    def get_request(self, request_id: str) -> Optional[Request]:
        return self.running.get(request_id) or self.finished.get(request_id)

    def abort_request(self, request_id: str) -> None:
        # Unlike the reference (scheduler.py:345-359), which returns after
        # popping a running request, also drop it from the queue: a preempted
        # request is in both.
        req = self.running.pop(request_id, None)
        self._unqueue(request_id)
        if req is not None:
            req.status = RequestStatus.FAILED
            self.finished[request_id] = req

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.priority_queue or self.running)

    def get_stats(self) -> dict:
        return {
            "waiting": len(self.waiting) + len(self.priority_queue),
            "running": len(self.running),
            "finished": len(self.finished),
            "total_processed": self._num_processed,
            "total_tokens": self._total_tokens,
            "policy": self.config.policy,
            "batch_dynamics": self.batch_dynamics.get_stats(),
        }

    def clear_finished(self, max_age: float = 300.0) -> None:
        cutoff = time.time() - max_age
        self.finished = {k: v for k, v in self.finished.items()
                         if v.finish_time and v.finish_time > cutoff}
