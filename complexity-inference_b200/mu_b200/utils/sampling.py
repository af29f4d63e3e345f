"""Batched GPU sampling (K7) with the reference's sampling semantics.

``BatchSampler`` keeps one repetition-penalty bitmap row per live request
on the device.  Every step it marks the step's input tokens (prompt tokens
at prefill, the previously sampled token at decode) in the owning rows, so
the bitmap always equals ``set(prompt + generated)`` — the ``past_tokens``
of mu_inference/utils/sampling.py:47-53 — without any host round trip, then
launches one sampler CTA per sequence.  Only the [B] chosen ids come back.

``prepare_logits`` / ``sample_token`` keep the reference's single-row API
(sampling.py:20-120) on top of the same kernel.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import zlib

import numpy as np
import torch

from .. import _lib
from .. import kernels as K
from ..core.config import SamplingParams


class SampleHandle:
    """Tokens of one launched sampling step: ``dev`` (int32 on the device,
    valid for the next step's inputs) and a pinned host copy that is ready
    once ``event`` has completed.  ``err`` (pinned, optional) receives the
    device error word as of the end of the step; ``wait`` raises
    :class:`~mu_b200._lib.DeviceError` when it is set, so a device-side
    time-out or bad index fails the step instead of returning its tokens."""

    __slots__ = ("dev", "host", "event", "err")

    def __init__(self, dev: torch.Tensor, host: torch.Tensor, event,
                 err: Optional[torch.Tensor] = None):
        self.dev, self.host, self.event, self.err = dev, host, event, err

    def wait(self) -> List[int]:
        if self.event is not None:
            self.event.synchronize()
        if self.err is not None:
            code = int(self.err[0])
            if code:
                raise _lib.DeviceError(code, "sampled step")
        return self.host.tolist()


class BatchSampler:
    # per row in the parameter blob (int32 words): temperature, top_p,
    # repetition_penalty (f32), top_k, bitmap row (i32), seed, offset (i64)
    _WORDS = 9

    def __init__(self, vocab_size: int, max_rows: int, device="cuda"):
        self.vocab = vocab_size
        self.words = (vocab_size + 31) // 32
        self.device = torch.device(device)
        self.seen = torch.zeros(max_rows, self.words, dtype=torch.int32, device=self.device)
        self.free_rows: List[int] = list(range(max_rows - 1, -1, -1))
        self.row_of: Dict[str, int] = {}
        self._seed_of: Dict[str, int] = {}
        # (comm, col0, cols) under a vocabulary-parallel LM head: the logits
        # buffer holds only this rank's columns until they are combined
        self.tp = None
        self._cap = 0
        self._alloc(256)

    def _alloc(self, n: int) -> None:
        if self._cap and self.device.type == "cuda":  # queued copies still use the old buffers
            torch.cuda.current_stream(self.device).synchronize()
        n = (n + 3) // 4 * 4
        self._cap = n
        pin = torch.cuda.is_available()
        # two pinned parameter blobs and token buffers, used alternately: the
        # host stages step i+1 while step i's copies may still be queued
        self._blob_h = [torch.zeros(self._WORDS * n, dtype=torch.int32, pin_memory=pin)
                        for _ in range(2)]
        self._blob_ev: List[Optional[torch.cuda.Event]] = [None, None]
        self._out_h = [torch.zeros(n, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._err_h = [torch.zeros(4, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._cur = 0
        self._blob_d = torch.zeros(self._WORDS * n, dtype=torch.int32, device=self.device)
        d = self._blob_d
        self.d_temp, self.d_topp, self.d_rep = (d[i * n:(i + 1) * n].view(torch.float32)
                                                for i in range(3))
        self.d_topk, self.d_rows = d[3 * n:4 * n], d[4 * n:5 * n]
        self.d_seed = d[5 * n:7 * n].view(torch.int64)
        self.d_off = d[7 * n:9 * n].view(torch.int64)
        self.d_out = torch.zeros(n, dtype=torch.int32, device=self.device)

    # ---- request rows -------------------------------------------------------
    def add(self, request_id: str) -> int:
        if request_id in self.row_of:
            return self.row_of[request_id]
        if not self.free_rows:
            grow = self.seen.shape[0]
            self.seen = torch.cat([self.seen, torch.zeros_like(self.seen)], 0)
            self.free_rows = list(range(2 * grow - 1, grow - 1, -1))
        row = self.free_rows.pop()
        self.seen[row].zero_()
        self.row_of[request_id] = row
        return row

    def remove(self, request_id: str) -> None:
        row = self.row_of.pop(request_id, None)
        self._seed_of.pop(request_id, None)
        if row is not None:
            self.free_rows.append(row)

    # ---- per step -------------------------------------------------------------
    def mark_inputs(self, token_rows: torch.Tensor, input_ids: torch.Tensor, n: int) -> None:
        """Set the bits of this step's input tokens in their requests' rows."""
        K.mark_seen(self.seen, token_rows, input_ids, self.vocab, n=n)

    def _seed(self, rid: str, p: SamplingParams) -> int:
        if p.seed is not None:
            return p.seed
        s = self._seed_of.get(rid)
        if s is None:
            s = self._seed_of[rid] = zlib.crc32(rid.encode())
        return s

    def launch(self, logits: torch.Tensor, request_ids: Sequence[str],
               params: Sequence[SamplingParams], steps: Sequence[int],
               token_rows: Optional[torch.Tensor] = None, input_ids: Optional[torch.Tensor] = None,
               num_tokens: int = 0) -> SampleHandle:
        """Enqueue (optional) bitmap marking of the step's input tokens, one
        sampling launch and the copy of the chosen ids to pinned host memory;
        returns without waiting."""
        B = len(request_ids)
        if B > self._cap:
            self._alloc(max(B, 2 * self._cap))
        n, k = self._cap, self._cur
        ev = self._blob_ev[k]
        if ev is not None:  # the copy that last read this blob must have run
            ev.synchronize()
        blob = self._blob_h[k].numpy()
        f = blob[:3 * n].view(np.float32)
        l = blob[5 * n:].view(np.int64)
        f[:B] = [p.temperature for p in params]
        f[n:n + B] = [p.top_p for p in params]
        f[2 * n:2 * n + B] = [p.repetition_penalty for p in params]
        blob[3 * n:3 * n + B] = [p.top_k for p in params]
        row_of = self.row_of
        blob[4 * n:4 * n + B] = [row_of[r] for r in request_ids]
        l[:B] = [self._seed(r, p) for r, p in zip(request_ids, params)]
        l[n:n + B] = steps
        stream = torch.cuda.current_stream(self.device)
        self._blob_d.copy_(self._blob_h[k], non_blocking=True)
        ev = self._blob_ev[k] or torch.cuda.Event()
        ev.record(stream)
        self._blob_ev[k] = ev
        if token_rows is not None and num_tokens > 0:
            self.mark_inputs(token_rows, input_ids, num_tokens)
        self.device_sample(logits, B, all(p.temperature <= 0 for p in params))
        host = self._out_h[k][:B]
        host.copy_(self.d_out[:B], non_blocking=True)
        err = self._err_h[k]
        _lib.call_status("muk_device_error_async", err.data_ptr(), stream.cuda_stream)
        done = torch.cuda.Event()
        done.record(stream)
        self._cur ^= 1
        return SampleHandle(self.d_out[:B], host, done, err)

    def device_sample(self, logits: torch.Tensor, B: int, greedy: bool) -> None:
        """The sampling launches of one step (parameters already in the
        device blob) into d_out.  Under a vocabulary-parallel head, an
        all-greedy step exchanges one (value, index) pair per row and rank;
        any other step all-gathers the columns first."""
        if self.tp is not None:
            comm, c0, n = self.tp
            if greedy:
                comm.greedy_(logits, B, c0, n, self.d_rep, self.seen, self.d_rows, self.d_out)
                return
            comm.allgather_cols_(logits, B, c0, n)
        K.sample(logits, self.d_temp, self.d_topk, self.d_topp, self.d_rep, self.seen,
                 self.d_seed, self.d_off, self.d_out, num_rows=B, seen_rows=self.d_rows)

    def sample(self, logits: torch.Tensor, request_ids: Sequence[str],
               params: Sequence[SamplingParams], steps: Sequence[int],
               copy_to_host: bool = True) -> torch.Tensor:
        """One token per logits row; returns a host (pinned) or device int32 tensor."""
        h = self.launch(logits, request_ids, params, steps)
        if not copy_to_host:
            return h.dev
        h.event.synchronize()
        return h.host


# ---- reference single-row API ------------------------------------------------
def prepare_logits(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0,
                   top_p: float = 1.0, repetition_penalty: float = 1.0,
                   past_tokens: Optional[List[int]] = None) -> torch.Tensor:
    """Processed logits [B, V] as the reference returns them (sampling.py:20-87):
    repetition penalty on row 0's past tokens (the reference indexes
    ``logits[0, id]``), temperature, top-k and top-p with removed entries at
    -inf.  Computed by the GPU sampler's filter (muk_prepare_logits); the
    result is returned on the input's device."""
    src = logits.detach()
    x = src.reshape(-1, src.shape[-1]).float()
    dev = x.device if x.is_cuda else torch.device("cuda")
    x = x.to(dev).contiguous()
    B, V = x.shape
    words = (V + 31) // 32
    seen = torch.zeros(2, words, dtype=torch.int32, device=dev)
    rows = torch.ones(B, dtype=torch.int32, device=dev)
    rows[0] = 0
    if past_tokens and repetition_penalty != 1.0:
        ids = sorted(set(int(i) for i in past_tokens if 0 <= int(i) < V))
        if ids:
            ids_t = torch.as_tensor(ids, dtype=torch.int32, device=dev)
            K.mark_seen(seen, torch.zeros_like(ids_t), ids_t, V)
    out = torch.empty_like(x)
    K.prepare_logits(x, torch.full((B,), float(temperature), device=dev),
                     torch.full((B,), int(top_k), device=dev, dtype=torch.int32),
                     torch.full((B,), float(top_p), device=dev),
                     torch.full((B,), float(repetition_penalty), device=dev), seen, out,
                     seen_rows=rows)
    return out.reshape(src.shape).to(src.device)


def sample_token(logits: torch.Tensor, do_sample: bool = True, seed: int = 0, step: int = 0) -> int:
    """One token from processed logits [1, V] (sampling.py:90-120): a draw from
    softmax(logits) (Gumbel-max with Philox noise keyed by ``seed`` and
    ``step``; -inf entries are never drawn, and a row that is all -inf gives
    token 0), or the argmax when ``do_sample`` is False."""
    dev = logits.device if logits.is_cuda else torch.device("cuda")
    V = logits.shape[-1]
    x = logits.reshape(-1, V)[:1].float().contiguous().to(dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    one = torch.ones(1, device=dev, dtype=torch.float32)
    K.sample(x, torch.tensor([1.0 if do_sample else 0.0], device=dev), torch.zeros(1, device=dev,
             dtype=torch.int32), one, one, None,
             torch.tensor([seed], device=dev, dtype=torch.int64),
             torch.tensor([step], device=dev, dtype=torch.int64), out)
    return int(out.item())
