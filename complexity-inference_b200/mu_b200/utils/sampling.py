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

from .. import kernels as K
from ..core.config import SamplingParams


class BatchSampler:
    def __init__(self, vocab_size: int, max_rows: int, device="cuda"):
        self.vocab = vocab_size
        self.words = (vocab_size + 31) // 32
        self.device = torch.device(device)
        self.seen = torch.zeros(max_rows, self.words, dtype=torch.int32, device=self.device)
        self.free_rows: List[int] = list(range(max_rows - 1, -1, -1))
        self.row_of: Dict[str, int] = {}
        self._cap = 0
        self._alloc(256)

    def _alloc(self, n: int) -> None:
        self._cap = n
        pin = torch.cuda.is_available()
        # host staging: temp f32, top_p f32, rep f32, top_k i32, rows i32, seeds i64, offsets i64
        self.h_f = torch.zeros(3, n, dtype=torch.float32, pin_memory=pin)
        self.h_i = torch.zeros(2, n, dtype=torch.int32, pin_memory=pin)
        self.h_l = torch.zeros(2, n, dtype=torch.int64, pin_memory=pin)
        self.d_f = torch.zeros(3, n, dtype=torch.float32, device=self.device)
        self.d_i = torch.zeros(2, n, dtype=torch.int32, device=self.device)
        self.d_l = torch.zeros(2, n, dtype=torch.int64, device=self.device)
        self.d_out = torch.zeros(n, dtype=torch.int32, device=self.device)
        self.h_out = torch.zeros(n, dtype=torch.int32, pin_memory=pin)
        self.d_seen_seq = torch.zeros(n, dtype=torch.int32, device=self.device)

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
        if row is not None:
            self.free_rows.append(row)

    # ---- per step -------------------------------------------------------------
    def mark_inputs(self, token_rows: torch.Tensor, input_ids: torch.Tensor, n: int) -> None:
        """Set the bits of this step's input tokens in their requests' rows."""
        K.mark_seen(self.seen, token_rows, input_ids, self.vocab, n=n)

    def sample(self, logits: torch.Tensor, request_ids: Sequence[str],
               params: Sequence[SamplingParams], steps: Sequence[int],
               copy_to_host: bool = True) -> torch.Tensor:
        """One token per logits row; returns a host (pinned) or device int32 tensor."""
        B = len(request_ids)
        if B > self._cap:
            self._alloc(max(B, 2 * self._cap))
        hf, hi, hl = self.h_f.numpy(), self.h_i.numpy(), self.h_l.numpy()
        for b, (rid, p, st) in enumerate(zip(request_ids, params, steps)):
            hf[0, b] = p.temperature
            hf[1, b] = p.top_p
            hf[2, b] = p.repetition_penalty
            hi[0, b] = p.top_k
            hi[1, b] = self.row_of[rid]
            hl[0, b] = p.seed if p.seed is not None else zlib.crc32(rid.encode())
            hl[1, b] = st
        self.d_f[:, :B].copy_(self.h_f[:, :B], non_blocking=True)
        self.d_i[:, :B].copy_(self.h_i[:, :B], non_blocking=True)
        self.d_l[:, :B].copy_(self.h_l[:, :B], non_blocking=True)
        K.sample(logits, self.d_f[0], self.d_i[0], self.d_f[1], self.d_f[2], self.seen,
                 self.d_l[0], self.d_l[1], self.d_out, num_rows=B, seen_rows=self.d_i[1])
        if not copy_to_host:
            return self.d_out[:B]
        self.h_out[:B].copy_(self.d_out[:B], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return self.h_out[:B]


# ---- reference single-row API ------------------------------------------------
def prepare_logits(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0,
                   top_p: float = 1.0, repetition_penalty: float = 1.0,
                   past_tokens: Optional[List[int]] = None) -> torch.Tensor:
    """Reference-compatible filtered logits [1, V] (sampling.py:20-87).

    Returned as a lazy record: the filtering itself happens inside the GPU
    sampler when ``sample_token`` consumes it."""
    out = logits.detach().float().reshape(1, -1)
    out._mu_params = (temperature, top_k, top_p, repetition_penalty, list(past_tokens or []))
    return out


def sample_token(logits: torch.Tensor, do_sample: bool = True, seed: int = 0, step: int = 0) -> int:
    """One token from [1, V] logits (sampling.py:90-120) via the GPU sampler."""
    t, k, p, rp, past = getattr(logits, "_mu_params", (1.0, 0, 1.0, 1.0, []))
    if not do_sample:
        t = 0.0
    dev = logits.device
    V = logits.shape[-1]
    x = logits.reshape(1, V).float().contiguous().to(dev)
    words = (V + 31) // 32
    seen = torch.zeros(1, words, dtype=torch.int32, device=dev)
    if past and rp != 1.0:
        ids = torch.as_tensor(sorted(set(i for i in past if 0 <= i < V)), dtype=torch.int32, device=dev)
        if ids.numel():
            K.mark_seen(seen, torch.zeros_like(ids), ids, V)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    K.sample(x, torch.tensor([t], device=dev, dtype=torch.float32),
             torch.tensor([k], device=dev, dtype=torch.int32),
             torch.tensor([p], device=dev, dtype=torch.float32),
             torch.tensor([rp], device=dev, dtype=torch.float32), seen,
             torch.tensor([seed], device=dev, dtype=torch.int64),
             torch.tensor([step], device=dev, dtype=torch.int64), out)
    return int(out.item())
