"""Packing of one continuous-batching step into flat GPU arrays.

A step is a list of sequences, decode sequences (one new token) first, then
prefill sequences (whole prompts) — the order MuScheduler.schedule emits
(mu_inference/core/scheduler.py:206-236).  The packer fills one pinned int32
staging buffer and issues a single host-to-device copy into a device buffer
whose segment offsets are fixed by the packer's capacity, so every
StepBatch view keeps the same device address from step to step (needed to
replay a captured CUDA graph):

    input_ids[T] positions[T] slot_mapping[T] seq_lens[B] cu_seqlens_q[B+1]
    prefill_cu[B+1] last_token_idx[B] block_tables[B][max_blocks]
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np
import torch


@dataclass
class SeqWork:
    """One sequence's share of a step."""

    request_id: str
    token_ids: np.ndarray      # new tokens of this step (int32)
    start_pos: int             # tokens already cached before this step
    slots: np.ndarray          # cache slots of the new tokens (int32)
    block_table: Sequence[int]


@dataclass
class StepBatch:
    num_tokens: int
    num_seqs: int
    num_decode: int
    max_q_len: int             # longest prefill in the step (0 if none)
    max_seq_len: int           # longest context after the step
    decode_len_bound: int      # grid bound for decode attention (>= every decode context)
    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    seq_lens: torch.Tensor
    cu_seqlens_q: torch.Tensor
    prefill_cu: torch.Tensor
    last_token_idx: torch.Tensor
    block_tables: torch.Tensor
    request_ids: List[str] = field(default_factory=list)


def _al(n: int) -> int:
    return (n + 3) // 4 * 4


class StepPacker:
    """Fixed-capacity staging for StepBatch (capacity grows on demand)."""

    def __init__(self, device, max_tokens: int, max_seqs: int, max_blocks: int):
        self.device = torch.device(device)
        self.generation = 0
        self._alloc(max_tokens, max_seqs, max_blocks)

    def _alloc(self, T: int, B: int, MB: int) -> None:
        self.cap_t, self.cap_b, self.cap_mb = T, B, MB
        o = {}
        off = 0
        for name, n in (("ids", T), ("pos", T), ("slots", T), ("lens", B), ("cu", B + 1),
                        ("pcu", B + 1), ("last", B), ("bt", B * MB)):
            o[name] = off
            off += _al(n)
        self.off, self.size = o, off
        pin = torch.cuda.is_available()
        self.host = torch.zeros(off, dtype=torch.int32, pin_memory=pin)
        self.host_np = self.host.numpy()
        self.dev = torch.zeros(off, dtype=torch.int32, device=self.device)
        self.generation += 1

    def ensure(self, T: int, B: int, MB: int) -> bool:
        if T <= self.cap_t and B <= self.cap_b and MB <= self.cap_mb:
            return False
        self._alloc(max(T, self.cap_t), max(B, self.cap_b), max(MB, self.cap_mb))
        return True

    def _view(self, name: str, n: int) -> torch.Tensor:
        return self.dev[self.off[name]:self.off[name] + n]

    def fill_host(self, seqs: List[SeqWork], num_decode: int):
        """Write the step into the pinned staging buffer; returns (T, B, maxb, qlens, ctx)."""
        B = len(seqs)
        qlens = np.fromiter((len(s.token_ids) for s in seqs), dtype=np.int64, count=B)
        T = int(qlens.sum())
        ctx = np.fromiter((s.start_pos + len(s.token_ids) for s in seqs), dtype=np.int64, count=B)
        maxb = max((len(s.block_table) for s in seqs), default=1)
        self.ensure(T, B, maxb)
        h, o = self.host_np, self.off
        cu = np.zeros(B + 1, dtype=np.int64)
        np.cumsum(qlens, out=cu[1:])
        if B:
            h[o["ids"]:o["ids"] + T] = np.concatenate([s.token_ids for s in seqs])
            h[o["slots"]:o["slots"] + T] = np.concatenate([s.slots for s in seqs])
            starts = np.fromiter((s.start_pos for s in seqs), dtype=np.int64, count=B)
            h[o["pos"]:o["pos"] + T] = np.arange(T) - np.repeat(cu[:-1] - starts, qlens)
        h[o["lens"]:o["lens"] + B] = ctx
        h[o["cu"]:o["cu"] + B + 1] = cu
        h[o["pcu"]:o["pcu"] + B - num_decode + 1] = cu[num_decode:] - cu[num_decode]
        h[o["last"]:o["last"] + B] = cu[1:] - 1
        bt = h[o["bt"]:o["bt"] + self.cap_b * self.cap_mb].reshape(self.cap_b, self.cap_mb)
        for i, s in enumerate(seqs):
            n = len(s.block_table)
            bt[i, :n] = s.block_table
            bt[i, n:maxb] = 0
        return T, B, maxb, qlens, ctx

    def pack(self, seqs: List[SeqWork], num_decode: int, decode_len_bound: Optional[int] = None,
             stream: Optional[torch.cuda.Stream] = None) -> StepBatch:
        T, B, maxb, qlens, ctx = self.fill_host(seqs, num_decode)
        # one copy covering the used prefix of every segment (block tables last)
        end = self.off["bt"] + B * self.cap_mb
        if self.device.type == "cuda":
            st = stream or torch.cuda.current_stream()
            with torch.cuda.stream(st):
                self.dev[:end].copy_(self.host[:end], non_blocking=True)
        else:
            self.dev[:end].copy_(self.host[:end])
        return self.batch_view(T, B, num_decode, qlens, ctx, decode_len_bound,
                               [s.request_id for s in seqs])

    def batch_view(self, T, B, num_decode, qlens, ctx, decode_len_bound=None,
                   request_ids=None) -> StepBatch:
        o = self.off
        max_q = int(qlens[num_decode:].max()) if B > num_decode else 0
        max_ctx = int(ctx.max()) if B else 0
        bound = decode_len_bound if decode_len_bound is not None else max_ctx
        return StepBatch(
            num_tokens=T, num_seqs=B, num_decode=num_decode, max_q_len=max_q, max_seq_len=max_ctx,
            decode_len_bound=max(bound, 1),
            input_ids=self._view("ids", T), positions=self._view("pos", T),
            slot_mapping=self._view("slots", T), seq_lens=self._view("lens", B),
            cu_seqlens_q=self._view("cu", B + 1), prefill_cu=self._view("pcu", B - num_decode + 1),
            last_token_idx=self._view("last", B),
            block_tables=self.dev[o["bt"]:o["bt"] + self.cap_b * self.cap_mb].view(self.cap_b,
                                                                                self.cap_mb),
            request_ids=list(request_ids or []),
        )
