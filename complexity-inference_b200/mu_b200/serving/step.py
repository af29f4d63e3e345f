"""Packing of one continuous-batching step into flat GPU arrays.

A step is a list of sequences, decode sequences (one new token) first, then
prefill sequences (whole prompts) — the order MuScheduler.schedule emits
(mu_inference/core/scheduler.py:206-236).  The packer fills one pinned int32
staging buffer and issues a single host-to-device copy into a device buffer
whose segment offsets are fixed by the packer's capacity, so every
StepBatch view keeps the same device address from step to step (needed to
replay a captured CUDA graph):

    input_ids[T] positions[T] slot_mapping[T] token_rows[T] decode_src[B]
    seq_lens[B] cu_seqlens_q[B+1] prefill_cu[B+1] last_token_idx[B]
    block_tables[B][max_blocks]

``token_rows`` names each token's repetition-bitmap row (the sampler's row
of its request); ``decode_src[j] >= 0`` says decode sequence j's input token
is entry ``decode_src[j]`` of the previous step's sampled tokens on the
device, patched in by ``muk_fill_decode_inputs`` after the copy.

There are two pinned staging buffers used alternately, each guarded by a
CUDA event recorded after its copy was enqueued: the host may pack step i+1
while the copy of step i is still queued behind earlier GPU work.
"""

from __future__ import annotations

import itertools
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
    src: int = -1              # decode input = previous step's sampled token [src]
    row: int = 0               # repetition-bitmap row of the request


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
    token_rows: Optional[torch.Tensor] = None
    decode_src: Optional[torch.Tensor] = None
    request_ids: List[str] = field(default_factory=list)


def _al(n: int) -> int:
    return (n + 3) // 4 * 4


class StepPacker:
    """Fixed-capacity staging for StepBatch (capacity grows on demand)."""

    SEGMENTS = ("ids", "pos", "slots", "trow", "src", "lens", "cu", "pcu", "last", "bt")

    def __init__(self, device, max_tokens: int, max_seqs: int, max_blocks: int):
        self.device = torch.device(device)
        self.generation = 0
        self._alloc(max_tokens, max_seqs, max_blocks)

    def _alloc(self, T: int, B: int, MB: int) -> None:
        self.cap_t, self.cap_b, self.cap_mb = T, B, MB
        sizes = {"ids": T, "pos": T, "slots": T, "trow": T, "src": B, "lens": B, "cu": B + 1,
                 "pcu": B + 1, "last": B, "bt": B * MB}
        o = {}
        off = 0
        for name in self.SEGMENTS:
            o[name] = off
            off += _al(sizes[name])
        self.off, self.size = o, off
        pin = torch.cuda.is_available()
        self._hosts = [torch.zeros(off, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._events: List[Optional[torch.cuda.Event]] = [None, None]
        self._cur = 0
        self.dev = torch.zeros(off, dtype=torch.int32, device=self.device)
        self.generation += 1

    @property
    def host(self) -> torch.Tensor:
        """The staging buffer the next fill_host writes."""
        return self._hosts[self._cur]

    @property
    def host_np(self) -> np.ndarray:
        return self._hosts[self._cur].numpy()

    def ensure(self, T: int, B: int, MB: int) -> bool:
        if T <= self.cap_t and B <= self.cap_b and MB <= self.cap_mb:
            return False
        if self.device.type == "cuda":  # queued copies still read the old buffers
            torch.cuda.current_stream(self.device).synchronize()
        self._alloc(max(T, self.cap_t), max(B, self.cap_b), max(MB, self.cap_mb))
        return True

    def _view(self, name: str, n: int) -> torch.Tensor:
        return self.dev[self.off[name]:self.off[name] + n]

    def fill_host(self, seqs: List[SeqWork], num_decode: int):
        """Write the step into the pinned staging buffer; returns (T, B, maxb, qlens, ctx)."""
        B = len(seqs)
        qlens = np.fromiter((len(s.token_ids) for s in seqs), dtype=np.int64, count=B)
        T = int(qlens.sum())
        tlen = np.fromiter((len(s.block_table) for s in seqs), dtype=np.int64, count=B)
        maxb = int(tlen.max()) if B else 1
        self.ensure(T, B, maxb)
        ev = self._events[self._cur]
        if ev is not None:  # the copy that last read this buffer must have run
            ev.synchronize()
        h, o = self.host_np, self.off
        starts = np.fromiter((s.start_pos for s in seqs), dtype=np.int64, count=B)
        ctx = starts + qlens
        cu = np.zeros(B + 1, dtype=np.int64)
        np.cumsum(qlens, out=cu[1:])
        if B:
            h[o["ids"]:o["ids"] + T] = np.concatenate([s.token_ids for s in seqs])
            h[o["slots"]:o["slots"] + T] = np.concatenate([s.slots for s in seqs])
            h[o["pos"]:o["pos"] + T] = np.arange(T) - np.repeat(cu[:-1] - starts, qlens)
            rows = np.fromiter((s.row for s in seqs), dtype=np.int32, count=B)
            h[o["trow"]:o["trow"] + T] = np.repeat(rows, qlens)
            h[o["src"]:o["src"] + B] = np.fromiter((s.src for s in seqs), dtype=np.int32, count=B)
        h[o["lens"]:o["lens"] + B] = ctx
        h[o["cu"]:o["cu"] + B + 1] = cu
        h[o["pcu"]:o["pcu"] + B - num_decode + 1] = cu[num_decode:] - cu[num_decode]
        h[o["last"]:o["last"] + B] = cu[1:] - 1
        bt = h[o["bt"]:o["bt"] + self.cap_b * self.cap_mb].reshape(self.cap_b, self.cap_mb)
        if B:
            bt[:B, :maxb] = 0
            total = int(tlen.sum())
            flat = np.fromiter(itertools.chain.from_iterable(s.block_table for s in seqs),
                               dtype=np.int32, count=total)
            tcu = np.zeros(B + 1, dtype=np.int64)
            np.cumsum(tlen, out=tcu[1:])
            dst = np.arange(total) + np.repeat(np.arange(B) * self.cap_mb - tcu[:-1], tlen)
            bt.reshape(-1)[dst] = flat
        return T, B, maxb, qlens, ctx

    def upload(self, end: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Copy the used prefix of the current staging buffer to the device
        buffer and switch to the other staging buffer."""
        src = self._hosts[self._cur]
        if self.device.type == "cuda":
            st = stream or torch.cuda.current_stream(self.device)
            with torch.cuda.stream(st):
                self.dev[:end].copy_(src[:end], non_blocking=True)
                ev = self._events[self._cur] or torch.cuda.Event()
                ev.record(st)
            self._events[self._cur] = ev
        else:
            self.dev[:end].copy_(src[:end])
        self._cur ^= 1

    def pack(self, seqs: List[SeqWork], num_decode: int, decode_len_bound: Optional[int] = None,
             stream: Optional[torch.cuda.Stream] = None) -> StepBatch:
        T, B, maxb, qlens, ctx = self.fill_host(seqs, num_decode)
        # one copy covering the used prefix of every segment (block tables last)
        self.upload(self.off["bt"] + B * self.cap_mb, stream)
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
            token_rows=self._view("trow", T), decode_src=self._view("src", B),
            request_ids=list(request_ids or []),
        )
