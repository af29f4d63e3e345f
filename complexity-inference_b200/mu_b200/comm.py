"""Tensor-parallel all-reduce over NVLink peer memory (libmuk's
``muk_allreduce_f32``), the replacement for the NCCL all-reduce after the
row-parallel projections.

Each rank allocates one symmetric buffer (PyTorch memory; the same size and
layout on every rank), exports it through CUDA IPC and maps every peer's
buffer.  The model writes its partial projection outputs into the buffer;
``all_reduce_(t)`` then sums ``t`` (a view of the buffer) across the ranks in
place (two kernels: NVLink stores of each share to its owner, then the
owner's rank-ordered sum stored to every rank, with the cross-GPU barriers
inside the kernels), so the call is stream-ordered like any other kernel and
can be captured in a CUDA graph.
The handle exchange uses the torch.distributed process group once, at
construction.  There is no counterpart in the reference, which has no
multi-GPU path.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib


class PeerAllReduce:
    def __init__(self, group, max_elems: int, device, x_elems: int = 0, logits_elems: int = 0,
                 pair_rows: int = 0):
        import torch.distributed as dist

        self.group = group
        # rows pushed to their owner rank as bf16 (MU_TP_PUSH_BF16=1; default
        # f32: bf16 saved 1.5 us of a ~68 us exchange at C3's step size)
        self.push_bf16 = os.environ.get("MU_TP_PUSH_BF16", "0") == "1"
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("PeerAllReduce supports at most 8 ranks")
        lib = _lib.load()
        flag_words = int(lib.muk_allreduce_flag_bytes()) // 4
        self.max_elems = (int(max_elems) + 63) // 64 * 64
        # row-owned shares of the fused GEMM + all-reduce round rows up per
        # rank: room for one extra row per rank at the widest hidden size
        self.scratch_elems = (int(lib.muk_allreduce_scratch_elems(self.max_elems, self.world))
                              + self.world * 16384 + 63) // 64 * 64
        # [data | scratch (world shares) | flags | x rows], f32 words; the flag
        # area starts zeroed.  The x area (bf16) receives every rank's
        # normalised rows from muk_tp_residual_norm.
        self.flag_words = flag_words
        self.x_words = (int(x_elems) + 1) // 2 + 15 & ~15
        # [... | logits (f32, the vocabulary-parallel LM head) | greedy pairs
        # (2 parities x world x pair_rows x 8 bytes)]
        self.logits_words = int(logits_elems) + 15 & ~15
        self.pair_rows = int(pair_rows)
        self.pair_words = 2 * self.world * self.pair_rows * 2 + 15 & ~15
        self.buf = torch.zeros(self.max_elems + self.scratch_elems + flag_words + self.x_words
                               + self.logits_words + self.pair_words,
                               dtype=torch.float32, device=device)
        torch.cuda.synchronize(device)
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_uint64()
        _lib.call_status("muk_ipc_get_handle", self.buf.data_ptr(), ctypes.addressof(handle),
                         ctypes.byref(off))
        mine = (bytes(handle), int(off.value))
        objs = [None] * self.world
        dist.all_gather_object(objs, mine, group=group)
        self._bases = []
        self._data_arrays = {}
        ptrs = []
        for r, (h, o) in enumerate(objs):
            if r == self.rank:
                ptrs.append(self.buf.data_ptr())
                continue
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            p, base = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.call_status("muk_ipc_open_handle", ctypes.addressof(hb), o, ctypes.byref(p),
                             ctypes.byref(base))
            ptrs.append(p.value)
            self._bases.append(base.value)
        self.ptrs = ptrs
        self.scratch_ptrs = [p + self.max_elems * 4 for p in ptrs]
        self.flag_ptrs = [p + (self.max_elems + self.scratch_elems) * 4 for p in ptrs]
        self._x_off = self.max_elems + self.scratch_elems + flag_words
        self.x_ptrs = [p + self._x_off * 4 for p in ptrs]
        self._xs = (ctypes.c_void_p * self.world)(*self.x_ptrs)
        self._lg_off = self._x_off + self.x_words
        self._lgs = (ctypes.c_void_p * self.world)(*[p + self._lg_off * 4 for p in ptrs])
        self._pr_off = self._lg_off + self.logits_words
        self._prs = (ctypes.c_void_p * self.world)(*[p + self._pr_off * 4 for p in ptrs])
        self._scratch = (ctypes.c_void_p * self.world)(*self.scratch_ptrs)
        self._flags = (ctypes.c_void_p * self.world)(*self.flag_ptrs)
        dist.barrier(group=group)

    def view(self, n: int) -> torch.Tensor:
        """The first n elements of this rank's buffer (the model writes partials here)."""
        if n > self.max_elems:
            raise ValueError(f"PeerAllReduce: {n} elements > capacity {self.max_elems}")
        return self.buf[:n]

    def x_view(self, rows: int, cols: int) -> torch.Tensor | None:
        """[rows, cols] bf16 in this rank's x area (None if it does not fit):
        the activation buffer that muk_tp_residual_norm fills on every rank."""
        if rows * cols > 2 * self.x_words:
            return None
        x = self.buf[self._x_off:self._x_off + self.x_words].view(torch.bfloat16)
        return x[: rows * cols].view(rows, cols)

    def logits_view(self, rows: int, cols: int) -> torch.Tensor | None:
        """[rows, cols] f32 in this rank's logits area (None if it does not
        fit): the buffer the vocabulary-parallel LM head writes its column
        slice into and the column all-gather fills."""
        if rows * cols > self.logits_words:
            return None
        return self.buf[self._lg_off:self._lg_off + rows * cols].view(rows, cols)

    def allgather_cols_(self, logits: torch.Tensor, rows: int, col0: int, cols: int) -> None:
        """Store this rank's columns [col0, col0 + cols) of rows [0, rows) of
        ``logits`` (a logits_view) into every rank's buffer
        (``muk_tp_allgather_cols``)."""
        if logits.data_ptr() != self.buf.data_ptr() + self._lg_off * 4:
            raise ValueError("allgather_cols_: logits must be the logits_view")
        _lib.call("muk_tp_allgather_cols", ctypes.addressof(self._lgs),
                  ctypes.addressof(self._flags), self.rank, self.world, rows, logits.stride(0),
                  col0, cols, torch.cuda.current_stream().cuda_stream)

    def greedy_(self, logits: torch.Tensor, rows: int, col0: int, cols: int, rep_penalty,
                seen_bits, seen_rows, out: torch.Tensor) -> None:
        """out[:rows] = the argmax of every full row (with the repetition
        penalty) from this rank's column slice and the peers' (value, index)
        pairs (``muk_tp_greedy``)."""
        if rows > self.pair_rows:
            raise ValueError(f"greedy_: {rows} rows > pair capacity {self.pair_rows}")
        _lib.call("muk_tp_greedy", logits.data_ptr(), logits.stride(0), rows, col0, cols,
                  None if rep_penalty is None else rep_penalty.data_ptr(),
                  None if seen_bits is None else seen_bits.data_ptr(),
                  0 if seen_bits is None else seen_bits.stride(0),
                  None if seen_rows is None else seen_rows.data_ptr(),
                  ctypes.addressof(self._prs), self.pair_rows, ctypes.addressof(self._flags),
                  self.rank, self.world, out.data_ptr(), torch.cuda.current_stream().cuda_stream)

    def residual_norm_(self, part: torch.Tensor, resid: torch.Tensor, norm_w, eps: float,
                       x: torch.Tensor, clamp, clamp_delta: bool, clamp_sum: bool,
                       clamp_norm: bool) -> None:
        """Reduce-scatter the split-K partials ``part`` [S, T, H] (a view at the
        start of the buffer), add the owned rows' sums to ``resid`` and
        all-gather their norm into every rank's x (``muk_tp_residual_norm``)."""
        S, T, H = part.shape
        if part.data_ptr() != self.buf.data_ptr() or x.data_ptr() != self.x_ptrs[self.rank]:
            raise ValueError("residual_norm_: partials / x must live in the peer buffer")
        bufs = self._data_arrays.get(0)
        if bufs is None:
            bufs = self._data_arrays[0] = (ctypes.c_void_p * self.world)(*self.ptrs)
        _lib.call("muk_tp_residual_norm", ctypes.addressof(bufs), ctypes.addressof(self._scratch),
                  ctypes.addressof(self._flags), self.rank, self.world, T, H, S, T * H,
                  resid.data_ptr(), None if norm_w is None else norm_w.data_ptr(), eps,
                  ctypes.addressof(self._xs), x.stride(0), int(clamp_delta and clamp.enabled),
                  int(clamp_sum and clamp.enabled), int(clamp_norm and clamp.enabled), clamp.mu,
                  clamp.clamp_min, clamp.clamp_max, torch.cuda.current_stream().cuda_stream)

    def gemm_residual_norm_(self, A: torch.Tensor, W: torch.Tensor, M: int, resid: torch.Tensor,
                            norm_w, eps: float, x: torch.Tensor, clamp, clamp_delta: bool,
                            clamp_sum: bool, clamp_norm: bool) -> None:
        """:meth:`residual_norm_` with the projection GEMM in front, its
        epilogue pushing rows to their owners (``muk_gemm_tp_residual_norm``)."""
        N, K = W.shape[0], A.shape[1]
        lib = _lib.load()
        need = int(lib.muk_gemm_allreduce_scratch_elems(M, N, self.world))
        if M * N > self.max_elems or need > self.scratch_elems:
            raise ValueError(f"PeerAllReduce: {M}x{N} does not fit the peer buffers")
        if x.data_ptr() != self.x_ptrs[self.rank]:
            raise ValueError("gemm_residual_norm_: x must live in the peer buffer")
        bufs = self._data_arrays.get(0)
        if bufs is None:
            bufs = self._data_arrays[0] = (ctypes.c_void_p * self.world)(*self.ptrs)
        _lib.call("muk_gemm_tp_residual_norm", A.data_ptr(), A.stride(0), W.data_ptr(),
                  W.stride(0), M, N, K, ctypes.addressof(bufs), ctypes.addressof(self._scratch),
                  ctypes.addressof(self._flags), self.rank, self.world, resid.data_ptr(),
                  None if norm_w is None else norm_w.data_ptr(), eps, ctypes.addressof(self._xs),
                  x.stride(0), int(clamp_delta and clamp.enabled), int(clamp_sum and clamp.enabled),
                  int(clamp_norm and clamp.enabled), clamp.mu, clamp.clamp_min, clamp.clamp_max,
                  int(self.push_bf16), torch.cuda.current_stream().cuda_stream)

    def owns(self, t: torch.Tensor) -> bool:
        p = t.data_ptr()
        return (self.buf.data_ptr() <= p and p + t.numel() * 4 <= self.buf.data_ptr()
                + self.max_elems * 4 and t.is_contiguous())

    def all_reduce_(self, t: torch.Tensor, slices: int = 1) -> torch.Tensor:
        """Sum ``t`` (a contiguous f32 view of the buffer) over the ranks, in
        place.  With ``slices`` > 1, ``t`` is [slices, ...] split-K partials:
        they are folded first and the sum lands in ``t[0]``, which is returned
        (else ``t``)."""
        if not self.owns(t):
            raise ValueError("PeerAllReduce.all_reduce_: tensor is not a view of the buffer")
        n = t.numel() // slices
        off = t.data_ptr() - self.buf.data_ptr()
        bufs = self._data_arrays.get(off)
        if bufs is None:
            bufs = self._data_arrays[off] = (ctypes.c_void_p * self.world)(
                *[p + off for p in self.ptrs])
        _lib.call("muk_allreduce_f32", ctypes.addressof(bufs), ctypes.addressof(self._scratch),
                  ctypes.addressof(self._flags), self.rank, self.world, n, slices, n,
                  torch.cuda.current_stream().cuda_stream)
        return t[0] if slices > 1 else t

    def gemm_all_reduce(self, A: torch.Tensor, W: torch.Tensor, M: int) -> torch.Tensor:
        """out = Σ_ranks A_r · W_rᵀ as f32 [M, N] in every rank's buffer (start
        of the data range, returned as [1, M, N]): the row-parallel GEMM whose
        epilogue pushes each row to its owner rank, then the owners' sums
        stored to every rank (``muk_gemm_allreduce_f32``)."""
        N, K = W.shape[0], A.shape[1]
        lib = _lib.load()
        need = int(lib.muk_gemm_allreduce_scratch_elems(M, N, self.world))
        if M * N > self.max_elems or need > self.scratch_elems:
            raise ValueError(f"PeerAllReduce: {M}x{N} does not fit the peer buffers")
        bufs = self._data_arrays.get(0)
        if bufs is None:
            bufs = self._data_arrays[0] = (ctypes.c_void_p * self.world)(*self.ptrs)
        _lib.call("muk_gemm_allreduce_f32", A.data_ptr(), A.stride(0), W.data_ptr(), W.stride(0),
                  M, N, K, ctypes.addressof(bufs), ctypes.addressof(self._scratch),
                  ctypes.addressof(self._flags), self.rank, self.world,
                  torch.cuda.current_stream().cuda_stream)
        return self.buf[:M * N].view(1, M, N)

    def rows_view(self, T: int, H: int) -> torch.Tensor:
        """[T, H] bf16 rows at the start of this rank's data range: where the
        expert-parallel combine expects each rank's expert rows."""
        n = T * H
        if (n + 1) // 2 > self.max_elems:
            raise ValueError(f"PeerAllReduce: {T}x{H} bf16 rows do not fit the peer buffer")
        return self.buf[:(n + 1) // 2].view(torch.bfloat16)[:n].view(T, H)

    def ep_gather_(self, rows: torch.Tensor, expert_offsets: torch.Tensor, e_lo: int,
                   e_hi: int) -> torch.Tensor:
        """Expert-parallel combine: this rank's rows [offs[e_lo], offs[e_hi]) of
        ``rows`` (a rows_view) copied into the same rows of every rank, so that
        every rank ends with every expert's rows (``muk_ep_gather_bf16``)."""
        if rows.data_ptr() != self.buf.data_ptr() or rows.dtype != torch.bfloat16:
            raise ValueError("PeerAllReduce.ep_gather_: rows must be a rows_view")
        bufs = self._data_arrays.get(0)
        if bufs is None:
            bufs = self._data_arrays[0] = (ctypes.c_void_p * self.world)(*self.ptrs)
        _lib.call("muk_ep_gather_bf16", ctypes.addressof(bufs), ctypes.addressof(self._flags),
                  self.rank, self.world, expert_offsets.data_ptr(), e_lo, e_hi, rows.shape[1],
                  torch.cuda.current_stream().cuda_stream)
        return rows

    def reset_flags(self) -> None:
        """Zero this rank's flag words (pushed / done epochs and its own
        epoch).  Only safe while no all-reduce kernel runs on any rank: the
        caller synchronises every rank and puts host barriers on both sides
        (MuWorker.tp_reset)."""
        self.buf[self.max_elems + self.scratch_elems:self._x_off].zero_()

    def close(self) -> None:
        torch.cuda.synchronize()
        for b in self._bases:
            _lib.call_status("muk_ipc_close_handle", b)
        self._bases = []
