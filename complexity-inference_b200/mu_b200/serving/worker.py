"""MuWorker: the drop-in step boundary (mu_inference/serving/worker.py).

``execute(List[WorkerRequest]) -> List[WorkerOutput]`` keeps the reference
signature, request/response types, order-preserving output and per-request
error mapping (worker.py:150-209).  The difference is underneath: the
reference runs one batch-1 forward per request with private contiguous KV
tensors; here all requests of the call form ONE flat step — decode requests
first, then prefills — over the paged KV pool, and the logits of all
sequences come out of a single LM-head GEMM.

``run_step`` is the batched entry used by the engines: it takes
(request id, new token ids) pairs, returns the [B, vocab] f32 logits on the
device and never copies logits to the host.  Pure-decode steps are replayed
from CUDA graphs captured per batch-size bucket (padded with inert
sequences: slot -1, one cached token), which removes the per-kernel launch
cost of the Python layer loop.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import _lib
from .. import kernels as K
from ..core.cache import PagedKVCache
from ..core.config import EngineConfig, ModelConfig
from ..models.loader import build_model, config_from_dict, detect_architecture, load_config
from ..models.weights import load_state_dict
from .step import SeqWork, StepBatch, StepPacker

logger = logging.getLogger(__name__)

GRAPH_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)


def _bucket(n: int) -> int:
    return next((b for b in GRAPH_BUCKETS if b >= n), n)


@dataclass
class StagedStep:
    """A step packed into the staging buffer, ready for run_staged."""

    B: int                 # real sequences (logits rows returned)
    T: int                 # tokens incl. padding
    Bp: int                # sequences incl. padding
    num_decode: int
    qlens: np.ndarray
    ctx: np.ndarray
    end: int               # used prefix of the staging buffer (int32 elements)
    graph: bool
    request_ids: List[str]
    patch: int = 0         # leading decode rows whose input comes from the previous samples
    real_tokens: int = 0   # tokens of the real sequences (padding excluded)


@dataclass
class WorkerRequest:
    """Request for the worker (worker.py:28-34)."""

    request_id: str
    input_ids: torch.Tensor  # [1, seq_len]
    position_ids: Optional[torch.Tensor] = None
    is_prefill: bool = True


@dataclass
class WorkerOutput:
    """Output of the worker (worker.py:37-43)."""

    request_id: str
    logits: torch.Tensor  # [1, vocab_size]
    finished: bool = False
    error: Optional[str] = None


class MuWorker:
    def __init__(self, config: EngineConfig, device: str = "cuda", tp_group=None):
        """``tp_group``: torch.distributed group of the tensor-parallel ranks
        (defaults to the world group when config.tensor_parallel_size > 1)."""
        self.config = config
        self.tp_group = tp_group
        self.device = torch.device(device)
        self.model = None
        self.cache: Optional[PagedKVCache] = None
        self.packer: Optional[StepPacker] = None
        self.active_requests: Dict[str, Dict] = {}
        self.stats = {"requests_processed": 0, "tokens_generated": 0, "prefill_tokens": 0}
        self.use_graphs = True
        self._graphs: Dict[int, Tuple[torch.cuda.CUDAGraph, int]] = {}
        self._graph_key = None
        # host-side (gloo) group of the tensor-parallel ranks, used to agree on
        # every step's success so that all ranks fail the same steps
        self._agree_group = None

    # ---- loading ---------------------------------------------------------------
    def load_model(self, model_path: str) -> None:
        """Load a local model dir (config.json + weights) and size the cache."""
        cfg_dict = load_config(model_path)
        arch = detect_architecture(cfg_dict)
        mcfg = self.config.model
        if mcfg is None or mcfg.hidden_size != cfg_dict.get("hidden_size", mcfg.hidden_size):
            mcfg = config_from_dict(cfg_dict)
            self.config.model = mcfg
        if int(self.config.tensor_parallel_size or 1) > 1:
            # read only this rank's slices of every tensor from disk
            from ..models.sharding import load_sharded_state_dict

            rank, tp, ep = self._tp_coords()
            sd, _ = load_sharded_state_dict(model_path, mcfg, arch, rank, tp, ep)
            self.load_state_dict(arch, mcfg, sd, sharded=True)
        else:
            self.load_state_dict(arch, mcfg, load_state_dict(model_path))

    def _tp_coords(self):
        import torch.distributed as dist

        tp = int(self.config.tensor_parallel_size or 1)
        if not dist.is_initialized():
            raise RuntimeError("tensor_parallel_size > 1 needs torch.distributed initialised")
        if dist.get_world_size(self.tp_group) != tp:
            raise RuntimeError(f"tensor_parallel_size {tp} != group size "
                               f"{dist.get_world_size(self.tp_group)}")
        return (dist.get_rank(self.tp_group), tp,
                bool(getattr(self.config, "expert_parallel", False)))

    def load_state_dict(self, arch: str, model_config: ModelConfig, sd, sharded: bool = False
                        ) -> None:
        """Build the model from a full state dict (sharded here when
        tensor-parallel) or, with ``sharded``, from this rank's shard."""
        self.config.model = model_config
        tp = int(self.config.tensor_parallel_size or 1)
        local = model_config
        if tp > 1:
            from ..models.sharding import local_config, shard_state_dict
            from ..models.weights import is_routed

            rank, tp, ep = self._tp_coords()
            if sharded:
                local = local_config(model_config, arch, tp, ep and is_routed(arch, model_config))
            else:
                sd, local = shard_state_dict(sd, model_config, arch, rank, tp, ep)
        self.model = build_model(arch, local, sd, self.config.mu, str(self.device))
        if tp > 1:
            import torch.distributed as dist

            from ..models.sharding import expert_range

            self.model.tp_group = self.tp_group or dist.group.WORLD
            if getattr(self.model, "local_experts", 0) and ep:
                self.model.expert_lo = expert_range(model_config, rank, tp)[0]
            if os.environ.get("MU_TP_STEP_AGREE", "1") != "0" and self._agree_group is None:
                ranks = dist.get_process_group_ranks(self.model.tp_group)
                self._agree_group = dist.new_group(ranks, backend="gloo")
        self._init_cache()

    # ---- tensor-parallel step agreement ----------------------------------------
    def tp_agree(self, ok: bool) -> bool:
        """True when every tensor-parallel rank read its copy of the step's
        results (one host-side all-reduce over gloo, no GPU work); always
        ``ok`` on a single GPU.  A device error or peer time-out on any rank
        thereby fails the same step, and the same requests, on all ranks, so
        their schedulers stay identical."""
        if self._agree_group is None:
            return ok
        import torch.distributed as dist

        t = torch.tensor([0 if ok else 1], dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self._agree_group)
        return int(t[0]) == 0

    def tp_reset(self) -> None:
        """After an agreed step failure: let every rank's kernels end (their
        cross-GPU waits are bounded), clear this GPU's error word, then zero
        the peer all-reduce flags and epoch on every rank between two host
        barriers, so no late store from the failed step meets a later call
        and all ranks restart their epochs together."""
        if self._agree_group is None:
            return
        import torch.distributed as dist

        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            _lib.device_error()
        dist.barrier(group=self._agree_group)
        comm = getattr(self.model, "comm", None)
        if comm is not None:
            comm.reset_flags()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self._agree_group)

    def _init_cache(self) -> None:
        mc, cc, sc = self.model.config, self.config.cache, self.config.scheduler
        nblocks = cc.num_gpu_blocks or cc.max_num_blocks
        self.cache = PagedKVCache(mc.num_hidden_layers, mc.num_key_value_heads, mc.head_dim,
                                  cc.block_size, nblocks, torch.bfloat16, str(self.device),
                                  self.config.mu)
        max_len = self.config.max_seq_len_hint or cc.max_seq_len
        max_blocks = (max_len + cc.block_size - 1) // cc.block_size + 1
        max_seqs = max(cc.max_num_seqs, sc.max_batch_size)
        max_tokens = max(sc.max_num_batched_tokens, max_seqs)
        if self.model.tp_group is not None and os.environ.get("MU_TP_COMM", "peer") == "peer":
            from ..comm import PeerAllReduce

            # partials of every step size this worker will run (the workspace
            # may round T up to a CUDA-graph bucket)
            rows = max(max_tokens, _bucket(max_seqs))
            cap = self.model.part_elems(rows)
            lg_rows = max(max_seqs, _bucket(max_seqs))
            vp = self.model.vocab_parallel_ok()
            self.model.comm = PeerAllReduce(
                self.model.tp_group, cap, self.device, x_elems=self.model.peer_x_elems(rows),
                logits_elems=lg_rows * mc.vocab_size if vp else 0,
                pair_rows=lg_rows if vp else 0)
        self.packer = StepPacker(self.device, max_tokens, max_seqs, max_blocks)
        self.model.ensure_workspace(max_tokens, max_seqs, max_blocks * cc.block_size)
        self._graphs.clear()

    # ---- request lifetime -------------------------------------------------------
    def allocate_request(self, request_id: str) -> bool:
        if not self.cache.allocate(request_id):
            return False
        self.active_requests[request_id] = {"seq_len": 0}
        return True

    def free_request(self, request_id: str) -> None:
        self.cache.free(request_id)
        self.active_requests.pop(request_id, None)

    # ---- batched step -----------------------------------------------------------
    def prepare(self, work: Sequence[Tuple], num_decode: int
                ) -> Tuple[List[SeqWork], List[Tuple[str, str]]]:
        """Reserve cache slots; returns the packable sequences and (id, error) pairs.

        ``work`` items are ``(request_id, new_token_ids)`` with optional
        ``src`` (index of the decode input among the previous step's sampled
        tokens on the device, -1 when the ids are given) and ``row``
        (repetition-bitmap row) appended."""
        seqs, errors = [], []
        cache = self.cache
        for item in work:
            rid, toks = item[0], item[1]
            st = self.active_requests.get(rid)
            if st is None:
                errors.append((rid, f"Request {rid} not allocated"))
                continue
            toks = np.asarray(toks, dtype=np.int32).reshape(-1)
            start = cache.get_seq_len(rid)
            slots = cache.reserve(rid, len(toks))
            if slots is None:
                errors.append((rid, "KV cache out of blocks"))
                continue
            st["seq_len"] = start + len(toks)
            seqs.append(SeqWork(rid, toks, start, slots, cache.block_table(rid),
                                item[2] if len(item) > 2 else -1,
                                item[3] if len(item) > 3 else 0))
        return seqs, errors

    def run_step(self, seqs: List[SeqWork], num_decode: int,
                 sampled: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, StepBatch]:
        """Pack and run one step; returns ([B, V] f32 logits on device, batch).

        ``sampled``: the previous step's sampled tokens on the device, read by
        decode sequences whose ``src`` is set."""
        st = self.stage(seqs, num_decode)
        self.packer.upload(st.end)
        return self.run_staged(st, sampled)

    def stage(self, seqs: List[SeqWork], num_decode: int) -> "StagedStep":
        """Reserve buffer room and fill the pinned host staging buffer for a step.

        Pure-decode steps are padded to their CUDA-graph bucket with inert
        sequences (slot -1, one cached token in block 0, outputs ignored)."""
        T = sum(len(s.token_ids) for s in seqs)
        B = len(seqs)
        grew = self.packer.ensure(max(T, _bucket(B)), max(B, _bucket(B)), max((len(s.block_table) for s in seqs),
                                                               default=1))
        # decode scratch is sized for the packer's block-table width (the graph bound)
        grew |= self.model.ensure_workspace(max(T, self.packer.cap_b), self.packer.cap_b,
                                            self._decode_bound())
        if grew:
            self._graphs.clear()
        # Tensor-parallel steps with the NCCL all-reduce run eagerly: replaying
        # graphs that captured the torch NCCL all-reduce gave wrong results
        # after the first replays.  The peer-memory all-reduce is graph-safe.
        tp_ok = self.model.tp_group is None or self.model.comm is not None
        graph = self.use_graphs and tp_ok and num_decode == B and B > 0
        allseq = seqs
        if graph:
            bucket = _bucket(B)
            allseq = list(seqs) + [SeqWork("", np.zeros(1, np.int32), 0, np.full(1, -1, np.int32),
                                           [0]) for _ in range(bucket - B)]
            num_decode = bucket
        Tp, Bp, _, qlens, ctx = self.packer.fill_host(allseq, num_decode)
        end = self.packer.off["bt"] + Bp * self.packer.cap_mb
        patch = max((i + 1 for i, s in enumerate(seqs) if s.src >= 0), default=0)
        return StagedStep(B, Tp, Bp, num_decode, qlens, ctx, end, graph,
                          [s.request_id for s in allseq], patch, T)

    def run_staged(self, st: "StagedStep", sampled: Optional[torch.Tensor] = None
                   ) -> Tuple[torch.Tensor, StepBatch]:
        """Run a step whose arrays are already in the packer's device buffer."""
        bound = self._decode_bound() if st.graph else None
        batch = self.packer.batch_view(st.T, st.Bp, st.num_decode, st.qlens, st.ctx, bound,
                                       st.request_ids)
        if st.patch:
            if sampled is None:
                raise ValueError("step has decode inputs from the previous samples; pass sampled")
            K.fill_decode_inputs(batch.input_ids, batch.decode_src, sampled, st.patch)
        if not st.graph:
            return self.model.forward_step(batch, self.cache), batch
        key = (self.packer.generation, id(self.model.ws))
        if self._graph_key != key:
            self._graphs.clear()
            self._graph_key = key
        g = self._graphs.get(st.Bp)
        if g is None:
            # warm-up on a side stream, then capture (all buffers are static)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.model.forward_step(batch, self.cache)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            n0 = _lib.launch_count
            with torch.cuda.graph(graph):
                self.model.forward_step(batch, self.cache)
            g = self._graphs[st.Bp] = (graph, _lib.launch_count - n0)
            _lib.launch_count = n0
        g[0].replay()
        _lib.launch_count += g[1]
        return self.model.ws.logits[:st.B], batch

    def _decode_bound(self) -> int:
        return self.packer.cap_mb * self.config.cache.block_size

    # ---- reference entry point ---------------------------------------------------
    @torch.inference_mode()
    def execute(self, requests: List[WorkerRequest]) -> List[WorkerOutput]:
        """One flat step for all requests; outputs in request order."""
        if not requests:
            return []
        V = self.model.config.vocab_size
        dec = [r for r in requests if not r.is_prefill]
        pre = [r for r in requests if r.is_prefill]
        work = [(r.request_id, r.input_ids.reshape(-1).cpu().numpy()) for r in dec + pre]
        out: Dict[str, WorkerOutput] = {}
        try:
            seqs, errors = self.prepare(work, len(dec))
            for rid, err in errors:
                out[rid] = WorkerOutput(rid, torch.zeros(1, V), finished=True, error=err)
            ok_ids = {s.request_id for s in seqs}
            nd = sum(1 for r in dec if r.request_id in ok_ids)
            if seqs:
                logits, _ = self.run_step(seqs, nd)
                vs = self.model.vocab_slice()
                if vs is not None:  # each rank computed its vocabulary columns
                    self.model.comm.allgather_cols_(self.model.ws.logits, len(seqs), *vs)
                logits = logits.clone()
                for i, s in enumerate(seqs):
                    out[s.request_id] = WorkerOutput(s.request_id, logits[i:i + 1])
                self.stats["tokens_generated"] += nd
                self.stats["prefill_tokens"] += sum(len(s.token_ids) for s in seqs[nd:])
        except Exception as e:  # per-request error mapping as in worker.py:179-206
            logger.error("step failed: %s", e)
            for r in requests:
                if r.request_id not in out or out[r.request_id].error is None:
                    out[r.request_id] = WorkerOutput(r.request_id, torch.zeros(1, V), True, str(e))
        return [out[r.request_id] for r in requests]

    def sampling_tp(self):
        """(comm, col0, cols) when the LM head is vocabulary-parallel (the
        sampler then combines the ranks' columns), else None."""
        vs = self.model.vocab_slice() if self.model is not None else None
        return None if vs is None else (self.model.comm, vs[0], vs[1])

    def close(self) -> None:
        """Release CUDA graphs and peer mappings (before the process group goes)."""
        self._graphs.clear()
        comm = getattr(self.model, "comm", None) if self.model is not None else None
        if comm is not None:
            comm.close()
            self.model.comm = None

    def get_stats(self) -> Dict:
        return {
            **self.stats,
            "active_requests": len(self.active_requests),
            "cache": self.cache.get_stats() if self.cache else {},
            "device": str(self.device),
            "model_memory_mb": self.model.get_memory_footprint()["total_mb"] if self.model else 0,
            "cuda_graphs": sorted(self._graphs),
        }

    def reset_stats(self) -> None:
        self.stats = {"requests_processed": 0, "tokens_generated": 0, "prefill_tokens": 0}
