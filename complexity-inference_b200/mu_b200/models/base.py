"""Model base: the flat-batch forward step shared by the Llama and Deep models.

The reference runs one ``model.forward(input_ids[1, S], past_key_values)``
per request (mu_inference/models/base.py:107-129, serving/worker.py:249-331).
Here a whole continuous-batching step runs as one pass over a flat token
stream ``[T, H]`` (decode tokens first, then prefill tokens) with the KV
cache in the paged pool; :meth:`MuModelBase.forward_step` returns the f32
logits of each sequence's last token, ``[B, vocab]``.

Numerics: weights and GEMM operands are bf16 with f32 accumulation; the
residual stream, norms and INL dynamics stay f32; RoPE uses the f32 cos/sin
table built exactly as RotaryEmbeddingCompat builds it (layers.py:286-299).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from .. import kernels as K
from ..core.config import ModelConfig, MuConfig
from ..kernels import Clamp

PAD_MULT = 64  # SwiGLU weights are interleaved in 64-row gate/up groups
# Row-parallel GEMM with the reduce-scatter in its epilogue pays while the
# GEMM has few rows (decode steps: 68 vs 79 us at 256 x 4096 x 2048 on 2
# GPUs); with more rows the epilogue's row-per-lane NVLink stores lose to a
# local GEMM plus the coalesced push kernel (117 vs 91 us at 1000 rows).
# Steps of at most this many rows run a row-parallel projection under
# peer-memory TP as one GEMM whose epilogue pushes rows to their owners
# (MU_TP_FUSED_MAX_ROWS overrides); larger steps run split-K, then a push
# kernel.  With the epilogue's stores staged through shared memory (whole
# 128-byte rows per NVLink store) the fused form wins at every C3 step size
# (2 GPUs: 16,842 vs 16,316-16,396 tokens/s with a 512-row limit).
FUSED_TP_MAX_ROWS = int(os.environ.get("MU_TP_FUSED_MAX_ROWS", str(1 << 20)))


@dataclass
class MuModelOutput:
    """Output record with the reference's fields (mu_inference/models/base.py:22-47)."""

    logits: torch.Tensor
    hidden_states: Optional[torch.Tensor] = None
    attentions: Optional[Dict[int, torch.Tensor]] = None
    router_logits: Optional[Dict[int, torch.Tensor]] = None
    mu_stats: Optional[Dict[str, float]] = None


def pad_to(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, pad: int) -> torch.Tensor:
    """[I, K] gate and up -> [2*pad, K] in 64-row groups g0 u0 g1 u1 ... (zero rows past I)."""
    I, Kd = gate.shape
    g = torch.zeros(pad, Kd, dtype=gate.dtype, device=gate.device)
    u = torch.zeros_like(g)
    g[:I] = gate
    u[:I] = up
    return torch.stack([g.view(pad // PAD_MULT, PAD_MULT, Kd), u.view(pad // PAD_MULT, PAD_MULT, Kd)],
                       1).reshape(2 * pad, Kd).contiguous()


def pad_cols(w: torch.Tensor, cols: int) -> torch.Tensor:
    if w.shape[1] == cols:
        return w.contiguous()
    out = torch.zeros(w.shape[0], cols, dtype=w.dtype, device=w.device)
    out[:, : w.shape[1]] = w
    return out


def choose_split(M: int, N: int, K: int, max_rows: int) -> int:
    """Split-K factor for an f32-partial GEMM, from libmuk's shape planner
    (the same model the launcher uses to pick tile shapes), bounded so the
    partials fit ``max_rows`` rows of the workspace."""
    from .. import _lib

    max_s = max(1, min(16, max_rows // max(M, 1)))
    return int(_lib.load().muk_gemm_plan_split(M, N, K, _lib.MUK_EPI_F32, max_s))


class Workspace:
    """Activation buffers sized for ``max_tokens`` tokens / ``max_seqs`` sequences.

    Buffer addresses stay fixed for the life of the workspace, which is what
    lets a decode step be captured in a CUDA graph and replayed."""

    def __init__(self, model: "MuModelBase", max_tokens: int, max_seqs: int, max_seq_len: int):
        cfg = model.config
        dev = model.device
        H, D = cfg.hidden_size, cfg.head_dim
        Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        T = max_tokens
        self.max_tokens, self.max_seqs, self.max_seq_len = T, max_seqs, max_seq_len
        bf, f32 = torch.bfloat16, torch.float32
        self.resid = torch.empty(T, H, device=dev, dtype=f32)
        # [x | mu_prev] for Deep; under peer-memory TP the model may keep x in
        # the peer-mapped area, where every rank's normalised rows land
        comm = getattr(model, "comm", None)
        px = comm.x_view(T, 2 * H) if comm is not None and model.peer_x_elems(T) else None
        self.shared_x = px is not None
        self.x = px if px is not None else torch.zeros(T, 2 * H, device=dev, dtype=bf)
        self.qkv = torch.empty(T, (Hq + 2 * Hkv) * D, device=dev, dtype=bf)
        self.attn = torch.empty(T, Hq * D, device=dev, dtype=bf)
        self.part_rows = max(T, 2048)
        n = self.part_rows * model.max_part_width()
        # under tensor parallelism the partials live in the peer-mapped buffer
        # that the all-reduce kernel sums in place
        self.shared_part = comm is not None and n <= comm.max_elems
        self.part = comm.view(n) if self.shared_part else torch.empty(n, device=dev, dtype=f32)
        self.act = torch.empty(T, model.act_width(), device=dev, dtype=bf)
        self.xl = torch.empty(max_seqs, H, device=dev, dtype=bf)
        # under a vocabulary-parallel LM head the logits live in the peer
        # buffer (each rank writes its columns, the samplers combine them)
        lg = comm.logits_view(max_seqs, cfg.vocab_size) \
            if comm is not None and model.vocab_parallel_ok() else None
        self.shared_logits = lg is not None
        self.logits = lg if lg is not None else torch.empty(max_seqs, cfg.vocab_size, device=dev,
                                                            dtype=f32)
        nbytes = K.decode_attn_workspace_size(max_seqs, Hq, D, max_seq_len)
        self.attn_ws = torch.empty(max(nbytes // 4, 4), device=dev, dtype=f32)
        model.extra_workspace(self, T)

    def part_view(self, splits: int, rows: int, cols: int) -> torch.Tensor:
        return self.part[: splits * rows * cols].view(splits, rows, cols)


class MuModelBase:
    """Common state and the attention / LM-head pieces of the step."""

    arch = "base"

    def __init__(self, config: ModelConfig, mu_config: Optional[MuConfig] = None,
                 device: str = "cuda"):
        self.config = config
        self.mu_config = mu_config or MuConfig()
        self.clamp = Clamp.from_mu_config(self.mu_config)
        self.device = torch.device(device)
        self.dtype = torch.bfloat16
        self.ws: Optional[Workspace] = None
        self.rope_cos: Optional[torch.Tensor] = None
        self.rope_sin: Optional[torch.Tensor] = None
        self._rope_len = 0
        self._fused_rope = os.environ.get("MU_FUSED_ROPE", "1") != "0"
        self._tp_fused = os.environ.get("MU_TP_FUSED", "1") != "0"
        self.tp_group = None   # torch.distributed group when tensor-parallel
        self.comm = None       # mu_b200.comm.PeerAllReduce when tensor-parallel over NVLink
        self.ensure_rope(max(config.max_position_embeddings, 16))

    # ---- overridable sizes ---------------------------------------------------
    def act_width(self) -> int:
        raise NotImplementedError

    def max_part_width(self) -> int:
        return self.config.hidden_size

    def part_elems(self, max_tokens: int) -> int:
        """f32 elements of the partial buffer for a workspace of max_tokens rows."""
        return max(max_tokens, 2048) * self.max_part_width()

    def extra_workspace(self, ws: Workspace, T: int) -> None:
        pass

    def vocab_parallel_ok(self) -> bool:
        """Whether the LM head can run vocabulary-parallel: peer-memory tensor
        parallelism and V a multiple of 4 x ranks (MU_TP_VOCAB=0: every rank
        computes the full head)."""
        if self.tp_group is None or os.environ.get("MU_TP_COMM", "peer") != "peer":
            return False
        if os.environ.get("MU_TP_VOCAB", "1") == "0":
            return False
        import torch.distributed as dist

        return self.config.vocab_size % (4 * dist.get_world_size(self.tp_group)) == 0

    def vocab_slice(self):
        """(col0, cols) of this rank's vocabulary columns when the LM head is
        vocabulary-parallel, else None."""
        ws = self.ws
        if self.comm is None or ws is None or not ws.shared_logits:
            return None
        cols = self.config.vocab_size // self.comm.world
        return self.comm.rank * cols, cols

    def peer_x_elems(self, max_tokens: int) -> int:
        """bf16 elements of the activation rows kept in peer memory under
        tensor parallelism (0: x stays private)."""
        return 0

    # ---- setup -----------------------------------------------------------------
    def ensure_rope(self, n: int) -> None:
        """f32 cos/sin [n, head_dim/2], built like RotaryEmbeddingCompat._build_cache."""
        if n <= self._rope_len:
            return
        D = self.config.head_dim
        inv = 1.0 / (self.config.rope_theta ** (torch.arange(0, D, 2).float() / D))
        t = torch.arange(n).float()
        f = torch.outer(t, inv)
        self.rope_cos = f.cos().to(self.device).contiguous()
        self.rope_sin = f.sin().to(self.device).contiguous()
        self._rope_len = n

    def ensure_workspace(self, max_tokens: int, max_seqs: int, max_seq_len: int) -> bool:
        """(Re)allocate buffers if a step needs more room; True if reallocated."""
        ws = self.ws
        if (ws is not None and ws.max_tokens >= max_tokens and ws.max_seqs >= max_seqs
                and ws.max_seq_len >= max_seq_len):
            return False
        if ws is not None:
            max_tokens = max(max_tokens, ws.max_tokens)
            max_seqs = max(max_seqs, ws.max_seqs)
            max_seq_len = max(max_seq_len, ws.max_seq_len)
        self.ws = None
        self.ws = Workspace(self, max_tokens, max_seqs, max_seq_len)
        self.ensure_rope(max_seq_len + 1)
        return True

    # ---- shared pieces of the step ---------------------------------------------
    def row_parallel(self, A: torch.Tensor, W: torch.Tensor, T: int, N: int) -> torch.Tensor:
        """A row-parallel projection (O, down) summed over the TP ranks; returns
        the [S, T, N] f32 slices the consumer reads.  Under peer-memory TP the
        GEMM and the reduce-scatter are one kernel (``muk_gemm_allreduce_f32``;
        MU_TP_FUSED=0: GEMM, then ``muk_allreduce_f32``); otherwise split-K
        partials, all-reduced by NCCL under TP."""
        ws = self.ws
        if self.comm is not None and ws.shared_part and self._tp_fused and T <= FUSED_TP_MAX_ROWS:
            return self.comm.gemm_all_reduce(A, W, T)
        s = choose_split(T, N, A.shape[1], ws.part_rows)
        part = ws.part_view(s, T, N)
        K.gemm(A, W, part, K.MUK_EPI_F32, split_k=s, M=T)
        return self.reduce_partials(part)

    def reduce_partials(self, part: torch.Tensor) -> torch.Tensor:
        """Sum a row-parallel projection's output over the TP ranks and return
        what the consumer reads: in place through peer memory when the
        partials sit in the shared buffer (``muk_allreduce_f32``; split-K
        slices [S, T, N] are folded first and the sum returned as [1, T, N]),
        else with an NCCL all-reduce of every slice."""
        if self.tp_group is None:
            return part
        if self.comm is not None and self.comm.owns(part):
            if part.dim() == 3:
                return self.comm.all_reduce_(part, slices=part.shape[0]).unsqueeze(0) \
                    if part.shape[0] > 1 else self.comm.all_reduce_(part)
            return self.comm.all_reduce_(part)
        import torch.distributed as dist

        dist.all_reduce(part, group=self.tp_group)
        return part

    def fused_rope(self) -> bool:
        """RoPE + KV append in the q|k|v GEMM's epilogue (MU_FUSED_ROPE=0: separate kernel)."""
        return self._fused_rope and self.config.head_dim in (64, 128)

    def qkv_proj(self, layer: int, x: torch.Tensor, w: torch.Tensor, batch, cache,
                 q_norm_w=None, k_norm_w=None, rownorm=None) -> None:
        """q|k|v projection of the step's tokens, RoPE'd, with k/v appended to
        the paged cache and q left in ws.qkv for the attention kernels
        (``rownorm``: finish the input's RMSNorm in the GEMM, fused path only)."""
        cfg, ws = self.config, self.ws
        T, Hq, Hkv, D = batch.num_tokens, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        kc, vc = cache.k_cache(layer), cache.v_cache(layer)
        if self.fused_rope():
            K.gemm_qkv_rope(x, w, ws.qkv, batch.positions, batch.slot_mapping, self.rope_cos,
                            self.rope_sin, Hq, Hkv, D, kc, vc, q_norm_w, k_norm_w, 1e-6, M=T,
                            rownorm=rownorm)
            return
        assert rownorm is None, "row-norm scaling needs the fused q|k|v epilogue"
        K.gemm(x, w, ws.qkv, K.MUK_EPI_BF16, M=T)
        K.rope_kv_append(ws.qkv, batch.positions, batch.slot_mapping, self.rope_cos, self.rope_sin,
                         Hq, Hkv, D, kc, vc, q_norm_w, k_norm_w, 1e-6, num_tokens=T)

    def attention(self, layer: int, batch, cache) -> torch.Tensor:
        """Paged decode / varlen prefill attention over the cache -> ws.attn
        (q in ws.qkv, k/v already appended by qkv_proj)."""
        cfg, ws = self.config, self.ws
        Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        kc, vc = cache.k_cache(layer), cache.v_cache(layer)
        nd, B = batch.num_decode, batch.num_seqs
        bt = batch.block_tables
        if nd > 0:
            bound = min(batch.decode_len_bound, bt.shape[1] * 16)
            K.decode_attn(ws.qkv[:, : Hq * D], ws.attn, kc, vc, bt, batch.seq_lens, Hq, Hkv, D,
                          bound, workspace=ws.attn_ws, num_seqs=nd)
        if B > nd:
            # decode sequences own exactly one token each, so prefill rows start at nd
            K.prefill_attn(ws.qkv[nd:, : Hq * D], ws.attn[nd:], kc, vc, bt[nd:],
                           batch.seq_lens[nd:], batch.prefill_cu, batch.max_q_len, Hq, Hkv, D,
                           num_seqs=B - nd)
        return ws.attn

    def lm_head(self, batch, final_norm_w: torch.Tensor, lm_w: torch.Tensor) -> torch.Tensor:
        ws, B = self.ws, batch.num_seqs
        K.rmsnorm_rows(ws.resid, batch.last_token_idx[:B], final_norm_w, self.config.rms_norm_eps,
                       ws.xl, self.clamp)
        return self.lm_gemm(lm_w, B)

    def lm_gemm(self, lm_w: torch.Tensor, B: int) -> torch.Tensor:
        """logits = xl · lm_wᵀ; under a vocabulary-parallel head only this
        rank's columns (rows [col0, col0 + cols) of lm_w) are computed, into
        the same columns of the shared [B, V] buffer, which is returned."""
        ws = self.ws
        vs = self.vocab_slice()
        if vs is None:
            K.gemm(ws.xl, lm_w, ws.logits, K.MUK_EPI_F32, M=B)
        else:
            c0, n = vs
            K.gemm(ws.xl, lm_w[c0:c0 + n], ws.logits[:, c0:c0 + n], K.MUK_EPI_F32, M=B)
        return ws.logits[:B]

    def forward_step(self, batch, cache) -> torch.Tensor:
        raise NotImplementedError

    # ---- reference-style helpers ------------------------------------------------
    def get_memory_footprint(self) -> Dict[str, float]:
        tot = sum(t.numel() * t.element_size() for t in self.weight_tensors())
        return {"total_mb": tot / 2**20}

    def weight_tensors(self) -> List[torch.Tensor]:
        return []

    def num_parameters(self) -> int:
        return sum(t.numel() for t in self.weight_tensors())
