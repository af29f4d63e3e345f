"""Torch-facing wrappers over the libmuk C ABI.

Each wrapper checks dtypes/devices/contiguity, then passes raw device
pointers and the current CUDA stream to the matching ``muk_*`` entry point.
PyTorch only provides memory and streams here; all arithmetic runs in the
sm_100a kernels.  Errors surface as :class:`mu_b200._lib.MukError`.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import MUK_EPI_BF16, MUK_EPI_BIAS_SILU, MUK_EPI_F32, MUK_EPI_ROPE_KV, MUK_EPI_SWIGLU, call

__all__ = [
    "Clamp", "MUK_EPI_BF16", "MUK_EPI_F32", "MUK_EPI_SWIGLU", "MUK_EPI_BIAS_SILU",
    "embed", "residual_rmsnorm", "rmsnorm_rows", "rope_kv_append", "decode_attn_workspace_size",
    "decode_attn", "prefill_attn", "gemm", "grouped_gemm", "route_permute", "gather_rows",
    "inl_dynamics", "reduce_clamp", "sample", "mark_seen", "fill_decode_inputs", "gemm_plan_info",
    "gemm_set_stream_k", "gemm_qkv_rope",
]


@dataclass(frozen=True)
class Clamp:
    """mu_clamp parameters (mu_inference/core/config.py:25-65, MuConfig)."""

    enabled: bool = False
    mu: float = 0.0
    clamp_min: float = -10.0
    clamp_max: float = 10.0

    @classmethod
    def from_mu_config(cls, cfg) -> "Clamp":
        if cfg is None:
            return cls()
        return cls(bool(cfg.enabled), float(cfg.mu), float(cfg.clamp_min), float(cfg.clamp_max))


NO_CLAMP = Clamp()


def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name}: must be a CUDA tensor")


def _row_stride(t: torch.Tensor, name: str) -> int:
    if t.dim() < 2 or t.stride(-1) != 1:
        raise ValueError(f"{name}: last dimension must be contiguous")
    return t.stride(-2)


# ---------------------------------------------------------------------------
def embed(ids: torch.Tensor, table: torch.Tensor, resid: torch.Tensor, clamp: Clamp = NO_CLAMP):
    _check(ids, torch.int32, "ids")
    _check(table, torch.bfloat16, "table")
    _check(resid, torch.float32, "resid")
    T, H = resid.shape
    call("muk_embed", _p(ids), _p(table), _row_stride(table, "table"), _p(resid), T, H,
         table.shape[0], int(clamp.enabled), clamp.mu, clamp.clamp_min, clamp.clamp_max, _stream())


def residual_rmsnorm(resid: torch.Tensor, partials: torch.Tensor | None, norm_w: torch.Tensor | None,
                     eps: float, out: torch.Tensor | None, *, clamp: Clamp = NO_CLAMP,
                     clamp_delta: bool = False, clamp_sum: bool = False, clamp_norm: bool = False,
                     delta_rows: torch.Tensor | None = None):
    """resid += mu_clamp?(Σ partials); out = mu_clamp?(RMSNorm(resid)).

    ``partials`` is [P, rows, H] (or [rows, H]) f32, or one [rows, H] bf16
    slice; ``delta_rows`` optionally gathers partial rows per token."""
    _check(resid, torch.float32, "resid")
    T, H = resid.shape
    en = clamp.enabled
    if partials is not None and partials.dtype == torch.bfloat16:
        ostride = 0 if out is None else _row_stride(out, "out")
        call("muk_residual_rmsnorm_bf16", _p(resid), _p(partials), _row_stride(partials, "partials"),
             _p(delta_rows), _p(norm_w), eps, _p(out), ostride, T, H, int(en and clamp_delta),
             int(en and clamp_sum), int(en and clamp_norm), clamp.mu, clamp.clamp_min,
             clamp.clamp_max, _stream())
        return
    np_, pstride, prow = 0, 0, 0
    if partials is not None:
        _check(partials, torch.float32, "partials")
        if partials.dim() == 2:
            partials = partials.unsqueeze(0)
        np_ = partials.shape[0]
        pstride = partials.stride(0)
        prow = partials.stride(1)
    ostride = 0
    if out is not None:
        _check(out, torch.bfloat16, "out")
        ostride = _row_stride(out, "out")
    call("muk_residual_rmsnorm", _p(resid), _p(partials), pstride, prow, np_, _p(delta_rows),
         _p(norm_w), eps, _p(out), ostride, T, H, int(en and clamp_delta), int(en and clamp_sum),
         int(en and clamp_norm), clamp.mu, clamp.clamp_min, clamp.clamp_max, _stream())


def rmsnorm_rows(resid: torch.Tensor, rows: torch.Tensor, norm_w: torch.Tensor, eps: float,
                 out: torch.Tensor, clamp: Clamp = NO_CLAMP):
    _check(resid, torch.float32, "resid")
    _check(out, torch.bfloat16, "out")
    H = resid.shape[1]
    call("muk_rmsnorm_rows", _p(resid), _p(rows), rows.numel(), _p(norm_w), eps, _p(out),
         _row_stride(out, "out"), H, int(clamp.enabled), clamp.mu, clamp.clamp_min,
         clamp.clamp_max, _stream())


def rope_kv_append(qkv: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                   rope_cos: torch.Tensor, rope_sin: torch.Tensor, num_q_heads: int,
                   num_kv_heads: int, head_dim: int, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                   qk_eps: float = 1e-6, num_tokens: int | None = None):
    _check(qkv, torch.bfloat16, "qkv")
    _check(k_cache, torch.bfloat16, "k_cache")
    T = qkv.shape[0] if num_tokens is None else num_tokens
    num_blocks, _, block_size, _ = k_cache.shape
    call("muk_rope_kv_append", _p(qkv), _row_stride(qkv, "qkv"), _p(positions), _p(slot_mapping),
         _p(rope_cos), _p(rope_sin), rope_cos.shape[0], T, num_q_heads, num_kv_heads, head_dim,
         _p(q_norm_w), _p(k_norm_w), qk_eps, _p(k_cache), _p(v_cache), num_blocks, block_size,
         _stream())


def decode_attn_workspace_size(num_seqs: int, num_q_heads: int, head_dim: int, max_seq_len: int,
                               block_size: int = 16) -> int:
    return int(_lib.load().muk_decode_attn_workspace_size(num_seqs, num_q_heads, head_dim,
                                                          max_seq_len, block_size))


def decode_attn(q: torch.Tensor, out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                block_tables: torch.Tensor, seq_lens: torch.Tensor, num_q_heads: int,
                num_kv_heads: int, head_dim: int, max_seq_len: int,
                workspace: torch.Tensor | None = None, scale: float | None = None,
                num_seqs: int | None = None):
    """Paged decode attention; q/out rows are [num_seqs, Hq*D] (row strides honoured)."""
    _check(q, torch.bfloat16, "q")
    _check(out, torch.bfloat16, "out")
    B = seq_lens.numel() if num_seqs is None else num_seqs
    num_blocks, _, block_size, _ = k_cache.shape
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    call("muk_paged_decode_attn", _p(q), _row_stride(q, "q"), _p(out), _row_stride(out, "out"),
         _p(k_cache), _p(v_cache), _p(block_tables), block_tables.stride(0), _p(seq_lens), B,
         num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, scale, max_seq_len,
         _p(workspace), ws_bytes, _stream())


def prefill_attn(q: torch.Tensor, out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 block_tables: torch.Tensor, seq_lens: torch.Tensor, cu_seqlens_q: torch.Tensor,
                 max_q_len: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 scale: float | None = None, num_seqs: int | None = None):
    _check(q, torch.bfloat16, "q")
    _check(out, torch.bfloat16, "out")
    B = seq_lens.numel() if num_seqs is None else num_seqs
    num_blocks, _, block_size, _ = k_cache.shape
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    call("muk_paged_prefill_attn", _p(q), _row_stride(q, "q"), _p(out), _row_stride(out, "out"),
         _p(k_cache), _p(v_cache), _p(block_tables), block_tables.stride(0), _p(seq_lens),
         _p(cu_seqlens_q), B, max_q_len, num_q_heads, num_kv_heads, head_dim, block_size,
         num_blocks, scale, _stream())


def gemm(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, epilogue: int = MUK_EPI_BF16,
         split_k: int = 1, bias: torch.Tensor | None = None, M: int | None = None):
    """C = epilogue(A · Bᵀ).  A [M, K] bf16, B [N, K] bf16 (nn.Linear layout)."""
    _check(A, torch.bfloat16, "A")
    _check(B, torch.bfloat16, "B")
    M = A.shape[0] if M is None else M
    N, K = B.shape[0], A.shape[1]
    if B.shape[1] != K:
        raise ValueError(f"gemm: K mismatch A{tuple(A.shape)} B{tuple(B.shape)}")
    ldc = C.stride(-2)
    args = ("muk_gemm_bf16", _p(A), _row_stride(A, "A"), _p(B), _row_stride(B, "B"), _p(C), ldc, M,
            N, K, epilogue, split_k, _p(bias), _stream())
    if gemm_probe is None:
        call(*args)
    else:
        with gemm_probe(2.0 * M * N * K):
            call(*args)


# Optional timing hook: a callable(flops) -> context manager wrapped around
# every muk_gemm_bf16 launch (the benchmark uses it to time each launch with
# CUDA events on the launching stream).
gemm_probe = None


def grouped_gemm(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, expert_offsets: torch.Tensor,
                 num_experts: int, N: int, epilogue: int, max_rows: int | None = None):
    """Rows of A in expert order times expert weights B [E*N, K]."""
    _check(A, torch.bfloat16, "A")
    _check(B, torch.bfloat16, "B")
    K = A.shape[1]
    max_rows = A.shape[0] if max_rows is None else max_rows
    call("muk_grouped_gemm_bf16", _p(A), _row_stride(A, "A"), _p(B), _row_stride(B, "B"), _p(C),
         C.stride(-2), _p(expert_offsets), num_experts, max_rows, N, K, epilogue, _stream())


def route_permute(expert_ids: torch.Tensor, num_experts: int, offsets: torch.Tensor,
                  perm: torch.Tensor, inv_perm: torch.Tensor, num_tokens: int | None = None):
    T = expert_ids.numel() if num_tokens is None else num_tokens
    call("muk_route_permute", _p(expert_ids), T, num_experts, _p(offsets), _p(perm),
         _p(inv_perm), _stream())


def gather_rows(src: torch.Tensor, rows: torch.Tensor, dst: torch.Tensor, num_rows: int | None = None):
    n = rows.numel() if num_rows is None else num_rows
    call("muk_gather_rows_bf16", _p(src), _row_stride(src, "src"), _p(rows), n, _p(dst),
         _row_stride(dst, "dst"), src.shape[1], _stream())


def reduce_bias_silu(partials: torch.Tensor, bias: torch.Tensor, out: torch.Tensor,
                     num_rows: int | None = None):
    """out = bf16(silu(sum of the [S, T, N] f32 partials + bias))."""
    if partials.dim() == 2:
        partials = partials.unsqueeze(0)
    T = out.shape[0] if num_rows is None else num_rows
    N = out.shape[1]
    call("muk_reduce_bias_silu", _p(partials), partials.stride(0), partials.shape[0], _p(bias),
         _p(out), _row_stride(out, "out"), T, N, _stream())


def reduce_clamp(partials: torch.Tensor, dst: torch.Tensor, dst_bf16: torch.Tensor | None,
                 clamp: Clamp = NO_CLAMP, num_tokens: int | None = None):
    if partials.dim() == 2:
        partials = partials.unsqueeze(0)
    T = dst.shape[0] if num_tokens is None else num_tokens
    H = dst.shape[1]
    call("muk_reduce_clamp", _p(partials), partials.stride(0), partials.shape[0], _p(dst),
         _p(dst_bf16), 0 if dst_bf16 is None else _row_stride(dst_bf16, "dst_bf16"), T, H,
         int(clamp.enabled), clamp.mu, clamp.clamp_min, clamp.clamp_max, _stream())


def inl_dynamics(h, ctrl_raw, ctrl_bias, muproj, mu_param, dt, v, v_bf16, resid, mu_out, norm_w,
                 eps, norm_out, token_ids=None, router_w=None, num_experts=0, vocab=0,
                 expert_ids=None, clamp: Clamp = NO_CLAMP, num_tokens: int | None = None,
                 v_zero: bool = False):
    """v_zero: read the incoming velocity as zero (the first layer) instead of v."""
    T = h.shape[0] if num_tokens is None else num_tokens
    H = h.shape[1]
    call("muk_inl_dynamics", _p(h), _p(ctrl_raw), _p(ctrl_bias), _p(muproj), _p(mu_param), dt,
         _p(v), int(v_zero), _p(v_bf16), 0 if v_bf16 is None else _row_stride(v_bf16, "v_bf16"), _p(resid),
         _p(mu_out), 0 if mu_out is None else _row_stride(mu_out, "mu_out"), _p(norm_w), eps,
         _p(norm_out), 0 if norm_out is None else _row_stride(norm_out, "norm_out"), _p(token_ids),
         _p(router_w), num_experts, vocab, _p(expert_ids), T, H, int(clamp.enabled), clamp.mu,
         clamp.clamp_min, clamp.clamp_max, _stream())


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
           top_p: torch.Tensor, rep_penalty: torch.Tensor, seen_bits: torch.Tensor | None,
           seeds: torch.Tensor, offsets: torch.Tensor, out: torch.Tensor, num_rows: int | None = None,
           seen_rows: torch.Tensor | None = None):
    """One token per logits row; bitmap row of row b is seen_bits[seen_rows[b]] (or b)."""
    _check(logits, torch.float32, "logits")
    B = logits.shape[0] if num_rows is None else num_rows
    V = logits.shape[1]
    call("muk_sample", _p(logits), _row_stride(logits, "logits"), B, V, _p(temperature), _p(top_k),
         _p(top_p), _p(rep_penalty), _p(seen_bits), 0 if seen_bits is None else seen_bits.stride(0),
         _p(seen_rows), _p(seeds), _p(offsets), _p(out), _stream())


def prepare_logits(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                   top_p: torch.Tensor, rep_penalty: torch.Tensor, seen_bits: torch.Tensor | None,
                   out: torch.Tensor, seen_rows: torch.Tensor | None = None):
    """prepare_logits per row (mu_inference/utils/sampling.py:20-87): out gets the
    penalised, temperature-scaled logits where kept and -inf where removed."""
    _check(logits, torch.float32, "logits")
    _check(out, torch.float32, "out")
    B, V = logits.shape
    call("muk_prepare_logits", _p(logits), _row_stride(logits, "logits"), B, V, _p(temperature),
         _p(top_k), _p(top_p), _p(rep_penalty), _p(seen_bits),
         0 if seen_bits is None else seen_bits.stride(0), _p(seen_rows), _p(out),
         _row_stride(out, "out"), _stream())


def mark_seen(seen_bits: torch.Tensor, rows: torch.Tensor, tokens: torch.Tensor, vocab: int,
              n: int | None = None):
    n = tokens.numel() if n is None else n
    call("muk_mark_seen", _p(seen_bits), seen_bits.stride(0), _p(rows), _p(tokens), n, vocab,
         _stream())


def fill_decode_inputs(input_ids: torch.Tensor, src: torch.Tensor, sampled: torch.Tensor, n: int):
    """input_ids[j] = sampled[src[j]] where src[j] >= 0, for j < n (int32 tensors)."""
    for t, name in ((input_ids, "input_ids"), (src, "src"), (sampled, "sampled")):
        _check(t, torch.int32, name)
    call("muk_fill_decode_inputs", _p(input_ids), _p(src), _p(sampled), n, _stream())


def gemm_plan_info(M: int, N: int, K: int, epilogue: int, split_k: int = 1) -> dict:
    """The launch muk_gemm_bf16 makes for a shape (kernel, tile width, schedule)."""
    import ctypes

    out = (ctypes.c_int32 * 7)()
    lib = _lib.load()
    rc = lib.muk_gemm_plan_info(M, N, K, epilogue, split_k, ctypes.addressof(out))
    if rc != 0:
        raise _lib.MukError("muk_gemm_plan_info", rc, _lib.last_error())
    keys = ("kernel", "bn", "split", "stream_k", "dp_tiles", "sk_tiles", "workers")
    return dict(zip(keys, list(out)))


def set_peer_timeout_ms(ms: int) -> None:
    """Bound of the collectives' cross-GPU waits on the current device."""
    _lib.call_status("muk_set_peer_timeout_ms", int(ms))


def gemm_set_stream_k(mode: int) -> int:
    """GEMM stream-K planning mode (0 off, 1 on, 2 auto = only for launches
    that would leave most SMs idle); returns the previous mode."""
    return int(_lib.load().muk_gemm_set_stream_k(int(mode)))


def gemm_qkv_rope(A: torch.Tensor, B: torch.Tensor, q_out: torch.Tensor, positions: torch.Tensor,
                  slot_mapping: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                  num_q_heads: int, num_kv_heads: int, head_dim: int, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, q_norm_w: torch.Tensor | None = None,
                  k_norm_w: torch.Tensor | None = None, qk_eps: float = 1e-6,
                  M: int | None = None, rownorm: "_lib.MukRowNorm | None" = None):
    """q|k|v projection with RoPE (+QK-norm) and the paged-KV append fused in
    the GEMM epilogue: q heads -> q_out, k/v heads -> the caches.  With
    ``rownorm`` (see :func:`row_norm`) each input row is first scaled by its
    RMSNorm factor from a producer's partial sums."""
    _check(A, torch.bfloat16, "A")
    _check(B, torch.bfloat16, "B")
    _check(k_cache, torch.bfloat16, "k_cache")
    M = A.shape[0] if M is None else M
    K = A.shape[1]
    num_blocks, _, block_size, _ = k_cache.shape
    name = "muk_gemm_qkv_rope" if rownorm is None else "muk_gemm_qkv_rope_rownorm"
    args = (name, _p(A), _row_stride(A, "A"), _p(B), _row_stride(B, "B"),
            _p(q_out), _row_stride(q_out, "q_out"), M, K, _p(positions), _p(slot_mapping),
            _p(rope_cos), _p(rope_sin), rope_cos.shape[0], num_q_heads, num_kv_heads, head_dim,
            _p(q_norm_w), _p(k_norm_w), qk_eps, _p(k_cache), _p(v_cache), num_blocks, block_size) + \
        ((_stream(),) if rownorm is None else (ctypes.byref(rownorm), _stream()))
    if gemm_probe is None:
        call(*args)
    else:
        with gemm_probe(2.0 * M * (num_q_heads + 2 * num_kv_heads) * head_dim * K):
            call(*args)


def row_norm(sumsq: torch.Tensor, hidden: int, eps: float) -> "_lib.MukRowNorm":
    """The consumer side of an RMSNorm split across two GEMMs: ``sumsq``
    [hidden / 128, stride] f32 holds the producer's (:func:`gemm_residual_norm`)
    per-128-column partial sums of r^2 for each row."""
    _check(sumsq, torch.float32, "sumsq")
    if sumsq.dim() != 2 or sumsq.stride(1) != 1 or sumsq.shape[0] != hidden // 128:
        raise ValueError(f"row_norm: sumsq must be [{hidden // 128}, rows], got {tuple(sumsq.shape)}")
    return _lib.MukRowNorm(sumsq.data_ptr(), sumsq.stride(0), sumsq.shape[0], hidden, eps)


def gemm_residual_norm(A: torch.Tensor, B: torch.Tensor, resid: torch.Tensor,
                       norm_w: torch.Tensor | None, x_out: torch.Tensor | None,
                       sumsq: torch.Tensor | None, M: int | None = None):
    """resid[:M] += A · Bᵀ (f32, in place); with ``norm_w``, also
    x_out = bf16(norm_w * resid) and the per-128-column partial sums of
    resid^2 into ``sumsq`` [N / 128, stride] — the first half of the next
    RMSNorm, finished by a consumer GEMM given :func:`row_norm`."""
    _check(A, torch.bfloat16, "A")
    _check(B, torch.bfloat16, "B")
    _check(resid, torch.float32, "resid")
    M = A.shape[0] if M is None else M
    N, K = B.shape[0], A.shape[1]
    if norm_w is not None:
        _check(norm_w, torch.float32, "norm_w")
        _check(x_out, torch.bfloat16, "x_out")
        _check(sumsq, torch.float32, "sumsq")
        if sumsq.dim() != 2 or sumsq.shape[0] != N // 128 or sumsq.shape[1] < M:
            raise ValueError(f"gemm_residual_norm: sumsq must be [{N // 128}, >= {M}]")
    args = ("muk_gemm_residual_norm", _p(A), _row_stride(A, "A"), _p(B), _row_stride(B, "B"), M,
            N, K, _p(resid), _row_stride(resid, "resid"), _p(norm_w), _p(x_out),
            _row_stride(x_out, "x_out") if x_out is not None else 0, _p(sumsq),
            sumsq.stride(0) if sumsq is not None else 0, _stream())
    if gemm_probe is None:
        call(*args)
    else:
        with gemm_probe(2.0 * M * N * K):
            call(*args)


def gemm_clamp_dual(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, C_bf16: torch.Tensor,
                    clamp: Clamp = NO_CLAMP, M: int | None = None):
    """C = mu_clamp?(A · Bᵀ) in f32 and its bf16 copy C_bf16, in one GEMM
    (split-K 1)."""
    _check(A, torch.bfloat16, "A")
    _check(B, torch.bfloat16, "B")
    _check(C, torch.float32, "C")
    _check(C_bf16, torch.bfloat16, "C_bf16")
    M = A.shape[0] if M is None else M
    N, K = B.shape[0], A.shape[1]
    args = ("muk_gemm_clamp_dual", _p(A), _row_stride(A, "A"), _p(B), _row_stride(B, "B"), _p(C),
            _row_stride(C, "C"), _p(C_bf16), _row_stride(C_bf16, "C_bf16"), M, N, K,
            int(clamp.enabled), clamp.mu, clamp.clamp_min, clamp.clamp_max, _stream())
    if gemm_probe is None:
        call(*args)
    else:
        with gemm_probe(2.0 * M * N * K):
            call(*args)


def gemm_swiglu_rownorm(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                        rownorm: "_lib.MukRowNorm | None", M: int | None = None):
    """:func:`gemm` with MUK_EPI_SWIGLU, each input row first scaled by its
    RMSNorm factor (``rownorm`` from :func:`row_norm`; None: unscaled)."""
    _check(A, torch.bfloat16, "A")
    _check(B, torch.bfloat16, "B")
    M = A.shape[0] if M is None else M
    N, K = B.shape[0], A.shape[1]
    args = ("muk_gemm_swiglu_rownorm", _p(A), _row_stride(A, "A"), _p(B), _row_stride(B, "B"),
            _p(C), C.stride(-2), M, N, K, None if rownorm is None else ctypes.byref(rownorm),
            _stream())
    if gemm_probe is None:
        call(*args)
    else:
        with gemm_probe(2.0 * M * N * K):
            call(*args)
