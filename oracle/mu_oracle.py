"""Numpy restatement of the reference forward step (TEST INFRASTRUCTURE ONLY).

Every function cites the reference code it restates (paths inside the
Complexity-ML/complexity-inference project).  Arithmetic is float32 like the
reference's fp32 path; matrices use the reference's own layouts
(nn.Linear weight = [out, in]; token-routed experts = [E, H, 2I] / [E, I, H]).
Nothing in the product package imports this module.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np

F32 = np.float32


def round_bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.astype(np.uint32).view(F32)


def _ident(x):
    return x

__all__ = [
    "MuCfg", "ModelShape", "mu_clamp", "soft_clamp", "rmsnorm", "rope_tables", "apply_rope",
    "sdpa", "OracleModel", "PagedAllocatorOracle", "prepare_logits", "route_experts",
    "inl_dynamics", "greedy_generate", "teacher_forced_logits", "round_bf16",
]


# ---------------------------------------------------------------------------
# mu dynamics — mu_inference/core/mu.py:30-107
# ---------------------------------------------------------------------------
@dataclass
class MuCfg:
    enabled: bool = False
    mu: float = 0.0
    clamp_min: float = -10.0
    clamp_max: float = 10.0


def soft_clamp(x, min_val: float, max_val: float):
    """tanh((x - c) / r) * r + c with c, r the centre and half-range (mu.py:30-68)."""
    if max_val <= min_val:
        return np.full_like(np.asarray(x, dtype=F32), (max_val + min_val) / 2)
    r = F32((max_val - min_val) * 0.5)
    c = F32((max_val + min_val) * 0.5)
    return (np.tanh((np.asarray(x, dtype=F32) - c) / r) * r + c).astype(F32)


def mu_clamp(x, mu: float = 0.0, clamp_min: float = -10.0, clamp_max: float = 10.0):
    """mu + soft_clamp(x - mu) (mu.py:71-107)."""
    x = np.asarray(x, dtype=F32)
    return (F32(mu) + soft_clamp(x - F32(mu), clamp_min, clamp_max)).astype(F32)


def _clamp(x, cfg: MuCfg):
    return mu_clamp(x, cfg.mu, cfg.clamp_min, cfg.clamp_max) if cfg.enabled else x


# ---------------------------------------------------------------------------
# layers — mu_inference/models/layers.py
# ---------------------------------------------------------------------------
def rmsnorm(x, w, eps: float, cfg: Optional[MuCfg] = None):
    """MuRMSNorm.forward (layers.py:149-164); nn.RMSNorm for QK-norm (cfg=None)."""
    x = x.astype(F32)
    var = np.mean(x * x, axis=-1, keepdims=True)
    y = (w.astype(F32) * (x / np.sqrt(var + F32(eps)))).astype(F32)
    return _clamp(y, cfg) if cfg is not None else y


def rope_tables(head_dim: int, theta: float, n: int):
    """RotaryEmbeddingCompat cos/sin (layers.py:286-299), halves only: [n, D/2]."""
    inv = (1.0 / (F32(theta) ** (np.arange(0, head_dim, 2, dtype=F32) / F32(head_dim)))).astype(F32)
    t = np.arange(n, dtype=F32)
    f = np.outer(t, inv).astype(F32)
    return np.cos(f).astype(F32), np.sin(f).astype(F32)


def apply_rope(x, cos, sin, pos):
    """x·cos + rotate_half(x)·sin with rotate_half = cat(-x2, x1) (layers.py:323-387).

    x: [S, H, D]; pos: [S] absolute positions."""
    D = x.shape[-1]
    c = np.concatenate([cos[pos], cos[pos]], -1)[:, None, :]
    s = np.concatenate([sin[pos], sin[pos]], -1)[:, None, :]
    rot = np.concatenate([-x[..., D // 2:], x[..., : D // 2]], -1)
    return (x * c + rot * s).astype(F32)


def sdpa(q, k, v, causal: bool, round_p=_ident):
    """GQA via repeat_interleave + scaled dot-product attention (layers.py:706-723).

    q [Hq, Sq, D], k/v [Hkv, Sk, D].  ``causal`` is the reference rule
    is_causal = (q_len == k_len); with q_len < k_len nothing is masked.
    ``round_p`` (bf16 emulation only) rounds the unnormalised probabilities
    before P·V while their sum stays float32."""
    Hq, Sq, D = q.shape
    G = Hq // k.shape[0]
    k = np.repeat(k, G, axis=0)
    v = np.repeat(v, G, axis=0)
    Sk = k.shape[1]
    mask = np.tril(np.ones((Sq, Sk), dtype=bool)) if causal else None
    out = np.empty((Hq, Sq, v.shape[2]), dtype=F32)
    step = max(1, (1 << 26) // max(1, Sq * Sk))  # heads per chunk: ~256 MB of scores
    for h0 in range(0, Hq, step):  # per-head math; chunks only bound host memory
        hs = slice(h0, min(Hq, h0 + step))
        s = np.matmul(q[hs], k[hs].transpose(0, 2, 1)).astype(F32) / F32(np.sqrt(D))
        if causal:
            s = np.where(mask[None], s, -np.inf)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        if round_p is _ident:
            p = p / p.sum(-1, keepdims=True)
            out[hs] = np.matmul(p.astype(F32), v[hs])
        else:
            out[hs] = np.matmul(round_p(p), v[hs]) / p.sum(-1, keepdims=True)
    return out


def _silu(x):
    return (x / (F32(1) + np.exp(-x))).astype(F32)


def _sigmoid(x):
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def _softplus(x):
    # torch.nn.functional.softplus, beta=1, threshold=20
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(F32)


def inl_dynamics(h, v, p: Dict[str, np.ndarray], prefix: str, dt: float, R=_ident):
    """INLDynamics.forward (layers.py:81-127).  Returns h_next, v_next, mu_contextual.

    ``R`` (bf16 emulation only) rounds the matmul inputs: [h, v] and the
    controller's hidden layer, and h before mu_proj."""
    H = h.shape[-1]
    if v is None:
        v = np.zeros_like(h)
    hv = np.concatenate([R(h), R(v)], -1)
    ch = R(_silu(hv @ p[prefix + "controller_in.weight"].T + p[prefix + "controller_in.bias"]))
    co = (ch @ p[prefix + "controller_out.weight"].T + p[prefix + "controller_out.bias"]).astype(F32)
    alpha = _sigmoid(co[:, :H])
    beta = np.minimum(_softplus(co[:, H:2 * H]), F32(2.0))
    gate = _sigmoid(co[:, 2 * H:])
    mu_c = (p[prefix + "mu"] + R(h) @ p[prefix + "mu_proj.weight"].T).astype(F32)
    v_next = np.clip(alpha * v - beta * (h - mu_c), -10.0, 10.0).astype(F32)
    h_next = (h + F32(dt) * gate * v_next).astype(F32)
    return h_next, v_next, mu_c


def route_experts(token_ids, mu, router_w, num_experts: int, vocab: int):
    """MuTokenRoutedMLP routing (layers.py:504-528): id % E, mu-guided argmax."""
    ids = np.clip(np.asarray(token_ids), 0, vocab - 1)
    base = ids % num_experts
    if mu is None:
        return base.astype(np.int64)
    logits = np.eye(num_experts, dtype=F32)[base] * F32(10.0) + (mu @ router_w.T).astype(F32)
    return np.argmax(logits, -1).astype(np.int64)


# ---------------------------------------------------------------------------
# models — mu_inference/models/llama.py and deep.py
# ---------------------------------------------------------------------------
@dataclass
class ModelShape:
    arch: str                 # "llama" | "deep"
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-6
    theta: float = 10000.0
    experts: int = 0
    qk_norm: bool = False
    tie: bool = True
    dt: float = 0.1
    max_pos: int = 2048


class OracleModel:
    """Per-request forward with a dense per-layer KV cache, as the reference runs it.

    ``forward(ids, past)`` restates LlamaForCausalLM.forward (llama.py:184-245)
    or DeepForCausalLM.forward (deep.py:232-333): returns the last-token
    logits and the grown cache.  past is a list of (K, V) [Hkv, P, D] or None.
    """

    def __init__(self, shape: ModelShape, params: Dict[str, np.ndarray], mu: MuCfg,
                 bf16_activations: bool = False):
        """``bf16_activations``: emulate a bf16 engine (not the reference):
        round to bfloat16 every value such an engine stores as bf16 between
        its f32-accumulating matmuls (matmul inputs, q/k after RoPE and v as
        cached, attention probabilities before P·V, the attention output,
        the final norm).  The residual stream and all accumulations stay
        float32.  Used by tests to measure the rounding floor of bf16
        activations at a given width."""
        self.R = round_bf16 if bf16_activations else _ident
        self.s = shape
        # set to a list to record each routed layer's expert ids per forward
        self.expert_trace: Optional[List[np.ndarray]] = None
        self.p = {k: np.asarray(v, dtype=F32) for k, v in params.items()}
        self.mu = mu
        self.cos, self.sin = rope_tables(shape.head_dim, shape.theta, max(shape.max_pos, 8192))
        if shape.tie or "lm_head.weight" not in self.p:
            self.p["lm_head.weight"] = self.p["embed_tokens.weight"]

    def _attention(self, l, x, segs, pasts, mu_prev):
        """Attention of every request's rows: x [T, H] holds the requests'
        new tokens back to back (segs = (start, length) per request), pasts
        their caches.  Projections are row-wise, so they run on all rows at
        once; RoPE positions and SDPA are per request (layers.py:626-741)."""
        s, p, R = self.s, self.p, self.R
        pre = f"layers.{l}.self_attn."
        T = x.shape[0]
        x = R(x)
        if mu_prev is not None:
            mu_prev = R(mu_prev)
        k = x @ p[pre + "k_proj.weight"].T
        q = x @ p[pre + "q_proj.weight"].T
        v = x @ p[pre + "v_proj.weight"].T
        if mu_prev is not None:  # layers.py:666-669
            k = k + mu_prev @ p[pre + "mu_to_k.weight"].T
            q = q + mu_prev @ p[pre + "mu_to_q.weight"].T
            v = v + mu_prev @ p[pre + "mu_to_v.weight"].T
        q = q.reshape(T, s.heads, s.head_dim).astype(F32)
        k = k.reshape(T, s.kv_heads, s.head_dim).astype(F32)
        v = v.reshape(T, s.kv_heads, s.head_dim).astype(F32)
        if s.qk_norm:  # layers.py:677-679
            q = rmsnorm(q, p[pre + "q_norm.weight"], 1e-6)
            k = rmsnorm(k, p[pre + "k_norm.weight"], 1e-6)
        o = np.empty((T, s.heads * s.head_dim), dtype=F32)
        kvs = []
        for (a, S), past in zip(segs, pasts):
            past_len = 0 if past is None else past[0].shape[1]
            pos = np.arange(past_len, past_len + S)
            qr = R(apply_rope(q[a:a + S], self.cos, self.sin, pos))
            kr = R(apply_rope(k[a:a + S], self.cos, self.sin, pos))
            K = kr.transpose(1, 0, 2)
            V = R(v[a:a + S]).transpose(1, 0, 2)
            if past is not None:
                K = np.concatenate([past[0], K], 1)
                V = np.concatenate([past[1], V], 1)
            orow = sdpa(qr.transpose(1, 0, 2), K, V, causal=(S == K.shape[1]), round_p=R)
            o[a:a + S] = R(orow.transpose(1, 0, 2).reshape(S, -1))
            kvs.append((K, V))
        out = _clamp((o @ p[pre + "o_proj.weight"].T).astype(F32), self.mu)
        return out, kvs

    def _mlp(self, l, x, token_ids, mu_cur):
        s, p = self.s, self.p
        pre = f"layers.{l}.mlp."
        if s.arch == "deep" and s.experts and s.experts > 1:
            e = route_experts(token_ids, mu_cur, p[pre + "mu_router.weight"], s.experts, s.vocab)
            if self.expert_trace is not None:
                self.expert_trace.append(e.copy())
            gu_w = p[pre + "gate_up_proj"]
            d_w = p[pre + "down_proj"]
            I = d_w.shape[1]
            out = np.empty_like(x)
            # layers.py:534-547 gathers each token's expert weights and runs a
            # per-token bmm; tokens are independent, so the rows of one
            # expert are computed together here (same products, one matmul)
            xr = self.R(x)
            for ex in np.unique(e):
                rows = np.nonzero(e == ex)[0]
                gu = xr[rows] @ gu_w[ex]
                inter = self.R(_silu(gu[:, :I]) * gu[:, I:])
                out[rows] = inter @ d_w[ex]
            return _clamp(out.astype(F32), self.mu)
        xr = self.R(x)
        gate = _silu(xr @ p[pre + "gate_proj.weight"].T)
        up = xr @ p[pre + "up_proj.weight"].T
        act = self.R(gate * up)
        return _clamp((act @ p[pre + "down_proj.weight"].T).astype(F32), self.mu)

    def forward(self, ids: Sequence[int], past=None, return_hidden: bool = False):
        """One request: last-token logits [V] and its grown cache."""
        logits, pasts, hn = self.forward_batch([ids], [past])
        if return_hidden:
            return logits[0], pasts[0], hn
        return logits[0], pasts[0]

    def forward_batch(self, ids_list: Sequence[Sequence[int]], past_list=None):
        """Several requests at once, each with its own new tokens and cache.

        Every request's rows get exactly the per-request math of the
        reference's batch-1 forward (all matmuls, norms, INL, routing and the
        MLP act row by row; attention and RoPE positions per request).
        Returns (last-token logits [R, V], new caches, final-norm rows)."""
        s, p, mu = self.s, self.p, self.mu
        if past_list is None:
            past_list = [None] * len(ids_list)
        seqs = [np.asarray(i, dtype=np.int64).reshape(-1) for i in ids_list]
        segs, a = [], 0
        for q in seqs:
            segs.append((a, len(q)))
            a += len(q)
        ids = np.concatenate(seqs)
        h = _clamp(p["embed_tokens.weight"][ids].astype(F32), mu)
        new_past = [[] for _ in seqs]
        v_state, mu_prev = None, None
        for l in range(s.layers):
            pre = f"layers.{l}."
            res = h
            x = rmsnorm(h, p[pre + "input_layernorm.weight"], s.eps, mu)
            attn, kvs = self._attention(l, x, segs,
                                        [None if pp is None else pp[l] for pp in past_list],
                                        mu_prev if s.arch == "deep" else None)
            for r, kv in enumerate(kvs):
                new_past[r].append(kv)
            if s.arch == "deep":  # deep.py:151-176
                h_next, v_state, mu_cur = inl_dynamics(attn, v_state, p, pre + "dynamics.", s.dt,
                                                       self.R)
                h = res + h_next
                res = h
                x2 = rmsnorm(h, p[pre + "post_attention_layernorm.weight"], s.eps, mu)
                h = res + self._mlp(l, x2, ids, mu_cur)
                h = _clamp(h, mu)
                mu_prev = mu_cur
            else:  # llama.py:100-128
                h = res + attn
                res = h
                x2 = rmsnorm(h, p[pre + "post_attention_layernorm.weight"], s.eps, mu)
                h = _clamp(res + self._mlp(l, x2, ids, None), mu)
        hn = rmsnorm(h, p["norm.weight"], s.eps, mu)
        last = np.array([a + n - 1 for a, n in segs])
        logits = (self.R(hn[last]) @ p["lm_head.weight"].T).astype(F32)
        return logits, new_past, hn


def greedy_generate(model: OracleModel, prompt: Sequence[int], n: int):
    """Prefill then n-1 decode steps with fp32 argmax (the MuEngine loop,
    mu_inference/serving/engine.py:188-237, with greedy selection)."""
    logits, past = model.forward(prompt)
    toks, all_logits = [], []
    for i in range(n):
        all_logits.append(logits)
        t = int(np.argmax(logits))
        toks.append(t)
        if i + 1 < n:
            logits, past = model.forward([t], past)
    return toks, np.stack(all_logits)


def teacher_forced_logits(model: OracleModel, prompt: Sequence[int], forced: Sequence[int]):
    """Logits at every step when the generated tokens are forced to ``forced``."""
    logits, past = model.forward(prompt)
    out = [logits]
    for t in forced[:-1]:
        logits, past = model.forward([t], past)
        out.append(logits)
    return np.stack(out)


# ---------------------------------------------------------------------------
# paged allocator — mu_inference/core/cache.py:257-462 (MuPagedCache)
# ---------------------------------------------------------------------------
class PagedAllocatorOracle:
    """Block bookkeeping of MuPagedCache: LIFO free list ``list(range(N))``
    popped from the end (cache.py:301, 317), one block taken at allocate
    (cache.py:311-320), a new block only when the next token arrives with
    pos == block_size (cache.py:360-367), free() extends the free list in
    table order (cache.py:424-429).  ``append(rid, n)`` is one layer-0
    append of n tokens and returns their slots (block*bs + offset)."""

    def __init__(self, num_blocks: int, block_size: int = 16):
        self.bs = block_size
        self.n = num_blocks
        self.free_blocks: List[int] = list(range(num_blocks))
        self.blocks: Dict[str, List[int]] = {}
        self.pos: Dict[str, int] = {}

    def allocate(self, rid: str) -> bool:
        if not self.free_blocks:
            return False
        self.blocks[rid] = [self.free_blocks.pop()]
        self.pos[rid] = 0
        return True

    def append(self, rid: str, n: int) -> Optional[List[int]]:
        if rid not in self.blocks:
            return None
        blocks, pos = self.blocks[rid], self.pos[rid]
        slots = []
        for _ in range(n):
            if pos >= self.bs:
                if not self.free_blocks:
                    self.pos[rid] = pos
                    return None
                blocks.append(self.free_blocks.pop())
                pos = 0
            slots.append(blocks[-1] * self.bs + pos)
            pos += 1
        self.pos[rid] = pos
        return slots

    def seq_len(self, rid: str) -> int:
        b = self.blocks.get(rid)
        return 0 if not b else (len(b) - 1) * self.bs + self.pos[rid]

    def free(self, rid: str) -> None:
        self.free_blocks.extend(self.blocks.pop(rid, []))
        self.pos.pop(rid, None)


# ---------------------------------------------------------------------------
# sampling — mu_inference/utils/sampling.py:20-87
# ---------------------------------------------------------------------------
def prepare_logits(logits, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0,
                   past_tokens=None):
    """Processed logits for one row [V] (the reference works on [1, V])."""
    x = np.array(logits, dtype=F32, copy=True)
    V = x.shape[-1]
    if repetition_penalty != 1.0 and past_tokens:
        for t in set(past_tokens):
            if t < V:
                x[t] = x[t] / F32(repetition_penalty) if x[t] > 0 else x[t] * F32(repetition_penalty)
    if temperature != 1.0:
        x = (x / F32(max(temperature, 1e-8))).astype(F32)
    if 0 < top_k < V:
        kth = np.sort(x)[::-1][top_k - 1]
        x = np.where(x < kth, F32(-np.inf), x).astype(F32)
    if top_p < 1.0:
        order = np.argsort(-x, kind="stable")
        sx = x[order]
        e = np.exp(sx - sx.max())
        # torch.cumsum on a CPU float tensor accumulates in double and stores
        # float; a float32 running sum drifts by ~1e-5 over 1e5 tokens
        cum = np.cumsum((e / e.sum()).astype(F32), dtype=np.float64).astype(F32)
        remove = cum > top_p
        remove[1:] = remove[:-1].copy()
        remove[0] = False
        x[order[remove]] = -np.inf
    return x
