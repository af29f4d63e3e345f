"""LlamaForCausalLM (and the Mistral / Qwen2 / Gemma aliases) on libmuk.

Same computation as mu_inference/models/llama.py:38-245 — pre-norm RMSNorm,
GQA attention with rotate-half RoPE, SwiGLU MLP, mu_clamp on the embedding,
every norm output, the attention and MLP outputs and the layer output when
MuConfig.enabled — restated as one flat-batch step per call:

    embed ─▶ [norm] ─▶ QKV GEMM ─▶ RoPE+append ─▶ decode/prefill attention
          ─▶ O GEMM (split-K f32 partials) ─▶ reduce+residual+clamp+norm
          ─▶ gate|up GEMM with SwiGLU epilogue ─▶ down GEMM (split-K)
          ─▶ reduce+residual+clamp+next norm ─▶ ... ─▶ last-row norm ─▶ LM head

Weight layouts prepared at load: q|k|v fused into one [(Hq+2Hkv)·D, H]
matrix; gate and up interleaved in 64-row groups for the SwiGLU epilogue,
intermediate padded with zero rows/columns to a multiple of 64 (exact).
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional

import torch

from .. import _lib
from .. import kernels as K
from ..core.config import ModelConfig, MuConfig
from .base import (FUSED_TP_MAX_ROWS, PAD_MULT, MuModelBase, choose_split, interleave_gate_up,
                   pad_cols, pad_to)
from .registry import register_model


@register_model("llama")
class LlamaForCausalLM(MuModelBase):
    arch = "llama"

    def __init__(self, config: ModelConfig, mu_config: Optional[MuConfig] = None,
                 device: str = "cuda"):
        super().__init__(config, mu_config, device)
        self.i_pad = pad_to(config.intermediate_size, PAD_MULT)
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.embed = None
        self.norm_w = None
        self.lm_w = None
        # whole step issued by libmuk's native executor (muk_llama_forward);
        # MU_NATIVE_STEP=0 keeps the per-kernel Python path
        self.native = os.environ.get("MU_NATIVE_STEP", "1") != "0"
        self._native_key = None
        self._native_model = None
        # RMSNorm split across the projection before it and the GEMM after it,
        # in steps of at least MU_FUSED_NORM_MIN_ROWS tokens (MU_FUSED_NORM=0:
        # separate residual + norm kernels always).  Below that the O / down
        # projections keep split-K, which the fused epilogue cannot use
        # (B200, M 256: 48 us fused vs 36 us split-K + norm; M 857: 44 vs 47).
        self._fused_norm = os.environ.get("MU_FUSED_NORM", "1") != "0"
        self.fused_norm_min_rows = int(os.environ.get("MU_FUSED_NORM_MIN_ROWS", "512"))

    def act_width(self) -> int:
        return self.i_pad

    def extra_workspace(self, ws, T: int) -> None:
        H = self.config.hidden_size
        ws.sumsq = torch.empty(max(H // 128, 1), T, device=self.device, dtype=torch.float32)

    def peer_x_elems(self, max_tokens: int) -> int:
        if os.environ.get("MU_TP_NORM", "1") == "0" or self.config.hidden_size % 8:
            return 0
        return max_tokens * 2 * self.config.hidden_size

    def tp_norm(self) -> bool:
        """Under peer-memory TP: reduce-scatter + residual/RMSNorm on each
        rank's rows + all-gather of x (muk_tp_residual_norm) in place of an
        all-reduce followed by a replicated residual/norm."""
        ws = self.ws
        return (self.tp_group is not None and self.comm is not None and ws is not None
                and ws.shared_part and ws.shared_x)

    def fused_norm(self) -> bool:
        """Residual add + RMSNorm in the O / down projection's epilogue and the
        row scale in the next GEMM: one GPU, no mu_clamp (its clamp of the norm
        output does not commute with the matmul), hidden a multiple of 128,
        RoPE in the q|k|v epilogue."""
        return (self._fused_norm and self.tp_group is None and not self.clamp.enabled
                and self.config.hidden_size % 128 == 0 and self.fused_rope())

    # ---- weights -------------------------------------------------------------
    @classmethod
    def from_state_dict(cls, config: ModelConfig, sd: Dict[str, torch.Tensor],
                        mu_config: Optional[MuConfig] = None, device: str = "cuda"):
        m = cls(config, mu_config, device)
        dev, bf = m.device, torch.bfloat16

        def w(name):
            return sd[name].to(dev, bf).contiguous()

        def f(name):
            return sd[name].to(dev, torch.float32).contiguous()

        m.embed = w("embed_tokens.weight")
        for l in range(config.num_hidden_layers):
            p = f"layers.{l}."
            a = p + "self_attn."
            m.layers.append({
                "w_in": f(p + "input_layernorm.weight"),
                "wqkv": torch.cat([w(a + "q_proj.weight"), w(a + "k_proj.weight"),
                                   w(a + "v_proj.weight")], 0).contiguous(),
                "wo": w(a + "o_proj.weight"),
                "w_post": f(p + "post_attention_layernorm.weight"),
                "wgu": interleave_gate_up(w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight"),
                                          m.i_pad),
                "wd": pad_cols(w(p + "mlp.down_proj.weight"), m.i_pad),
            })
        m.norm_w = f("norm.weight")
        if config.tie_word_embeddings or "lm_head.weight" not in sd:
            m.lm_w = m.embed
        else:
            m.lm_w = w("lm_head.weight")
        return m

    def weight_tensors(self):
        ts = [self.embed, self.norm_w] + ([] if self.lm_w is self.embed else [self.lm_w])
        for L in self.layers:
            ts.extend(L.values())
        return ts

    # ---- step ------------------------------------------------------------------
    def _native_ok(self) -> bool:
        if not self.native:
            return False
        if self.tp_group is None:
            return True
        return self.comm is not None and self.ws.shared_part  # peer all-reduce only

    def _native(self, cache) -> "_lib.MukLlamaModel":
        """The executor's model struct (rebuilt when a buffer moves)."""
        ws, cfg = self.ws, self.config
        key = (id(ws), cache.block_pool.data_ptr(), self.rope_cos.data_ptr(), id(self.comm),
               self.fused_rope(), self._tp_fused, self.fused_norm(), self.fused_norm_min_rows,
               self.tp_norm(), self.vocab_slice())
        if key == self._native_key:
            return self._native_model
        layers = (_lib.MukLlamaLayer * len(self.layers))()
        for i, L in enumerate(self.layers):
            layers[i] = _lib.MukLlamaLayer(L["w_in"].data_ptr(), L["wqkv"].data_ptr(),
                                           L["wo"].data_ptr(), L["w_post"].data_ptr(),
                                           L["wgu"].data_ptr(), L["wd"].data_ptr())
        cl = self.clamp
        m = _lib.MukLlamaModel()
        m.num_layers, m.hidden = len(self.layers), cfg.hidden_size
        m.num_q_heads, m.num_kv_heads = cfg.num_attention_heads, cfg.num_key_value_heads
        m.head_dim, m.inter_pad, m.vocab = cfg.head_dim, self.i_pad, cfg.vocab_size
        m.eps = cfg.rms_norm_eps
        m.clamp, m.mu, m.clamp_min, m.clamp_max = int(cl.enabled), cl.mu, cl.clamp_min, cl.clamp_max
        m.layers = layers
        vs = self.vocab_slice()
        m.embed, m.final_norm = self.embed.data_ptr(), self.norm_w.data_ptr()
        m.lm_head = self.lm_w.data_ptr() + (0 if vs is None else vs[0] * self.lm_w.stride(0) * 2)
        m.rope_cos, m.rope_sin, m.rope_len = (self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
                                              self.rope_cos.shape[0])
        m.kv_pool, m.num_blocks, m.block_size = (cache.block_pool.data_ptr(), cache.max_num_blocks,
                                                 cache.block_size)
        m.resid, m.x, m.x_stride = ws.resid.data_ptr(), ws.x.data_ptr(), ws.x.stride(0)
        m.qkv, m.attn, m.act = ws.qkv.data_ptr(), ws.attn.data_ptr(), ws.act.data_ptr()
        m.part, m.part_rows = ws.part.data_ptr(), ws.part_rows
        m.xl, m.logits = ws.xl.data_ptr(), ws.logits.data_ptr()
        m.lm_rows, m.logits_ld = cfg.vocab_size, ws.logits.stride(0)
        vs = self.vocab_slice()
        if vs is not None:  # this rank's vocabulary columns only
            c0, n = vs
            m.lm_rows = n
            m.logits = ws.logits.data_ptr() + 4 * c0
        m.attn_ws, m.attn_ws_bytes = ws.attn_ws.data_ptr(), ws.attn_ws.numel() * 4
        m.fused_rope = int(self.fused_rope())
        m.tp_fused = FUSED_TP_MAX_ROWS if self._tp_fused else 0
        m.fused_norm = max(1, self.fused_norm_min_rows) if self.fused_norm() else 0
        m.sumsq = ws.sumsq.data_ptr()
        m.tp_norm = int(self.tp_norm())
        m.tp_push_bf16 = int(self.comm.push_bf16) if self.comm is not None else 0
        m.tp_world, m.tp_rank = 1, 0
        if self.comm is not None:
            c = self.comm
            m.tp_world, m.tp_rank = c.world, c.rank
            for r in range(c.world):
                m.ar_data[r], m.ar_scratch[r], m.ar_flags[r] = (c.ptrs[r], c.scratch_ptrs[r],
                                                                 c.flag_ptrs[r])
                m.x_peer[r] = c.x_ptrs[r]
        m._keep = layers  # the layer array must outlive the struct
        self._native_key, self._native_model = key, m
        return m

    def _forward_native(self, batch, cache) -> torch.Tensor:
        m = self._native(cache)
        T, B, nd = batch.num_tokens, batch.num_seqs, batch.num_decode
        b = _lib.MukStepBatch(T, B, nd, batch.max_q_len, batch.decode_len_bound,
                              batch.input_ids.data_ptr(), batch.positions.data_ptr(),
                              batch.slot_mapping.data_ptr(), batch.seq_lens.data_ptr(),
                              batch.prefill_cu.data_ptr(), batch.last_token_idx.data_ptr(),
                              batch.block_tables.data_ptr(), batch.block_tables.stride(0))
        # two all-reduces per layer: fused (GEMM + finish: one extra kernel each)
        # or separate (push + finish: two each)
        attn = (2 if nd > 0 else 0) + (1 if B > nd else 0)
        if m.tp_world > 1 and m.tp_norm:
            # q|k|v (+RoPE), attention, 2 x (projection + finish [+ push]), SwiGLU
            per_layer = (1 if m.fused_rope else 2) + attn + 1 + \
                (4 if (m.tp_fused and T <= m.tp_fused) else 6)
            n = 2 + per_layer * m.num_layers + 2
        else:
            tp = (2 if (m.tp_fused and T <= m.tp_fused) else 4) if m.tp_world > 1 else 0
            fused = m.fused_norm > 0 and T >= m.fused_norm
            per_layer = (4 if fused else 6 if m.fused_rope else 7) + attn + tp
            n = 4 + per_layer * m.num_layers
        _lib.call_counted("muk_llama_forward", n, ctypes.byref(m),
                          ctypes.byref(b), torch.cuda.current_stream().cuda_stream)
        return self.ws.logits[:B]

    def forward_step(self, batch, cache) -> torch.Tensor:
        if self._native_ok():
            return self._forward_native(batch, cache)
        cfg, ws, cl = self.config, self.ws, self.clamp
        T, H, eps = batch.num_tokens, cfg.hidden_size, cfg.rms_norm_eps
        resid, x = ws.resid[:T], ws.x[:T, :H]
        K.embed(batch.input_ids, self.embed, resid, cl)
        K.residual_rmsnorm(resid, None, self.layers[0]["w_in"], eps, x, clamp=cl, clamp_norm=True)
        nl = len(self.layers)
        if self.tp_norm():
            # reduce-scatter + residual/norm on the owned rows + all-gather of x;
            # the residual stays row-sharded and the last layer applies the
            # final norm (the LM head reads each sequence's last row of x)
            c = self.comm
            fused_tp = self._tp_fused and T <= FUSED_TP_MAX_ROWS

            def project_norm(A, W, norm_w, clamp_sum):
                if fused_tp:
                    c.gemm_residual_norm_(A, W, T, resid, norm_w, eps, x, cl, True, clamp_sum,
                                          True)
                    return
                s = choose_split(T, H, A.shape[1], ws.part_rows)
                part = ws.part_view(s, T, H)
                K.gemm(A, W, part, K.MUK_EPI_F32, split_k=s, M=T)
                c.residual_norm_(part, resid, norm_w, eps, x, cl, True, clamp_sum, True)

            for l, L in enumerate(self.layers):
                self.qkv_proj(l, x, L["wqkv"], batch, cache)
                attn = self.attention(l, batch, cache)
                project_norm(attn[:T], L["wo"], L["w_post"], False)
                K.gemm(x, L["wgu"], ws.act, K.MUK_EPI_SWIGLU, M=T)
                last = l + 1 == nl
                project_norm(ws.act[:T], L["wd"],
                             self.norm_w if last else self.layers[l + 1]["w_in"], True)
            B = batch.num_seqs
            K.gather_rows(x, batch.last_token_idx[:B], ws.xl, num_rows=B)
            return self.lm_gemm(self.lm_w, B)
        if self.fused_norm() and T >= max(1, self.fused_norm_min_rows):
            # x holds bf16(w * h); the GEMM that reads it scales each row by
            # rsqrt(mean(h^2) + eps) from the producer's partial sums
            rn = K.row_norm(ws.sumsq, H, eps)
            for l, L in enumerate(self.layers):
                self.qkv_proj(l, x, L["wqkv"], batch, cache, rownorm=rn if l > 0 else None)
                attn = self.attention(l, batch, cache)
                K.gemm_residual_norm(attn[:T], L["wo"], resid, L["w_post"], x, ws.sumsq, M=T)
                K.gemm_swiglu_rownorm(x, L["wgu"], ws.act, rn, M=T)
                last = l + 1 == nl
                K.gemm_residual_norm(ws.act[:T], L["wd"], resid,
                                     None if last else self.layers[l + 1]["w_in"],
                                     None if last else x, None if last else ws.sumsq, M=T)
            return self.lm_head(batch, self.norm_w, self.lm_w)
        for l, L in enumerate(self.layers):
            self.qkv_proj(l, x, L["wqkv"], batch, cache)
            attn = self.attention(l, batch, cache)
            part = self.row_parallel(attn[:T], L["wo"], T, H)
            # h += clamp(attn_out); x = clamp(norm_post(h))    (llama.py:111-115)
            K.residual_rmsnorm(resid, part, L["w_post"], eps, x, clamp=cl, clamp_delta=True,
                               clamp_norm=True)
            K.gemm(x, L["wgu"], ws.act, K.MUK_EPI_SWIGLU, M=T)
            part = self.row_parallel(ws.act[:T], L["wd"], T, H)
            # h = clamp(h + clamp(mlp_out)); x = clamp(norm_in_next(h))   (llama.py:116-126)
            last = l + 1 == nl
            K.residual_rmsnorm(resid, part, None if last else self.layers[l + 1]["w_in"], eps,
                               None if last else x, clamp=cl, clamp_delta=True, clamp_sum=True,
                               clamp_norm=True)
        return self.lm_head(batch, self.norm_w, self.lm_w)


@register_model("mistral")
class MistralForCausalLM(LlamaForCausalLM):
    """Same architecture as Llama (mu_inference/models/llama.py:270-279)."""


@register_model("qwen")
class Qwen2ForCausalLM(LlamaForCausalLM):
    """Same architecture as Llama (mu_inference/models/llama.py:282-289)."""


@register_model("gemma")
class GemmaForCausalLM(LlamaForCausalLM):
    """Same architecture as Llama (mu_inference/models/llama.py:292-299)."""
