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

from typing import Dict, List, Optional

import torch

from .. import kernels as K
from ..core.config import ModelConfig, MuConfig
from .base import PAD_MULT, MuModelBase, choose_split, interleave_gate_up, pad_cols, pad_to
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

    def act_width(self) -> int:
        return self.i_pad

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
    def forward_step(self, batch, cache) -> torch.Tensor:
        cfg, ws, cl = self.config, self.ws, self.clamp
        T, H, eps = batch.num_tokens, cfg.hidden_size, cfg.rms_norm_eps
        resid, x = ws.resid[:T], ws.x[:T, :H]
        K.embed(batch.input_ids, self.embed, resid, cl)
        K.residual_rmsnorm(resid, None, self.layers[0]["w_in"], eps, x, clamp=cl, clamp_norm=True)
        nl = len(self.layers)
        for l, L in enumerate(self.layers):
            K.gemm(x, L["wqkv"], ws.qkv, K.MUK_EPI_BF16, M=T)
            attn = self.attention(l, batch, cache)
            s = choose_split(T, H, attn.shape[1], ws.part_rows)
            part = ws.part_view(s, T, H)
            K.gemm(attn, L["wo"], part, K.MUK_EPI_F32, split_k=s, M=T)
            part = self.reduce_partials(part)
            # h += clamp(attn_out); x = clamp(norm_post(h))    (llama.py:111-115)
            K.residual_rmsnorm(resid, part, L["w_post"], eps, x, clamp=cl, clamp_delta=True,
                               clamp_norm=True)
            K.gemm(x, L["wgu"], ws.act, K.MUK_EPI_SWIGLU, M=T)
            s = choose_split(T, H, self.i_pad, ws.part_rows)
            part = ws.part_view(s, T, H)
            K.gemm(ws.act, L["wd"], part, K.MUK_EPI_F32, split_k=s, M=T)
            part = self.reduce_partials(part)
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
