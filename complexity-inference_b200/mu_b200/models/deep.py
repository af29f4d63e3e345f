"""DeepForCausalLM (Pacific-Prime) on libmuk: mu-guided attention, INL
dynamics and the token-routed MLP as one flat-batch step.

Restates mu_inference/models/deep.py:36-333 with layers.py:21-127 (INL),
427-559 (token-routed MLP) and 562-741 (mu-guided attention):

    x|mu_prev ─▶ fused [q|k|v ; mu_to_q|k|v] GEMM (K = 2H; H on layer 0)
             ─▶ QK-norm + RoPE + append ─▶ attention ─▶ O GEMM ─▶ clamp
             ─▶ controller_in GEMM (bias+SiLU epilogue) ─▶ controller_out GEMM
             ─▶ mu_proj GEMM ─▶ INL kernel (v', h', residual, mu_c, post-norm,
                mu-guided routing) ─▶ stable sort by expert ─▶ row gather
             ─▶ grouped gate|up GEMM (SwiGLU) ─▶ grouped down GEMM
             ─▶ un-permute + clamp + residual + clamp + next norm

The reference gathers a private copy of the expert weights per token
(layers.py:534-536); here tokens are bucketed per expert so each expert's
weights stream once per step.  Expert weights are transposed at load to
K-major ([E·2I, H] interleaved gate/up, [E·H, I]).
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
from .weights import expert_intermediate, is_routed


@register_model("deep")
class DeepForCausalLM(MuModelBase):
    arch = "deep"

    def __init__(self, config: ModelConfig, mu_config: Optional[MuConfig] = None,
                 device: str = "cuda"):
        super().__init__(config, mu_config, device)
        self.routed = is_routed("deep", config)
        inner = expert_intermediate(config) if self.routed else config.intermediate_size
        self.i_pad = pad_to(inner, PAD_MULT)
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.embed = self.norm_w = self.lm_w = None
        # expert parallelism: this GPU holds experts [expert_lo, expert_lo + local_experts)
        self.local_experts = config.num_experts if self.routed else 0
        self.expert_lo = 0
        # how expert outputs reach every GPU under expert parallelism with the
        # peer-memory collectives: "gather" (each GPU's expert rows in bf16,
        # muk_ep_gather_bf16) or "allreduce" (full-width f32 all-reduce)
        self.ep_combine = os.environ.get("MU_EP_COMBINE", "gather")
        # whole step issued by libmuk's native executor (muk_deep_forward);
        # MU_NATIVE_STEP=0 (or native = False) issues it kernel by kernel
        self.native = os.environ.get("MU_NATIVE_STEP", "1") != "0"
        self._native_key = None
        self._native_model = None

    def act_width(self) -> int:
        return self.i_pad

    def extra_workspace(self, ws, T: int) -> None:
        cfg, dev = self.config, self.device
        H, C = cfg.hidden_size, cfg.dynamics_controller_hidden
        ws.h = torch.empty(T, H, device=dev, dtype=torch.float32)
        ws.hv = torch.zeros(T, 2 * H, device=dev, dtype=torch.bfloat16)
        ws.v = torch.zeros(T, H, device=dev, dtype=torch.float32)
        ws.ch = torch.empty(T, C, device=dev, dtype=torch.bfloat16)
        ws.ctrl = torch.empty(T, 3 * H, device=dev, dtype=torch.float32)
        ws.mp = torch.empty(T, H, device=dev, dtype=torch.float32)
        ws.x2 = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        ws.xs = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        # the expert MLP's output is reduced over TP ranks like the partials:
        # under peer-memory TP it shares their buffer (the O partials are
        # consumed before the down GEMM writes it)
        ws.dpart = (ws.part[:T * H].view(T, H) if ws.shared_part
                    else torch.empty(T, H, device=dev, dtype=torch.float32))
        ws.eids = torch.zeros(T, device=dev, dtype=torch.int32)
        ws.offs = torch.zeros(max(cfg.num_experts, 1) + 1, device=dev, dtype=torch.int32)
        ws.perm = torch.arange(T, device=dev, dtype=torch.int32)
        ws.inv = torch.arange(T, device=dev, dtype=torch.int32)

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
            d = p + "dynamics."
            wx = torch.cat([w(a + "q_proj.weight"), w(a + "k_proj.weight"), w(a + "v_proj.weight")], 0)
            wm = torch.cat([w(a + "mu_to_q.weight"), w(a + "mu_to_k.weight"),
                            w(a + "mu_to_v.weight")], 0)
            L = {
                "w_in": f(p + "input_layernorm.weight"),
                "wcat": torch.cat([wx, wm], 1).contiguous(),  # [(Hq+2Hkv)D, 2H]
                "wo": w(a + "o_proj.weight"),
                "w_post": f(p + "post_attention_layernorm.weight"),
                "wci": w(d + "controller_in.weight"),
                "bci": f(d + "controller_in.bias"),
                "wco": w(d + "controller_out.weight"),
                "bco": f(d + "controller_out.bias"),
                "wmu": w(d + "mu_proj.weight"),
                "mu": f(d + "mu"),
            }
            if config.use_qk_norm:
                L["qn"] = f(a + "q_norm.weight")
                L["kn"] = f(a + "k_norm.weight")
            if m.routed:
                gu = sd[p + "mlp.gate_up_proj"].to(dev, bf)   # [E, H, 2I] (local experts)
                dn = sd[p + "mlp.down_proj"].to(dev, bf)      # [E, I, H]
                E = m.local_experts = gu.shape[0]
                Ie = gu.shape[2] // 2
                L["wgu"] = torch.cat([interleave_gate_up(gu[e, :, :Ie].t(), gu[e, :, Ie:].t(), m.i_pad)
                                      for e in range(E)], 0).contiguous()
                L["wd"] = torch.cat([pad_cols(dn[e].t(), m.i_pad) for e in range(E)], 0).contiguous()
                L["router"] = w(p + "mlp.mu_router.weight")
            else:
                L["wgu"] = interleave_gate_up(w(p + "mlp.gate_proj.weight"),
                                              w(p + "mlp.up_proj.weight"), m.i_pad)
                L["wd"] = pad_cols(w(p + "mlp.down_proj.weight"), m.i_pad)
            m.layers.append(L)
        m.norm_w = f("norm.weight")
        tied = config.tie_word_embeddings or "lm_head.weight" not in sd
        m.lm_w = m.embed if tied else w("lm_head.weight")
        return m

    def weight_tensors(self):
        ts = [self.embed, self.norm_w] + ([] if self.lm_w is self.embed else [self.lm_w])
        for L in self.layers:
            ts.extend(L.values())
        return ts

    # ---- step ------------------------------------------------------------------
    def _ctrl_split(self, T: int, N: int, K: int) -> int:
        """Split-K factor of the controller's input layer (the partials live
        in ws.ctrl, [T, 3H] f32)."""
        cap = (3 * self.config.hidden_size) // max(N, 1)
        return int(_lib.load().muk_gemm_plan_split(T, N, K, _lib.MUK_EPI_F32, max(1, min(16, cap))))

    def _native_ok(self) -> bool:
        if not self.native:
            return False
        if self.tp_group is None:
            return True
        return self.comm is not None and self.ws.shared_part  # peer all-reduce only

    def _native(self, cache) -> "_lib.MukDeepModel":
        """The executor's model struct (rebuilt when a buffer moves)."""
        ws, cfg, cl = self.ws, self.config, self.clamp
        key = (id(ws), cache.block_pool.data_ptr(), self.rope_cos.data_ptr(), id(self.comm),
               self.fused_rope(), self._tp_fused, self.vocab_slice(), self.expert_lo,
               self.ep_combine)
        if key == self._native_key:
            return self._native_model
        H = cfg.hidden_size

        def p(t):
            return 0 if t is None else t.data_ptr()

        layers = (_lib.MukDeepLayer * len(self.layers))()
        for i, L in enumerate(self.layers):
            # the executor assumes the fused layouts from_state_dict builds
            assert L["wcat"].stride(0) == 2 * H and L["wci"].stride(0) == 2 * H
            layers[i] = _lib.MukDeepLayer(
                p(L["w_in"]), p(L["wcat"]), p(L["wo"]), p(L["w_post"]), p(L["wci"]),
                p(L["bci"]), p(L["wco"]), p(L["bco"]), p(L["wmu"]), p(L["mu"]), p(L.get("qn")),
                p(L.get("kn")), p(L["wgu"]), p(L["wd"]), p(L.get("router")))
        m = _lib.MukDeepModel()
        m.num_layers, m.hidden = len(self.layers), H
        m.num_q_heads, m.num_kv_heads = cfg.num_attention_heads, cfg.num_key_value_heads
        m.head_dim, m.inter_pad, m.vocab = cfg.head_dim, self.i_pad, cfg.vocab_size
        m.ctrl_hidden = self.layers[0]["wci"].shape[0]
        m.num_experts = cfg.num_experts if self.routed else 0
        m.local_experts, m.expert_lo = self.local_experts, self.expert_lo
        m.ep_gather = int(self.ep_combine == "gather")
        m.eps, m.dt = cfg.rms_norm_eps, cfg.dynamics_dt
        m.clamp, m.mu, m.clamp_min, m.clamp_max = int(cl.enabled), cl.mu, cl.clamp_min, cl.clamp_max
        m.layers = layers
        m.embed, m.final_norm = self.embed.data_ptr(), self.norm_w.data_ptr()
        vs = self.vocab_slice()
        m.lm_head = self.lm_w.data_ptr() + (0 if vs is None else vs[0] * self.lm_w.stride(0) * 2)
        m.rope_cos, m.rope_sin, m.rope_len = (self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
                                              self.rope_cos.shape[0])
        m.kv_pool, m.num_blocks, m.block_size = (cache.block_pool.data_ptr(), cache.max_num_blocks,
                                                 cache.block_size)
        m.resid, m.x, m.x_stride = ws.resid.data_ptr(), ws.x.data_ptr(), ws.x.stride(0)
        m.qkv, m.attn, m.act = ws.qkv.data_ptr(), ws.attn.data_ptr(), ws.act.data_ptr()
        m.part, m.part_rows = ws.part.data_ptr(), ws.part_rows
        m.h, m.hv, m.v, m.ch = ws.h.data_ptr(), ws.hv.data_ptr(), ws.v.data_ptr(), ws.ch.data_ptr()
        m.ctrl, m.mp, m.x2, m.xs = (ws.ctrl.data_ptr(), ws.mp.data_ptr(), ws.x2.data_ptr(),
                                    ws.xs.data_ptr())
        m.dpart, m.eids, m.offs = ws.dpart.data_ptr(), ws.eids.data_ptr(), ws.offs.data_ptr()
        m.perm, m.inv = ws.perm.data_ptr(), ws.inv.data_ptr()
        m.xl, m.logits = ws.xl.data_ptr(), ws.logits.data_ptr()
        m.lm_rows, m.logits_ld = cfg.vocab_size, ws.logits.stride(0)
        if vs is not None:  # this rank's vocabulary columns only
            c0, n = vs
            m.lm_rows = n
            m.logits = ws.logits.data_ptr() + 4 * c0
        m.attn_ws, m.attn_ws_bytes = ws.attn_ws.data_ptr(), ws.attn_ws.numel() * 4
        m.fused_rope = int(self.fused_rope())
        m.tp_world, m.tp_rank = 1, 0
        m.tp_fused = FUSED_TP_MAX_ROWS if self._tp_fused else 0
        if self.comm is not None:
            c = self.comm
            m.tp_world, m.tp_rank = c.world, c.rank
            for r in range(c.world):
                m.ar_data[r], m.ar_scratch[r], m.ar_flags[r] = (c.ptrs[r], c.scratch_ptrs[r],
                                                                 c.flag_ptrs[r])
        m._keep = layers  # the layer array must outlive the struct
        self._native_key, self._native_model = key, m
        return m

    def _forward_native(self, batch, cache) -> torch.Tensor:
        m = self._native(cache)
        b = _lib.MukStepBatch(batch.num_tokens, batch.num_seqs, batch.num_decode,
                              batch.max_q_len, batch.decode_len_bound,
                              batch.input_ids.data_ptr(), batch.positions.data_ptr(),
                              batch.slot_mapping.data_ptr(), batch.seq_lens.data_ptr(),
                              batch.prefill_cu.data_ptr(), batch.last_token_idx.data_ptr(),
                              batch.block_tables.data_ptr(), batch.block_tables.stride(0))
        _lib.call_native("muk_deep_forward", ctypes.byref(m), ctypes.byref(b),
                         torch.cuda.current_stream().cuda_stream)
        return self.ws.logits[:batch.num_seqs]

    def forward_step(self, batch, cache) -> torch.Tensor:
        if self._native_ok():
            return self._forward_native(batch, cache)
        cfg, ws, cl = self.config, self.ws, self.clamp
        T, H, eps = batch.num_tokens, cfg.hidden_size, cfg.rms_norm_eps
        E, V = cfg.num_experts, cfg.vocab_size
        resid = ws.resid[:T]
        xcat = ws.x[:T]             # [x | mu_prev]
        K.embed(batch.input_ids, self.embed, resid, cl)
        K.residual_rmsnorm(resid, None, self.layers[0]["w_in"], eps, xcat[:, :H], clamp=cl,
                           clamp_norm=True)
        nl = len(self.layers)
        for l, L in enumerate(self.layers):
            kdim = H if l == 0 else 2 * H  # layer 0 has no mu_prev (deep.py:296)
            self.qkv_proj(l, xcat[:, :kdim], L["wcat"][:, :kdim], batch, cache, L.get("qn"),
                          L.get("kn"))
            attn = self.attention(l, batch, cache)
            # h = clamp(o_proj(attn)) in f32 (INL input) and bf16 (controller / mu GEMMs)
            if self.tp_group is None and H % 32 == 0 and \
                    choose_split(T, H, attn.shape[1], ws.part_rows) == 1:
                K.gemm_clamp_dual(attn[:T], L["wo"], ws.h, ws.hv[:, :H], cl, M=T)
            else:
                part = self.row_parallel(attn[:T], L["wo"], T, H)
                K.reduce_clamp(part, ws.h, ws.hv[:, :H], cl, num_tokens=T)
            # controller input [h | v]: the velocity starts at zero
            # (layers.py:99-100), so layer 0 multiplies the h half only
            kc = H if l == 0 else 2 * H
            a_ci, w_ci = ws.hv[:, :kc], L["wci"][:, :kc]
            nc = w_ci.shape[0]
            # the narrow (64-wide) layer is a few tiles over a long K: split-K
            # partials (in ws.ctrl, written only later by controller_out) and a
            # bias + SiLU pass keep every SM streaming
            s = self._ctrl_split(T, nc, kc) if nc <= 128 else 1
            if s > 1:
                part = ws.ctrl.view(-1)[: s * T * nc].view(s, T, nc)
                K.gemm(a_ci, w_ci, part, K.MUK_EPI_F32, split_k=s, M=T)
                K.reduce_bias_silu(part, L["bci"], ws.ch, num_rows=T)
            else:
                K.gemm(a_ci, w_ci, ws.ch, K.MUK_EPI_BIAS_SILU, bias=L["bci"], M=T)
            K.gemm(ws.ch, L["wco"], ws.ctrl, K.MUK_EPI_F32, M=T)
            K.gemm(ws.hv[:, :H], L["wmu"], ws.mp, K.MUK_EPI_F32, M=T)
            K.inl_dynamics(ws.h, ws.ctrl, L["bco"], ws.mp, L["mu"], cfg.dynamics_dt, ws.v,
                           ws.hv[:, H:], ws.resid, ws.x[:, H:], L["w_post"], eps, ws.x2,
                           batch.input_ids, L.get("router"), E if self.routed else 0, V,
                           ws.eids, cl, num_tokens=T, v_zero=l == 0)
            last = l + 1 == nl
            nxt_w = None if last else self.layers[l + 1]["w_in"]
            nxt_out = None if last else xcat[:, :H]
            if self.routed:
                K.route_permute(ws.eids, E, ws.offs, ws.perm, ws.inv, num_tokens=T)
                K.gather_rows(ws.x2, ws.perm, ws.xs, num_rows=T)
                El, e0 = self.local_experts, self.expert_lo
                offs = ws.offs[e0:e0 + El + 1]   # rows of this GPU's experts (sorted order)
                K.grouped_gemm(ws.xs, L["wgu"], ws.act, offs, El, 2 * self.i_pad,
                               K.MUK_EPI_SWIGLU, max_rows=T)
                if El < E and self.comm is not None and self.ep_combine == "gather":
                    # expert parallel: every rank holds every token, so dispatch
                    # is local; the combine copies each rank's expert rows (bf16)
                    # into every rank's buffer over NVLink
                    rows = self.comm.rows_view(T, H)
                    K.grouped_gemm(ws.act, L["wd"], rows, offs, El, H, K.MUK_EPI_BF16, max_rows=T)
                    self.comm.ep_gather_(rows, ws.offs, e0, e0 + El)
                    delta = rows
                else:
                    if El < E:  # other experts' rows arrive through the all-reduce
                        ws.dpart[:T].zero_()
                    K.grouped_gemm(ws.act, L["wd"], ws.dpart, offs, El, H, K.MUK_EPI_F32,
                                   max_rows=T)
                    self.reduce_partials(ws.dpart[:T])  # same expert order on every rank
                    delta = ws.dpart[:T]
                K.residual_rmsnorm(resid, delta, nxt_w, eps, nxt_out, clamp=cl,
                                   clamp_delta=True, clamp_sum=True, clamp_norm=True,
                                   delta_rows=ws.inv)
            else:
                K.gemm(ws.x2, L["wgu"], ws.act, K.MUK_EPI_SWIGLU, M=T)
                part = self.row_parallel(ws.act[:T], L["wd"], T, H)
                K.residual_rmsnorm(resid, part, nxt_w, eps, nxt_out, clamp=cl, clamp_delta=True,
                                   clamp_sum=True, clamp_norm=True)
        return self.lm_head(batch, self.norm_w, self.lm_w)
