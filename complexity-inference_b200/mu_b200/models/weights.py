"""Seeded random weights in the reference's state-dict naming, and model dirs.

``random_state_dict`` draws every parameter from one seeded torch.Generator
in a fixed order, so the same (config, seed) gives the same tensors on any
machine with this torch build: matrices and embeddings ~ N(0, 0.02), norm
weights 1, INL ``dynamics.mu`` 0 and the controller_out bias at the values
INLDynamics.__init__ derives from the alpha/beta/gate settings
(mu_inference/models/layers.py:65-76).  Names follow the reference modules
(``layers.{i}.self_attn.q_proj.weight`` ...), so the same dict loads into the
reference with ``load_state_dict``.
"""

from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Dict

import torch

from ..core.config import ModelConfig

STD = 0.02


def expert_intermediate(cfg: ModelConfig) -> int:
    """Per-expert width: intermediate_size // num_experts (layers.py:454)."""
    return cfg.intermediate_size // cfg.num_experts


def is_routed(arch: str, cfg: ModelConfig) -> bool:
    return arch == "deep" and bool(cfg.num_experts) and cfg.num_experts > 1


def random_state_dict(cfg: ModelConfig, arch: str, seed: int, device: str = "cpu",
                      dtype: torch.dtype = torch.float32, include_unused: bool = True
                      ) -> Dict[str, torch.Tensor]:
    """Seeded parameters for ``arch`` in {"llama", "deep"}.

    ``include_unused`` adds the reference's mu_to_q/k/v of Llama attention,
    which the Llama forward never uses (mu_prev is None there)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, D = cfg.hidden_size, cfg.head_dim
    Hq, Hkv, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.vocab_size
    sd: Dict[str, torch.Tensor] = {}

    def normal(name, *shape):
        sd[name] = (torch.randn(*shape, generator=g, device=device) * STD).to(dtype)

    def ones(name, n):
        sd[name] = torch.ones(n, device=device, dtype=dtype)

    normal("embed_tokens.weight", V, H)
    for l in range(cfg.num_hidden_layers):
        p = f"layers.{l}."
        ones(p + "input_layernorm.weight", H)
        normal(p + "self_attn.q_proj.weight", Hq * D, H)
        normal(p + "self_attn.k_proj.weight", Hkv * D, H)
        normal(p + "self_attn.v_proj.weight", Hkv * D, H)
        normal(p + "self_attn.o_proj.weight", H, Hq * D)
        if arch == "deep" or include_unused:
            normal(p + "self_attn.mu_to_q.weight", Hq * D, H)
            normal(p + "self_attn.mu_to_k.weight", Hkv * D, H)
            normal(p + "self_attn.mu_to_v.weight", Hkv * D, H)
        if arch == "deep" and cfg.use_qk_norm:
            ones(p + "self_attn.q_norm.weight", D)
            ones(p + "self_attn.k_norm.weight", D)
        ones(p + "post_attention_layernorm.weight", H)
        if is_routed(arch, cfg):
            E, Ie = cfg.num_experts, expert_intermediate(cfg)
            normal(p + "mlp.gate_up_proj", E, H, 2 * Ie)
            normal(p + "mlp.down_proj", E, Ie, H)
            normal(p + "mlp.mu_router.weight", E, H)
        else:
            I = cfg.intermediate_size
            normal(p + "mlp.gate_proj.weight", I, H)
            normal(p + "mlp.up_proj.weight", I, H)
            normal(p + "mlp.down_proj.weight", H, I)
        if arch == "deep":
            C = cfg.dynamics_controller_hidden
            q = p + "dynamics."
            sd[q + "mu"] = torch.zeros(H, device=device, dtype=dtype)
            normal(q + "mu_proj.weight", H, H)
            normal(q + "controller_in.weight", C, 2 * H)
            normal(q + "controller_in.bias", C)
            normal(q + "controller_out.weight", 3 * H, C)
            a = math.log(cfg.dynamics_alpha / (1.0 - cfg.dynamics_alpha + 1e-8))
            b = math.log(math.exp(cfg.dynamics_beta) - 1.0 + 1e-8)
            gt = math.log(cfg.dynamics_gate / (1.0 - cfg.dynamics_gate + 1e-8))
            sd[q + "controller_out.bias"] = torch.cat([
                torch.full((H,), a), torch.full((H,), b), torch.full((H,), gt)]).to(device, dtype)
    ones("norm.weight", H)
    if not cfg.tie_word_embeddings:
        normal("lm_head.weight", V, H)
    return sd


def config_dict(cfg: ModelConfig, arch: str) -> dict:
    """config.json content that both this package and the reference parse identically."""
    name = {"deep": "DeepForCausalLM", "llama": "LlamaForCausalLM"}[arch]
    d = {
        "architectures": [name],
        "model_type": arch,
        "vocab_size": cfg.vocab_size,
        "hidden_size": cfg.hidden_size,
        "intermediate_size": cfg.intermediate_size,
        "num_hidden_layers": cfg.num_hidden_layers,
        "num_attention_heads": cfg.num_attention_heads,
        "num_key_value_heads": cfg.num_key_value_heads,
        "head_dim": cfg.head_dim,
        "max_position_embeddings": cfg.max_position_embeddings,
        "rope_theta": cfg.rope_theta,
        "rms_norm_eps": cfg.rms_norm_eps,
        "tie_word_embeddings": cfg.tie_word_embeddings,
        "use_qk_norm": cfg.use_qk_norm,
        "dynamics_alpha": cfg.dynamics_alpha,
        "dynamics_beta": cfg.dynamics_beta,
        "dynamics_gate": cfg.dynamics_gate,
        "dynamics_dt": cfg.dynamics_dt,
        "dynamics_controller_hidden": cfg.dynamics_controller_hidden,
    }
    if arch == "deep":
        d["num_experts"] = cfg.num_experts
    return d


def write_model_dir(path, cfg: ModelConfig, arch: str, state_dict: Dict[str, torch.Tensor]) -> Path:
    """Write config.json + model.safetensors (contiguous CPU copies)."""
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(config_dict(cfg, arch), indent=2))
    save_file({k: v.detach().cpu().contiguous() for k, v in state_dict.items()},
              str(path / "model.safetensors"))
    return path


def load_state_dict(path) -> Dict[str, torch.Tensor]:
    """All tensors of a model dir (safetensors first, else .bin/.pt), with the
    reference's prefix stripping ("model.", "transformer.", "decoder.";
    mu_inference/models/loader.py:188-227)."""
    path = Path(path)
    files = sorted(path.glob("*.safetensors"))
    sd: Dict[str, torch.Tensor] = {}
    if files:
        from safetensors.torch import load_file

        for f in files:
            sd.update(load_file(str(f), device="cpu"))
    else:
        for f in sorted(list(path.glob("*.bin")) + list(path.glob("*.pt"))):
            sd.update(torch.load(str(f), map_location="cpu", weights_only=True))
    if not sd:
        raise FileNotFoundError(f"no weight files in {path}")
    return {strip_prefix(k): v for k, v in sd.items()}


def strip_prefix(name: str) -> str:
    """Parameter name without the "model." / "transformer." / "decoder."
    prefix (mu_inference/models/loader.py:188-227)."""
    for pre in ("model.", "transformer.", "decoder."):
        if name.startswith(pre):
            return name[len(pre):]
    return name


def state_dict_digest(sd: Dict[str, torch.Tensor]) -> float:
    """Order-independent checksum used to pin golden fixtures to their weights."""
    tot = 0.0
    for i, k in enumerate(sorted(sd)):
        t = sd[k].double()
        tot += float(t.sum()) * (i + 1) + float((t * t).sum())
    return tot
