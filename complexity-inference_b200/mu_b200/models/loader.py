"""Model loading with the reference's API (mu_inference/models/loader.py:33-303).

Local directories only (config.json + safetensors / .bin / .pt): the hub
download path of the reference needs a network and is not part of the
forward step.  Weights are cast to bf16 and re-laid-out for the kernels by
the model's ``from_state_dict``.
"""

from __future__ import annotations

import json
import os
from typing import Any, Dict, Optional

import torch

from ..core.config import ModelConfig, ModelType, MuConfig
from .registry import MODEL_REGISTRY, detect_architecture, get_model_class
from .weights import load_state_dict


def load_config(model_path: str) -> Dict[str, Any]:
    path = os.path.abspath(model_path)
    cfg = os.path.join(path, "config.json")
    if not os.path.isfile(cfg):
        raise FileNotFoundError(f"No config.json found in {path}")
    with open(cfg) as f:
        return json.load(f)


def config_from_dict(d: Dict[str, Any]) -> ModelConfig:
    """The reference's second config parser (loader.py:64-97): reads head_dim,
    num_local_experts and qk_norm, which ModelConfig.from_dict does not."""
    arch = detect_architecture(d)
    mt = ModelType[arch.upper()] if arch and arch.upper() in ModelType.__members__ else ModelType.AUTO
    heads = d.get("num_attention_heads", 16)
    return ModelConfig(
        model_type=mt,
        vocab_size=d.get("vocab_size", 32000),
        hidden_size=d.get("hidden_size", 2048),
        intermediate_size=d.get("intermediate_size", 5632),
        num_hidden_layers=d.get("num_hidden_layers", 24),
        num_attention_heads=heads,
        num_key_value_heads=d.get("num_key_value_heads", heads),
        head_dim=d.get("head_dim", d.get("hidden_size", 2048) // heads),
        max_position_embeddings=d.get("max_position_embeddings", 2048),
        rms_norm_eps=d.get("rms_norm_eps", 1e-6),
        rope_theta=d.get("rope_theta", 10000.0),
        num_experts=d.get("num_experts", d.get("num_local_experts")),
        use_qk_norm=d.get("use_qk_norm", d.get("qk_norm", False)),
        tie_word_embeddings=d.get("tie_word_embeddings", True),
        dynamics_alpha=d.get("dynamics_alpha", 0.9),
        dynamics_beta=d.get("dynamics_beta", 0.1),
        dynamics_gate=d.get("dynamics_gate", 0.5),
        dynamics_dt=d.get("dynamics_dt", 0.1),
        dynamics_controller_hidden=d.get("dynamics_controller_hidden", 64),
    )


def build_model(arch: str, config: ModelConfig, state_dict: Dict[str, torch.Tensor],
                mu_config: Optional[MuConfig] = None, device: str = "cuda"):
    cls = get_model_class(arch)
    if cls is None:
        raise ValueError(f"Unsupported model type: {arch}. Supported: {list(MODEL_REGISTRY)}")
    return cls.from_state_dict(config, state_dict, mu_config or MuConfig(), device)


def load_model(model_path: str, model_type: Optional[str] = None,
               config: Optional[ModelConfig] = None, mu_config: Optional[MuConfig] = None,
               device: str = "cuda", dtype: torch.dtype = torch.bfloat16, **kwargs):
    """Load a local model directory onto ``device``.  ``dtype`` is accepted for
    API compatibility; the kernels always hold weights in bf16."""
    cfg_dict = load_config(model_path)
    if config is None:
        config = config_from_dict(cfg_dict)
    if model_type is None:
        model_type = detect_architecture(cfg_dict)
        if model_type is None:
            raise ValueError("Could not detect model architecture. Please specify model_type.")
    return build_model(model_type, config, load_state_dict(model_path), mu_config, device)
