"""Model registry with the reference's API (mu_inference/models/registry.py:17-141)."""

from __future__ import annotations

import logging
from typing import Callable, Dict, Optional, Type

logger = logging.getLogger(__name__)

MODEL_REGISTRY: Dict[str, Type] = {}

# HuggingFace architecture names -> registry keys (registry.py:20-47).  "phi"
# is listed there without a registered class; it stays unsupported here too.
ARCHITECTURE_ALIASES = {
    "DeepForCausalLM": "deep",
    "DeepseekForCausalLM": "deep",
    "PacificPrimeForCausalLM": "deep",
    "LlamaForCausalLM": "llama",
    "Llama2ForCausalLM": "llama",
    "Llama3ForCausalLM": "llama",
    "CodeLlamaForCausalLM": "llama",
    "MistralForCausalLM": "mistral",
    "Mixtral": "mistral",
    "Qwen2ForCausalLM": "qwen",
    "QwenForCausalLM": "qwen",
    "PhiForCausalLM": "phi",
    "Phi3ForCausalLM": "phi",
    "GemmaForCausalLM": "gemma",
    "Gemma2ForCausalLM": "gemma",
}

_TYPE_MAPPING = {
    "llama": "llama", "mistral": "mistral", "qwen": "qwen", "qwen2": "qwen", "phi": "phi",
    "phi3": "phi", "gemma": "gemma", "gemma2": "gemma", "deep": "deep", "deepseek": "deep",
}


def register_model(name: str) -> Callable:
    def deco(cls: Type) -> Type:
        MODEL_REGISTRY[name.lower()] = cls
        logger.debug("registered model %s -> %s", name, cls.__name__)
        return cls

    return deco


def get_model_class(model_type: str) -> Optional[Type]:
    _ensure_models()
    key = model_type.lower()
    if key in MODEL_REGISTRY:
        return MODEL_REGISTRY[key]
    for alias, canonical in ARCHITECTURE_ALIASES.items():
        if alias.lower() == key:
            return MODEL_REGISTRY.get(canonical)
    return None


def detect_architecture(config_dict: dict) -> Optional[str]:
    for arch in config_dict.get("architectures", []) or []:
        if arch in ARCHITECTURE_ALIASES:
            return ARCHITECTURE_ALIASES[arch]
    mt = str(config_dict.get("model_type", "")).lower()
    for key, val in _TYPE_MAPPING.items():
        if key in mt:
            return val
    if config_dict.get("num_experts") is not None:
        return "deep"
    return None


def list_supported_models() -> list:
    _ensure_models()
    return list(MODEL_REGISTRY.keys())


def is_supported(model_type: str) -> bool:
    return get_model_class(model_type) is not None


def _ensure_models() -> None:
    from . import deep, llama  # noqa: F401  (registers the classes)
