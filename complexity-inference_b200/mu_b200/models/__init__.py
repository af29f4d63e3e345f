"""Model registry, weights and the flat-batch Llama / Deep steps."""

from .registry import MODEL_REGISTRY, register_model  # noqa: F401
