"""mu_b200 — the mu_inference continuous-batching forward step on B200 (sm_100a).

Public surface mirrors ``mu_inference`` (Complexity-ML/complexity-inference,
mu_inference/__init__.py:36-78): ``MuEngine``, ``MuBatchEngine``,
``SamplingParams`` and the config types, ``MODEL_REGISTRY`` /
``register_model``, ``load_model``, ``mu_clamp`` / ``soft_clamp`` /
``MuDynamics``.  Every tensor operation of the step runs in libmuk.so
(hand-written sm_100a kernels behind a C ABI, ``include/muk.h``); importing
the engines requires that library and a CUDA device.
"""

__version__ = "0.1.0"

from .core.config import (CacheConfig, EngineConfig, ModelConfig, ModelType, MuConfig,
                          SamplingParams, SchedulerConfig)
from .core.mu import MuDynamics, mu_clamp, soft_clamp
from .models.base import MuModelBase, MuModelOutput
from .models.loader import load_model
from .models.registry import MODEL_REGISTRY, register_model

__all__ = [
    "__version__", "mu_clamp", "soft_clamp", "MuDynamics", "MuConfig", "EngineConfig",
    "SamplingParams", "ModelConfig", "ModelType", "CacheConfig", "SchedulerConfig",
    "MuModelBase", "MuModelOutput", "load_model", "MODEL_REGISTRY", "register_model",
    "MuEngine", "MuBatchEngine",
]


def __getattr__(name):
    if name in ("MuEngine", "MuBatchEngine"):
        from .serving import engine

        return getattr(engine, name)
    raise AttributeError(name)
