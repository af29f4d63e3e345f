"""Configuration types, field-for-field compatible with mu_inference.core.config.

The dataclasses keep the reference's names, defaults and validation
(mu_inference/core/config.py:25-345) so existing callers construct them
unchanged.  Additions, all optional: ``CacheConfig.num_gpu_blocks``
(pool size override used by the paged cache),
``EngineConfig.max_seq_len_hint`` (sizes decode scratch for graph capture),
``EngineConfig.expert_parallel`` and ``SchedulerConfig.step_token_alignment``
(tile-aligned step sizes under chunked prefill).
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Dict, List, Literal, Optional


class ModelType(str, Enum):
    """Architectures the reference names (config.py:12-20)."""

    DEEP = "deep"
    LLAMA = "llama"
    MISTRAL = "mistral"
    QWEN = "qwen"
    PHI = "phi"
    GEMMA = "gemma"
    AUTO = "auto"


@dataclass
class MuConfig:
    """mu_clamp settings (config.py:25-65).  Disabled by default, as in the reference."""

    enabled: bool = False
    mu: float = 0.0
    clamp_min: float = -10.0
    clamp_max: float = 10.0
    velocity_min: float = -10.0
    velocity_max: float = 10.0
    beta: float = 1.0
    beta_min: float = 0.0
    beta_max: float = 2.0
    ema_alpha: float = 0.3
    apply_to_attention: bool = True
    apply_to_mlp: bool = True
    apply_to_layernorm: bool = True
    apply_to_kv_cache: bool = True


@dataclass
class SamplingParams:
    """Per-request sampling knobs (config.py:68-116), same defaults and checks.

    ``seed`` is honoured here (the reference ignores it): it keys the
    counter-based RNG of the GPU sampler."""

    temperature: float = 0.8
    top_k: int = 50
    top_p: float = 0.9
    repetition_penalty: float = 1.1
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    max_tokens: int = 512
    min_tokens: int = 0
    stop_sequences: List[str] = field(default_factory=list)
    stop_token_ids: List[int] = field(default_factory=list)
    seed: Optional[int] = None
    logprobs: bool = False
    top_logprobs: int = 0
    skip_special_tokens: bool = True

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.repetition_penalty < 1:
            raise ValueError("repetition_penalty must be >= 1")


@dataclass
class ModelConfig:
    """Architecture description (config.py:119-218)."""

    model_type: ModelType = ModelType.AUTO
    vocab_size: int = 32000
    hidden_size: int = 2048
    intermediate_size: int = 5632
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: Optional[int] = None
    max_position_embeddings: int = 2048
    rope_theta: float = 10000.0
    rope_scaling: Optional[Dict[str, Any]] = None
    rms_norm_eps: float = 1e-6
    hidden_act: str = "silu"
    use_token_routed_mlp: bool = False
    num_experts: int = 4
    use_qk_norm: bool = False
    tie_word_embeddings: bool = True
    pad_token_id: int = 0
    bos_token_id: int = 1
    eos_token_id: int = 2
    dynamics_alpha: float = 0.9
    dynamics_beta: float = 0.1
    dynamics_gate: float = 0.5
    dynamics_dt: float = 0.1
    dynamics_controller_hidden: int = 64

    def __post_init__(self):
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        """HF config.json -> ModelConfig, the reference's first parser (config.py:172-218)."""
        arch = d.get("architectures", [""])[0]
        mt = ModelType.AUTO
        for key, val in (("Deep", ModelType.DEEP), ("Llama", ModelType.LLAMA),
                         ("Mistral", ModelType.MISTRAL), ("Qwen", ModelType.QWEN),
                         ("Phi", ModelType.PHI), ("Gemma", ModelType.GEMMA)):
            if key in arch:
                mt = val
                break
        heads = d.get("num_attention_heads", 16)
        return cls(
            model_type=mt,
            vocab_size=d.get("vocab_size", 32000),
            hidden_size=d.get("hidden_size", 2048),
            intermediate_size=d.get("intermediate_size", 5632),
            num_hidden_layers=d.get("num_hidden_layers", 24),
            num_attention_heads=heads,
            num_key_value_heads=d.get("num_key_value_heads", heads),
            max_position_embeddings=d.get("max_position_embeddings", 2048),
            rope_theta=d.get("rope_theta", 10000.0),
            rms_norm_eps=d.get("rms_norm_eps", 1e-6),
            hidden_act=d.get("hidden_act", "silu"),
            use_token_routed_mlp=d.get("use_token_routed_mlp", False),
            num_experts=d.get("num_experts", 4),
            use_qk_norm=d.get("use_qk_norm", False),
            tie_word_embeddings=d.get("tie_word_embeddings", True),
            pad_token_id=d.get("pad_token_id", 0),
            bos_token_id=d.get("bos_token_id", 1),
            eos_token_id=d.get("eos_token_id", 2),
            dynamics_alpha=d.get("dynamics_alpha", 0.9),
            dynamics_beta=d.get("dynamics_beta", 0.1),
            dynamics_gate=d.get("dynamics_gate", 0.5),
            dynamics_dt=d.get("dynamics_dt", 0.1),
            dynamics_controller_hidden=d.get("dynamics_controller_hidden", 64),
        )


@dataclass
class CacheConfig:
    """Paged KV cache settings (config.py:221-245)."""

    max_seq_len: int = 2048
    block_size: int = 16
    max_num_blocks: int = 2048
    max_num_seqs: int = 256
    dtype: Literal["float16", "bfloat16", "float32"] = "float16"
    use_paged: bool = True
    mu_enabled: bool = True
    num_gpu_blocks: Optional[int] = None


@dataclass
class SchedulerConfig:
    """Scheduler settings (config.py:248-275)."""

    max_batch_size: int = 64
    max_num_batched_tokens: int = 8192
    max_waiting_requests: int = 1000
    policy: Literal["fcfs", "priority", "fair"] = "fcfs"
    enable_preemption: bool = True
    preemption_mode: Literal["recompute", "swap"] = "recompute"
    enable_chunked_prefill: bool = True
    max_prefill_tokens: int = 4096
    # With chunked prefill: trim the step's last prefill chunk so that the
    # step's token count is a multiple of this (0 = off).  GEMM tiles cover
    # 128 or 256 rows, so rows past the last full tile cost a whole tile; the
    # trimmed tokens run first in the next step.  Not in the reference.
    step_token_alignment: int = 0
    enable_continuous_batching: bool = True
    batch_wait_time_ms: float = 5.0
    min_batch_size: int = 1


@dataclass
class EngineConfig:
    """Top-level engine configuration (config.py:278-345)."""

    model_path: str = ""
    model: ModelConfig = field(default_factory=ModelConfig)
    mu: MuConfig = field(default_factory=MuConfig)
    sampling: SamplingParams = field(default_factory=SamplingParams)
    cache: CacheConfig = field(default_factory=CacheConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    device: str = "cuda"
    dtype: Literal["float16", "bfloat16", "float32"] = "float16"
    tensor_parallel_size: int = 1
    # token-routed experts distributed whole over the tensor-parallel ranks
    # (expert e on rank e // (E / P)) instead of split column-wise
    expert_parallel: bool = False
    host: str = "0.0.0.0"
    port: int = 8080
    log_level: Literal["DEBUG", "INFO", "WARNING", "ERROR"] = "INFO"
    use_torch_compile: bool = False
    compile_mode: Literal["default", "reduce-overhead", "max-autotune"] = "reduce-overhead"
    max_seq_len_hint: Optional[int] = None

    @classmethod
    def from_pretrained(cls, model_path: str, **kwargs) -> "EngineConfig":
        """Local model directory -> EngineConfig (no hub download: offline)."""
        cfg_path = Path(model_path) / "config.json"
        with open(cfg_path) as f:
            model_config = ModelConfig.from_dict(json.load(f))
        return cls(model_path=str(model_path), model=model_config,
                   cache=CacheConfig(max_seq_len=model_config.max_position_embeddings), **kwargs)
