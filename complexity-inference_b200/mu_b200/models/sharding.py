"""Tensor-parallel sharding of the reference state dict.

Rank r of P keeps:
* attention: query heads [r·Hq/P, (r+1)·Hq/P) and KV heads [r·Hkv/P, ...)
  — rows of q/k/v_proj and mu_to_q/k/v (column-parallel), the matching
  input columns of o_proj (row-parallel); QK-norm weights are per head-dim
  and replicated;
* MLP: rows [r·I/P, (r+1)·I/P) of gate/up (column-parallel) and those
  columns of down (row-parallel); for token-routed experts the same split is
  applied inside every expert ([E, H, 2I] / [E, I, H] keep E whole);
* with ``expert_parallel``, token-routed experts are instead kept whole and
  distributed: rank r holds experts [r·E/P, (r+1)·E/P) (one per GPU when
  P = E), so expert e lives on GPU e // (E/P).  Every rank routes every token
  (the routing inputs are replicated), runs its own experts' tokens through
  the grouped GEMMs and leaves the other rows zero;
* everything else (embeddings, norms, LM head, INL dynamics, router) whole.

After a row-parallel projection (or the expert MLP) each rank holds a
partial sum of the full [T, H] output; one all-reduce per projection (two
per layer) restores it, so all ranks carry identical residual streams and
sample identical tokens.  Expert parallelism therefore needs no all-to-all:
the tokens are already on every GPU (attention is head-parallel), and the
all-reduce that follows the MLP carries each token's expert output from the
GPU that owns the expert.
The shard has the same names as the full dict and a ModelConfig whose head
and intermediate counts are the local ones.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Tuple

import torch

from ..core.config import ModelConfig
from .weights import expert_intermediate, is_routed


def local_config(cfg: ModelConfig, arch: str, tp: int, expert_parallel: bool = False
                 ) -> ModelConfig:
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if Hq % tp or Hkv % tp:
        raise ValueError(f"tensor_parallel_size {tp} must divide heads {Hq}/{Hkv}")
    if expert_parallel and is_routed(arch, cfg):
        if cfg.num_experts % tp:
            raise ValueError(f"tensor_parallel_size {tp} must divide num_experts {cfg.num_experts}")
        inter = cfg.intermediate_size  # experts stay whole
    elif is_routed(arch, cfg):
        ie = expert_intermediate(cfg)
        if ie % tp:
            raise ValueError(f"tensor_parallel_size {tp} must divide the expert width {ie}")
        inter = cfg.intermediate_size // tp
    else:
        if cfg.intermediate_size % tp:
            raise ValueError(f"tensor_parallel_size {tp} must divide {cfg.intermediate_size}")
        inter = cfg.intermediate_size // tp
    return dataclasses.replace(cfg, num_attention_heads=Hq // tp, num_key_value_heads=Hkv // tp,
                               intermediate_size=inter, head_dim=cfg.head_dim)


def expert_range(cfg: ModelConfig, rank: int, tp: int) -> Tuple[int, int]:
    """Experts [lo, hi) held by ``rank`` under expert parallelism."""
    n = cfg.num_experts // tp
    return rank * n, (rank + 1) * n


def shard_index(name: str, cfg: ModelConfig, arch: str, rank: int, tp: int,
                expert_parallel: bool = False) -> Optional[Tuple[int, List[tuple]]]:
    """How rank ``rank`` of ``tp`` slices parameter ``name``: None for the
    whole tensor, else (concat dim, [index tuples]) — the rank's shard is the
    concatenation of ``t[idx]`` over the tuples.  One rule set serves both a
    tensor in memory and a lazy safetensors slice read from disk."""
    if tp == 1:
        return None
    D = cfg.head_dim
    hq = cfg.num_attention_heads // tp
    hkv = cfg.num_key_value_heads // tp
    q0, k0 = rank * hq * D, rank * hkv * D
    routed = is_routed(arch, cfg)
    ep = expert_parallel and routed
    if routed:
        ie = expert_intermediate(cfg)
        il = ie // tp
    else:
        il = cfg.intermediate_size // tp
    i0 = rank * il
    leaf = name.split(".", 2)[-1] if name.startswith("layers.") else name
    all_ = slice(None)
    if leaf in ("self_attn.q_proj.weight", "self_attn.mu_to_q.weight"):
        return 0, [(slice(q0, q0 + hq * D),)]
    if leaf in ("self_attn.k_proj.weight", "self_attn.v_proj.weight",
                "self_attn.mu_to_k.weight", "self_attn.mu_to_v.weight"):
        return 0, [(slice(k0, k0 + hkv * D),)]
    if leaf == "self_attn.o_proj.weight":
        return 1, [(all_, slice(q0, q0 + hq * D))]
    if leaf in ("mlp.gate_proj.weight", "mlp.up_proj.weight"):
        return 0, [(slice(i0, i0 + il),)]
    if leaf == "mlp.down_proj.weight" and not routed:
        return 1, [(all_, slice(i0, i0 + il))]
    if leaf in ("mlp.gate_up_proj", "mlp.down_proj") and ep:   # whole experts [e0, e1)
        e0, e1 = expert_range(cfg, rank, tp)
        return 0, [(slice(e0, e1),)]
    if leaf == "mlp.gate_up_proj":   # [E, H, 2I]: gate cols [0, I), up cols [I, 2I)
        return 2, [(all_, all_, slice(i0, i0 + il)), (all_, all_, slice(ie + i0, ie + i0 + il))]
    if leaf == "mlp.down_proj" and routed:   # [E, I, H]
        return 1, [(all_, slice(i0, i0 + il), all_)]
    return None


def _take(t, spec) -> torch.Tensor:
    if spec is None:
        return t[:] if not isinstance(t, torch.Tensor) else t
    dim, idxs = spec
    parts = [t[idx] for idx in idxs]
    return parts[0] if len(parts) == 1 else torch.cat(parts, dim)


def shard_state_dict(sd: Dict[str, torch.Tensor], cfg: ModelConfig, arch: str, rank: int,
                     tp: int, expert_parallel: bool = False
                     ) -> Tuple[Dict[str, torch.Tensor], ModelConfig]:
    """The rank's shard of a full state dict plus its local ModelConfig."""
    if tp == 1:
        return dict(sd), cfg
    ep = expert_parallel and is_routed(arch, cfg)
    lcfg = local_config(cfg, arch, tp, ep)
    out = {name: _take(t, shard_index(name, cfg, arch, rank, tp, ep)) for name, t in sd.items()}
    return {k: v.contiguous() for k, v in out.items()}, lcfg


def load_sharded_state_dict(path, cfg: ModelConfig, arch: str, rank: int, tp: int,
                            expert_parallel: bool = False
                            ) -> Tuple[Dict[str, torch.Tensor], ModelConfig]:
    """Read only this rank's shard of every parameter from a model dir's
    safetensors files (lazy slices; the full tensors are never materialised),
    with the reference's prefix stripping (mu_inference/models/loader.py:188-227).
    Directories without safetensors fall back to loading and slicing in memory."""
    from pathlib import Path

    from .weights import load_state_dict, strip_prefix

    files = sorted(Path(path).glob("*.safetensors"))
    if not files:
        return shard_state_dict(load_state_dict(path), cfg, arch, rank, tp, expert_parallel)
    from safetensors import safe_open

    ep = expert_parallel and is_routed(arch, cfg)
    out: Dict[str, torch.Tensor] = {}
    for f in files:
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for key in h.keys():
                name = strip_prefix(key)
                spec = shard_index(name, cfg, arch, rank, tp, ep)
                out[name] = (h.get_tensor(key) if spec is None
                             else _take(h.get_slice(key), spec)).contiguous()
    if not out:
        raise FileNotFoundError(f"no weight files in {path}")
    return out, (local_config(cfg, arch, tp, ep) if tp > 1 else cfg)
