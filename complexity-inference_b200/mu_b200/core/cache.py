"""Paged KV cache: a GPU block pool with MuPagedCache-compatible bookkeeping.

Pool layout (one allocation): ``[num_layers][2][num_blocks][num_kv_heads]
[block_size][head_dim]``, so the K (or V) tile of one (block, kv head) is a
contiguous ``block_size * head_dim`` run for the attention kernels, and a
layer's K and V are plain 4-D views.

Block bookkeeping reproduces mu_inference/core/cache.py:257-462 exactly:
the free list starts as ``list(range(N))`` and is popped from the end
(LIFO); ``allocate`` takes one block even for an empty request; a new block
is taken only when a token arrives while the last block is full; ``free``
returns blocks in table order.  Block tables and slot mappings therefore
match the reference allocator bit for bit.

One deliberate difference: the reference advances a request's position on
every ``append`` call, i.e. once per layer (cache.py:340, 374), so a
multi-layer model spreads one token over several slots.  Here slots are
reserved once per token per step (:meth:`PagedKVCache.reserve`) and shared
by all layers; the reference-style ``append(request_id, layer_idx, k, v)``
keeps its signature and reuses the slots reserved by the layer-0 call.
"""

from __future__ import annotations

import threading
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .config import MuConfig
from .mu import mu_clamp


class PagedKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, block_size: int = 16,
                 max_num_blocks: int = 2048, dtype: torch.dtype = torch.bfloat16,
                 device: str = "cuda", mu_config: Optional[MuConfig] = None):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.max_num_blocks = max_num_blocks
        self.dtype = dtype
        self.device = device
        self.mu_config = mu_config or MuConfig()
        self.block_pool = torch.zeros(num_layers, 2, max_num_blocks, num_kv_heads, block_size,
                                      head_dim, dtype=dtype, device=device)
        self.free_blocks: List[int] = list(range(max_num_blocks))
        self.request_blocks: Dict[str, List[int]] = {}
        self.request_pos: Dict[str, int] = {}
        self._pending: Dict[str, np.ndarray] = {}
        self._lock = threading.RLock()

    # ---- device views ------------------------------------------------------
    def k_cache(self, layer: int) -> torch.Tensor:
        return self.block_pool[layer, 0]

    def v_cache(self, layer: int) -> torch.Tensor:
        return self.block_pool[layer, 1]

    # ---- reference API (cache.py:311-453) -----------------------------------
    def allocate(self, request_id: str) -> bool:
        """Give a new request its first block (LIFO pop); False when full."""
        with self._lock:
            if not self.free_blocks:
                return False
            self.request_blocks[request_id] = [self.free_blocks.pop()]
            self.request_pos[request_id] = 0
            return True

    def reserve(self, request_id: str, num_tokens: int) -> Optional[np.ndarray]:
        """Slots (block*block_size + offset) for the next ``num_tokens`` tokens.

        All-or-nothing: returns None (state unchanged) when the request is
        unknown or the pool cannot hold the tokens."""
        with self._lock:
            blocks = self.request_blocks.get(request_id)
            if blocks is None:
                return None
            bs = self.block_size
            pos = self.request_pos[request_id]
            n = int(num_tokens)
            if n <= 0:
                return np.empty(0, dtype=np.int32)
            first = min(n, bs - pos) if pos < bs else 0
            rest = n - first
            need = (rest + bs - 1) // bs
            if need > len(self.free_blocks):
                return None
            out = np.empty(n, dtype=np.int32)
            if first:
                out[:first] = blocks[-1] * bs + pos + np.arange(first, dtype=np.int32)
            if need:
                new = [self.free_blocks.pop() for _ in range(need)]
                blocks.extend(new)
                idx = np.arange(rest, dtype=np.int32)
                out[first:] = np.asarray(new, dtype=np.int32)[idx // bs] * bs + idx % bs
                self.request_pos[request_id] = rest - (need - 1) * bs
            else:
                self.request_pos[request_id] = pos + first
            return out

    def blocks_needed(self, request_id: str, num_tokens: int) -> int:
        """New blocks a reserve(request_id, num_tokens) would take."""
        pos = self.request_pos.get(request_id, 0)
        first = min(num_tokens, self.block_size - pos) if pos < self.block_size else 0
        return (num_tokens - first + self.block_size - 1) // self.block_size

    def append(self, request_id: str, layer_idx: int, keys: torch.Tensor,
               values: torch.Tensor) -> int:
        """Reference-compatible append of [1, T, Hkv, D] keys/values for one layer.

        Layer 0 reserves T new slots; other layers write the same slots.
        mu_clamp is applied when enabled with apply_to_kv_cache, as in
        cache.py:342-355.  This API path is a convenience for callers of the
        reference interface; the forward step writes the cache with the
        fused RoPE+append kernel instead.  Returns the sequence length, or
        -1 on failure."""
        with self._lock:
            if request_id not in self.request_blocks:
                return -1
            T = keys.shape[1]
            slots = self._pending.get(request_id)
            if layer_idx == 0 or slots is None or len(slots) != T:
                slots = self.reserve(request_id, T)
                if slots is None:
                    return -1
                self._pending[request_id] = slots
            if self.mu_config.enabled and self.mu_config.apply_to_kv_cache:
                c = self.mu_config
                keys = mu_clamp(keys, c.mu, c.clamp_min, c.clamp_max)
                values = mu_clamp(values, c.mu, c.clamp_min, c.clamp_max)
            s = torch.as_tensor(slots, dtype=torch.long, device=self.block_pool.device)
            blk, off = s // self.block_size, s % self.block_size
            self.block_pool[layer_idx, 0, blk, :, off] = keys[0].to(self.dtype)
            self.block_pool[layer_idx, 1, blk, :, off] = values[0].to(self.dtype)
            return self.get_seq_len(request_id)

    def get(self, request_id: str, layer_idx: int
            ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """All cached K, V of a request/layer as [1, T, Hkv, D] (cache.py:377-413)."""
        with self._lock:
            blocks = self.request_blocks.get(request_id)
            if not blocks:
                return None, None
            n = self.get_seq_len(request_id)
            if n == 0:
                return None, None
            idx = torch.as_tensor(blocks, dtype=torch.long, device=self.block_pool.device)
            k = self.block_pool[layer_idx, 0, idx].transpose(1, 2).reshape(-1, self.num_kv_heads,
                                                                           self.head_dim)[:n]
            v = self.block_pool[layer_idx, 1, idx].transpose(1, 2).reshape(-1, self.num_kv_heads,
                                                                           self.head_dim)[:n]
            return k.unsqueeze(0), v.unsqueeze(0)

    def get_seq_len(self, request_id: str) -> int:
        with self._lock:
            blocks = self.request_blocks.get(request_id)
            if not blocks:
                return 0
            return (len(blocks) - 1) * self.block_size + self.request_pos[request_id]

    def block_table(self, request_id: str) -> List[int]:
        return self.request_blocks.get(request_id, [])

    def free(self, request_id: str) -> None:
        with self._lock:
            self.free_blocks.extend(self.request_blocks.pop(request_id, []))
            self.request_pos.pop(request_id, None)
            self._pending.pop(request_id, None)

    def clear(self) -> None:
        with self._lock:
            self.request_blocks.clear()
            self.request_pos.clear()
            self._pending.clear()
            self.free_blocks = list(range(self.max_num_blocks))

    def get_stats(self) -> dict:
        with self._lock:
            used = self.max_num_blocks - len(self.free_blocks)
            return {
                "type": "paged",
                "active_requests": len(self.request_blocks),
                "used_blocks": used,
                "free_blocks": len(self.free_blocks),
                "max_blocks": self.max_num_blocks,
                "block_size": self.block_size,
                "total_tokens": sum(self.get_seq_len(r) for r in self.request_blocks),
                "utilization": used / self.max_num_blocks if self.max_num_blocks else 0,
                "memory_mb": self.block_pool.numel() * self.block_pool.element_size() / 2**20,
            }


# Reference class name kept for drop-in callers.
MuPagedCache = PagedKVCache


def create_cache(config, num_layers: int, num_kv_heads: int, head_dim: int, device: str = "cuda",
                 mu_config: Optional[MuConfig] = None, dtype: Optional[torch.dtype] = None):
    """Factory mirroring cache.py:465-515.  Only the paged cache exists here:
    the dense MuKVCache alternative is not on the paged forward path."""
    if not config.use_paged:
        raise NotImplementedError("mu_b200 implements the paged KV cache only (use_paged=True)")
    dtype_map = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
    dt = dtype or dtype_map.get(config.dtype, torch.bfloat16)
    nblocks = config.num_gpu_blocks or config.max_num_blocks
    return PagedKVCache(num_layers, num_kv_heads, head_dim, config.block_size, nblocks, dt, device,
                        mu_config)
