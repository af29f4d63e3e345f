"""mu_clamp / soft_clamp and the scalar MuDynamics controller.

Host-side counterparts of mu_inference/core/mu.py:30-304.  The tensor path
never calls these: on the GPU, mu_clamp is fused into the kernels (libmuk).
They serve the scheduler (priority smoothing) and the public API
(``from mu_b200 import mu_clamp``).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import List, Optional, Union

import torch

Number = Union[float, torch.Tensor]


def soft_clamp(value: Number, min_val: float, max_val: float) -> Number:
    """tanh((x - c)/r)·r + c, c = (max+min)/2, r = (max-min)/2; constant c if max <= min."""
    if max_val <= min_val:
        c = (max_val + min_val) / 2
        return torch.full_like(value, c) if isinstance(value, torch.Tensor) else c
    r = (max_val - min_val) * 0.5
    c = (max_val + min_val) * 0.5
    if isinstance(value, torch.Tensor):
        return torch.tanh((value - c) / r) * r + c
    return math.tanh((value - c) / r) * r + c


def mu_clamp(value: Number, mu: float = 0.0, clamp_min: float = -10.0,
             clamp_max: float = 10.0) -> Number:
    """mu + soft_clamp(value - mu, clamp_min, clamp_max)."""
    return mu + soft_clamp(value - mu, clamp_min, clamp_max)


def apply_mu_dynamics(tensor: torch.Tensor, mu: float = 0.0, clamp_min: float = -10.0,
                      clamp_max: float = 10.0, enabled: bool = True) -> torch.Tensor:
    return mu_clamp(tensor, mu, clamp_min, clamp_max) if enabled else tensor


@dataclass
class MuState:
    current_value: float = 0.0
    target_mu: float = 0.0
    velocity: float = 0.0
    acceleration: float = 0.0
    integral_error: float = 0.0
    previous_error: float = 0.0
    last_update_time: float = field(default_factory=time.time)
    value_history: List[float] = field(default_factory=list)
    max_history: int = 20


class MuDynamics:
    """EMA + velocity tracker returning mu-clamped values (mu.py:160-304)."""

    def __init__(self, mu: float = 0.0, clamp_min: float = -10.0, clamp_max: float = 10.0,
                 velocity_min: float = -10.0, velocity_max: float = 10.0, beta: float = 1.0,
                 ema_alpha: float = 0.3, enabled: bool = True):
        self.mu = mu
        self.clamp_min = clamp_min
        self.clamp_max = clamp_max
        self.velocity_min = velocity_min
        self.velocity_max = velocity_max
        self.beta = beta
        self.ema_alpha = ema_alpha
        self.enabled = enabled
        self.state = MuState(target_mu=mu)

    def update(self, new_value: float, dt: Optional[float] = None) -> float:
        if not self.enabled:
            return new_value
        now = time.time()
        if dt is None:
            dt = now - self.state.last_update_time
        if dt <= 0:
            return new_value
        st = self.state
        if st.current_value != 0:
            st.velocity = soft_clamp((new_value - st.current_value) / dt, self.velocity_min,
                                     self.velocity_max)
        st.current_value = self.ema_alpha * new_value + (1 - self.ema_alpha) * st.current_value
        st.value_history.append(new_value)
        if len(st.value_history) > st.max_history:
            st.value_history.pop(0)
        st.last_update_time = now
        return mu_clamp(st.current_value, self.mu, self.clamp_min, self.clamp_max)

    def get_equilibrium_force(self) -> float:
        dev = self.state.current_value - self.mu
        return soft_clamp(-self.beta * dev - 0.3 * self.state.velocity, -2.0, 2.0)

    def should_intervene(self) -> bool:
        if not self.enabled:
            return False
        if abs(self.state.velocity) >= self.velocity_max * 0.9:
            return True
        return abs(self.state.current_value - self.mu) > self.clamp_max * 0.8

    def reset(self) -> None:
        self.state = MuState(target_mu=self.mu)

    def get_stats(self) -> dict:
        return {
            "enabled": self.enabled,
            "mu": self.mu,
            "current_value": self.state.current_value,
            "velocity": self.state.velocity,
            "equilibrium_force": self.get_equilibrium_force(),
            "should_intervene": self.should_intervene(),
        }
