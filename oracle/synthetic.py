"""Seeded synthetic MoE-layer inputs (test infrastructure, CPU generator).

The reference ships no data: its tests draw unseeded ``torch.randn`` inputs
(``MoE/tests/dist_moe_test.py:211,483``).  The workloads here are seeded stand-ins with the
shapes and distributions of the benchmark configurations: activations N(0, x_std),
router and expert weights N(0, w_std).  A CPU ``torch.Generator`` makes them identical on
every machine with the same torch version.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class LayerInputs:
    x: torch.Tensor        # [T, d]
    w_r: torch.Tensor      # [E, d]   router (nn.Linear(d, E).weight)
    gate: torch.Tensor     # [E, I, d] gate_proj.weight per expert
    up: torch.Tensor       # [E, I, d] up_proj.weight per expert
    down: torch.Tensor     # [E, d, I] down_proj.weight per expert


def make_layer_inputs(T: int, d: int, E: int, I: int, seed: int, dtype: torch.dtype = torch.float32,
                      x_std: float = 1.0, w_std: float = 0.02, x_mean: float = 0.0,
                      r_std: Optional[float] = None) -> LayerInputs:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, d, generator=g) * x_std + x_mean
    w_r = torch.randn(E, d, generator=g) * (w_std if r_std is None else r_std)
    gate = torch.randn(E, I, d, generator=g) * w_std
    up = torch.randn(E, I, d, generator=g) * w_std
    down = torch.randn(E, d, I, generator=g) * w_std
    return LayerInputs(x.to(dtype), w_r.to(dtype), gate.to(dtype), up.to(dtype), down.to(dtype))
