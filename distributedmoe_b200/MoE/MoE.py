"""Expert MLP module and the single-GPU MoE block (reference ``MoE/MoE.py``).

``Qwen3MoEMLP`` keeps the reference's parameters and math, ``down(act(gate(x)) * up(x))`` with
ReLU by default (``MoE.py:10-28``).  ``Qwen3SparseMoEBlock`` is the local (no transfer engine)
layer of ``MoE.py:31-105``; here its forward is the fused kernel chain :func:`moe_layer_forward`
(router -> routing plan -> gather -> tcgen05 grouped MLP -> weighted combine), on one stream
with no host synchronisation.  Experts live in an ``nn.ModuleList`` so ``.to()`` moves them
(the reference keeps a plain list, which ``.to()`` skips).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from distributedmoe_b200 import _native as N

_ACT = {"relu": N.ACT_RELU, "silu": N.ACT_SILU}


class Qwen3MoEMLP(nn.Module):
    def __init__(self, hidden_features: int, intermediate_features: int, dtype: torch.dtype = torch.float16,
                 activation: str = "relu"):
        super().__init__()
        self.hidden_features = hidden_features
        self.intermediate_features = intermediate_features
        self.gate_proj = nn.Linear(hidden_features, intermediate_features, bias=False, dtype=dtype)
        self.up_proj = nn.Linear(hidden_features, intermediate_features, bias=False, dtype=dtype)
        self.down_proj = nn.Linear(intermediate_features, hidden_features, bias=False, dtype=dtype)
        self.activation = nn.ReLU() if activation == "relu" else nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.activation(self.gate_proj(x)) * self.up_proj(x))


def moe_layer_forward(x: torch.Tensor, w_router: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
                      down: torch.Tensor, top_k: int, *, activation: int = N.ACT_RELU, renormalize: bool = False,
                      router_mode: int = N.ROUTER_SOFTMAX, scale: float = 1.0, score_bias: Optional[torch.Tensor] = None,
                      n_group: int = 1, topk_group: int = 1, out: Optional[torch.Tensor] = None,
                      work: Optional[Dict[str, torch.Tensor]] = None) -> torch.Tensor:
    """One MoE layer on the current stream, through the library kernels only.

    x [T, d]; w_router [E, d]; gate/up [E, I, d]; down [E, d, I] (one dtype, f16 or bf16).
    The per-expert segment table for the grouped MLP stays on the device (the plan's
    offsets), so nothing synchronises with the host.  ``work`` caches the permuted buffers
    between calls of the same shape."""
    T, d = x.shape
    E = gate.shape[0]
    idx, w, _ = N.router(x, w_router, top_k, mode=router_mode, renormalize=renormalize, scale=scale,
                         score_bias=score_bias, n_group=n_group, topk_group=topk_group, w_dtype=torch.float32)
    plan = N.route_plan(idx, None, E, want_slot=False, want_weight=False)
    n = T * top_k
    if work is not None and work.get("rows") is not None and work["rows"].shape == (n, d) and work["rows"].dtype == x.dtype:
        xbuf, ybuf = work["rows"], work["out_rows"]
    else:
        xbuf = torch.empty(n, d, dtype=x.dtype, device=x.device)
        ybuf = torch.empty(n, d, dtype=x.dtype, device=x.device)
        if work is not None:
            work["rows"], work["out_rows"] = xbuf, ybuf
    N.permute_rows(x, xbuf, [0], [0], [n], row_map=plan["perm_token"])
    seg_expert = work.get("seg_expert") if work is not None else None
    if seg_expert is None or seg_expert.numel() != E or seg_expert.device != x.device:
        seg_expert = torch.arange(E, dtype=torch.int32, device=x.device)
        if work is not None:
            work["seg_expert"] = seg_expert
    N.grouped_gated_mlp(xbuf, gate, up, down, seg_expert, plan["offsets"][1:], activation, ybuf)
    if out is None:
        out = torch.empty(T, d, dtype=x.dtype, device=x.device)
    N.combine(ybuf, plan["inverse"], w, out)
    return out


class Qwen3SparseMoEBlock(nn.Module):
    def __init__(self, number_of_experts: int, top_k: int, hidden_features: int, intermediate_features: int,
                 dtype: torch.dtype = torch.float16, activation: str = "relu", renormalize: bool = False):
        super().__init__()
        self.number_of_experts = number_of_experts
        self.top_k = top_k
        self.hidden_features = hidden_features
        self.intermediate_features = intermediate_features
        self.activation = activation
        self.renormalize = renormalize
        self.gate = nn.Linear(hidden_features, number_of_experts, bias=False, dtype=dtype)
        self.experts = nn.ModuleList(Qwen3MoEMLP(hidden_features, intermediate_features, dtype, activation)
                                     for _ in range(number_of_experts))
        self._stacked: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None
        self._stacked_key = None
        self._work: Dict[str, torch.Tensor] = {}

    def stacked_weights(self) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Contiguous [E, I, d] / [E, I, d] / [E, d, I] stacks (rebuilt if a weight moved)."""
        key = tuple((m.gate_proj.weight.data_ptr(), m.up_proj.weight.data_ptr(), m.down_proj.weight.data_ptr())
                    for m in self.experts)
        if self._stacked is None or key != self._stacked_key:
            with torch.no_grad():
                self._stacked = (torch.stack([m.gate_proj.weight for m in self.experts]).contiguous(),
                                 torch.stack([m.up_proj.weight for m in self.experts]).contiguous(),
                                 torch.stack([m.down_proj.weight for m in self.experts]).contiguous())
            self._stacked_key = key
        return self._stacked

    def forward(self, input_batch: torch.Tensor, experts_latency_benchmark=None) -> torch.Tensor:
        shape = input_batch.shape
        x = input_batch.reshape(-1, self.hidden_features).contiguous()
        g, u, dn = self.stacked_weights()
        with torch.no_grad():
            y = moe_layer_forward(x, self.gate.weight.detach(), g, u, dn, self.top_k, activation=_ACT[self.activation],
                                  renormalize=self.renormalize, work=self._work)
        return y.reshape(shape)
