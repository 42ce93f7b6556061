"""Protocol identifiers and per-expert routing metadata (reference ``MoE/DistMoE.py:9-32``)."""

from __future__ import annotations

from collections import deque
from enum import Enum
from typing import Any, Deque, List, Optional, Tuple

import torch


class P2PHeaders(Enum):  # [1000; 1999]; 4738 is reserved by the transfer engine
    Ping = 1001
    Pong = 1002
    DispatchSubmit = 1038  # from moe block
    CombineSubmit = 1039  # from moe block
    CombineRequest = 1139  # from experts block
    IOTransferDescriptorsRequest = 1200  # from experts block
    IOTransferDescriptorsSubmit = 1201  # from moe block
    HostOutputBufferUnlocked = 1432  # from experts block
    HostInputBufferUnlocked = 1587  # from experts block
    ExpertsBlockStop = 1999  # from moe block


class SegmentQueue:
    """FIFO of pending (l, r) activation segments of one expert, with the ``queue.Queue``
    methods the dispatch path uses (single event-loop thread, so no locking)."""

    __slots__ = ("_q",)

    def __init__(self, items=()):
        self._q: Deque[Tuple[int, int]] = deque(items)

    def empty(self) -> bool:
        return not self._q

    def qsize(self) -> int:
        return len(self._q)

    def get_nowait(self) -> Tuple[int, int]:
        return self._q.popleft()

    get = get_nowait

    def put_nowait(self, item: Tuple[int, int]) -> None:
        self._q.append(item)

    put = put_nowait

    def items(self) -> List[Tuple[int, int]]:
        return list(self._q)

    def has_rows(self) -> bool:
        """True if a queued segment still holds rows.  Dispatch re-queues a segment after
        taking rows from it even when it is used up (``MoE/PipelineTask.py:218``), so
        ``empty()`` alone does not mean there is work left."""
        return any(r > l for l, r in self._q)


class ExpertMetaData:
    """Per-expert routing state of one forward pass (reference dataclass, same fields).

    The token list and weights are views of the routing plan's permuted arrays
    (``expert_base`` .. ``expert_base + expert_total_activations``), materialised on first
    access so that a forward over many experts does no per-expert tensor work."""

    def __init__(self, block_indexes: List[int], expert_shared_rate: int, expert_weights: Optional[torch.Tensor],
                 expert_token_indexes: Optional[torch.Tensor], expert_total_activations: int, expert_offsets: Any):
        self.block_indexes = block_indexes
        self.expert_shared_rate = expert_shared_rate
        self._weights = expert_weights
        self._tokens = expert_token_indexes
        self.expert_total_activations = expert_total_activations
        self.expert_offsets = expert_offsets
        self.expert_base = 0
        self._plan = None

    def bind(self, plan: dict, base: int, count: int) -> None:
        self._plan = plan
        self.expert_base = base
        self.expert_total_activations = count
        self._tokens = None
        self._weights = None
        self.expert_offsets = SegmentQueue([(0, count)])

    @property
    def expert_token_indexes(self) -> torch.Tensor:
        if self._tokens is None and self._plan is not None:
            b, n = self.expert_base, self.expert_total_activations
            self._tokens = self._plan["perm_token"][b:b + n]
        return self._tokens

    @expert_token_indexes.setter
    def expert_token_indexes(self, v: torch.Tensor) -> None:
        self._tokens = v

    @property
    def expert_weights(self) -> torch.Tensor:
        if self._weights is None and self._plan is not None:
            b, n = self.expert_base, self.expert_total_activations
            self._weights = self._plan["perm_weight"][b:b + n, None]
        return self._weights

    @expert_weights.setter
    def expert_weights(self, v: torch.Tensor) -> None:
        self._weights = v
