"""Alive/dead state and selection of expert blocks (reference ``MoE/pools/ExpertBlocksPool.py``).

``policy="fifo"`` (default) is the reference behaviour: a FIFO of alive block indexes;
``aquire`` pops the next index and silently drops dead ones, ``mark_alive`` re-queues a
block (``ExpertBlocksPool.py:37-62``).  ``policy="least_loaded"`` (extension) returns the
alive block with the fewest activations in flight, ties to the lower index; callers report
load with ``add_load``/``sub_load``.
"""

from __future__ import annotations

import asyncio
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple


@dataclass
class ExpertBlockMetaData:
    is_alive: bool
    alive_event: asyncio.Event
    experts_block_index: int
    expert_indexes: List[int]


class ExpertBlocksPool:
    def __init__(self, expert_blocks: List[List[int]], policy: str = "fifo") -> None:
        if policy not in ("fifo", "least_loaded"):
            raise ValueError(f"unknown expert block selection policy {policy!r}")
        self.policy = policy
        self.number_of_expert_blocks = len(expert_blocks)
        self.expert_blocks_metadata: List[ExpertBlockMetaData] = []
        self.expert_block_indexes_pool: asyncio.Queue = asyncio.Queue()
        self.load: List[int] = [0] * self.number_of_expert_blocks
        for b in range(self.number_of_expert_blocks):
            md = ExpertBlockMetaData(True, asyncio.Event(), b, list(expert_blocks[b]))
            md.alive_event.set()
            self.expert_blocks_metadata.append(md)
            self.expert_block_indexes_pool.put_nowait(b)

    async def aquire(self, candidates: Optional[Sequence[int]] = None) -> Tuple[int, ExpertBlockMetaData]:
        if self.policy == "least_loaded":
            while True:
                pool = candidates if candidates is not None else range(self.number_of_expert_blocks)
                alive = [b for b in pool if self.expert_blocks_metadata[b].alive_event.is_set()]
                if alive:
                    b = min(alive, key=lambda i: (self.load[i], i))
                    return b, self.expert_blocks_metadata[b]
                await asyncio.sleep(0.001)
        while True:
            try:
                b: int = await self.expert_block_indexes_pool.get()
            except (asyncio.QueueEmpty, AttributeError):
                raise RuntimeError("Expert blocks async queue is corrupted.")
            md = self.expert_blocks_metadata[b]
            if md.alive_event.is_set():
                return b, md

    # the reference spells it "aquire"; both names work
    acquire = aquire

    def release(self, experts_block_index: int) -> None:
        if self.policy == "fifo" and self.expert_blocks_metadata[experts_block_index].alive_event.is_set():
            self.expert_block_indexes_pool.put_nowait(experts_block_index)

    def add_load(self, experts_block_index: int, n: int) -> None:
        self.load[experts_block_index] += n

    def sub_load(self, experts_block_index: int, n: int) -> None:
        self.load[experts_block_index] = max(0, self.load[experts_block_index] - n)

    def mark_alive(self, experts_block_index: int) -> None:
        md = self.expert_blocks_metadata[experts_block_index]
        if not md.alive_event.is_set():
            md.alive_event.set()
            if self.policy == "fifo":
                self.expert_block_indexes_pool.put_nowait(experts_block_index)
        md.is_alive = True

    def mark_dead(self, experts_block_index: int) -> None:
        md = self.expert_blocks_metadata[experts_block_index]
        if md.alive_event.is_set():
            md.alive_event.clear()
        md.is_alive = False

    def close(self) -> None:
        while not self.expert_block_indexes_pool.empty():
            try:
                b = self.expert_block_indexes_pool.get_nowait()
                self.expert_blocks_metadata[b].alive_event.clear()
            except Exception:
                break
