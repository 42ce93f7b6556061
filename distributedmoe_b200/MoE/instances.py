"""Expert instances of the device-driven (NVLinkDirect) data plane.

An instance is one copy of an expert's weights on one rank: expert block b of
``DistMoEBlockConfig.expert_blocks`` lives on rank ``block_ranks[b]`` and contributes one
instance per expert it holds (the reference places blocks on ``eb_devices``,
``MoE/DistMoEBlock.py:45,64``; an expert listed in several blocks has several instances,
which is how the reference expresses replicas, ``:199-207``).  Instances are numbered rank
by rank; inside a rank in the order of that rank's weight stack (its blocks in index order,
each block's experts in list order), so rank r owns the contiguous range
``[inst_first[r], inst_first[r+1])`` and instance i sits at stack position ``inst_slot[i]``.

Which instances a host may send to is its ``ExpertBlocksPool``'s business
(``MoE/pools/ExpertBlocksPool.py:37-71``): :meth:`InstanceTable.alive_arrays` turns the
pool's alive flags into the per-expert candidate lists the placement kernel reads.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Sequence, Tuple

from distributedmoe_b200._native import EP_MAX_INSTANCES, EP_MAX_RANKS, EP_MAX_REPLICAS


@dataclass
class InstanceTable:
    world: int
    num_experts: int
    inst_rank: List[int] = field(default_factory=list)
    inst_slot: List[int] = field(default_factory=list)
    inst_expert: List[int] = field(default_factory=list)
    inst_block: List[int] = field(default_factory=list)
    inst_first: List[int] = field(default_factory=list)

    @classmethod
    def from_blocks(cls, expert_blocks: Sequence[Sequence[int]], block_ranks: Sequence[int], world: int,
                    num_experts: int) -> "InstanceTable":
        if len(block_ranks) != len(expert_blocks):
            raise ValueError("one rank per expert block is required")
        if not 1 <= world <= EP_MAX_RANKS:
            raise ValueError(f"world size {world} not in [1, {EP_MAX_RANKS}]")
        t = cls(world, num_experts)
        for r in range(world):
            t.inst_first.append(len(t.inst_rank))
            slot = 0
            for b, experts in enumerate(expert_blocks):
                if block_ranks[b] != r:
                    continue
                for e in experts:
                    if not 0 <= e < num_experts:
                        raise ValueError(f"block {b} lists expert {e} outside [0, {num_experts})")
                    t.inst_rank.append(r)
                    t.inst_slot.append(slot)
                    t.inst_expert.append(e)
                    t.inst_block.append(b)
                    slot += 1
        t.inst_first.append(len(t.inst_rank))
        if any(not 0 <= r < world for r in block_ranks):
            raise ValueError("a block is placed on a rank outside the world")
        if not 1 <= len(t.inst_rank) <= EP_MAX_INSTANCES:
            raise ValueError(f"{len(t.inst_rank)} expert instances; 1..{EP_MAX_INSTANCES} supported")
        per_expert = [0] * num_experts
        for e in t.inst_expert:
            per_expert[e] += 1
        if max(per_expert) > EP_MAX_REPLICAS:
            raise ValueError(f"an expert has more than {EP_MAX_REPLICAS} instances")
        return t

    @property
    def n_inst(self) -> int:
        return len(self.inst_rank)

    def local_count(self, rank: int) -> int:
        return self.inst_first[rank + 1] - self.inst_first[rank]

    def local_blocks(self, rank: int) -> List[int]:
        """Blocks of `rank` in stack order (each once)."""
        out: List[int] = []
        for i in range(self.inst_first[rank], self.inst_first[rank + 1]):
            if not out or out[-1] != self.inst_block[i]:
                out.append(self.inst_block[i])
        return out

    def alive_arrays(self, alive_blocks: Sequence[bool]) -> Tuple[List[int], List[int]]:
        """(alive_n [E], alive_inst [E * EP_MAX_REPLICAS]): per expert, its instances whose
        block is alive, in instance order (unused entries 0)."""
        E = self.num_experts
        n = [0] * E
        inst = [0] * (E * EP_MAX_REPLICAS)
        for i, (e, b) in enumerate(zip(self.inst_expert, self.inst_block)):
            if alive_blocks[b]:
                inst[e * EP_MAX_REPLICAS + n[e]] = i
                n[e] += 1
        return n, inst
