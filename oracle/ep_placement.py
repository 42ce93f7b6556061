"""CPU restatement of the expert-parallel placement (test infrastructure only).

TEST INFRASTRUCTURE ONLY: only ``tests/`` use this module, as the checker of the exchange
kernels' bookkeeping (``dmoe_ep_plan`` / ``dmoe_ep_dispatch``).

The reference has no such step: its host packs tasks for one expert block at a time and
the block copies the rows it is told about (``MoE/PipelineTask.py:162-218,459``).  With
every rank dispatching at once, the rows of one expert instance from all senders must land
in one contiguous run of the owner's receive buffer.  This module states that layout in
plain Python so the device results can be compared bit for bit:

* sender r splits expert e's n_e rows (its routing-plan order) over e's alive instances:
  "rotate" sends all of them to instance ``alive[(epoch + r) % n_alive]``, "split" sends
  rows ``[q*n/na, (q+1)*n/na)`` to the q-th alive instance;
* the owner lays out its instances in stack order, and inside an instance the senders in
  rank order: sender r's rows of instance i start at
  ``sum(tot[i'] for earlier i' of that rank) + sum(M[r'][i] for r' < r)``;
* activation p of sender r (expert e, i-th row of e) goes to (rank, row) or is dropped
  when e has no alive instance.
"""

from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

POLICY_ROTATE = 0
POLICY_SPLIT = 1


def split_rows(n: int, alive: Sequence[int], policy: int, epoch: int, rank: int) -> List[Tuple[int, int, int]]:
    """(instance, first row, end row) parts of one expert's n rows for one sender."""
    na = len(alive)
    if na == 0:
        return []
    if policy == POLICY_SPLIT:
        return [(alive[q], q * n // na, (q + 1) * n // na) for q in range(na)]
    return [(alive[(epoch + rank) % na], 0, n)]


def placement(counts: Sequence[Sequence[int]], alive: Sequence[Sequence[Sequence[int]]], inst_rank: Sequence[int],
              inst_first: Sequence[int], policy: int, epoch: int, cap: int) -> Dict[str, object]:
    """counts[r][e]: sender r's rows of expert e; alive[r][e]: the instances sender r may use
    for e.  Returns send matrix M[r][i], per-rank dest_off[r][i], seg_end[g][j] and the parts
    of every sender."""
    G = len(counts)
    E = len(counts[0]) if G else 0
    n_inst = len(inst_rank)
    M = [[0] * n_inst for _ in range(G)]
    parts = [[split_rows(counts[r][e], alive[r][e], policy, epoch, r) for e in range(E)] for r in range(G)]
    for r in range(G):
        for e in range(E):
            for inst, lo, hi in parts[r][e]:
                M[r][inst] = hi - lo
    tot = [sum(M[r][i] for r in range(G)) for i in range(n_inst)]
    base = [0] * n_inst
    for g in range(len(inst_first) - 1):
        run = 0
        for i in range(inst_first[g], inst_first[g + 1]):
            base[i] = run
            run += tot[i]
    dest_off = [[min(base[i] + sum(M[q][i] for q in range(r)), cap) for i in range(n_inst)] for r in range(G)]
    seg_end = [[min(base[i] + tot[i], cap) for i in range(inst_first[g], inst_first[g + 1])]
               for g in range(len(inst_first) - 1)]
    return {"M": M, "parts": parts, "dest_off": dest_off, "seg_end": seg_end, "base": base, "tot": tot}


def destinations(plan_counts: Sequence[int], parts, inst_rank: Sequence[int], dest_off: Sequence[int],
                 cap: int) -> List[Tuple[int, int]]:
    """(rank, row) of each activation of one sender in its routing-plan order ((-1, -1) if
    dropped).  plan_counts[e]: the sender's rows of expert e (experts in index order)."""
    out: List[Tuple[int, int]] = []
    for e, n in enumerate(plan_counts):
        ps = parts[e]
        for i in range(n):
            hit = None
            for inst, lo, hi in ps:
                if lo <= i < hi:
                    hit = (inst, lo)
            if hit is None:
                out.append((-1, -1))
                continue
            inst, lo = hit
            row = dest_off[inst] + (i - lo)
            out.append((inst_rank[inst], row) if row < cap else (-1, -1))
    return out
