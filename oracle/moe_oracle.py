"""CPU oracle for the DistributedMoE MoE-layer hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``distributedmoe_b200``) may import
this module; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, and only as the checker or as the timed CPU baseline.

It restates, with torch CPU ops, the algorithm of the reference path
(slivanovich/DistributedMoE, ``src/python``):

* routing              -- ``MoE/DistMoEBlock.py:553-562`` (gate, fp32 softmax, top-k, cast)
* per-expert grouping  -- ``MoE/DistMoEBlock.py:568-605`` (one-hot mask, ``torch.where``:
                          slot-major, token-ascending order within an expert)
* dispatch packing     -- ``MoE/PipelineTask.py:162-218`` (block list order, capacity,
                          optional alignment by bisect, uint16 packet fields)
* expert grouped MLP   -- ``MoE/PipelineTask.py:478-520`` (``grouped_mm`` x3, act*mul)
* combine              -- ``MoE/PipelineTask.py:322-346`` (weighted ``scatter_add_``)
* local reference      -- ``MoE/tests/dist_moe_test.py:173-197`` (``local_experts``)

Extensions that the reference does not have (top-k renormalisation, SiLU activation, the
sigmoid / group-limited / biased / scaled router of DeepSeek-V3, Zipf logit bias) are
switches here, written from the published method descriptions and labelled as
extensions.  With the switches off, the oracle follows the reference exactly.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own code on CPU (with
stubs for its absent transfer libraries) and ``tests/test_oracle_golden.py`` checks this
module against those vectors.
"""

from __future__ import annotations

import bisect
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

ACT_RELU = 0
ACT_SILU = 1

ROUTER_SOFTMAX = 0
ROUTER_SIGMOID_GROUP = 1


# ---------------------------------------------------------------------------------------
# routing
# ---------------------------------------------------------------------------------------
def router_logits(x: torch.Tensor, w_r: torch.Tensor, *, fp32_logits: bool = True,
                  logit_bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``router_logits = self.gate(input_batch)`` (``MoE/DistMoEBlock.py:556``; gate defined at
    ``:134`` as ``nn.Linear(d, E, bias=False)``).

    With ``fp32_logits`` the product is taken in fp32 (the operands are upcast exactly), which
    is the router the benchmark configurations ask for; otherwise the logits are in the model
    dtype, as the reference computes them.  ``logit_bias`` (shape [E]) models the
    ``nn.Linear(d, E, bias=True)`` gate replacement that the reference documents at ``:133``
    (used for the skewed-load Zipf bias)."""
    if fp32_logits:
        logits = x.float() @ w_r.float().t()
        if logit_bias is not None:
            logits = logits + logit_bias.float()
    else:
        logits = F.linear(x, w_r, None if logit_bias is None else logit_bias.to(x.dtype))
    return logits


def route(logits: torch.Tensor, top_k: int, out_dtype: torch.dtype, *, mode: int = ROUTER_SOFTMAX,
          renormalize: bool = False, score_bias: Optional[torch.Tensor] = None,
          scale: float = 1.0, n_group: int = 1, topk_group: int = 1) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k selection; returns (weights [T,k] out_dtype, selected_experts [T,k] int64).

    ``mode == ROUTER_SOFTMAX`` with ``renormalize=False, scale=1`` is the reference:
    ``softmax(logits, dtype=float)`` -> ``torch.topk`` -> ``.to(dtype)``
    (``MoE/DistMoEBlock.py:557-562``).  Renormalisation divides the k selected fp32
    probabilities by their sum before the cast (extension).

    ``mode == ROUTER_SIGMOID_GROUP`` is the DeepSeek-V3 router (extension, from the
    published description): scores = sigmoid(logits); selection uses scores + bias;
    experts are split in ``n_group`` groups, a group's score is the sum of its two best
    biased scores, the best ``topk_group`` groups are kept, and the top-k biased scores
    among the kept experts are selected; the weights are the unbiased scores of the
    selected experts, optionally renormalised, times ``scale``."""
    if mode == ROUTER_SOFTMAX:
        probs = F.softmax(logits.float(), dim=1, dtype=torch.float)
        weights, selected = torch.topk(probs, top_k, dim=-1)
        if renormalize:
            weights = weights / weights.sum(dim=-1, keepdim=True)
        if scale != 1.0:
            weights = weights * scale
        return weights.to(out_dtype), selected
    if mode == ROUTER_SIGMOID_GROUP:
        T, E = logits.shape
        scores = torch.sigmoid(logits.float())
        biased = scores + (score_bias.float() if score_bias is not None else 0.0)
        per_group = E // n_group
        grouped = biased.view(T, n_group, per_group)
        group_score = grouped.topk(2, dim=-1).values.sum(dim=-1)             # [T, n_group]
        keep_groups = group_score.topk(topk_group, dim=-1).indices           # [T, topk_group]
        group_mask = torch.zeros(T, n_group, dtype=torch.bool, device=logits.device)
        group_mask.scatter_(1, keep_groups, True)
        expert_mask = group_mask.unsqueeze(-1).expand(T, n_group, per_group).reshape(T, E)
        masked = biased.masked_fill(~expert_mask, float("-inf"))
        selected = masked.topk(top_k, dim=-1).indices
        weights = scores.gather(1, selected)
        if renormalize:
            weights = weights / weights.sum(dim=-1, keepdim=True)
        weights = weights * scale
        return weights.to(out_dtype), selected
    raise ValueError(f"unknown router mode {mode}")


# ---------------------------------------------------------------------------------------
# per-expert grouping (the routing plan)
# ---------------------------------------------------------------------------------------
@dataclass
class RoutePlan:
    """The per-expert state ``_setup_forward_pass`` builds (``MoE/DistMoEBlock.py:568-605``,
    ``MoE/DistMoE.py:23-32``), plus the concatenated permuted order."""
    experts_hit: List[int]
    counts: torch.Tensor          # [E] int64
    offsets: torch.Tensor         # [E+1] int64, exclusive prefix of counts
    perm_token: torch.Tensor      # [T*k] int64: token of each permuted activation
    perm_slot: torch.Tensor       # [T*k] int64: top-k slot of each permuted activation
    inverse: torch.Tensor         # [T, k] int64: permuted position of (token, slot)
    token_indexes: Dict[int, torch.Tensor] = field(default_factory=dict)
    weights: Dict[int, torch.Tensor] = field(default_factory=dict)


def route_plan(selected: torch.Tensor, routing_weights: torch.Tensor, num_experts: int) -> RoutePlan:
    """Per-expert activation lists exactly as ``MoE/DistMoEBlock.py:568-605`` builds them.

    ``expert_mask = one_hot(selected, E).permute(2, 1, 0)`` is [E, k, T]; for each hit expert
    ``torch.where(expert_mask[e])`` yields (slot, token) pairs in row-major order, i.e.
    slot-major and token-ascending within a slot; the expert's weights are
    ``routing_weights[token, slot]``.  The top_k == 1 branch (``:606-632``) yields the same
    lists.  The permuted order concatenates the experts in index order."""
    T, k = selected.shape
    expert_mask = F.one_hot(selected, num_classes=num_experts).permute(2, 1, 0)
    hit = torch.greater(expert_mask.sum(dim=(-1, -2)), 0).nonzero().flatten().tolist()
    counts = torch.zeros(num_experts, dtype=torch.int64)
    perm_token, perm_slot = [], []
    token_indexes: Dict[int, torch.Tensor] = {}
    weights: Dict[int, torch.Tensor] = {}
    for e in range(num_experts):
        if e in hit:
            slot, tok = torch.where(expert_mask[e])
            token_indexes[e] = tok
            weights[e] = routing_weights[tok, slot, None]
            counts[e] = tok.numel()
            perm_token.append(tok)
            perm_slot.append(slot)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    pt = torch.cat(perm_token) if perm_token else torch.zeros(0, dtype=torch.int64)
    ps = torch.cat(perm_slot) if perm_slot else torch.zeros(0, dtype=torch.int64)
    inverse = torch.empty(T, k, dtype=torch.int64)
    inverse[pt, ps] = torch.arange(pt.numel(), dtype=torch.int64)
    return RoutePlan(hit, counts, offsets, pt, ps, inverse, token_indexes, weights)


def route_plan_fast(selected: torch.Tensor, num_experts: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Vectorised equivalent of :func:`route_plan` (``MoE/DistMoEBlock.py:568-605``) for large
    inputs: a stable sort of the slot-major flattened (slot, token) list by expert.  Returns (counts, offsets,
    perm_token, perm_slot)."""
    T, k = selected.shape
    flat = selected.t().reshape(-1)                                   # slot-major order
    order = torch.sort(flat, stable=True).indices
    perm_token = order % T
    perm_slot = order // T
    counts = torch.bincount(flat, minlength=num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    return counts, offsets, perm_token, perm_slot


# ---------------------------------------------------------------------------------------
# dispatch packing (host side of HostPipelineTask.dispatch)
# ---------------------------------------------------------------------------------------
def alignment_candidates(io_buffer_size: int) -> List[int]:
    """``MoE/DistMoEBlock.py:262-265``: multiples of io_buffer_size // 1024, then the size."""
    step = io_buffer_size // 1024
    out = list(range(step, io_buffer_size, step))
    out.append(io_buffer_size)
    return out


@dataclass
class PackedTask:
    """One host task's packing (``MoE/PipelineTask.py:137-218``)."""
    block: int
    # (expert, buffer_offset, padded_size, actual_size, expert_offset_l)
    segments: List[Tuple[int, int, int, int, int]]
    used_activations: int


def pack_dispatch(block_experts: Sequence[int], experts_hit: Sequence[int],
                  expert_offsets: Dict[int, List[Tuple[int, int]]], buffer_size: int,
                  candidates: Optional[List[int]]) -> List[Tuple[int, int, int, int, int]]:
    """One task's packing loop, ``MoE/PipelineTask.py:162-218``.

    ``expert_offsets[e]`` is the FIFO of pending (l, r) segments of expert e (mutated).
    Returns (expert, buffer_offset, padded_size, actual_size, l) per packed segment."""
    used_padded = 0
    segs = []
    hit = set(experts_hit)
    for e in block_experts:
        if e not in hit:
            continue
        if used_padded >= buffer_size:
            break
        q = expert_offsets[e]
        if not q:
            continue
        l, r = q.pop(0)
        remaining = buffer_size - used_padded
        actual = min(r - l, remaining)
        size = actual
        if size <= 0:
            q.append((l, r))
            continue
        if candidates is not None and len(candidates) > 0:
            i = bisect.bisect_left(candidates, actual)
            if i < len(candidates):
                opt = candidates[i]
                if opt > remaining:
                    q.append((l, r))
                    continue
                size = opt
            else:
                q.append((l, r))
                continue
        segs.append((e, used_padded, size, actual, l))
        used_padded += size
        q.append((l + actual, r))
    return segs


def plan_forward_tasks(counts: Sequence[int], expert_blocks: Sequence[Sequence[int]], buffer_size: int,
                       top_k: int, num_tokens: int, using_alignment: bool = False,
                       alive: Optional[Sequence[bool]] = None) -> List[PackedTask]:
    """The dispatch waves of ``DistMoEBlock.async_forward`` (``MoE/DistMoEBlock.py:701-718``)
    with blocks chosen FIFO round-robin among alive blocks (``MoE/pools/ExpertBlocksPool.py:37-49``;
    ``MoE/PipelineTask.py:137-145``), assuming every task completes.  Tasks that pack nothing
    are skipped, as ``MoE/PipelineTask.py:277-279`` does."""
    E = len(counts)
    hit = [e for e in range(E) if counts[e] > 0]
    offsets = {e: [(0, int(counts[e]))] for e in hit}
    cands = alignment_candidates(buffer_size) if using_alignment else None
    total = top_k * num_tokens
    alive = list(alive) if alive is not None else [True] * len(expert_blocks)
    rr = [b for b in range(len(expert_blocks)) if alive[b]]
    transferred = 0
    tasks: List[PackedTask] = []
    stall = 0
    while transferred < total:
        # A wave creates all its tasks before any of them runs (MoE/DistMoEBlock.py:638-668),
        # so every task of the wave takes (and rotates) a block even when it packs nothing.
        n_disp = max(-(-(total - transferred) // buffer_size), 1)
        progressed = False
        for _ in range(n_disp):
            b = rr.pop(0)
            rr.append(b)
            segs = pack_dispatch(expert_blocks[b], hit, offsets, buffer_size, cands)
            used = sum(s[3] for s in segs)
            if segs:
                tasks.append(PackedTask(b, segs, used))
                transferred += used
                progressed = progressed or used > 0
        stall = 0 if progressed else stall + 1
        if stall > len(expert_blocks) + 1:
            raise RuntimeError("dispatch packing made no progress")
    return tasks


def encode_dispatch_packet(task_name: bytes, using_grouped_gemm: bool,
                           segs: Sequence[Tuple[int, int, int, int, int]],
                           in_id: bytes, out_id: bytes) -> List[Tuple[int, bytes]]:
    """DispatchSubmit body, ``MoE/PipelineTask.py:125-150,208-210,262-263``."""
    import struct
    body: List[Tuple[int, bytes]] = [(len(task_name), task_name), (1, struct.pack("!B", int(using_grouped_gemm))),
                                     (2, struct.pack("!H", len(segs)))]
    for e, off, size, _actual, _l in segs:
        body += [(2, struct.pack("!H", e)), (2, struct.pack("!H", off)), (2, struct.pack("!H", size))]
    body += [(len(in_id), in_id), (len(out_id), out_id)]
    return body


def serialize_p2p_packet(header: int, body) -> bytes:
    """``TensorTransferEngine/TensorTransferEngine.py:194-207``."""
    import struct
    parts = [struct.pack("!H", header)]
    if isinstance(body, list):
        parts.append(struct.pack("!H", len(body)))
        for size, meta in body:
            parts.append(struct.pack("!H", size))
            parts.append(meta)
    else:
        parts.append(struct.pack("!H", 1))
        parts.append(struct.pack("!H", body[0]))
        parts.append(body[1])
    return b"".join(parts)


# ---------------------------------------------------------------------------------------
# expert compute and combine
# ---------------------------------------------------------------------------------------
def _act(g: torch.Tensor, act: int) -> torch.Tensor:
    """The expert activation: ReLU as the reference's expert (``MoE/MoE.py:25-28``), or SiLU
    (SwiGLU extension)."""
    return F.relu(g) if act == ACT_RELU else F.silu(g)


def expert_grouped_mlp(X: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor, down_w: torch.Tensor,
                       seg_expert: Sequence[int], seg_end: Sequence[int], act: int = ACT_RELU) -> torch.Tensor:
    """Grouped path of ``ExpertsBlockPipelineTask.run`` (``MoE/PipelineTask.py:478-520``).

    ``gate_w, up_w`` are the stacked ``[E, I, d]`` projections and ``down_w`` ``[E, d, I]``
    (``MoE/DistExpertsBlock.py:168-177``); ``seg_end`` are the cumulative (padded) ends
    (``offs``).  Rows beyond ``seg_end[-1]`` are not computed.  Computation is in the dtype of
    X like the reference's ``grouped_mm`` (fp32 accumulation inside the library)."""
    n = int(seg_end[-1]) if len(seg_end) else 0
    if n == 0:
        return X[:0].clone()
    pos = list(seg_expert)
    offs = torch.tensor(list(seg_end), dtype=torch.int32)
    g = torch.nn.functional.grouped_mm(X[:n], gate_w[pos].transpose(1, 2), offs=offs)
    u = torch.nn.functional.grouped_mm(X[:n], up_w[pos].transpose(1, 2), offs=offs)
    h = _act(g, act) * u
    return torch.nn.functional.grouped_mm(h, down_w[pos].transpose(1, 2), offs=offs)


def quantize_rows_e4m3(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Row-wise e4m3 quantisation of the 8-bit expert path: s = amax(|row|) / 448 (1 for a
    zero row), q = round-to-nearest-even(x / s) saturated to +-448, in fp32 on the CPU.  The
    reference's benchmark only casts tensors to an 8-bit float (precision "fp8",
    ``MoE/benchmarks/bench.py:184-185``); the scales are this implementation's, so the pin is
    torch's own e4m3 rounding."""
    xf = x.float().cpu()
    s = xf.abs().amax(-1) / 448.0
    s = torch.where(s > 0, s, torch.ones_like(s))
    q = (xf / s[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q, s


def dequantize_rows_e4m3(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """q * s[row] in fp32."""
    return q.float() * s[..., None]


def expert_mlp_fp32(X: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor, act: int) -> torch.Tensor:
    """One expert ``down(act(gate(x)) * up(x))`` (``MoE/MoE.py:27-28``) in fp32."""
    X = X.float()
    return (_act(X @ wg.float().t(), act) * (X @ wu.float().t())) @ wd.float().t()


def combine_task(output_batch: torch.Tensor, out_buf: torch.Tensor, snapshots: Sequence[Tuple[int, int, int, int]],
                 token_indexes: Dict[int, torch.Tensor], weights: Dict[int, torch.Tensor]) -> None:
    """``HostPipelineTask.combine`` (``MoE/PipelineTask.py:322-346``): for each snapshot
    (expert, expert_offset, padded_size, actual_size) scatter-add weighted rows; the buffer
    offset advances by the padded size."""
    o = 0
    for e, l, padded, actual in snapshots:
        tok = token_indexes[e][l:l + actual]
        src = out_buf[o:o + actual] * weights[e][l:l + actual]
        output_batch.scatter_add_(0, tok.unsqueeze(-1).expand(-1, output_batch.size(-1)), src)
        o += padded


# ---------------------------------------------------------------------------------------
# whole layer
# ---------------------------------------------------------------------------------------
def moe_forward_reference_order(x: torch.Tensor, w_r: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor,
                                down_w: torch.Tensor, top_k: int, expert_blocks: Sequence[Sequence[int]],
                                io_buffer_size: int, *, using_alignment: bool = False, act: int = ACT_RELU,
                                fp32_logits: bool = False, renormalize: bool = False,
                                logits: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The layer as the reference's distributed path computes it, in its own arithmetic
    order: routing, packed dispatch tasks, grouped MLP per task, per-task weighted
    scatter-add in the model dtype (``MoE/DistMoEBlock.py:553`` zero-initialises the output
    in dtype).  Block-local stacks: expert e of block b is ``gate_w[e]`` etc."""
    dtype = x.dtype
    T = x.shape[0]
    E = gate_w.shape[0]
    if logits is None:
        logits = router_logits(x, w_r, fp32_logits=fp32_logits)
    rw, sel = route(logits, top_k, dtype, renormalize=renormalize)
    plan = route_plan(sel, rw, E)
    tasks = plan_forward_tasks(plan.counts.tolist(), expert_blocks, io_buffer_size, top_k, T, using_alignment)
    out = torch.zeros(T, x.shape[1], dtype=dtype)
    for task in tasks:
        buf = torch.zeros(io_buffer_size, x.shape[1], dtype=dtype)
        seg_expert, seg_end = [], []
        for e, off, size, actual, l in task.segments:
            buf[off:off + actual] = x[plan.token_indexes[e][l:l + actual]]
            seg_expert.append(e)
            seg_end.append(off + size)
        y = expert_grouped_mlp(buf, gate_w, up_w, down_w, seg_expert, seg_end, act)
        ybuf = torch.zeros_like(buf)
        ybuf[:y.shape[0]] = y
        combine_task(out, ybuf, [(e, l, size, actual) for e, off, size, actual, l in task.segments],
                     plan.token_indexes, plan.weights)
    return out


def local_experts(x: torch.Tensor, logits: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor,
                  down_w: torch.Tensor, top_k: int, *, act: int = ACT_RELU, renormalize: bool = False,
                  mode: int = ROUTER_SOFTMAX, score_bias: Optional[torch.Tensor] = None, scale: float = 1.0,
                  n_group: int = 1, topk_group: int = 1, shared: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
                  compute_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``local_experts`` (``MoE/tests/dist_moe_test.py:173-197``): per hit expert, run the MLP
    on its tokens, weight, ``index_add_`` into a zero output in the model dtype.

    ``compute_dtype=torch.float32`` gives the fp32 reference used for bf16 tolerance checks:
    the MLP and the accumulation run in fp32 on the same (bf16-valued) operands, the routing
    weights are the fp32 weights (before the cast).  ``shared`` adds an always-on shared
    expert (DeepSeek-V3 extension) with weight 1."""
    dtype = x.dtype if compute_dtype is None else compute_dtype
    E = gate_w.shape[0]
    rw, sel = route(logits, top_k, dtype if compute_dtype is None else torch.float32, mode=mode,
                    renormalize=renormalize, score_bias=score_bias, scale=scale, n_group=n_group, topk_group=topk_group)
    out = torch.zeros(x.shape, dtype=dtype, device=x.device)
    xin = x.to(dtype)
    mask = F.one_hot(sel, num_classes=E).permute(2, 1, 0)
    hit = torch.greater(mask.sum(dim=(-1, -2)), 0).nonzero().flatten().tolist()
    for e in hit:
        slot, tok = torch.where(mask[e])
        xe = xin[tok]
        if compute_dtype is None:
            ye = F.linear(_act(F.linear(xe, gate_w[e]), act) * F.linear(xe, up_w[e]), down_w[e])
        else:
            ye = expert_mlp_fp32(xe, gate_w[e], up_w[e], down_w[e], act)
        out.index_add_(0, tok, (ye * rw[tok, slot, None]).to(dtype))
    if shared is not None:
        sg, su, sd = shared
        if compute_dtype is None:
            out = out + F.linear(_act(F.linear(xin, sg), act) * F.linear(xin, su), sd)
        else:
            out = out + expert_mlp_fp32(xin, sg, su, sd, act)
    return out


def combine_from_permuted(y_perm: torch.Tensor, inverse: torch.Tensor, weights: torch.Tensor,
                          out_dtype: torch.dtype) -> torch.Tensor:
    """Gather form of the combine: out[t] = sum_s w[t,s] * y_perm[inverse[t,s]] in fp32, cast
    once.  Equal to the reference's weighted scatter-add (``MoE/PipelineTask.py:326-346``) up
    to summation order."""
    T, k = inverse.shape
    acc = torch.zeros(T, y_perm.shape[1], dtype=torch.float32)
    for s in range(k):
        acc += y_perm[inverse[:, s]].float() * weights[:, s:s + 1].float()
    return acc.to(out_dtype)
