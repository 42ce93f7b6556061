"""Edge cases of the oracle's routing, packing and combine on the CPU: empty and ragged
batches, a single expert, every expert hit by every token, a segment larger than a buffer,
alignment padding, dead blocks with replicas."""

import pytest
import torch

from oracle import moe_oracle as O


@pytest.mark.parametrize("T,k,E", [(0, 2, 8), (1, 1, 1), (7, 2, 8), (333, 8, 64), (50, 4, 4)])
def test_route_plan_orders_agree(T, k, E):
    g = torch.Generator().manual_seed(T * 31 + k * 7 + E)
    logits = torch.randn(T, E, generator=g)
    w, sel = O.route(logits, k, torch.float32)
    plan = O.route_plan(sel, w, E)
    counts, offsets, pt, ps = O.route_plan_fast(sel, E)
    assert torch.equal(plan.counts, counts)
    assert torch.equal(plan.offsets, offsets)
    assert torch.equal(plan.perm_token, pt) and torch.equal(plan.perm_slot, ps)
    assert int(counts.sum()) == T * k
    if T:
        # inverse is a permutation of the T*k activations
        assert torch.equal(plan.inverse.flatten().sort().values, torch.arange(T * k))


def test_route_plan_every_expert_hit_by_every_token():
    T, E = 9, 4
    logits = torch.randn(T, E, generator=torch.Generator().manual_seed(3))
    w, sel = O.route(logits, E, torch.float32)
    plan = O.route_plan(sel, w, E)
    assert plan.counts.tolist() == [T] * E
    for e in range(E):
        toks = plan.token_indexes[e].tolist()
        assert sorted(toks) == list(range(T))  # every token once
        b = int(plan.offsets[e])
        pairs = list(zip(plan.perm_slot[b:b + T].tolist(), plan.perm_token[b:b + T].tolist()))
        assert pairs == sorted(pairs)  # slot-major, tokens ascending within a slot


def test_pack_dispatch_splits_a_segment_larger_than_the_buffer():
    offsets = {0: [(0, 10)], 1: [(0, 3)]}
    segs = O.pack_dispatch([0, 1], [0, 1], offsets, 4, None)
    assert segs == [(0, 0, 4, 4, 0)]
    assert offsets[0] == [(4, 10)] and offsets[1] == [(0, 3)]
    segs = O.pack_dispatch([0, 1], [0, 1], offsets, 8, None)
    assert segs == [(0, 0, 6, 6, 4), (1, 6, 2, 2, 0)]
    assert offsets[0] == [(10, 10)] and offsets[1] == [(2, 3)]  # used-up segment is re-queued


def test_pack_dispatch_pads_to_alignment_candidates():
    cands = O.alignment_candidates(1024 * 4)  # multiples of 4 up to 4096
    assert cands[:3] == [4, 8, 12] and cands[-1] == 4096
    offsets = {0: [(0, 5)], 1: [(0, 9)]}
    segs = O.pack_dispatch([0, 1], [0, 1], offsets, 4096, cands)
    assert segs == [(0, 0, 8, 5, 0), (1, 8, 12, 9, 0)]


def test_plan_forward_tasks_covers_every_activation_and_skips_dead_blocks():
    counts = [300, 0, 1200, 45, 700, 5, 0, 2000]
    blocks = [[0, 1, 2, 3], [4, 5, 6, 7], [0, 1, 2, 3, 4, 5, 6, 7]]
    T, k = 2125, 2
    tasks = O.plan_forward_tasks(counts, blocks, 1024, k, T)
    assert sum(t.used_activations for t in tasks) == T * k
    covered = {}
    for t in tasks:
        for e, _off, _size, actual, l in t.segments:
            covered.setdefault(e, []).append((l, l + actual))
    for e, c in enumerate(counts):
        spans = sorted(covered.get(e, []))
        assert sum(b - a for a, b in spans) == c
    dead = O.plan_forward_tasks(counts, blocks, 1024, k, T, alive=[True, False, True])
    assert all(t.block != 1 for t in dead)
    assert sum(t.used_activations for t in dead) == T * k


def test_combine_from_permuted_matches_per_expert_scatter():
    T, k, E, d = 37, 3, 6, 16
    g = torch.Generator().manual_seed(9)
    w, sel = O.route(torch.randn(T, E, generator=g), k, torch.float32)
    plan = O.route_plan(sel, w, E)
    y_perm = torch.randn(T * k, d, generator=g)
    out = O.combine_from_permuted(y_perm, plan.inverse, w, torch.float32)
    ref = torch.zeros(T, d, dtype=torch.float64)
    for e in plan.experts_hit:
        b = int(plan.offsets[e])
        rows = y_perm[b:b + int(plan.counts[e])].double()
        ref.index_add_(0, plan.token_indexes[e], rows * plan.weights[e].double())
    assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-5)


def test_nan_logit_row_routes_to_valid_experts():
    """A token whose logits hold a NaN still gets k expert indices in [0, E) from torch.topk
    (the softmax spreads the NaN over the whole row, so which k it picks is not specified);
    its weights are NaN and only its own output row turns NaN."""
    E, k = 8, 2
    logits = torch.randn(4, E)
    logits[1, 3] = float("nan")
    logits[2, :] = float("nan")
    w, sel = O.route(logits, k, torch.float32)
    assert sel.min().item() >= 0 and sel.max().item() < E
    assert torch.isnan(w[1]).all() and torch.isnan(w[2]).all()
    assert torch.isfinite(w[0]).all() and torch.isfinite(w[3]).all()
    plan = O.route_plan(sel, w, E)
    assert sorted(plan.inverse.flatten().tolist()) == list(range(4 * k))


def test_e4m3_row_quantisation_known_values():
    """The 8-bit restatement: a row whose amax is 448 keeps scale 1 and e4m3's own codes
    (448 -> 0x7e, 1.0 -> 0x38, -1.0 -> 0xb8, 2^-4 -> 0x18, the halfway 1.0625 rounds to even
    1.0); a zero row gets scale 1; another row scales its amax to 448."""
    x = torch.tensor([[448.0, 1.0, -1.0, 0.0625, 1.0625, 0.0, 0.0, 0.0],
                      [0.0] * 8,
                      [2.0, -1.0, 0.5, 0.0, 0.0, 0.0, 0.0, 0.0]])
    q, s = O.quantize_rows_e4m3(x)
    assert s.tolist() == [1.0, 1.0, torch.tensor(2.0 / 448.0, dtype=torch.float32).item()]
    codes = q.view(torch.uint8)
    assert codes[0, :5].tolist() == [0x7E, 0x38, 0xB8, 0x18, 0x38]
    assert codes[1].tolist() == [0] * 8
    assert codes[2, 0].item() == 0x7E and codes[2, 1].item() == 0xF6  # 448, -224
    back = O.dequantize_rows_e4m3(q, s)
    assert torch.allclose(back[2, :3], torch.tensor([2.0, -1.0, 0.5]), rtol=1e-6, atol=0)
