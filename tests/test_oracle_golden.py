"""The oracle restatement checked against golden vectors made by the reference's own code.

The fixtures in ``tests/golden/`` come from ``tests/golden/make_golden.py``, which runs the
reference's ``_setup_forward_pass``, ``HostPipelineTask.dispatch/combine`` and
``ExpertsBlockPipelineTask.run`` on CPU.  These tests need no GPU.
"""

import glob
import os
import struct

import pytest
import torch

from oracle import moe_oracle as O
from oracle.synthetic import make_layer_inputs

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAMES = sorted(os.path.basename(p)[:-3] for p in glob.glob(os.path.join(GOLDEN, "*.pt")))
DT = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16}


def _load(name):
    return torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)


def _inputs(cfg):
    return make_layer_inputs(cfg["T"], cfg["d"], cfg["E"], cfg["I"], cfg["seed"], DT[cfg["dtype"]])


def test_fixtures_present():
    assert {"tiny_e8k2", "split_2blocks", "align_pad", "topk1", "replicas", "e16k4_sparse", "bf16_small",
            "silu_ext", "plumbing"} <= set(NAMES)


@pytest.mark.parametrize("name", NAMES)
def test_routing_matches_reference(name):
    g = _load(name)
    cfg = g["config"]
    inp = _inputs(cfg)
    dtype = DT[cfg["dtype"]]
    logits = O.router_logits(inp.x, inp.w_r, fp32_logits=False)
    if g["logits"] is not None:
        assert torch.equal(logits, g["logits"])
    else:
        assert torch.equal(logits[::8], g["logits_rows"])
    w, sel = O.route(logits, cfg["k"], dtype)
    assert torch.equal(sel, g["selected"])
    assert torch.equal(w, g["routing_weights"].to(dtype))
    plan = O.route_plan(sel, w, cfg["E"])
    assert plan.experts_hit == g["experts_hit"]
    for e, pe in g["per_expert"].items():
        assert torch.equal(plan.token_indexes[e], pe["tokens"]), f"expert {e} token order"
        assert torch.equal(plan.weights[e].flatten(), pe["weights"])
    # The vectorised plan gives the same permutation.
    counts, offsets, pt, ps = O.route_plan_fast(sel, cfg["E"])
    assert torch.equal(counts, plan.counts)
    assert torch.equal(pt, plan.perm_token) and torch.equal(ps, plan.perm_slot)


@pytest.mark.parametrize("name", NAMES)
def test_dispatch_packing_matches_reference(name):
    g = _load(name)
    cfg = g["config"]
    counts = [0] * cfg["E"]
    for e, pe in g["per_expert"].items():
        counts[e] = pe["tokens"].numel()
    tasks = O.plan_forward_tasks(counts, cfg["blocks"], cfg["io"], cfg["k"], cfg["T"], cfg["align"])
    assert len(tasks) == len(g["tasks"])
    for mine, ref in zip(tasks, g["tasks"]):
        assert mine.block == ref["block"]
        assert [(e, off, size) for e, off, size, _a, _l in mine.segments] == [tuple(s) for s in ref["packet_segments"]]
        assert [(e, l, size, a) for e, _o, size, a, l in mine.segments] == [tuple(s) for s in ref["snapshot"]]
        assert mine.used_activations == ref["used"]
        # The DispatchSubmit wire format, minus the random task name and the buffer ids.
        name_len = 8
        body = O.encode_dispatch_packet(ref["packet"][6:6 + name_len], True, mine.segments,
                                        ref["packet"][-2:], ref["packet"][-2:])
        pkt = O.serialize_p2p_packet(1038, body)
        assert pkt[:-8] == ref["packet"][:-8]


@pytest.mark.parametrize("name", [n for n in NAMES if n != "plumbing"])
def test_task_buffers_match_reference(name):
    """Gathered input rows and grouped-MLP output rows of each task, when the fixture keeps them."""
    g = _load(name)
    cfg = g["config"]
    if "in_rows" not in g["tasks"][0]:
        pytest.skip("fixture keeps no buffer rows")
    inp = _inputs(cfg)
    dtype = DT[cfg["dtype"]]
    logits = O.router_logits(inp.x, inp.w_r, fp32_logits=False)
    w, sel = O.route(logits, cfg["k"], dtype)
    plan = O.route_plan(sel, w, cfg["E"])
    act = O.ACT_SILU if cfg["act"] == "silu" else O.ACT_RELU
    for tr in g["tasks"]:
        blk = cfg["blocks"][tr["block"]]
        used = sum(s[2] for s in tr["packet_segments"])
        buf = torch.zeros(used, cfg["d"], dtype=dtype)
        pos, ends = [], []
        for (e, off, size), (_e, l, _s, actual) in zip(tr["packet_segments"], tr["snapshot"]):
            buf[off:off + actual] = inp.x[plan.token_indexes[e][l:l + actual]]
            pos.append(blk.index(e))
            ends.append(off + size)
        assert torch.equal(buf, tr["in_rows"])
        stack_g = inp.gate[blk]
        stack_u = inp.up[blk]
        stack_d = inp.down[blk]
        y = O.expert_grouped_mlp(buf, stack_g, stack_u, stack_d, pos, ends, act)
        assert torch.equal(y, tr["out_rows"])


@pytest.mark.parametrize("name", NAMES)
def test_layer_output_matches_reference(name):
    g = _load(name)
    cfg = g["config"]
    inp = _inputs(cfg)
    act = O.ACT_SILU if cfg["act"] == "silu" else O.ACT_RELU
    if len(cfg["blocks"]) == 1 and cfg["blocks"][0] == list(range(cfg["E"])):
        out = O.moe_forward_reference_order(inp.x, inp.w_r, inp.gate, inp.up, inp.down, cfg["k"], cfg["blocks"],
                                            cfg["io"], using_alignment=cfg["align"], act=act)
        ref = g["output"]
        if name == "plumbing":
            assert torch.equal(out[::8], ref)
            assert torch.allclose(out.double().sum(1), g["output_row_sum"], rtol=0, atol=1e-9)
        else:
            assert torch.equal(out, ref)
    # local_experts restatement against the reference's local_experts
    logits = O.router_logits(inp.x, inp.w_r, fp32_logits=False)
    loc = O.local_experts(inp.x, logits, inp.gate, inp.up, inp.down, cfg["k"], act=act)
    if name == "plumbing":
        loc = loc[::8]
    assert torch.equal(loc, g["local"])


def test_fp32_reference_close_to_plumbing_output():
    """The fp32 compute path used as the bf16 tolerance reference agrees with the fp32 layer."""
    g = _load("plumbing")
    cfg = g["config"]
    inp = _inputs(cfg)
    logits = O.router_logits(inp.x, inp.w_r, fp32_logits=False)
    loc = O.local_experts(inp.x, logits, inp.gate, inp.up, inp.down, cfg["k"], compute_dtype=torch.float32)
    assert torch.allclose(loc[::8], g["output"], atol=1e-5, rtol=1e-5)


def test_deepseek_router_properties():
    """Extension (DeepSeek-V3 router): selections stay inside the kept groups; weights renormalise to scale."""
    T, E, k = 64, 256, 8
    gen = torch.Generator().manual_seed(2)
    logits = torch.randn(T, E, generator=gen)
    bias = torch.randn(E, generator=gen) * 0.01
    w, sel = O.route(logits, k, torch.float32, mode=O.ROUTER_SIGMOID_GROUP, renormalize=True, score_bias=bias,
                     scale=2.5, n_group=8, topk_group=4)
    assert torch.allclose(w.sum(-1), torch.full((T,), 2.5), atol=1e-5)
    groups = sel // (E // 8)
    assert all(len(set(r.tolist())) <= 4 for r in groups)
    # Each selection is among the best biased scores of the kept groups.
    s = torch.sigmoid(logits) + bias
    for t in range(4):
        kept = set(groups[t].tolist())
        cand = sorted([(s[t, e].item(), e) for e in range(E) if e // 32 in kept], reverse=True)
        assert set(sel[t].tolist()) <= {e for _, e in cand[:k]} | set()
