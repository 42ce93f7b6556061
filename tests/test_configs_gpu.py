"""The layer at the shapes and routing modes of the benchmark configurations, end to end
through the drop-in API on one GPU, against the oracle:

* DeepSeek-V3 routing: sigmoid scores with a selection-only bias, group-limited top-k
  (8 groups, top-4 groups), renormalised and scaled, plus an always-on shared expert; once
  at small dimensions and once at the DeepSeek expert shape (d=7168, I=2048).
* Qwen3-30B-A3B decode: E=128, k=8, d=2048, I=768 at T = 16, 64, 256, eight blocks of 16
  experts (the 8-GPU layout, here on one GPU).
* Skewed load with replicas: Zipf-biased router logits, every expert in two blocks, the
  least-loaded replica policy, one block lost half-way through the steps.

Large shapes are built on the GPU and checked against the oracle's expert math run in fp32
on the GPU (the routing itself is checked bit-exact elsewhere); small ones run the oracle on
the CPU.  Tolerances are the layer's: rel-L2 1e-2 and max-abs 2e-2 (scaled by the output
range when it exceeds 1).
"""

import math

import pytest
import torch

from oracle import moe_oracle as O

gpu = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _check(y, ref):
    y = y.reshape(ref.shape).double()
    ref = ref.double()
    rel = ((y - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    mx = (y - ref).abs().max().item()
    assert rel < 1e-2, f"rel-L2 {rel}"
    assert mx <= 2e-2 * max(1.0, ref.abs().max().item()), f"max-abs {mx}"


def _weights(E, d, I, seed, w_std, device):
    g = torch.Generator(device=device).manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g, device=device) * w_std).to(torch.bfloat16)
    return mk(E, I, d), mk(E, I, d), mk(E, d, I), g


def _cluster(E, blocks, k, d, gate, up, down, io, **opts):
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    stacked = [(gate[b].contiguous(), up[b].contiguous(), down[b].contiguous()) for b in blocks]
    return LocalCluster(E, blocks, k, d, torch.bfloat16, DEV, [DEV] * len(blocks), stacked=stacked,
                        io_buffer_size=io, number_of_io_buffers=4, **opts)


def _deepseek(T, d, E, I, I_s, blocks, io, seed, oracle_device):
    from distributedmoe_b200 import _native as N
    k, n_group, topk_group, scale = 8, 8, 4, 2.5
    gate, up, down, g = _weights(E, d, I, seed, 0.006, DEV)
    sg, su, sd = [(torch.randn(*s, generator=g, device=DEV) * 0.006).to(torch.bfloat16)
                  for s in ((I_s, d), (I_s, d), (d, I_s))]
    w_r = (torch.randn(E, d, generator=g, device=DEV) * 0.006).to(torch.bfloat16)
    bias = torch.randn(E, generator=g, device=DEV) * 0.01
    x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
    cl = _cluster(E, blocks, k, d, gate, up, down, io, activation="silu", renormalize=True,
                  router_mode="sigmoid_group", routed_scaling_factor=scale, n_group=n_group, topk_group=topk_group)
    try:
        moe = cl.moe
        with torch.no_grad():
            moe.gate.weight.copy_(w_r)
        moe.score_bias = bias
        moe.set_shared_expert(sg, su, sd)
        ys = [moe(x) for _ in range(2)]
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    _, _, logits = N.router(x, w_r, k, want_logits=True)
    od = oracle_device
    ref = O.local_experts(x.to(od), logits.to(od), gate.to(od), up.to(od), down.to(od), k, act=O.ACT_SILU,
                          renormalize=True, mode=O.ROUTER_SIGMOID_GROUP, score_bias=bias.to(od), scale=scale,
                          n_group=n_group, topk_group=topk_group, shared=(sg.to(od), su.to(od), sd.to(od)),
                          compute_dtype=torch.float32)
    for y in ys:
        _check(y.to(od), ref)


@gpu
def test_deepseek_routing_with_shared_expert_small():
    _deepseek(T=400, d=256, E=64, I=128, I_s=192, blocks=[list(range(0, 64, 2)), list(range(1, 64, 2))], io=2048,
              seed=31, oracle_device="cpu")


@gpu
def test_deepseek_expert_shape():
    """d=7168, I=2048 (the DeepSeek-V3 expert and shared-expert shape), 32 routed experts in
    two blocks (the full 256 do not change the kernels' shapes, only the segment count,
    which the routing-plan and grouped-MLP tests cover)."""
    _deepseek(T=256, d=7168, E=32, I=2048, I_s=2048, blocks=[list(range(16)), list(range(16, 32))], io=4096,
              seed=32, oracle_device=DEV)


@gpu
@pytest.mark.parametrize("T", [16, 64, 256])
def test_qwen3_decode_shape(T):
    from distributedmoe_b200 import _native as N
    E, k, d, I = 128, 8, 2048, 768
    gate, up, down, g = _weights(E, d, I, 33, 0.02, DEV)
    w_r = (torch.randn(E, d, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
    blocks = [list(range(16 * b, 16 * b + 16)) for b in range(8)]
    cl = _cluster(E, blocks, k, d, gate, up, down, 4096, activation="silu", renormalize=True)
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        ys = [cl.moe(x) for _ in range(2)]
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    _, _, logits = N.router(x, w_r, k, want_logits=True)
    ref = O.local_experts(x, logits, gate, up, down, k, act=O.ACT_SILU, renormalize=True, compute_dtype=torch.float32)
    for y in ys:
        _check(y, ref)


@gpu
def test_skewed_load_replicas_block_lost_midway():
    """Zipf(s=1.2) bias on the router logits (a fixed permutation of expert ranks), every
    expert in two of eight blocks, least-loaded replica choice; block 3 is disabled after
    five of ten steps and every step still matches the oracle."""
    from distributedmoe_b200 import _native as N
    T, d, E, k, I = 1024, 256, 8, 2, 512
    gate, up, down, g = _weights(E, d, I, 34, 0.02, DEV)
    w_r = (torch.randn(E, d, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    ranks = torch.randperm(E, generator=torch.Generator().manual_seed(4)) + 1
    zipf = torch.tensor([-1.2 * math.log(float(r)) for r in ranks], device=DEV)
    blocks = [[b, (b + 1) % E] for b in range(8)]
    cl = _cluster(E, blocks, k, d, gate, up, down, 1024, activation="silu", renormalize=True,
                  expert_block_policy="least_loaded")
    try:
        moe = cl.moe
        lin = torch.nn.Linear(d, E, bias=True, dtype=torch.bfloat16, device=DEV)
        with torch.no_grad():
            lin.weight.copy_(w_r)
            lin.bias.copy_(zipf.to(torch.bfloat16))
        moe.gate = lin
        outs = []
        for step in range(10):
            if step == 5:
                moe.disable_experts_block(3)
            x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
            outs.append((x, moe(x)))
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    bias32 = lin.bias.detach().float()
    for x, y in outs:
        _, _, logits = N.router(x, w_r, k, logit_bias=bias32, want_logits=True)
        ref = O.local_experts(x.cpu(), logits.cpu(), gate.cpu(), up.cpu(), down.cpu(), k, act=O.ACT_SILU,
                              renormalize=True, compute_dtype=torch.float32)
        _check(y.float().cpu(), ref)
