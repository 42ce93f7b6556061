"""Every benchmark configuration at full size, built exactly as bench.py builds it
(``bench.Layer``: same seeds, weights, router, cluster and data plane), its whole output
checked against the oracle's expert math in fp32 on the GPU:

* Mixtral-8x7B shape on one GPU: T=4096, d=4096, E=8, top-2, I=14336, seed 1, on the
  device-driven plane (what the bench times) and on the reference's task protocol.
* DeepSeek-V3 shape on one GPU: all 256 routed experts plus the shared expert, T=8192,
  d=7168, I=2048, sigmoid / group-limited top-8 router, seed 2.
* Qwen3-30B-A3B decode shape: T = 16, 64, 256, d=2048, E=128, top-8, I=768, seed 3.
* Skewed-load fault tolerance: Mixtral shape, T=16384, every expert in two blocks, Zipf(1.2)
  router bias, even split over alive replicas, block 3 lost at step 50 of 100; every one of
  the 100 steps is checked.

Bars: rel-L2 <= 1e-2 and max-abs <= 2e-2 * max(1, |ref|_inf) (the scale term admits the
final bf16 rounding of outputs larger than 1).

Routing is also checked against the oracle's OWN fp32 logits (x.float() @ w_r.float().T,
``oracle/moe_oracle.py::router_logits``) and torch.topk over its probabilities: the kernel's
logits must agree with the oracle's within the worst-case error of two fp32 sums of the same
d exact products in different orders (2 (d-1) 2^-24 sum|x_i w_i|), and every token whose top-k differs
must be a near-tie: the oracle's router applied to the kernel's own logits reproduces the
kernel's picks exactly, and the oracle's values at the two choices differ by less than the
logit disagreement allows.  The count of such tokens is printed.
"""

import math

import pytest
import torch

import bench
from oracle import moe_oracle as O

gpu = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _exact_fp32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False  # the oracle's fp32 products stay fp32
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def _check(y, ref, what=""):
    y = y.reshape(ref.shape).double()
    ref = ref.double()
    rel = ((y - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    mx = (y - ref).abs().max().item()
    bar = 2e-2 * max(1.0, ref.abs().max().item())
    print(f"{what}: rel-L2 {rel:.3e}, max-abs {mx:.3e} (bar {bar:.3e})")
    assert rel < 1e-2, f"{what}: rel-L2 {rel}"
    assert mx <= bar, f"{what}: max-abs {mx}"


def _routing_vs_oracle_logits(layer: "bench.Layer", x: torch.Tensor, what: str) -> None:
    from distributedmoe_b200 import _native as N
    w = layer.w
    mode = O.ROUTER_SIGMOID_GROUP if w.router_mode == "sigmoid_group" else O.ROUTER_SOFTMAX
    kw = dict(mode=mode, renormalize=True, score_bias=layer.score_bias, scale=w.scale, n_group=w.n_group,
              topk_group=w.topk_group)
    ref_logits = O.router_logits(x, layer.w_r, fp32_logits=True, logit_bias=layer.logit_bias)
    _, ref_sel = O.route(ref_logits, w.k, torch.float32, **kw)
    nmode = N.ROUTER_SIGMOID_GROUP if mode == O.ROUTER_SIGMOID_GROUP else N.ROUTER_SOFTMAX
    idx, _, k_logits = N.router(x, layer.w_r, w.k, mode=nmode, renormalize=True, scale=w.scale,
                                logit_bias=layer.logit_bias, score_bias=layer.score_bias, n_group=w.n_group,
                                topk_group=w.topk_group, want_logits=True, w_dtype=torch.float32)
    diff = (k_logits - ref_logits).abs()
    # Both sides sum d exact fp32 products in different orders: each sum is within
    # (d - 1) * 2^-24 * sum|x_i w_i| of the exact value, so the two within twice that.
    mag = x.float().abs() @ layer.w_r.float().abs().t()
    tol = 2.0 * x.shape[1] * 2.0 ** -24 * mag + 1e-7
    assert bool((diff <= tol).all()), f"{what}: kernel logits differ from the oracle's by {diff.max().item():.3e}"
    mism = (idx != ref_sel).any(dim=1).nonzero().flatten()
    print(f"{what}: {mism.numel()} of {x.shape[0]} tokens pick a different top-{w.k} than torch.topk over the "
          f"oracle's fp32 logits (max |logit diff| {diff.max().item():.2e})")
    if mism.numel():
        # The oracle's own router on the kernel's logits gives exactly the kernel's picks ...
        _, sel_on_kernel = O.route(k_logits[mism], w.k, torch.float32, **kw)
        assert torch.equal(sel_on_kernel, idx[mism]), f"{what}: a mismatch is not explained by the logits"
        # ... and the choices differ only where the oracle's ranking values nearly tie.
        if mode == O.ROUTER_SOFTMAX:
            v = ref_logits[mism]
        else:
            v = torch.sigmoid(ref_logits[mism]) + layer.score_bias
        gap = (v.gather(1, ref_sel[mism]).sum(1) - v.gather(1, idx[mism]).sum(1)).abs()
        slack = 4 * w.k * diff[mism].max(dim=1).values + 1e-6
        if mode == O.ROUTER_SOFTMAX:
            assert bool((gap <= slack).all()), f"{what}: top-k gaps {gap.tolist()} exceed {slack.tolist()}"
    assert mism.numel() <= max(2, x.shape[0] // 1000), f"{what}: {mism.numel()} near-tie mismatches"


def _layer_check(name, data_plane="direct", tokens=None, forwards=2):
    w = bench.WORKLOADS[name]
    old = w.tokens
    if tokens is not None:
        w.tokens = tokens
    try:
        layer = bench.Layer(w, DEV, data_plane=data_plane)
    finally:
        w.tokens = old
    try:
        from distributedmoe_b200 import _native as N
        ys = [layer.moe(layer.x) for _ in range(forwards)]
        torch.cuda.synchronize()
        N.check_device_status(DEV)
        ref = bench.oracle_fp32(layer, layer.x)
        for i, y in enumerate(ys):
            _check(y, ref, f"{name}/{data_plane} T={layer.T} forward {i}")
        _routing_vs_oracle_logits(layer, layer.x, f"{name} T={layer.T}")
    finally:
        layer.close()


@gpu
@pytest.mark.parametrize("data_plane", ["direct", "tasks"])
def test_mixtral_layer_full_size(data_plane):
    _layer_check("mixtral", data_plane)


@gpu
def test_deepseek_layer_full_size_256_experts_and_shared():
    _layer_check("deepseek")


@gpu
@pytest.mark.parametrize("T", [16, 64, 256])
def test_qwen3_decode_layer(T):
    _layer_check("qwen3-decode", tokens=T, forwards=3)


@gpu
def test_skewed_fault_tolerance_full_size_every_step():
    """100 steps at T=16384 (fits one B200); block 3 is disabled before step 50 and stays
    lost; every step's whole output matches the oracle."""
    from distributedmoe_b200 import _native as N
    w = bench.WORKLOADS["skewed-ft"]
    layer = bench.Layer(w, DEV)
    g = torch.Generator(device=DEV).manual_seed(w.seed + 100)
    worst = 0.0
    try:
        _routing_vs_oracle_logits(layer, layer.x, "skewed-ft")
        for step in range(100):
            if step == 50:
                layer.moe.disable_experts_block(3)
            x = torch.randn(layer.T, w.d, generator=g, device=DEV).to(torch.bfloat16)
            y = layer.moe(x)
            ref = bench.oracle_fp32(layer, x)
            yd, rd = y.double(), ref.double()
            rel = ((yd - rd).norm() / rd.norm()).item()
            mx = (yd - rd).abs().max().item()
            worst = max(worst, rel)
            assert rel < 1e-2, f"step {step}: rel-L2 {rel}"
            assert mx <= 2e-2 * max(1.0, rd.abs().max().item()), f"step {step}: max-abs {mx}"
        torch.cuda.synchronize()
        N.check_device_status(DEV)
        loads = layer.moe.expert_blocks_pool.expert_blocks_metadata[3].is_alive
        assert not loads
    finally:
        layer.close()
    print(f"skewed-ft: 100 steps, worst rel-L2 {worst:.3e}")
