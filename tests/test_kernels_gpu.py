"""Parity of each sm_100a kernel with the oracle (GPU only).

Bars: bit-exact for indices, counts and permutation order (given identical fp32 logits);
bf16 floating point within max-abs 2e-2 (after scaling by the output's magnitude) and
rel-L2 1e-2 against an fp32 reference of the same op.
"""

import pytest
import torch

from oracle import moe_oracle as O

gpu = pytest.mark.gpu
DEV = "cuda:0"


def _nat():
    from distributedmoe_b200 import _native as N
    return N


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _assert_close_bf16(out, ref, rel_l2=1e-2, max_abs=2e-2):
    """bf16 bar: rel-L2 <= 1e-2 and max |out-ref| <= max_abs * max(1, max|ref|) (the scale
    term allows the final bf16 rounding of large outputs)."""
    out, ref = out.float().cpu(), ref.float().cpu()
    r = _rel_l2(out, ref)
    m = (out - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    assert r <= rel_l2, f"rel-L2 {r:.3e}"
    assert m <= max_abs * scale, f"max-abs {m:.3e} (scale {scale:.2f})"


def _status_ok():
    N = _nat()
    N.check_device_status(torch.device(DEV))


# ----------------------------------------------------------------------------- router
@gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("T,d,E,k", [(1, 64, 8, 2), (1000, 1024, 8, 2), (333, 2048, 128, 8), (64, 256, 4, 1)])
def test_router_softmax_matches_oracle(dtype, T, d, E, k):
    N = _nat()
    g = torch.Generator().manual_seed(T * 7 + E)
    x = torch.randn(T, d, generator=g).to(dtype)
    w_r = (torch.randn(E, d, generator=g) * 0.02).to(dtype)
    idx, w, logits = N.router(x.to(DEV), w_r.to(DEV), k, want_logits=True, w_dtype=dtype)
    torch.cuda.synchronize()
    ref_logits = O.router_logits(x, w_r, fp32_logits=True)
    assert torch.allclose(logits.cpu(), ref_logits, rtol=1e-4, atol=1e-4)
    # Routing from the kernel's own fp32 logits must be bit-exact.
    rw, sel = O.route(logits.cpu(), k, dtype)
    assert torch.equal(idx.cpu(), sel)
    assert torch.allclose(w.cpu().float(), rw.float(), rtol=1e-2 if dtype != torch.float32 else 1e-6, atol=1e-6)


@gpu
def test_router_from_logits_renorm_scale():
    N = _nat()
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(4096, 8, generator=g) * 3
    idx, w, _ = N.router(None, None, 2, logits_in=logits.to(DEV), renormalize=True, scale=1.0, w_dtype=torch.float32)
    rw, sel = O.route(logits, 2, torch.float32, renormalize=True)
    assert torch.equal(idx.cpu(), sel)
    assert torch.allclose(w.cpu(), rw, rtol=1e-6, atol=1e-7)


@gpu
@pytest.mark.parametrize("T", [1, 257, 2048])
def test_router_sigmoid_group_matches_oracle(T):
    """DeepSeek-V3 router (extension): sigmoid, bias for selection, 8 groups / top-4, top-8, renorm x2.5."""
    N = _nat()
    g = torch.Generator().manual_seed(2 + T)
    E, k = 256, 8
    logits = torch.randn(T, E, generator=g)
    bias = torch.randn(E, generator=g) * 0.01
    idx, w, _ = N.router(None, None, k, logits_in=logits.to(DEV), mode=N.ROUTER_SIGMOID_GROUP, renormalize=True,
                         scale=2.5, score_bias=bias.to(DEV), n_group=8, topk_group=4, w_dtype=torch.float32)
    rw, sel = O.route(logits, k, torch.float32, mode=O.ROUTER_SIGMOID_GROUP, renormalize=True, score_bias=bias,
                      scale=2.5, n_group=8, topk_group=4)
    assert torch.equal(idx.cpu(), sel)
    assert torch.allclose(w.cpu(), rw, rtol=1e-5, atol=1e-6)


@gpu
@pytest.mark.parametrize("T,d,E", [(600, 7168, 256), (40, 512, 64), (1, 2048, 128)])
def test_router_tensor_core_logits(T, d, E):
    """Many experts: the logits are a tcgen05 GEMM (pair tiles for T >= 128, single-SM tiles
    below), fp32 accumulation; selection from them is then bit-exact against the oracle."""
    N = _nat()
    g = torch.Generator().manual_seed(T + d + E)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, d, generator=g) * 0.006).to(torch.bfloat16)
    bias = torch.randn(E, generator=g) * 0.01
    idx, w, logits = N.router(x.to(DEV), w_r.to(DEV), 8, want_logits=True, mode=N.ROUTER_SIGMOID_GROUP,
                              renormalize=True, scale=2.5, score_bias=bias.to(DEV), n_group=8, topk_group=4,
                              w_dtype=torch.float32)
    torch.cuda.synchronize()
    _status_ok()
    ref_logits = x.double() @ w_r.double().t()
    assert torch.allclose(logits.cpu().double(), ref_logits, rtol=1e-4, atol=1e-4)
    rw, sel = O.route(logits.cpu(), 8, torch.float32, mode=O.ROUTER_SIGMOID_GROUP, renormalize=True, score_bias=bias,
                      scale=2.5, n_group=8, topk_group=4)
    assert torch.equal(idx.cpu(), sel)
    assert torch.allclose(w.cpu(), rw, rtol=1e-5, atol=1e-6)


@gpu
@pytest.mark.parametrize("T,d,E", [(1, 2048, 128), (64, 2048, 128), (256, 7168, 256), (100, 512, 64), (257, 2048, 128)])
@pytest.mark.parametrize("few", ["1", "0"])
def test_router_logits_few_tokens_and_tensor_cores(T, d, E, few, monkeypatch):
    """Router logits for E >= 32: the CUDA-core kernel for T <= 256 (eight experts per CTA)
    and the tensor-core GEMM (DMOE_LOGITS_FEW_TOKENS=0, or T > 256) both agree with the
    oracle's fp32 logits within the fp32 summation bound; selection from them is bit-exact."""
    monkeypatch.setenv("DMOE_LOGITS_FEW_TOKENS", few)
    N = _nat()
    g = torch.Generator().manual_seed(T + d + E + 1)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, d, generator=g) * 0.02).to(torch.bfloat16)
    idx, w, logits = N.router(x.to(DEV), w_r.to(DEV), 8, want_logits=True, renormalize=True, w_dtype=torch.float32)
    torch.cuda.synchronize()
    _status_ok()
    ref = O.router_logits(x, w_r, fp32_logits=True)
    mag = x.float().abs() @ w_r.float().abs().t()
    assert bool(((logits.cpu() - ref).abs() <= 2 * d * 2.0 ** -24 * mag + 1e-6).all())
    rw, sel = O.route(logits.cpu(), 8, torch.float32, renormalize=True)
    assert torch.equal(idx.cpu(), sel)
    assert torch.allclose(w.cpu(), rw, rtol=1e-6, atol=1e-7)


@gpu
def test_router_rejects_bad_args():
    N = _nat()
    x = torch.randn(4, 64, device=DEV)
    with pytest.raises(N.DMoEError):
        N.router(x, torch.randn(300, 64, device=DEV), 2)  # E > 256


# ----------------------------------------------------------------------------- plan
# Plan paths: one CTA, one ranking pass (E <= 16, T*k <= 32768); one CTA in rounds of 1024
# (E <= 64 up to 16384 activations, E <= 256 up to 8192); three launches otherwise.
_PLAN_PATHS = {"few": {}, "single": {"DMOE_PLAN_FEW": "0"}, "multi": {"DMOE_PLAN_FEW": "0", "DMOE_PLAN_SINGLE": "0"}}


@gpu
@pytest.mark.parametrize("T,k,E", [(1, 1, 1), (1, 2, 8), (37, 2, 8), (5, 4, 16), (4096, 2, 8), (8192, 8, 256),
                                   (4096, 8, 256), (16384, 2, 8), (3000, 8, 1024), (100, 1, 4), (16, 8, 128),
                                   (1000, 3, 13), (8192, 4, 16)])
@pytest.mark.parametrize("path", sorted(_PLAN_PATHS))
def test_route_plan_bit_exact(T, k, E, path, monkeypatch):
    """Every plan path (DMOE_PLAN_FEW=0 and DMOE_PLAN_SINGLE=0 switch the one-CTA paths off)
    gives the oracle's plan bit for bit wherever it applies."""
    for key, v in _PLAN_PATHS[path].items():
        monkeypatch.setenv(key, v)
    N = _nat()
    g = torch.Generator().manual_seed(T + 31 * k + E)
    # distinct experts per token, like top-k
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]) if k <= E else None
    w = torch.rand(T, k, generator=g).to(torch.bfloat16)
    res = N.route_plan(idx.to(DEV), w.to(DEV), E)
    torch.cuda.synchronize()
    counts, offsets, pt, ps = O.route_plan_fast(idx, E)
    assert torch.equal(res["counts"].cpu().long(), counts)
    assert torch.equal(res["offsets"].cpu().long(), offsets)
    assert torch.equal(res["perm_token"].cpu().long(), pt)
    assert torch.equal(res["perm_slot"].cpu().long(), ps)
    inv = torch.empty(T * k, dtype=torch.long)
    inv[pt * k + ps] = torch.arange(T * k)
    assert torch.equal(res["inverse"].cpu().long(), inv)
    assert torch.equal(res["perm_weight"].cpu(), w[pt, ps])


@gpu
@pytest.mark.parametrize("path", sorted(_PLAN_PATHS))
def test_route_plan_invalid_experts_are_left_out(path, monkeypatch):
    """Indices outside [0, E) get no position: counts cover only valid ones, inverse is -1."""
    for key, v in _PLAN_PATHS[path].items():
        monkeypatch.setenv(key, v)
    N = _nat()
    T, k, E = 3000, 2, 8
    g = torch.Generator().manual_seed(9)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    idx[7, 1] = -1
    idx[100, 0] = E
    res = N.route_plan(idx.to(DEV), None, E, want_weight=False)
    torch.cuda.synchronize()
    valid = (idx >= 0) & (idx < E)
    assert res["counts"].sum().item() == int(valid.sum())
    inv = res["inverse"].cpu().view(T, k)
    assert inv[7, 1].item() == -1 and inv[100, 0].item() == -1
    assert sorted(inv[valid].tolist()) == list(range(int(valid.sum())))
    pt = res["perm_token"].cpu()[:int(valid.sum())]
    off = res["offsets"].cpu()
    for e in range(E):
        toks = pt[off[e]:off[e + 1]]
        assert bool((idx[toks.long()] == e).any(dim=1).all())


@gpu
@pytest.mark.parametrize("T,d,E,k,dtype", [(4096, 4096, 8, 2, torch.bfloat16), (4097, 4096, 8, 2, torch.bfloat16),
                                           (33, 2048, 6, 3, torch.bfloat16), (500, 8192, 4, 2, torch.bfloat16),
                                           (17, 256, 2, 1, torch.bfloat16), (1, 1024, 8, 2, torch.bfloat16),
                                           (300, 5120, 8, 2, torch.bfloat16), (1000, 3072, 8, 2, torch.float16)])
@pytest.mark.parametrize("kernel", ["mma", "ring"])
def test_router_few_experts_kernels(T, d, E, k, dtype, kernel, monkeypatch):
    """The few-expert routers -- 16x8x16 tensor-core MMAs over 16-token groups (d a multiple
    of 1024 up to 5120), or weights in registers with token tiles through a bulk-copy ring
    (DMOE_ROUTER_MMA=0, and every other shape): logits within fp32 summation error of the
    oracle's, selection bit-exact from them, with a logit bias, renormalisation and a scale;
    also the Mixtral shape and a ragged last group."""
    if kernel == "ring":
        monkeypatch.setenv("DMOE_ROUTER_MMA", "0")
    N = _nat()
    g = torch.Generator().manual_seed(T + d + E)
    x = torch.randn(T, d, generator=g).to(dtype)
    w_r = (torch.randn(E, d, generator=g) * 0.02).to(dtype)
    bias = torch.randn(E, generator=g)
    idx, w, logits = N.router(x.to(DEV), w_r.to(DEV), k, want_logits=True, logit_bias=bias.to(DEV),
                              renormalize=True, scale=1.5, w_dtype=torch.float32)
    torch.cuda.synchronize()
    ref_logits = O.router_logits(x, w_r, fp32_logits=True, logit_bias=bias)
    mag = x.float().abs() @ w_r.float().abs().t()
    assert bool(((logits.cpu() - ref_logits).abs() <= 2 * d * 2.0 ** -24 * mag + 1e-6).all())
    rw, sel = O.route(logits.cpu(), k, torch.float32, renormalize=True, scale=1.5)
    assert torch.equal(idx.cpu(), sel)
    assert torch.allclose(w.cpu(), rw, rtol=1e-6, atol=1e-7)


@gpu
def test_route_plan_matches_reference_lists():
    """Per-expert lists equal the reference's torch.where lists (golden fixture)."""
    N = _nat()
    import os
    gold = torch.load(os.path.join(os.path.dirname(__file__), "golden", "replicas.pt"), weights_only=False)
    sel = gold["selected"]
    E = gold["config"]["E"]
    res = N.route_plan(sel.to(DEV), gold["routing_weights"].to(DEV), E)
    off = res["offsets"].cpu()
    pt = res["perm_token"].cpu().long()
    pw = res["perm_weight"].cpu()
    for e, pe in gold["per_expert"].items():
        assert torch.equal(pt[off[e]:off[e + 1]], pe["tokens"])
        assert torch.equal(pw[off[e]:off[e + 1]], pe["weights"].float())


# ----------------------------------------------------------------------------- permute / combine
@gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_permute_rows_gather_and_copy(dtype):
    N = _nat()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(500, 256, generator=g).to(dtype).to(DEV)
    row_map = torch.randint(0, 500, (900,), generator=g, dtype=torch.int32).to(DEV)
    dst = torch.zeros(1024, 256, dtype=dtype, device=DEV)
    seg_src, seg_dst, seg_len = [0, 300, 301, 800], [0, 310, 320, 1000], [300, 1, 0, 24]
    N.permute_rows(x, dst, seg_src, seg_dst, seg_len, row_map=row_map)
    ref = torch.zeros_like(dst)
    for s, dd, n in zip(seg_src, seg_dst, seg_len):
        ref[dd:dd + n] = x[row_map[s:s + n].long()]
    assert torch.equal(dst, ref)
    dst2 = torch.zeros_like(dst)
    N.permute_rows(dst, dst2, [310, 0], [0, 700], [10, 300])
    assert torch.equal(dst2[0:10], dst[310:320]) and torch.equal(dst2[700:1000], dst[0:300])


@gpu
@pytest.mark.parametrize("dtype,k", [(torch.bfloat16, 2), (torch.bfloat16, 8), (torch.float32, 2), (torch.float16, 1)])
def test_combine_matches_oracle(dtype, k):
    N = _nat()
    g = torch.Generator().manual_seed(4)
    T, d = 777, 512
    rows = torch.randn(T * k, d, generator=g).to(dtype)
    perm = torch.randperm(T * k, generator=g)
    inverse = perm.view(T, k)
    w = torch.rand(T, k, generator=g).to(dtype)
    out = torch.empty(T, d, dtype=dtype, device=DEV)
    N.combine(rows.to(DEV), inverse.to(torch.int32).to(DEV), w.to(DEV), out)
    ref = O.combine_from_permuted(rows, inverse, w, torch.float32)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(out.cpu().float(), ref, rtol=tol, atol=tol)
    # accumulate mode adds to the existing output
    out2 = out.clone()
    N.combine(rows.to(DEV), inverse.to(torch.int32).to(DEV), w.to(DEV), out2, accumulate=True)
    assert torch.allclose(out2.cpu().float(), 2 * ref, rtol=2 * tol, atol=2 * tol)


# ----------------------------------------------------------------------------- grouped MLP
def _mlp_case(seed, E, d, I, seg_sizes, dtype, act, w_std=0.02):
    g = torch.Generator().manual_seed(seed)
    M = sum(seg_sizes) + 7
    X = torch.randn(M, d, generator=g).to(dtype)
    wg = (torch.randn(E, I, d, generator=g) * w_std).to(dtype)
    wu = (torch.randn(E, I, d, generator=g) * w_std).to(dtype)
    wd = (torch.randn(E, d, I, generator=g) * w_std).to(dtype)
    experts = [int(torch.randint(0, E, (1,), generator=g)) for _ in seg_sizes]
    ends, acc = [], 0
    for s in seg_sizes:
        acc += s
        ends.append(acc)
    return X, wg, wu, wd, experts, ends


def _mlp_ref_fp32(X, wg, wu, wd, experts, ends, act):
    Y = torch.zeros(X.shape[0], X.shape[1], dtype=torch.float32)
    start = 0
    for e, en in zip(experts, ends):
        if en > start:
            Y[start:en] = O.expert_mlp_fp32(X[start:en], wg[e], wu[e], wd[e], act)
        start = en
    return Y


@gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("act", [O.ACT_RELU, O.ACT_SILU])
@pytest.mark.parametrize("E,d,I,sizes", [
    (1, 64, 128, [128]),
    (4, 256, 384, [1, 127, 128, 129, 0, 300]),
    (8, 200, 320, [5, 0, 260, 64]),          # K tail (200 % 64), N tails (I=320, d=200)
    (3, 512, 256, [1000]),
    # segments averaging >= 128 rows take the pair (2-SM) kernel
    (6, 256, 384, [1030, 1000, 300, 129, 0, 256, 511, 385]),
])
def test_grouped_mlp_matches_fp32_reference(dtype, act, E, d, I, sizes):
    N = _nat()
    X, wg, wu, wd, experts, ends = _mlp_case(11 + d + I, E, d, I, sizes, dtype, act)
    Y = torch.full((X.shape[0], d), 7.0, dtype=dtype, device=DEV)
    N.grouped_gated_mlp(X.to(DEV), wg.to(DEV), wu.to(DEV), wd.to(DEV), experts, ends, act, Y)
    torch.cuda.synchronize()
    _status_ok()
    ref = _mlp_ref_fp32(X, wg, wu, wd, experts, ends, act)
    n = ends[-1]
    _assert_close_bf16(Y[:n].cpu(), ref[:n])
    assert torch.all(Y[n:].cpu() == 7.0), "rows outside the segments must stay untouched"


@gpu
@pytest.mark.parametrize("env", [{"DMOE_GEMM_HYBRID": "1"}, {"DMOE_GEMM_RASTER": "0"}, {"DMOE_GEMM_RASTER": "1"},
                                 {"DMOE_GEMM_VARIANT": "1sm"}, {"DMOE_GEMM_HYBRID": "1", "DMOE_GEMM_RASTER": "1"},
                                 {"DMOE_GEMM2_RASTER": "1"}])
def test_grouped_mlp_launch_variants(env, monkeypatch):
    """The non-default launch shapes (pair tiles with single-SM remainders, the other tile
    orders, single-SM tiles only) give the same results."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    N = _nat()
    dtype, act = torch.bfloat16, O.ACT_SILU
    X, wg, wu, wd, experts, ends = _mlp_case(77, 6, 256, 384, [1030, 1000, 300, 129, 0, 256, 511, 385], dtype, act)
    Y = torch.zeros(X.shape[0], 256, dtype=dtype, device=DEV)
    N.grouped_gated_mlp(X.to(DEV), wg.to(DEV), wu.to(DEV), wd.to(DEV), experts, ends, act, Y)
    torch.cuda.synchronize()
    _status_ok()
    ref = _mlp_ref_fp32(X, wg, wu, wd, experts, ends, act)
    _assert_close_bf16(Y[:ends[-1]].cpu(), ref[:ends[-1]])


@gpu
@pytest.mark.parametrize("policy", [1, 2, 3])
@pytest.mark.parametrize("device_table", [False, True])
def test_grouped_mlp_tile_policies(policy, device_table):
    """Every tile policy (pair tiles, single-SM tiles, pairs with single-SM remainders) on a
    ragged table (empty, 1, 128, 129, 256, 257, 300, 384, 385, 511 rows) gives the same
    rows, with host and device segment tables; rows outside the segments stay untouched."""
    N = _nat()
    dtype, act = torch.bfloat16, O.ACT_SILU
    sizes = [257, 0, 300, 1, 128, 129, 256, 384, 385, 511]
    X, wg, wu, wd, experts, ends = _mlp_case(79 + policy, 10, 256, 384, sizes, dtype, act)
    Y = torch.full((X.shape[0] + 64, 256), 7.0, dtype=dtype, device=DEV)
    Xd = torch.cat([X, torch.zeros(64, X.shape[1], dtype=dtype)]).to(DEV)
    if device_table:
        se = torch.tensor(experts, dtype=torch.int32, device=DEV)
        sn = torch.tensor(ends, dtype=torch.int32, device=DEV)
    else:
        se, sn = experts, ends
    N.grouped_gated_mlp(Xd, wg.to(DEV), wu.to(DEV), wd.to(DEV), se, sn, act, Y, tile_policy=policy)
    torch.cuda.synchronize()
    _status_ok()
    ref = _mlp_ref_fp32(X, wg, wu, wd, experts, ends, act)
    n = ends[-1]
    _assert_close_bf16(Y[:n].cpu(), ref[:n])
    assert torch.all(Y[n:].cpu() == 7.0), "rows outside the segments must stay untouched"


@gpu
def test_grouped_mlp_with_sm_reserve():
    """Leaving SMs free shrinks the persistent grid; the results stay the same."""
    N = _nat()
    dtype, act = torch.bfloat16, O.ACT_SILU
    X, wg, wu, wd, experts, ends = _mlp_case(78, 6, 256, 384, [1030, 1000, 300, 129, 0, 256, 511, 385], dtype, act)
    ref = _mlp_ref_fp32(X, wg, wu, wd, experts, ends, act)
    try:
        for reserve in (8, 30):
            N.set_gemm_sm_reserve(reserve)
            Y = torch.zeros(X.shape[0], 256, dtype=dtype, device=DEV)
            N.grouped_gated_mlp(X.to(DEV), wg.to(DEV), wu.to(DEV), wd.to(DEV), experts, ends, act, Y)
            torch.cuda.synchronize()
            _status_ok()
            _assert_close_bf16(Y[:ends[-1]].cpu(), ref[:ends[-1]])
    finally:
        N.set_gemm_sm_reserve(0)


@gpu
def test_grouped_mlp_device_segment_table_and_reference_grouped_mm():
    """Device-resident segment table; compared with the reference's own bf16 grouped_mm path."""
    N = _nat()
    dtype = torch.bfloat16
    E, d, I = 8, 256, 512
    X, wg, wu, wd, experts, ends = _mlp_case(99, E, d, I, [40, 200, 1, 90, 0, 129], dtype, O.ACT_RELU)
    Y = torch.zeros(X.shape[0], d, dtype=dtype, device=DEV)
    se = torch.tensor(experts, dtype=torch.int32, device=DEV)
    sn = torch.tensor(ends, dtype=torch.int32, device=DEV)
    N.grouped_gated_mlp(X.to(DEV), wg.to(DEV), wu.to(DEV), wd.to(DEV), se, sn, O.ACT_RELU, Y)
    torch.cuda.synchronize()
    _status_ok()
    ref = O.expert_grouped_mlp(X, wg, wu, wd, experts, ends, O.ACT_RELU)  # reference arithmetic (bf16 grouped_mm)
    _assert_close_bf16(Y[:ends[-1]].cpu(), ref)


@gpu
def test_grouped_mlp_mixtral_shape_sampled_rows():
    """Full Mixtral expert shape (d=4096, I=14336, 8 experts, ~1024 rows each), checked on
    sampled rows of each segment against an fp32 GPU reference."""
    N = _nat()
    torch.manual_seed(1)
    dtype = torch.bfloat16
    E, d, I = 8, 4096, 14336
    sizes = [1024 + 37 * ((e * 5) % 7) - 100 for e in range(E)]
    M = sum(sizes)
    X = torch.randn(M, d, device=DEV, dtype=dtype)
    wg = (torch.randn(E, I, d, device=DEV) * 0.02).to(dtype)
    wu = (torch.randn(E, I, d, device=DEV) * 0.02).to(dtype)
    wd = (torch.randn(E, d, I, device=DEV) * 0.02).to(dtype)
    ends = torch.tensor(sizes).cumsum(0).tolist()
    experts = list(range(E))
    Y = torch.empty(M, d, device=DEV, dtype=dtype)
    N.grouped_gated_mlp(X, wg, wu, wd, experts, ends, O.ACT_SILU, Y)
    torch.cuda.synchronize()
    _status_ok()
    start = 0
    for e, en in zip(experts, ends):
        rows = torch.cat([torch.arange(start, start + 16), torch.arange(en - 16, en)]).to(DEV)
        xs = X[rows].float()
        h = torch.nn.functional.silu(xs @ wg[e].float().t()) * (xs @ wu[e].float().t())
        ref = h @ wd[e].float().t()
        _assert_close_bf16(Y[rows].cpu(), ref.cpu())
        start = en


# ----------------------------------------------------------------------------- completion flags
@gpu
def test_flag_signal_then_wait_and_bounded_timeout():
    """A wait whose value is already there returns at once; a wait for a value nothing
    writes gives up after its limit and reports DMOE_DEVERR_FLAG_TIMEOUT in the status word,
    leaving the stream and the context usable.  (Signaller and waiter never run as two
    kernels at the same time on this one GPU: the signal has finished before the wait.)"""
    N = _nat()
    dev = torch.device(DEV)
    flag = torch.zeros(1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    N.flag_signal(flag.data_ptr(), 5, s)
    torch.cuda.synchronize()
    assert int(flag.item()) == 5
    N.flag_wait(flag.data_ptr(), 5, 2_000_000_000, status.data_ptr(), s)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    N.flag_wait(flag.data_ptr(), 6, 2_000_000, status.data_ptr(), s)  # nothing writes 6: 2 ms limit
    torch.cuda.synchronize()
    assert int(status.item()) & 0x10
    y = torch.ones(4, device=dev) * 3  # the context still works
    assert float(y.sum().item()) == 12.0


@gpu
def test_router_nan_logits_pick_valid_experts():
    """A NaN logit ranks first (torch.topk's order) and every pick stays in [0, E), in both
    router modes; a NaN token's weights are NaN, the other tokens are unaffected."""
    from distributedmoe_b200 import _native as N
    T, E, k = 64, 32, 4
    g = torch.Generator(device=DEV).manual_seed(3)
    logits = torch.randn(T, E, generator=g, device=DEV)
    logits[5, 7] = float("nan")
    logits[9, :] = float("nan")
    for mode, kw in ((N.ROUTER_SOFTMAX, {}), (N.ROUTER_SIGMOID_GROUP, dict(n_group=4, topk_group=2))):
        idx, w, _ = N.router(None, None, k, logits_in=logits.contiguous(), mode=mode, renormalize=True,
                             w_dtype=torch.float32, **kw)
        torch.cuda.synchronize()
        assert idx.min().item() >= 0 and idx.max().item() < E
        assert idx[5, 0].item() == 7
        assert torch.isnan(w[9]).all()
        ok = [t for t in range(T) if t not in (5, 9)]
        assert torch.isfinite(w[ok]).all()


@gpu
def test_layer_with_a_nan_token_keeps_other_tokens_finite():
    """A NaN in one token's activations reaches only that token's output row: its rows are
    routed to valid experts and every expert row and plan entry stays in bounds."""
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.MoE import moe_layer_forward
    T, d, E, k, I = 200, 128, 8, 2, 256
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
    x[17, 3] = float("nan")
    w_r = (torch.randn(E, d, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    gate = (torch.randn(E, I, d, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    up = (torch.randn(E, I, d, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    down = (torch.randn(E, d, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    y = moe_layer_forward(x, w_r, gate, up, down, k, activation=N.ACT_SILU, renormalize=True)
    torch.cuda.synchronize()
    N.check_device_status(DEV)
    assert torch.isnan(y[17]).all()
    rest = torch.cat([y[:17], y[18:]])
    assert torch.isfinite(rest).all()
