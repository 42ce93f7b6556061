"""8-bit (e4m3) experts on the GPU.

* Row-wise quantisation bit for bit against the oracle's restatement (torch's own e4m3
  rounding on the CPU), for f32, f16 and bf16 rows, a zero row and an outlier.
* The e4m3 gate/up + bf16 down grouped MLP against an fp32 reference of the dequantised
  operands: rel-L2 <= 1e-2 and max-abs <= 2e-2 (scaled by the output range), the bf16 bar
  (the only differences are fp32 summation order and the bf16 rounding of h and of the
  output); every tile policy, ragged segments, K and N tails.
* Against the bf16 kernel on the unquantised operands: within e4m3's rounding.
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


@gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(1, 16), (37, 272), (300, 4096)])
def test_quantize_rows_bit_exact(dtype, rows, cols):
    N = _nat()
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = (torch.randn(rows, cols, generator=g) * torch.logspace(-3, 3, rows)[:, None]).to(dtype)
    x[rows // 2] = 0  # an all-zero row gets scale 1
    if rows > 2:
        x[1, 3] = 6e4  # one outlier sets its row's scale
    q, s = N.quantize_rows_e4m3(x.to(DEV))
    torch.cuda.synchronize()
    rq, rs = O.quantize_rows_e4m3(x)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


@gpu
def test_quantize_records_layout():
    """Records of the 8-bit exchange: row t's codes in bytes [0, d), its scale at byte d."""
    N = _nat()
    T, d = 50, 256
    x = torch.randn(T, d, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    rec = N.quantize_records(x.to(DEV)).cpu()
    rq, rs = O.quantize_rows_e4m3(x)
    assert rec.shape == (T, d + 16)
    assert torch.equal(rec[:, :d], rq.view(torch.uint8))
    assert torch.equal(rec[:, d:d + 4].contiguous().view(torch.float32).flatten(), rs)


def _fp8_case(seed, E, d, I, sizes, w_std=0.02):
    g = torch.Generator().manual_seed(seed)
    M = sum(sizes) + 5
    X = torch.randn(M, d, generator=g).to(torch.bfloat16)
    wg = (torch.randn(E, I, d, generator=g) * w_std).to(torch.bfloat16)
    wu = (torch.randn(E, I, d, generator=g) * w_std).to(torch.bfloat16)
    wd = (torch.randn(E, d, I, generator=g) * w_std).to(torch.bfloat16)
    experts = [int(torch.randint(0, E, (1,), generator=g)) for _ in sizes]
    ends, acc = [], 0
    for n in sizes:
        acc += n
        ends.append(acc)
    return X, wg, wu, wd, experts, ends


@gpu
@pytest.mark.parametrize("act", [O.ACT_SILU, O.ACT_RELU])
@pytest.mark.parametrize("policy", [0, 1, 2, 3])
@pytest.mark.parametrize("E,d,I,sizes", [
    (2, 128, 128, [128]),
    (5, 208, 320, [1, 0, 129, 257, 64]),             # K tail (208 % 128), N tail (320 % 128)
    (4, 1024, 768, [1030, 300, 0, 511, 256, 385]),  # pair tiles and remainders
])
def test_grouped_mlp_fp8_matches_dequantised_reference(act, policy, E, d, I, sizes):
    N = _nat()
    X, wg, wu, wd, experts, ends = _fp8_case(5 + d + I + policy, E, d, I, sizes)
    Xq, xs = N.quantize_rows_e4m3(X.to(DEV))
    ex = N.Fp8Experts(wg.to(DEV), wu.to(DEV), wd.to(DEV))
    Y = torch.full((X.shape[0], d), 7.0, dtype=torch.bfloat16, device=DEV)
    N.grouped_gated_mlp_fp8(Xq, xs, ex, experts, ends, act, Y, tile_policy=policy)
    torch.cuda.synchronize()
    N.check_device_status(torch.device(DEV))
    Xd = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(X))
    gd = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(wg))
    ud = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(wu))
    ref = torch.zeros(X.shape[0], d)
    start = 0
    for e, en in zip(experts, ends):
        if en > start:
            ref[start:en] = O.expert_mlp_fp32(Xd[start:en], gd[e], ud[e], wd[e].float(), act)
        start = en
    n = ends[-1]
    out = Y[:n].cpu().float()
    assert _rel_l2(out, ref[:n]) <= 1e-2
    assert (out - ref[:n]).abs().max().item() <= 2e-2 * max(1.0, ref[:n].abs().max().item())
    assert torch.all(Y[n:].cpu() == 7.0), "rows outside the segments must stay untouched"


@gpu
def test_grouped_mlp_fp8_device_table_and_close_to_bf16():
    """A device segment table gives the host table's rows; against the bf16 kernel on the
    unquantised operands the result stays within e4m3's rounding (3 mantissa bits)."""
    N = _nat()
    E, d, I, sizes = 4, 1024, 1024, [700, 300, 0, 1200]
    X, wg, wu, wd, experts, ends = _fp8_case(91, E, d, I, sizes)
    Y16 = torch.zeros(X.shape[0], d, dtype=torch.bfloat16, device=DEV)
    N.grouped_gated_mlp(X.to(DEV), wg.to(DEV), wu.to(DEV), wd.to(DEV), experts, ends, O.ACT_SILU, Y16)
    Xq, xs = N.quantize_rows_e4m3(X.to(DEV))
    ex = N.Fp8Experts(wg.to(DEV), wu.to(DEV), wd.to(DEV))
    Y8 = torch.zeros_like(Y16)
    N.grouped_gated_mlp_fp8(Xq, xs, ex, experts, ends, O.ACT_SILU, Y8)
    Y8d = torch.zeros_like(Y16)
    se = torch.tensor(experts, dtype=torch.int32, device=DEV)
    sn = torch.tensor(ends, dtype=torch.int32, device=DEV)
    N.grouped_gated_mlp_fp8(Xq, xs, ex, se, sn, O.ACT_SILU, Y8d)
    torch.cuda.synchronize()
    N.check_device_status(torch.device(DEV))
    n = ends[-1]
    assert torch.equal(Y8[:n], Y8d[:n])
    assert _rel_l2(Y8[:n].float().cpu(), Y16[:n].float().cpu()) <= 0.08
