"""The drop-in API end to end on a GPU: DistMoEBlock + DistExpertsBlock threads over the
NVLink/CUDA-IPC transfer engine, against the oracle (mirrors the reference's
``MoE/tests/dist_moe_test.py::test_forward``, which checks DistMoEBlock(x) against
``local_experts``)."""

import pytest
import torch

from oracle import moe_oracle as O
from oracle.synthetic import make_layer_inputs

gpu = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _rel_l2(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def _layers(inp, E, dtype):
    from distributedmoe_b200.MoE.MoE import Qwen3MoEMLP
    out = []
    for e in range(E):
        m = Qwen3MoEMLP(inp.x.shape[1], inp.gate.shape[1], dtype)
        with torch.no_grad():
            m.gate_proj.weight.copy_(inp.gate[e])
            m.up_proj.weight.copy_(inp.up[e])
            m.down_proj.weight.copy_(inp.down[e])
        out.append(m)
    return out


def _run(T, d, E, k, I, blocks, io, *, dtype=torch.bfloat16, seed=0, align=False, act="relu", renorm=False,
         shape3d=False, forwards=2, disable=None, x_mean=0.0, **opts):
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    inp = make_layer_inputs(T, d, E, I, seed, dtype, x_mean=x_mean)
    layers = _layers(inp, E, dtype)
    cl = LocalCluster(E, blocks, k, d, dtype, DEV, [DEV] * len(blocks),
                      expert_layers=[[layers[e] for e in b] for b in blocks], io_buffer_size=io,
                      number_of_io_buffers=4, activation=act, renormalize=renorm, **opts)
    try:
        moe = cl.moe
        with torch.no_grad():
            moe.gate.weight.copy_(inp.w_r.to(DEV))
        if disable is not None:
            moe.disable_experts_block(disable)
        x = inp.x.to(DEV)
        if shape3d:
            x = x.view(1, T, d)
        outs = [moe(x, using_alignment=align) for _ in range(forwards)]
        torch.cuda.synchronize()
        N.check_device_status(DEV)
        _, _, logits = N.router(inp.x.to(DEV), inp.w_r.to(DEV), k, want_logits=True)
        ref = O.local_experts(inp.x, logits.cpu(), inp.gate, inp.up, inp.down, k, act=O.ACT_SILU if act == "silu" else O.ACT_RELU,
                              renormalize=renorm, compute_dtype=torch.float32)
    finally:
        cl.close()
    for y in outs:
        assert y.shape == x.shape and y.dtype == dtype
        yy = y.reshape(T, d).float().cpu()
        assert _rel_l2(yy, ref) < 1e-2
        assert (yy - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
    return outs


@gpu
def test_forward_one_block():
    _run(300, 256, 8, 2, 512, [list(range(8))], 1024)


@gpu
def test_forward_reference_test_shape_fp16():
    """The reference test's layer shape (E=128, k=8, d=2048, I=6144, fp16, inputs randn+10),
    fewer tokens."""
    _run(512, 2048, 128, 8, 6144, [list(range(128))], 8192, dtype=torch.float16, x_mean=10.0, forwards=1)


@gpu
def test_forward_reference_test_shape_fp32():
    """The reference test's "--precision fp32" (MoE/tests/conftest.py:17-21): fp32 layer, the
    expert GEMMs on tf32 tensor cores (operands rounded to a 10-bit mantissa, fp32
    accumulation), within the same bars against fp32 math."""
    _run(512, 2048, 128, 8, 6144, [list(range(128))], 8192, dtype=torch.float32, x_mean=10.0, forwards=1)


@gpu
def test_forward_split_tasks_two_blocks_silu_renorm_3d():
    _run(700, 128, 8, 2, 256, [[0, 2, 4, 6], [1, 3, 5, 7]], 1024, act="silu", renorm=True, shape3d=True)


@gpu
def test_forward_alignment_padding():
    _run(1500, 128, 8, 2, 128, [list(range(8))], 2048, align=True)


@gpu
def test_forward_top1_and_sparse_experts():
    _run(50, 128, 4, 1, 128, [list(range(4))], 1024)
    _run(5, 128, 16, 4, 128, [list(range(16))], 1024)


@gpu
def test_forward_replica_survives_disabled_block():
    """Every expert lives in two blocks; with block 0 disabled, block 1 serves all of them
    (ExpertBlocksPool drops dead blocks, MoE/pools/ExpertBlocksPool.py:37-45)."""
    _run(600, 128, 8, 2, 128, [list(range(8)), list(range(8))], 1024, disable=0)


@gpu
def test_forward_least_loaded_policy():
    _run(600, 128, 8, 2, 128, [list(range(8)), list(range(8))], 1024, expert_block_policy="least_loaded")


@gpu
def test_local_sparse_moe_block_matches_oracle():
    from distributedmoe_b200.MoE.MoE import Qwen3SparseMoEBlock
    from distributedmoe_b200 import _native as N
    T, d, E, k, I = 333, 256, 8, 2, 384
    inp = make_layer_inputs(T, d, E, I, 5, torch.bfloat16)
    blk = Qwen3SparseMoEBlock(E, k, d, I, torch.bfloat16, activation="silu").to(DEV)
    with torch.no_grad():
        blk.gate.weight.copy_(inp.w_r)
        for e in range(E):
            blk.experts[e].gate_proj.weight.copy_(inp.gate[e])
            blk.experts[e].up_proj.weight.copy_(inp.up[e])
            blk.experts[e].down_proj.weight.copy_(inp.down[e])
    y = blk(inp.x.to(DEV).view(1, T, d))
    _, _, logits = N.router(inp.x.to(DEV), inp.w_r.to(DEV), k, want_logits=True)
    ref = O.local_experts(inp.x, logits.cpu(), inp.gate, inp.up, inp.down, k, act=O.ACT_SILU, compute_dtype=torch.float32)
    assert _rel_l2(y.view(T, d).float().cpu(), ref) < 1e-2


@gpu
def test_forward_timeout_returns_partial_result(monkeypatch):
    """A block that silently drops its task (no output, no acknowledgement, but still answers
    health checks) makes the host wait until forward_timeout and return the partial result:
    every token keeps the contributions of the experts whose tasks came back and loses those
    of the silent block's experts (the reference's SLA path, MoE/DistMoEBlock.py:709-718)."""
    import time

    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE import PipelineTask as PT
    from distributedmoe_b200.MoE.local_cluster import LocalCluster

    real_run = PT.ExpertsBlockPipelineTask.run

    async def run(self, experts_block_index, *a, **kw):
        if experts_block_index == 1:
            self.close()
            return  # the task is lost: nothing computed, nothing acknowledged
        return await real_run(self, experts_block_index, *a, **kw)

    monkeypatch.setattr(PT.ExpertsBlockPipelineTask, "run", run)
    T, d, E, k, I = 400, 128, 8, 2, 256
    inp = make_layer_inputs(T, d, E, I, 21, torch.bfloat16)
    layers = _layers(inp, E, torch.bfloat16)
    blocks = [[0, 1, 2, 3], [4, 5, 6, 7]]
    cl = LocalCluster(E, blocks, k, d, torch.bfloat16, DEV, [DEV, DEV],
                      expert_layers=[[layers[e] for e in b] for b in blocks], io_buffer_size=1024,
                      number_of_io_buffers=4, activation="silu", renormalize=True, forward_timeout=1500)
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(inp.w_r.to(DEV))
        t0 = time.monotonic()
        y = cl.moe(inp.x.to(DEV))
        waited = time.monotonic() - t0
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    assert waited >= 1.0, "the host returned before its forward timeout"
    _, _, logits = N.router(inp.x.to(DEV), inp.w_r.to(DEV), k, want_logits=True)
    down = inp.down.clone()
    down[4:] = 0  # the silent block's experts contribute nothing
    ref = O.local_experts(inp.x, logits.cpu(), inp.gate, inp.up, down, k, act=O.ACT_SILU, renormalize=True,
                          compute_dtype=torch.float32)
    yy = y.float().cpu()
    assert _rel_l2(yy, ref) < 1e-2
    assert (yy - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
