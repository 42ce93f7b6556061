"""The device-driven data plane (NVLinkDirect backend) on one GPU.

* The exchange kernels' bookkeeping (dmoe_ep_plan / dmoe_ep_dispatch) against the CPU
  restatement in ``oracle/ep_placement.py``, bit for bit: parts, receive offsets, segment
  table, per-activation destinations, the rows that land in the receive buffer and their
  return addresses in the back map.
* The layer through ``DistMoEBlock.forward`` on the direct plane against the oracle:
  one block, several blocks with replicas (even split over alive replicas, one block lost
  mid-run), rotation over replicas, an expert with no alive block (its rows leave the sum),
  a shared expert, an empty batch, a 3-D input.

Tolerances are the layer's: rel-L2 1e-2 and max-abs 2e-2 (scaled by the output range when
it exceeds 1), against fp32 expert math.
"""

import pytest
import torch

from oracle import ep_placement as P
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


def _weights(E, d, I, seed, w_std=0.02):
    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g, device=DEV) * w_std).to(torch.bfloat16)
    return mk(E, I, d), mk(E, I, d), mk(E, d, I), mk(E, d), g


def _cluster(E, blocks, k, d, gate, up, down, max_tokens, **opts):
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    from distributedmoe_b200.TensorTransferEngine import TensorTransferEngineBackend as B
    stacked = [(gate[b].contiguous(), up[b].contiguous(), down[b].contiguous()) for b in blocks]
    return LocalCluster(E, blocks, k, d, torch.bfloat16, DEV, [DEV] * len(blocks), stacked=stacked,
                        io_buffer_size=256, number_of_io_buffers=1, backend=B.NVLinkDirect, max_tokens=max_tokens,
                        **opts)


def _oracle(x, w_r, gate, up, down, k, drop_experts=(), logit_bias=None, **kw):
    from distributedmoe_b200 import _native as N
    _, _, logits = N.router(x, w_r, k, logit_bias=logit_bias, want_logits=True)
    if drop_experts:
        g, u, dn = gate.clone(), up.clone(), down.clone()
        for e in drop_experts:
            dn[e].zero_()  # an expert whose rows never come back adds nothing
        gate, up, down = g, u, dn
    return O.local_experts(x, logits, gate, up, down, k, act=O.ACT_SILU, renormalize=True, compute_dtype=torch.float32,
                           **kw)


@gpu
@pytest.mark.parametrize("policy", [P.POLICY_ROTATE, P.POLICY_SPLIT])
def test_exchange_bookkeeping_matches_restatement(policy):
    """ep_plan + ep_dispatch with one rank over 3 blocks (two experts replicated, one
    expert with no alive instance) vs oracle/ep_placement.py, bit for bit."""
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.instances import InstanceTable

    E, k, d, T = 6, 2, 64, 301
    blocks = [[0, 1, 2], [2, 3, 4], [4, 0]]
    inst = InstanceTable.from_blocks(blocks, [0, 0, 0], 1, E)
    alive_blocks = [True, True, False]  # block 2 lost: experts 4 and 0 keep one instance each
    n, alive_inst = inst.alive_arrays(alive_blocks)
    n[5] = 0  # expert 5 is in no block: its rows are dropped
    g = torch.Generator(device=DEV).manual_seed(5)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:k] for _ in range(T)])
    plan = N.route_plan(idx, None, E, want_slot=True, want_weight=False)
    counts = plan["counts"].cpu().tolist()
    cap = T * k
    x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
    recv = torch.zeros(cap, d, dtype=torch.bfloat16, device=DEV)
    back = torch.full((cap,), -1, dtype=torch.int32, device=DEV)
    rows_ret = torch.zeros(T * k, d, dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(N.ep_flags_bytes() // 8, dtype=torch.int64, device=DEV)
    win = N.ep_window(1, 0, [flags.data_ptr()], [0], [recv.data_ptr()], [back.data_ptr()], [rows_ret.data_ptr()])
    i32 = dict(dtype=torch.int32, device=DEV)
    R = N.EP_MAX_REPLICAS
    table = (torch.tensor(n, **i32), torch.tensor(alive_inst, **i32), torch.tensor(inst.inst_rank, **i32),
             torch.tensor(inst.inst_slot, **i32), torch.tensor(inst.inst_first, **i32))
    part_n, part_inst = torch.zeros(E, **i32), torch.zeros(E * R, **i32)
    part_start, dest_off = torch.zeros(E * (R + 1), **i32), torch.zeros(inst.n_inst, **i32)
    seg_expert, seg_end = torch.zeros(inst.n_inst, **i32), torch.zeros(inst.n_inst, **i32)
    ret, done = torch.empty(T * k, **i32), torch.zeros(1, **i32)
    for epoch in (1, 2, 3):  # the window's counter: one per ep_plan call
        N.ep_plan(win, plan["counts"], E, inst.n_inst, policy, table, cap, 10**9,
                  (part_n, part_inst, part_start, dest_off, seg_expert, seg_end))
        N.ep_dispatch(win, x, T, k, E, plan["offsets"], plan["perm_token"], plan["perm_slot"],
                      (part_n, part_inst, part_start, dest_off), table[2], cap, ret, done)
        torch.cuda.synchronize()
        N.check_device_status(DEV)
        assert flags[3 * N.EP_MAX_RANKS].item() == epoch
        alive = [[[alive_inst[e * R + q] for q in range(n[e])] for e in range(E)]]
        ref = P.placement([counts], alive, inst.inst_rank, inst.inst_first, policy, epoch, cap)
        assert dest_off.cpu().tolist() == ref["dest_off"][0]
        assert seg_end.cpu().tolist() == ref["seg_end"][0]
        assert seg_expert.cpu().tolist() == inst.inst_slot
        dests = P.destinations(counts, ref["parts"][0], inst.inst_rank, ref["dest_off"][0], cap)
        got = ret.cpu().tolist()
        want = [-1 if r < 0 else (r << 27) | row for r, row in dests]
        assert got == want
        assert done.item() == 0
        # the rows: recv[row] == x[perm_token[p]] for every placed activation
        pt = plan["perm_token"].cpu()
        rows = [(p, row) for p, (r, row) in enumerate(dests) if r >= 0]
        src = x[pt[[p for p, _ in rows]].to(DEV)]
        dst = recv[torch.tensor([row for _, row in rows], device=DEV)]
        assert torch.equal(src, dst)
        # ... and each placed row's return address (rank 0, token * k + slot) in the back map
        ps = plan["perm_slot"].cpu()
        bk = back.cpu()
        assert all(bk[row].item() == pt[p].item() * k + ps[p].item() for p, row in rows)
        assert sum(1 for r, _ in dests if r < 0) == counts[5]


@gpu
@pytest.mark.parametrize("T", [1, 300, 2049])
def test_direct_layer_one_block(T):
    E, k, d, I = 8, 2, 256, 512
    gate, up, down, w_r, g = _weights(E, d, I, 11)
    cl = _cluster(E, [list(range(E))], k, d, gate, up, down, 4096, activation="silu", renormalize=True)
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        xs = [torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16) for _ in range(3)]
        ys = [cl.moe(x) for x in xs]
        torch.cuda.synchronize()
        from distributedmoe_b200 import _native as N
        N.check_device_status(DEV)
    finally:
        cl.close()
    for x, y in zip(xs, ys):
        assert y.shape == x.shape and y.dtype == x.dtype
        _check(y, _oracle(x, w_r, gate, up, down, k))


@gpu
def test_direct_layer_3d_input_and_empty_batch():
    from distributedmoe_b200 import _native as N
    E, k, d, I = 8, 2, 128, 256
    gate, up, down, w_r, g = _weights(E, d, I, 12)
    cl = _cluster(E, [list(range(E))], k, d, gate, up, down, 512, activation="silu", renormalize=True)
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        x = torch.randn(2, 100, d, generator=g, device=DEV).to(torch.bfloat16)
        y = cl.moe(x)
        empty = cl.moe(torch.empty(0, d, dtype=torch.bfloat16, device=DEV))
        y2 = cl.moe(x)
        torch.cuda.synchronize()
        N.check_device_status(DEV)
        with pytest.raises(ValueError):
            cl.moe(torch.empty(513, d, dtype=torch.bfloat16, device=DEV))
    finally:
        cl.close()
    assert y.shape == (2, 100, d) and empty.shape == (0, d)
    ref = _oracle(x.reshape(-1, d), w_r, gate, up, down, k)
    _check(y, ref)
    _check(y2, ref)


@gpu
@pytest.mark.parametrize("policy", ["least_loaded", "fifo"])
def test_direct_replicas_block_lost_midway(policy):
    """Every expert in two of eight blocks; block 3 lost after four steps, back after eight;
    all twelve steps match the oracle (least_loaded splits an expert's rows evenly over its
    alive replicas, fifo rotates whole experts over them)."""
    from distributedmoe_b200 import _native as N
    E, k, d, I, T = 8, 2, 256, 384, 777
    gate, up, down, w_r, g = _weights(E, d, I, 13)
    blocks = [[b, (b + 1) % E] for b in range(E)]
    cl = _cluster(E, blocks, k, d, gate, up, down, T, activation="silu", renormalize=True,
                  expert_block_policy=policy)
    outs = []
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        for step in range(12):
            if step == 4:
                cl.moe.disable_experts_block(3)
            if step == 8:
                cl.moe.enable_experts_block(3)
            x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
            outs.append((x, cl.moe(x)))
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    for x, y in outs:
        _check(y, _oracle(x, w_r, gate, up, down, k))


@gpu
def test_direct_expert_without_alive_block_leaves_the_sum():
    """Blocks [0..3] and [4..7]; with block 1 disabled, experts 4..7 have no alive instance:
    their rows are dropped and every token keeps only its other experts' contributions, as
    the reference's partial result keeps only the tasks that came back."""
    from distributedmoe_b200 import _native as N
    E, k, d, I, T = 8, 2, 128, 256, 500
    gate, up, down, w_r, g = _weights(E, d, I, 14)
    cl = _cluster(E, [[0, 1, 2, 3], [4, 5, 6, 7]], k, d, gate, up, down, T, activation="silu", renormalize=True)
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        cl.moe.disable_experts_block(1)
        x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
        y = cl.moe(x)
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    _check(y, _oracle(x, w_r, gate, up, down, k, drop_experts=(4, 5, 6, 7)))


@gpu
def test_direct_deepseek_router_and_shared_expert():
    from distributedmoe_b200 import _native as N
    E, k, d, I, I_s, T = 64, 8, 256, 128, 192, 400
    gate, up, down, w_r, g = _weights(E, d, I, 15, 0.006)
    sg, su, sd = [(torch.randn(*s, generator=g, device=DEV) * 0.006).to(torch.bfloat16)
                  for s in ((I_s, d), (I_s, d), (d, I_s))]
    bias = torch.randn(E, generator=g, device=DEV) * 0.01
    blocks = [list(range(0, E, 2)), list(range(1, E, 2))]
    cl = _cluster(E, blocks, k, d, gate, up, down, T, activation="silu", renormalize=True,
                  router_mode="sigmoid_group", routed_scaling_factor=2.5, n_group=8, topk_group=4)
    try:
        moe = cl.moe
        with torch.no_grad():
            moe.gate.weight.copy_(w_r)
        moe.score_bias = bias
        moe.set_shared_expert(sg, su, sd)
        x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
        ys = [moe(x) for _ in range(2)]
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    _, _, logits = N.router(x, w_r, k, want_logits=True)
    ref = O.local_experts(x, logits, gate, up, down, k, act=O.ACT_SILU, renormalize=True,
                          mode=O.ROUTER_SIGMOID_GROUP, score_bias=bias, scale=2.5, n_group=8, topk_group=4,
                          shared=(sg, su, sd), compute_dtype=torch.float32)
    for y in ys:
        _check(y, ref)


@gpu
def test_direct_layer_cuda_graph_replays_match_eager():
    """cuda_graphs=True: the first forward of each token count runs eagerly and is captured;
    later ones replay the graph (new inputs through the static buffer).  Every output matches
    the oracle, a block lost between replays is routed around (the alive table is uploaded
    outside the graph), and the replays are counted as library launches."""
    from distributedmoe_b200 import _native as N
    E, k, d, I = 8, 2, 256, 512
    gate, up, down, w_r, g = _weights(E, d, I, 16)
    blocks = [[b, (b + 1) % E] for b in range(E)]
    stacked = [(gate[b].contiguous(), up[b].contiguous(), down[b].contiguous()) for b in blocks]
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    from distributedmoe_b200.TensorTransferEngine import TensorTransferEngineBackend as B
    cl = LocalCluster(E, blocks, k, d, torch.bfloat16, DEV, [DEV] * len(blocks), stacked=stacked, io_buffer_size=256,
                      number_of_io_buffers=1, backend=B.NVLinkDirect, max_tokens=512, cuda_graphs=True,
                      activation="silu", renormalize=True, expert_block_policy="least_loaded")
    outs = []
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        for i, T in enumerate([64, 64, 64, 300, 64, 300, 300, 64]):
            if i == 5:
                cl.moe.disable_experts_block(2)
            x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
            before = N.launch_count()
            y = cl.moe(x)
            outs.append((x, y, N.launch_count() - before))
        torch.cuda.synchronize()
        N.check_device_status(DEV)
        assert sorted(cl.moe._ep["graphs"]) == [64, 300]
    finally:
        cl.close()
    for x, y, launches in outs:
        _check(y, _oracle(x, w_r, gate, up, down, k))
        assert launches >= 6


@gpu
@pytest.mark.parametrize("graphs", [False, True])
def test_direct_layer_fp8_experts(graphs):
    """expert_precision="fp8": 8-bit records cross the window and the gate/up GEMM runs on
    e4m3 tensor cores.  Against the oracle on the dequantised operands (row-wise e4m3 of the
    tokens and of the gate/up weights, bf16 down projection) the layer meets the bf16 bar,
    with replicated blocks and graph replays; against the 16-bit oracle it stays within
    e4m3's rounding."""
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    from distributedmoe_b200.TensorTransferEngine import TensorTransferEngineBackend as B
    E, k, d, I = 8, 2, 256, 384
    gate, up, down, w_r, g = _weights(E, d, I, 23)
    blocks = [[0, 1, 2, 3], [4, 5, 6, 7], [1, 6]]
    stacked = [(gate[b].contiguous(), up[b].contiguous(), down[b].contiguous()) for b in blocks]
    cl = LocalCluster(E, blocks, k, d, torch.bfloat16, DEV, [DEV] * len(blocks), stacked=stacked, io_buffer_size=256,
                      number_of_io_buffers=1, backend=B.NVLinkDirect, max_tokens=1024, cuda_graphs=graphs,
                      expert_precision="fp8", activation="silu", renormalize=True)
    outs = []
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        for T in [1, 200, 1024, 200]:
            x = torch.randn(T, d, generator=g, device=DEV).to(torch.bfloat16)
            outs.append((x, cl.moe(x)))
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    gd = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(gate)).to(DEV)
    ud = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(up)).to(DEV)
    for x, y in outs:
        _, _, logits = N.router(x, w_r, k, want_logits=True)
        xd = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(x)).to(DEV)
        ref = O.local_experts(xd, logits, gd, ud, down, k, act=O.ACT_SILU, renormalize=True,
                              compute_dtype=torch.float32)
        assert y.shape == x.shape and y.dtype == torch.bfloat16
        _check(y, ref)
        ref16 = _oracle(x, w_r, gate, up, down, k)
        rel = ((y.double() - ref16.double()).norm() / ref16.double().norm()).item()
        assert rel < 0.08, rel


@gpu
def test_direct_layer_fp32():
    """An fp32 layer on the direct plane: fp32 rows cross the window, the expert GEMMs run on
    tf32 tensor cores, the combine accumulates fp32 rows; against fp32 math."""
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    from distributedmoe_b200.TensorTransferEngine import TensorTransferEngineBackend as B
    E, k, d, I = 8, 2, 256, 384
    gate, up, down, w_r, g = _weights(E, d, I, 31)
    gate, up, down, w_r = gate.float(), up.float(), down.float(), w_r.float()
    blocks = [[0, 1, 2, 3], [4, 5, 6, 7], [2, 5]]
    stacked = [(gate[b].contiguous(), up[b].contiguous(), down[b].contiguous()) for b in blocks]
    cl = LocalCluster(E, blocks, k, d, torch.float32, DEV, [DEV] * len(blocks), stacked=stacked, io_buffer_size=256,
                      number_of_io_buffers=1, backend=B.NVLinkDirect, max_tokens=1024, activation="silu",
                      renormalize=True, expert_block_policy="least_loaded")
    outs = []
    try:
        with torch.no_grad():
            cl.moe.gate.weight.copy_(w_r)
        for T in [1, 300, 1024]:
            x = torch.randn(T, d, generator=g, device=DEV)
            outs.append((x, cl.moe(x)))
        torch.cuda.synchronize()
        N.check_device_status(DEV)
    finally:
        cl.close()
    for x, y in outs:
        assert y.shape == x.shape and y.dtype == torch.float32
        _check(y, _oracle(x, w_r, gate, up, down, k))
