"""Generate golden vectors by running the reference's own code on CPU.

Usage (in a container where the reference's source tree is available):
    python tests/golden/make_golden.py /path/to/reference
    DISTRIBUTEDMOE_REFERENCE=/path/to/reference python tests/golden/make_golden.py

The reference (slivanovich/DistributedMoE) is pure Python.  Its transfer libraries (nixl,
mooncake) are absent here, so they are replaced by empty stub modules; its data path is
driven with duck-typed CPU buffers and a capturing transfer engine:

* ``DistMoEBlock._setup_forward_pass`` (``src/python/MoE/DistMoEBlock.py:540-636``) builds the
  routing and per-expert lists,
* ``HostPipelineTask.dispatch`` (``src/python/MoE/PipelineTask.py:111-304``) packs and gathers,
* ``ExpertsBlockPipelineTask.run`` (``src/python/MoE/PipelineTask.py:424-574``) runs the
  grouped MLP, ``HostPipelineTask.combine`` (``:306-370``) combines,
* ``local_experts`` (``src/python/MoE/tests/dist_moe_test.py:173-197``) gives the local result.

The dispatch waves follow ``DistMoEBlock.async_forward`` (``:701-718``).  Inputs come from
``oracle/synthetic.py`` (seeded), so only outputs are stored.  Each config writes
``tests/golden/<name>.pt``.  Configs marked ``ext`` swap the reference's ReLU for SiLU
(extension, not reference behaviour).
"""

from __future__ import annotations

import asyncio
import contextlib
import os
import struct
import sys
import types
from types import SimpleNamespace

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import torch  # noqa: E402

from oracle.synthetic import make_layer_inputs  # noqa: E402

CONFIGS = [
    # name, T, d, E, k, I, dtype, expert_blocks, io_buffer_size, using_alignment, seed, act
    dict(name="tiny_e8k2", T=37, d=64, E=8, k=2, I=128, dtype=torch.float32, blocks=[list(range(8))],
         io=1024, align=False, seed=10, act="relu"),
    dict(name="split_2blocks", T=700, d=32, E=8, k=2, I=64, dtype=torch.float32,
         blocks=[[0, 2, 4, 6], [1, 3, 5, 7]], io=1024, align=False, seed=11, act="relu"),
    dict(name="align_pad", T=1500, d=32, E=8, k=2, I=64, dtype=torch.float32, blocks=[list(range(8))],
         io=2048, align=True, seed=12, act="relu"),
    dict(name="topk1", T=50, d=64, E=4, k=1, I=64, dtype=torch.float32, blocks=[list(range(4))],
         io=1024, align=False, seed=13, act="relu"),
    dict(name="replicas", T=600, d=32, E=8, k=2, I=64, dtype=torch.float32,
         blocks=[[0, 1, 2, 3, 4, 5], [2, 3, 4, 5, 6, 7]], io=1024, align=False, seed=14, act="relu"),
    dict(name="e16k4_sparse", T=5, d=64, E=16, k=4, I=64, dtype=torch.float32, blocks=[list(range(16))],
         io=1024, align=False, seed=15, act="relu"),
    dict(name="bf16_small", T=64, d=128, E=8, k=2, I=128, dtype=torch.bfloat16, blocks=[list(range(8))],
         io=1024, align=False, seed=16, act="relu"),
    dict(name="silu_ext", T=37, d=64, E=8, k=2, I=128, dtype=torch.float32, blocks=[list(range(8))],
         io=1024, align=False, seed=10, act="silu"),
    # The CPU plumbing configuration (T=256, d=1024, E=8, k=2, I=2816, fp32, seed 0).
    dict(name="plumbing", T=256, d=1024, E=8, k=2, I=2816, dtype=torch.float32, blocks=[list(range(8))],
         io=1024, align=False, seed=0, act="relu"),
]


def _install_stubs(ref_python: str) -> None:
    os.environ.setdefault("ENABLE_FILE_LOGGING", "false")
    os.environ.setdefault("LOG_LEVEL", "ERROR")
    sys.path.insert(0, ref_python)

    class _Dummy:  # stands in for the absent transfer-library types
        pass

    def stub(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m

    stub("nixl")
    stub("nixl._bindings", nixlXferDList=_Dummy, nixlRegDList=_Dummy)
    stub("nixl._api", nixl_xfer_handle=_Dummy, nixl_agent=_Dummy, nixl_agent_config=_Dummy)
    stub("nixl._utils")
    stub("mooncake")
    stub("mooncake.engine", TransferEngine=_Dummy)
    import TensorTransferEngine as pkg  # namespace package: the upstream __init__.py is not committed
    from TensorTransferEngine.TensorTransferEngine import TensorTransferEngine, TensorTransferEngineConfig
    pkg.TensorTransferEngine = TensorTransferEngine
    pkg.TensorTransferEngineConfig = TensorTransferEngineConfig


class _FakeStream:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False

    def synchronize(self):
        pass


class _FakeBuffer:
    def __init__(self, size, hidden, dtype, bid: bytes):
        self.size = size
        self.data = torch.zeros(size, hidden, dtype=dtype)
        self.device = self.data.device
        self.cuda_stream = _FakeStream()
        self.id = bid

    async def read_from(self, remote_name, src_buffer):
        self.data.copy_(src_buffer.data)

    async def write_to(self, remote_name, dst_buffer):
        dst_buffer.data.copy_(self.data)


class _FakePool:
    def __init__(self, n, size, hidden, dtype, id0):
        self.buffer_size = size
        self.buffers = [_FakeBuffer(size, hidden, dtype, (id0 + i).to_bytes(2, "big")) for i in range(n)]
        self.free = list(range(n))

    async def acquire(self):
        i = self.free.pop(0)
        return i, self.buffers[i]

    def release(self, i):
        self.free.append(i)


class _CaptureTTE:
    def __init__(self, names):
        self.remote_names = names
        self.sent = []

    async def async_send_metadata_to(self, remote_name, header, body):
        self.sent.append((remote_name, header, body))


def run_config(cfg):
    from MoE.DistMoE import ExpertMetaData, P2PHeaders
    from MoE.DistMoEBlock import DistMoEBlock
    from MoE.DistExpertsBlock import DistExpertsBlock
    from MoE.MoE import Qwen3MoEMLP
    from MoE.PipelineTask import ExpertsBlockPipelineTask, HostPipelineTask
    from MoE.pools.ExpertBlocksPool import ExpertBlocksPool
    from MoE.tests.dist_moe_test import local_experts
    from TensorTransferEngine.TensorTransferEngine import TensorTransferEngine
    from queue import Queue

    T, d, E, k, I, dtype = cfg["T"], cfg["d"], cfg["E"], cfg["k"], cfg["I"], cfg["dtype"]
    inp = make_layer_inputs(T, d, E, I, cfg["seed"], dtype)
    act_silu = cfg["act"] == "silu"

    layers = []
    for e in range(E):
        m = Qwen3MoEMLP(d, I, dtype)
        with torch.no_grad():
            m.gate_proj.weight.copy_(inp.gate[e])
            m.up_proj.weight.copy_(inp.up[e])
            m.down_proj.weight.copy_(inp.down[e])
        if act_silu:
            m.activation = torch.nn.SiLU()
        layers.append(m)

    gate = torch.nn.Linear(d, E, bias=False, dtype=dtype)
    with torch.no_grad():
        gate.weight.copy_(inp.w_r)

    # --- routing: DistMoEBlock._setup_forward_pass called unbound on a namespace -------
    host = SimpleNamespace(dtype=dtype, device=torch.device("cpu"), hidden_features=d, gate=gate, top_k=k,
                           number_of_experts=E, experts_metadata={}, logger=None, output_batch=None)
    for e in range(E):
        host.experts_metadata[e] = ExpertMetaData(block_indexes=[], expert_shared_rate=0,
                                                  expert_weights=torch.empty(1, dtype=dtype),
                                                  expert_token_indexes=torch.empty(1, dtype=torch.int),
                                                  expert_total_activations=0, expert_offsets=Queue())
    with torch.no_grad():
        experts_hit, input_batch = DistMoEBlock._setup_forward_pass(host, inp.x)
        logits = gate(inp.x)
        probs = torch.nn.functional.softmax(logits, dim=1, dtype=torch.float)
        rw, sel = torch.topk(probs, k, dim=-1)

    # --- expert-block weights as DistExpertsBlock.initialize_expert_layers stacks them ---
    eb_states = []
    orig_stream = torch.cuda.Stream
    torch.cuda.Stream = lambda device=None: _FakeStream()  # CPU stand-in for per-expert streams
    try:
        for b, blk in enumerate(cfg["blocks"]):
            ns = SimpleNamespace(experts_block_index=b, device=torch.device("cpu"), expert_layers={}, expert_streams={})
            DistExpertsBlock.initialize_expert_layers(ns, cfg["blocks"], [layers[e] for e in blk])
            eb_states.append(ns)
    finally:
        torch.cuda.Stream = orig_stream

    # --- dispatch / expert run / combine, in the waves of async_forward ---------------
    io = cfg["io"]
    n_buf = 64
    remote_names = [f"eb{b}" for b in range(len(cfg["blocks"]))]
    host_tte = _CaptureTTE(remote_names)
    host_in = _FakePool(n_buf, io, d, dtype, 0)
    host_out = _FakePool(n_buf, io, d, dtype, n_buf)
    blocks_pool = ExpertBlocksPool(cfg["blocks"])
    candidates = []
    step = io // 1024
    candidates = list(range(step, io, step)) + [io]
    codec = SimpleNamespace(_serialized_size=2)

    tasks_record = []
    output_batch = torch.zeros(T, d, dtype=dtype)

    async def forward():
        lock = asyncio.Lock()
        active = [0]
        transferred = [0]
        eb_tasks = {}
        total = k * T
        combining = asyncio.Event()
        orig_cuda_stream_ctx = torch.cuda.stream
        orig_relu = torch.nn.functional.relu
        torch.cuda.stream = lambda s: contextlib.nullcontext()
        if act_silu:
            # Extension: the grouped path hard-codes ReLU (MoE/PipelineTask.py:518); swap it.
            torch.nn.functional.relu = torch.nn.functional.silu
        try:
            while transferred[0] < total:
                n_disp = max(-(-(total - transferred[0]) // io), 1)
                wave = []
                for _ in range(n_disp):
                    t = HostPipelineTask(host_tte, host_in, host_out, experts_hit, blocks_pool,
                                         host.experts_metadata, lock, None)
                    wave.append(t)
                for t in wave:
                    n_before = len(host_tte.sent)
                    await t.dispatch(input_batch, active, transferred, eb_tasks,
                                     candidates if cfg["align"] else None, True)
                    if len(host_tte.sent) == n_before:
                        continue
                    remote, header, body = host_tte.sent[-1]
                    assert header == P2PHeaders.DispatchSubmit.value
                    packet = TensorTransferEngine.serialize_p2p_packet(codec, header, body)
                    _, metadata = TensorTransferEngine.deserialize_p2p_packet(codec, packet)
                    b = remote_names.index(remote)
                    in_snapshot = t.input_buffer.data.clone()
                    eb = eb_states[b]
                    eb_tte = _CaptureTTE([f"host"])
                    eb_in = _FakePool(1, io, d, dtype, 0)
                    eb_out = _FakePool(1, io, d, dtype, 1)
                    run = ExpertsBlockPipelineTask(eb_tte, eb_in, eb_out, eb.expert_layers, eb.experts_combine_layer,
                                                   eb.expert_streams, "host", metadata, asyncio.Lock(), None)
                    host_in_descs = {t.input_buffer.id: t.input_buffer}
                    host_out_descs = {t.output_buffer.id: t.output_buffer}
                    await run.run(b, host_in_descs, host_out_descs)
                    assert eb_tte.sent and eb_tte.sent[-1][1] == P2PHeaders.HostOutputBufferUnlocked.value
                    out_snapshot = t.output_buffer.data.clone()
                    segs = []
                    n_exp = struct.unpack("!H", metadata[2][1])[0]
                    for i in range(n_exp):
                        segs.append(tuple(struct.unpack("!H", metadata[3 + 3 * i + j][1])[0] for j in range(3)))
                    await t.combine(active, output_batch, combining)
                    tasks_record.append(dict(block=b, packet_segments=segs,
                                             snapshot=list(t.experts_metadata_snapshot),
                                             used=t.used_activations, packet=packet,
                                             in_rows=in_snapshot, out_rows=out_snapshot))
        finally:
            torch.cuda.stream = orig_cuda_stream_ctx
            torch.nn.functional.relu = orig_relu

    asyncio.run(forward())

    with torch.no_grad():
        moe = SimpleNamespace(hidden_features=d, dtype=dtype, device=torch.device("cpu"), gate=gate, top_k=k,
                              number_of_experts=E)
        local = local_experts(moe, layers, inp.x.clone())

    per_expert = {e: dict(tokens=host.experts_metadata[e].expert_token_indexes.clone(),
                          weights=host.experts_metadata[e].expert_weights.flatten().clone())
                  for e in experts_hit}
    big = cfg["name"] == "plumbing"
    keep_rows = k * T <= 256
    rec = dict(
        config={key: (str(v) if key == "dtype" else v) for key, v in cfg.items()},
        experts_hit=list(experts_hit), logits=None if big else logits.clone(), selected=sel.clone(),
        routing_weights=rw.clone(), per_expert=per_expert,
        tasks=[{key: v for key, v in tr.items() if (keep_rows or key not in ("in_rows", "out_rows"))} for tr in tasks_record],
        output=output_batch.clone(), local=local.clone(),
    )
    if big:
        # Keep the fixture small: every 8th output row plus fp64 row sums / norms of all rows.
        rec["output"] = output_batch[::8].clone()
        rec["local"] = local[::8].clone()
        rec["output_row_sum"] = output_batch.double().sum(1)
        rec["output_row_norm"] = output_batch.double().norm(dim=1)
        rec["logits_rows"] = logits[::8].clone()
    for tr in rec["tasks"]:
        if "in_rows" in tr:
            used = sum(s[2] for s in tr["packet_segments"])
            tr["in_rows"] = tr["in_rows"][:used].clone()
            tr["out_rows"] = tr["out_rows"][:used].clone()
    return rec


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DISTRIBUTEDMOE_REFERENCE")
    if not ref:
        raise SystemExit("usage: make_golden.py /path/to/reference  (or set DISTRIBUTEDMOE_REFERENCE)")
    _install_stubs(os.path.join(ref, "src", "python"))
    cwd = os.getcwd()
    os.chdir("/tmp")  # the reference's logging may create ./logs
    try:
        for cfg in CONFIGS:
            rec = run_config(cfg)
            path = os.path.join(HERE, cfg["name"] + ".pt")
            torch.save(rec, path)
            print(f"{cfg['name']}: experts_hit={len(rec['experts_hit'])} tasks={len(rec['tasks'])} "
                  f"max|out-local|={(rec['output'].double() - rec['local'].double()).abs().max().item():.3e} -> {path}")
    finally:
        os.chdir(cwd)


if __name__ == "__main__":
    main()
