"""Host-side logic that needs no GPU: segment queues, expert-block selection, the engine's
descriptor and completion-notice packets, the expert-parallel port exchange over two
`gloo` ranks, and the benchmark's workload bookkeeping."""

import asyncio
import os
import socket
import struct

import pytest
import torch
import torch.multiprocessing as mp

from distributedmoe_b200.MoE.DistMoE import SegmentQueue
from distributedmoe_b200.MoE.pools.ExpertBlocksPool import ExpertBlocksPool


# ----------------------------------------------------------------------------- segment queue
def test_segment_queue_has_rows_ignores_used_up_segments():
    q = SegmentQueue([(0, 5)])
    assert not q.empty() and q.has_rows()
    l, r = q.get_nowait()
    q.put_nowait((r, r))  # dispatch re-queues a segment it used up (reference behaviour)
    assert not q.empty()
    assert not q.has_rows()
    q.put_nowait((7, 9))  # an aborted task's rows come back
    assert q.has_rows()
    assert q.items() == [(5, 5), (7, 9)]


# ----------------------------------------------------------------------------- block pool
def _run(coro):
    return asyncio.new_event_loop().run_until_complete(coro)


def test_fifo_pool_round_robin_skips_dead_blocks():
    pool = ExpertBlocksPool([[0, 1], [2, 3], [4, 5]])

    async def take(n):
        out = []
        for _ in range(n):
            b, _md = await pool.aquire()
            out.append(b)
            pool.release(b)
        return out

    assert _run(take(4)) == [0, 1, 2, 0]
    pool.mark_dead(1)
    assert _run(take(3)) == [2, 0, 2]
    pool.mark_alive(1)
    assert 1 in _run(take(3))


def test_least_loaded_pool_prefers_idle_candidates():
    pool = ExpertBlocksPool([[0], [1], [2]], policy="least_loaded")
    pool.add_load(0, 100)
    pool.add_load(1, 10)
    b, _ = _run(pool.aquire())
    assert b == 2
    b, _ = _run(pool.aquire([0, 1]))
    assert b == 1
    pool.mark_dead(1)
    b, _ = _run(pool.aquire([0, 1]))
    assert b == 0
    pool.sub_load(0, 1000)
    assert pool.load[0] == 0


def test_unknown_policy_is_rejected():
    with pytest.raises(ValueError):
        ExpertBlocksPool([[0]], policy="random")


# ----------------------------------------------------------------------------- engine packets
def _bare_engine(pid=1234):
    """An NVLink engine object without sockets or a GPU: enough for its packet code."""
    from distributedmoe_b200.TensorTransferEngine.NVLinkTensorTransferEngine import NVLinkTensorTransferEngine
    import threading

    e = object.__new__(NVLinkTensorTransferEngine)
    e.pid = pid
    e._serialized_size = 2
    e._lock = threading.Lock()
    e._notice_events = {}
    e._pending_notice = {}
    e._region_owner = {}
    e.remote_info = {}
    return e


def test_region_descriptors_round_trip():
    from distributedmoe_b200.TensorTransferEngine.NVLinkTensorTransferEngine import NVLinkRegion

    e = _bare_engine()
    regions = [NVLinkRegion(e.pid, 3, 0x7F0000001000 + i, 4096 * (i + 1), bytes([i]) * 64, 256 * i, 10 + i,
                            bytes([200 + i]) * 64) for i in range(3)]
    back = e.deserialize_descs(e.serialize_descs(regions))
    assert back == regions


def test_completion_notice_packet_names_owner_device_and_regions():
    from distributedmoe_b200.TensorTransferEngine.NVLinkTensorTransferEngine import NOTICE_HEADER, NVLinkRegion

    e = _bare_engine()
    e.remote_info = {"127.0.0.1:5000": (4321, 1, "box"), "127.0.0.1:6000": (999, 2, "box")}
    handle = bytes(range(64))
    stream_key = 0xABC
    e._notice_events[stream_key] = (1, 0xDEAD, handle)
    regions = [NVLinkRegion(4321, 1, 0, 16, b"\0" * 64, 0, tok, b"\0" * 64) for tok in (9, 3, 9)]
    for r in regions:
        owner = e._owner_name(r)
        assert owner == "127.0.0.1:5000"
        e._pending_notice.setdefault(owner, {}).setdefault(stream_key, set()).add(r.event_token)
    packets = e._take_notices("127.0.0.1:5000")
    assert len(packets) == 1 and e._take_notices("127.0.0.1:5000") == []
    header, body = e.deserialize_p2p_packet(packets[0])
    assert header == NOTICE_HEADER
    assert struct.unpack("!h", body[0][1]) == (1,)
    assert body[1][1] == handle
    assert [struct.unpack("!Q", raw)[0] for _, raw in body[2:]] == [3, 9]
    # a region of a process that is no peer of this engine has no owner
    assert e._owner_name(NVLinkRegion(777, 0, 0, 16, b"\0" * 64, 0, 1, b"\0" * 64)) is None


# ----------------------------------------------------------------------------- port exchange
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _port_worker(rank, world, port, results):
    import torch.distributed as dist
    from datetime import timedelta
    from distributedmoe_b200.MoE.sharded_cluster import _ports_collide, exchange_engine_ports

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        table = exchange_engine_ports("127.0.0.1", rank)
        results.put((rank, table, _ports_collide(table)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_engine_port_exchange_over_gloo_ranks(world):
    """Every rank gets the same table of engine ports, with no port used twice (4 ranks pick
    84 listener ports)."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_port_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, table, collide = results.get(timeout=120)
            out[rank] = (table, collide)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert sorted(out) == list(range(world))
    t0 = out[0][0]
    assert all(out[r][0] == t0 for r in range(world))  # every rank sees the same table
    assert not out[0][1]
    for r, row in enumerate(t0):
        assert row["device"] == r and row["address"] == "127.0.0.1"
        for key in ("host_p2p", "host_hc", "eb_port", "eb_p2p", "eb_hc"):
            assert len(row[key]) == world
    ports = [p for row in t0 for key in ("host_p2p", "host_hc", "eb_port", "eb_p2p", "eb_hc") for p in row[key]]
    ports += [row["host_port"] for row in t0]
    assert len(ports) == len(set(ports))


# ----------------------------------------------------------------------------- bench workloads
def test_bench_workloads():
    import bench

    mix, ds = bench.WORKLOADS["mixtral"], bench.WORKLOADS["deepseek"]
    # weak scaling: tokens per GPU fixed; strong: the step's tokens split over the GPUs
    assert mix.tokens_per_rank(8) == 4096 and ds.tokens_per_rank(8) == 1024
    assert mix.mlp_flops(4096 * 2) == 6.0 * 4096 * 2 * 4096 * 14336
    qwen = bench.WORKLOADS["qwen3-decode"]
    assert qwen.E == 128 and qwen.k == 8 and qwen.strong
    # one host's task buffers: every activation fits one wave; packet fields stay 16-bit
    for w in (mix, ds, qwen):
        for world in (1, 2, 4, 8):
            par = "experts" if world > 1 else "single"
            size, n = w.io(world, par)
            assert 256 <= size <= 65535
            per_host = w.tokens_per_rank(world) * w.k
            if par == "single":
                assert size * n >= per_host
            else:
                assert n == 2 * world and size >= per_host // world
            c = w.config(world, par, "tasks")
            assert c["io_buffer_size"] == size and c["io_buffers"] == n
            assert c["tokens_per_gpu"] * world == c["tokens_per_step"]
            c = w.config(world, par, "direct")
            assert c["transfer_engine"] == "NVLinkDirect" and "io_buffer_size" not in c
            blocks, ranks = w.blocks(world)
            assert ranks == list(range(world)) and sorted(e for b in blocks for e in b) == list(range(w.E))
    # skewed fault tolerance: every expert in exactly two blocks, on two different GPUs
    ft = bench.WORKLOADS["skewed-ft"]
    for world in (1, 2, 4, 8):
        blocks, ranks = ft.blocks(world)
        for e in range(ft.E):
            holders = [b for b, experts in enumerate(blocks) if e in experts]
            assert len(holders) == 2
            if world > 1:
                assert ranks[holders[0]] != ranks[holders[1]]
    assert ft.tokens_per_rank(8) == 2048 and ft.fail_block == 3


# ----------------------------------------------------------------------------- health checks
class _FakePair:
    """Health-check sockets of one block: pings are recorded; a pong comes back while the
    block is 'up', nothing while it is 'down'."""

    def __init__(self, engine):
        from distributedmoe_b200.MoE.DistMoE import P2PHeaders

        self.up = True
        self.pings = 0
        self._pong = engine.serialize_p2p_packet(P2PHeaders.Pong.value, [])
        outer = self

        class _Push:
            async def send(self, packet):
                outer.pings += 1

        class _Pull:
            async def recv(self):
                while not outer.up:
                    await asyncio.sleep(0.01)
                return outer._pong

        self.pusher, self.puller = _Push(), _Pull()


class _FakeTask:
    def __init__(self):
        self.aborted = False
        self.dispatch_done = True
        self.combine_done = False
        self.used_activations = 5

    def abort(self):
        self.aborted = True


def test_health_checker_marks_a_silent_block_dead_then_alive_and_aborts_its_tasks():
    """MoE/DistMoEBlock.py:312-414: a block that does not answer a ping within the P2P
    timeout (1 s here) is marked dead and the tasks dispatched to it are aborted (their
    activations go back to the queues); when it answers again it is marked alive."""
    import logging
    from distributedmoe_b200.MoE.DistMoEBlock import DistMoEBlock

    eng = _bare_engine()
    blk = object.__new__(DistMoEBlock)
    pair = _FakePair(eng)
    blk.monitoring_flag = True
    blk.health_check_timeout = 1000  # ms
    blk.disabled_expert_blocks = set()
    blk.health_check_p2p_pairs = {"eb0": pair}
    blk.tensor_transfer_engine = eng
    blk.expert_blocks_pool = ExpertBlocksPool([[0, 1], [2, 3]])
    blk.logger = logging.getLogger("test.health")
    task = _FakeTask()
    blk.pipeline_tasks = {b"t": task}
    blk.expert_block_tasks = {0: [b"t"]}
    blk.dispatch_tasks, blk.combine_tasks = {}, {}
    blk.transferred_activations = [5]
    blk.active_pipeline_tasks = [1]

    async def scenario():
        blk.async_lock = asyncio.Lock()
        blk.combining = asyncio.Event()
        checker = asyncio.create_task(blk._expert_block_health_checker(0, "eb0"))
        md = blk.expert_blocks_pool.expert_blocks_metadata[0]
        await asyncio.sleep(0.15)
        alive_before = md.is_alive
        pair.up = False
        await asyncio.sleep(1.4)
        dead_after_silence = not md.is_alive
        pair.up = True
        await asyncio.sleep(0.3)
        alive_again = md.is_alive
        blk.monitoring_flag = False
        checker.cancel()
        await asyncio.gather(checker, return_exceptions=True)
        return alive_before, dead_after_silence, alive_again

    alive_before, dead_after_silence, alive_again = _run(scenario())
    assert alive_before and dead_after_silence and alive_again
    assert pair.pings > 3
    assert task.aborted
    assert blk.transferred_activations == [0] and blk.active_pipeline_tasks == [0]
    assert blk.expert_block_tasks[0] == [] and b"t" not in blk.pipeline_tasks


# ----------------------------------------------------------------------------- wire format
class _FakeStream:
    cuda_stream = 0

    def wait_event(self, ev):
        pass


class _FakeBuffer:
    def __init__(self, i):
        self.id = i.to_bytes(length=2, byteorder="big")
        self.cuda_stream = _FakeStream()
        self.data = None

    def begin_use(self, s):
        pass

    def end_use(self, s):
        pass


class _FakePool:
    def __init__(self, size, first_id):
        self.buffer_size = size
        self._next = first_id

    async def acquire(self):
        self._next += 1
        return self._next, _FakeBuffer(self._next)

    def release(self, i):
        pass


class _CaptureEngine:
    def __init__(self, blocks):
        self.remote_names = [f"block-{b}" for b in range(blocks)]
        self.sent = []

    async def async_send_metadata_to(self, remote_name, header, body):
        self.sent.append((remote_name, header, body))


class _FakeEvent:
    def record(self, s=None):
        pass


@pytest.mark.parametrize("name", ["tiny_e8k2", "split_2blocks", "align_pad", "topk1", "replicas", "e16k4_sparse",
                                  "plumbing"])
def test_product_dispatch_packets_match_reference_bytes(name, monkeypatch):
    """The product's own HostPipelineTask.dispatch (not the oracle's encoder) produces, wave
    by wave, the reference's DispatchSubmit packets byte for byte (golden packets recorded
    from the reference's code), apart from the random task name and the buffer ids."""
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.DistMoE import ExpertMetaData, SegmentQueue
    from distributedmoe_b200.MoE.PipelineTask import ForwardState, HostPipelineTask
    from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import TensorTransferEngine

    g = torch.load(os.path.join(os.path.dirname(__file__), "golden", name + ".pt"), weights_only=False)
    cfg = g["config"]
    E, blocks, io, k, T = cfg["E"], cfg["blocks"], cfg["io"], cfg["k"], cfg["T"]
    monkeypatch.setattr(N, "permute_rows", lambda *a, **kw: None)
    monkeypatch.setattr(torch.cuda, "Event", _FakeEvent)
    counts = [0] * E
    for e, pe in g["per_expert"].items():
        counts[e] = pe["tokens"].numel()
    plan = {"perm_token": torch.zeros(max(sum(counts), 1), dtype=torch.int32)}
    md = {}
    base = 0
    for e in range(E):
        md[e] = ExpertMetaData([b for b in range(len(blocks)) if e in blocks[b]], 0, None, None, 0, SegmentQueue())
        if counts[e]:
            md[e].bind(plan, base, counts[e])
        base += counts[e]
    hit = [e for e in range(E) if counts[e]]
    pool = ExpertBlocksPool(blocks)
    engine = _CaptureEngine(len(blocks))
    fs = ForwardState(None, plan, [0] * (E + 1), None, None, None)
    candidates = list(range(io // 1024, io, io // 1024)) + [io] if cfg["align"] else None
    transferred, active = [0], [0]
    tasks_of_block = {}

    async def waves():
        lock = asyncio.Lock()
        while transferred[0] < k * T:
            n = max(-(-(k * T - transferred[0]) // io), 1)
            for _ in range(n):  # a wave's tasks run in creation order
                t = HostPipelineTask(engine, _FakePool(io, 0), _FakePool(io, 100), hit, pool, md, lock,
                                     forward_state=fs)
                await t.dispatch(None, active, transferred, tasks_of_block, candidates, True)

    asyncio.new_event_loop().run_until_complete(waves())
    sent = [(r, TensorTransferEngine.serialize_p2p_packet(None, h, body)) for r, h, body in engine.sent]
    assert len(sent) == len(g["tasks"])
    for (remote, pkt), ref in zip(sent, g["tasks"]):
        assert remote == f"block-{ref['block']}"
        assert pkt[:6] == ref["packet"][:6]            # header 1038, item count, name length
        assert pkt[14:-8] == ref["packet"][14:-8]      # grouped-gemm flag, expert count, segments
        assert len(pkt) == len(ref["packet"])          # same two 2-byte buffer ids at the end


# ----------------------------------------------------------------------------- direct plane host logic
def test_instance_table_layout_and_alive_lists():
    from distributedmoe_b200.MoE.instances import InstanceTable
    blocks = [[0, 1], [2, 3], [1, 2], [3, 0]]
    t = InstanceTable.from_blocks(blocks, [0, 1, 0, 1], 2, 4)
    # rank-major, each rank's blocks in index order, each block's experts in list order
    assert t.inst_rank == [0, 0, 0, 0, 1, 1, 1, 1]
    assert t.inst_expert == [0, 1, 1, 2, 2, 3, 3, 0]
    assert t.inst_slot == [0, 1, 2, 3, 0, 1, 2, 3]
    assert t.inst_first == [0, 4, 8] and t.local_blocks(0) == [0, 2] and t.local_blocks(1) == [1, 3]
    n, inst = t.alive_arrays([True, True, True, True])
    R = 4
    assert n == [2, 2, 2, 2]
    assert inst[0 * R:0 * R + 2] == [0, 7] and inst[1 * R:1 * R + 2] == [1, 2]
    n, inst = t.alive_arrays([True, False, True, True])  # block 1 (experts 2, 3 on rank 1) lost
    assert n == [2, 2, 1, 1] and inst[2 * R] == 3 and inst[3 * R] == 6
    with pytest.raises(ValueError):
        InstanceTable.from_blocks([[0, 1]] * 5, [0] * 5, 1, 2)  # five replicas of an expert
    with pytest.raises(ValueError):
        InstanceTable.from_blocks([[0, 9]], [0], 1, 4)


def test_placement_restatement_properties():
    """oracle/ep_placement.py: every sender's rows of an instance form one contiguous run of
    the owner's buffer, senders in rank order, instances in stack order, nothing overlaps, and
    each owner's segment table ends where its rows end."""
    import random

    from oracle import ep_placement as P
    rng = random.Random(0)
    E, G = 6, 3
    inst_rank = [0, 0, 0, 1, 1, 2, 2, 2]
    inst_first = [0, 3, 5, 8]
    inst_expert = [0, 1, 2, 3, 4, 5, 0, 1]
    for policy in (P.POLICY_ROTATE, P.POLICY_SPLIT):
        for epoch in (1, 2, 7):
            counts = [[rng.randrange(0, 50) for _ in range(E)] for _ in range(G)]
            alive = [[[i for i, e2 in enumerate(inst_expert) if e2 == e] for e in range(E)] for _ in range(G)]
            alive[1][0] = alive[1][0][:1]  # rank 1 sees one of expert 0's replicas as dead
            res = P.placement(counts, alive, inst_rank, inst_first, policy, epoch, cap=10**6)
            for g in range(G):
                used = set()
                for r in range(G):
                    for i in range(inst_first[g], inst_first[g + 1]):
                        rows = range(res["dest_off"][r][i], res["dest_off"][r][i] + res["M"][r][i])
                        assert not used & set(rows)
                        used |= set(rows)
                assert used == set(range(sum(res["tot"][inst_first[g]:inst_first[g + 1]])))
                assert res["seg_end"][g][-1] == len(used)
            for r in range(G):
                for e in range(E):
                    assert sum(hi - lo for _i, lo, hi in res["parts"][r][e]) == counts[r][e]
                dest = P.destinations(counts[r], res["parts"][r], inst_rank, res["dest_off"][r], 10**6)
                assert len(dest) == sum(counts[r]) and all(g >= 0 for g, _ in dest)


def _window_worker(rank, world, port, results):
    from datetime import timedelta

    import torch.distributed as dist

    from distributedmoe_b200.MoE.instances import InstanceTable
    from distributedmoe_b200.MoE.sharded_cluster import gather_window_descriptors
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        descs = gather_window_descriptors(struct.pack("!Q", 1000 + rank) + bytes([rank]) * 5)
        t = InstanceTable.from_blocks([[0, 1], [1, 2], [2, 0]][:world], list(range(world)), world, 3)
        results.put((rank, descs, t.inst_rank, t.inst_slot, t.inst_first))
    finally:
        dist.destroy_process_group()


def test_window_descriptors_and_instance_tables_agree_over_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_window_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, *rest = results.get(timeout=120)
            out[rank] = rest
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert out[0] == out[1]
    descs = out[0][0]
    assert [struct.unpack("!Q", d[:8])[0] for d in descs] == [1000, 1001]


def test_free_ports_are_distinct_bindable_and_outside_the_ephemeral_range():
    """Listener ports are picked below the kernel's ephemeral range (where outgoing
    connections take their source ports), distinct, and free to bind."""
    import socket
    from distributedmoe_b200.MoE.local_cluster import _ephemeral_range, free_ports

    ports = free_ports(41)
    assert len(set(ports)) == 41
    lo, _ = _ephemeral_range()
    if min(lo, 32000) - 20000 >= 8 * 41:
        assert all(20000 <= p < min(lo, 32000) for p in ports)
    for p in ports[:5]:
        s = socket.socket()
        s.bind(("127.0.0.1", p))
        s.close()


def test_blocking_metadata_exchange_gives_up_after_its_deadline():
    """The set-up hand-shake's blocking receive and send retry on socket timeouts, but for at
    most deadline_s seconds: a peer that never answers ends in TimeoutError, not a hang."""
    import asyncio
    import logging
    import time

    eng = _bare_engine()
    eng.logger = logging.getLogger("test.deadline")

    def never(_coro_fn):
        raise asyncio.TimeoutError

    eng._run_blocking = never
    t0 = time.monotonic()
    with pytest.raises(TimeoutError, match="no metadata from peer"):
        eng.get_metadata_from("peer", deadline_s=0.05)
    with pytest.raises(TimeoutError, match="could be sent to peer"):
        eng.send_metadata_to("peer", 0, (0, b""), deadline_s=0.05)
    assert time.monotonic() - t0 < 10
