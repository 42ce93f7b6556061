"""Host side of the distributed MoE layer (reference ``MoE/DistMoEBlock.py``).

Public API as in the reference: ``DistMoEBlockConfig``, ``DistMoEBlock(config, tte_config,
metrics_collector=None)``, ``forward(x, using_grouped_gemm=True, using_alignment=False)``,
``disable_experts_block``, ``enable_experts_block``, ``close``; the same control flow for
dispatch waves, the ``forward_timeout`` SLA (partial result on expiry), the ZeroMQ health
checker, the P2P handler, and abort + re-dispatch of a dead block's tasks.

Routing differs in where it runs: one router kernel (fp32 logits, softmax or the
sigmoid/group-limited router, top-k, optional renormalisation) and the routing-plan
kernels replace the gate GEMM, softmax, top-k, one-hot mask and the per-expert
``torch.where`` loop with its per-expert host synchronisations (``:553-605``).  The host
reads back only the E per-expert counts, once per forward.  The output is the gather-form
weighted combine of the permuted expert outputs, issued on the caller's stream.

With the ``NVLinkDirect`` backend and :meth:`setup_direct_plane`, a forward is device-driven
instead: router -> routing plan -> count exchange -> gather into the receivers' buffers over
NVLink -> one grouped MLP per GPU over every host's rows -> epoch flags -> combine by peer
loads, all on the caller's stream with no host synchronisation.  Every rank of the group
runs one forward per step.  Block choice (alive blocks only, FIFO rotation or an even split
over replicas) and dead-block exclusion keep the pool's semantics; rows of an expert with no
alive block are left out of the sum, as the reference's partial result leaves out the
tasks that never came back (``:716-718``).
"""

from __future__ import annotations

import asyncio
import math
import os
import struct
import threading
import timeit
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import zmq
import zmq.asyncio

from distributedmoe_b200 import _native as N
from distributedmoe_b200.MoE.DistMoE import ExpertMetaData, P2PHeaders, SegmentQueue
from distributedmoe_b200.MoE.instances import InstanceTable
from distributedmoe_b200.MoE.PipelineTask import ForwardState, HostPipelineTask
from distributedmoe_b200.MoE.pools.BuffersPool import BuffersPool
from distributedmoe_b200.MoE.pools.ExpertBlocksPool import ExpertBlocksPool
from distributedmoe_b200.TensorTransferEngine import create_transfer_engine
from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import (
    TensorTransferEngine,
    TensorTransferEngineBackend,
    TensorTransferEngineConfig,
)
from distributedmoe_b200.TensorTransferEngine.utils import P2PPair, join_host_port
from distributedmoe_b200.utils.logging_config import get_logger

ACTIVATIONS = {"relu": N.ACT_RELU, "silu": N.ACT_SILU}


@dataclass
class DistMoEBlockConfig:
    backend: TensorTransferEngineBackend
    number_of_experts: int
    expert_blocks: List[List[int]]
    number_of_io_buffers: int
    io_buffer_size: int
    top_k: int
    hidden_features: int
    dtype: torch.dtype
    moe_device: torch.device
    eb_devices: List[torch.device]
    forward_timeout: int
    host_health_check_ports: List[int]
    remote_health_check_ports: List[int]
    # ---- options this build adds; each default reproduces the reference except
    # router_fp32_logits, which defaults to fp32 logits (the reference's gate computes them in
    # the model dtype, and that rounding can change the top-k picks of near-ties) ----
    # expert activation: "relu" (reference, MoE/MoE.py:25) or "silu" (SwiGLU)
    activation: str = "relu"
    # divide the top-k routing weights by their sum (the reference does not)
    renormalize: bool = False
    # router logits in fp32 (False: in the model dtype, as the reference's gate computes them;
    # True is the one default that differs from the reference)
    router_fp32_logits: bool = True
    # "softmax" (reference) or "sigmoid_group" (DeepSeek-V3 style)
    router_mode: str = "softmax"
    routed_scaling_factor: float = 1.0
    n_group: int = 1
    topk_group: int = 1
    # expert block choice: "fifo" (reference round robin) or "least_loaded"
    expert_block_policy: str = "fifo"
    # every dispatch wave sends at least one task to each alive block that holds pending
    # activations (False: ceil(remaining / io_buffer_size) tasks per wave, as the reference,
    # which sends the blocks' work one wave after another when it fits one buffer)
    dispatch_all_blocks: bool = False


class DistMoEBlock(nn.Module):
    def __init__(self, config: DistMoEBlockConfig, tte_config: TensorTransferEngineConfig, metrics_collector=None):
        super().__init__()
        self.logger = get_logger("dist_moe.moe.block")
        self._is_closed = False
        self.metrics_collector = metrics_collector
        self.config = config
        self.device: torch.device = torch.device(config.moe_device)
        self.number_of_expert_blocks = len(config.expert_blocks)
        self.number_of_experts = config.number_of_experts
        self.top_k = config.top_k
        self.experts_hit: List[int] = []
        self.hidden_features = config.hidden_features
        self.dtype = config.dtype
        self.forward_timeout = config.forward_timeout
        self.host_health_check_ports = config.host_health_check_ports
        self.remote_health_check_ports = config.remote_health_check_ports
        self.health_check_timeout = tte_config.p2p_timeout_duration
        if config.activation not in ACTIVATIONS:
            raise ValueError(f"unknown activation {config.activation!r}")
        if config.router_mode not in ("softmax", "sigmoid_group"):
            raise ValueError(f"unknown router mode {config.router_mode!r}")

        self.event_loop = asyncio.new_event_loop()
        asyncio.set_event_loop(self.event_loop)
        self._loop_stopped = threading.Event()

        with torch.cuda.device(self.device):
            self.tensor_transfer_engine: TensorTransferEngine = create_transfer_engine(config.backend, tte_config)

        self.health_check_context = zmq.asyncio.Context()
        self.health_check_p2p_pairs: Dict[str, P2PPair] = {}
        self.setup_health_check(tte_config)

        # Router (replaceable like the reference's, :133-134); score_bias feeds the
        # selection of the sigmoid router only.
        self.gate: nn.Module = nn.Linear(self.hidden_features, self.number_of_experts, bias=False, dtype=self.dtype,
                                         device=self.device)
        self.score_bias: Optional[torch.Tensor] = None
        self.output_batch: torch.Tensor = torch.zeros(1, dtype=self.dtype, device=self.device)
        # Optional always-on shared expert (DeepSeek-V3 extension; the reference has none),
        # computed on this GPU beside the routed experts and added with weight 1.
        self.shared_expert: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None
        self._shared_stream: Optional[torch.cuda.Stream] = None

        self.expert_blocks: List[List[int]] = config.expert_blocks
        self.expert_blocks_pool = ExpertBlocksPool(self.expert_blocks, policy=config.expert_block_policy)
        self.initialize_metadata()

        self.number_of_io_buffers = config.number_of_io_buffers
        self.io_buffer_size = config.io_buffer_size
        if not (1 <= self.io_buffer_size <= 65535):
            raise ValueError("io_buffer_size must fit the 16-bit packet fields (1..65535)")
        self.activations_batch_size_candidates: List[int] = []
        self.initialize_io_buffers()

        self.async_lock = asyncio.Lock()
        self.combining = asyncio.Event()
        self.pipeline_tasks: Dict[bytes, HostPipelineTask] = {}
        self.dispatch_tasks: Dict[bytes, asyncio.Task] = {}
        self.combine_tasks: Dict[bytes, asyncio.Task] = {}
        self.expert_block_tasks: Dict[int, List[bytes]] = {}
        self.active_pipeline_tasks: List[int] = [0]
        self.transferred_activations: List[int] = [0]
        self.total_activations = 0
        self.forward_state: Optional[ForwardState] = None
        self._counts_host = torch.empty(self.number_of_experts, dtype=torch.int32, pin_memory=True)

        self.monitoring_flag = True
        self.monitoring_tasks: List[asyncio.Task] = []
        self.disabled_expert_blocks: set = set()
        self._ep: Optional[dict] = None  # device-driven data plane (setup_direct_plane)
        self.setup_monitoring()
        self.logger.info(f"DistMoEBlock initialized - Experts: {self.number_of_experts}, "
                         f"Blocks: {self.number_of_expert_blocks}, Device: {self.device}")

    # ------------------------------------------------------------------ setup
    def disable_experts_block(self, experts_block_index: int) -> None:
        self.disabled_expert_blocks.add(experts_block_index)
        self.expert_blocks_pool.mark_dead(experts_block_index)

    def enable_experts_block(self, experts_block_index: int) -> None:
        self.disabled_expert_blocks.discard(experts_block_index)
        self.expert_blocks_pool.mark_alive(experts_block_index)

    def setup_health_check(self, tte_config: TensorTransferEngineConfig) -> None:
        assert len(self.host_health_check_ports) == len(tte_config.remote_addresses)
        assert len(self.remote_health_check_ports) == len(tte_config.remote_addresses)
        for i in range(len(tte_config.remote_addresses)):
            remote_name = join_host_port(tte_config.remote_addresses[i], tte_config.remote_ports[i])
            pair = P2PPair(self.health_check_context.socket(zmq.PUSH), self.health_check_context.socket(zmq.PULL))
            pair.pusher.bind(join_host_port(tte_config.host_address, self.host_health_check_ports[i], "tcp"))
            pair.pusher.setsockopt(zmq.RCVTIMEO, self.health_check_timeout)
            pair.puller.connect(join_host_port(tte_config.remote_addresses[i], self.remote_health_check_ports[i], "tcp"))
            pair.puller.setsockopt(zmq.RCVTIMEO, self.health_check_timeout)
            self.health_check_p2p_pairs[remote_name] = pair

    def initialize_io_buffers(self) -> None:
        args = (self.tensor_transfer_engine, self.io_buffer_size, self.hidden_features, self.dtype, self.device)
        self.input_buffers_pool = BuffersPool(self.number_of_io_buffers, *args)
        self.output_buffers_pool = BuffersPool(self.number_of_io_buffers, *args)
        self.tensor_transfer_engine.handshake()  # synchronisation point, as in the reference (:246-247)
        packet = self._build_io_descriptors_packet()

        async def send_io_descriptors():
            for remote_name in self.tensor_transfer_engine.remote_names:
                await self.tensor_transfer_engine.async_send_metadata_to(
                    remote_name, P2PHeaders.IOTransferDescriptorsSubmit.value, packet)

        self.event_loop.run_until_complete(send_io_descriptors())
        step = max(self.io_buffer_size // 1024, 1)
        self.activations_batch_size_candidates = list(range(step, self.io_buffer_size, step)) + [self.io_buffer_size]

    def _build_io_descriptors_packet(self) -> List[Tuple[int, bytes]]:
        """``!H n`` then (2-byte id, serialized descriptors) per input then output buffer (``:269-289``)."""
        packet: List[Tuple[int, bytes]] = [(2, struct.pack("!H", self.number_of_io_buffers))]
        for i, b in enumerate(self.input_buffers_pool.buffers):
            b.id = i.to_bytes(length=2, byteorder="big")
            packet += [(2, b.id), b.serialized_transfer_descs]
        for i, b in enumerate(self.output_buffers_pool.buffers):
            b.id = (self.number_of_io_buffers + i).to_bytes(length=2, byteorder="big")
            packet += [(2, b.id), b.serialized_transfer_descs]
        return packet

    def initialize_metadata(self) -> None:
        self.experts_metadata: Dict[int, ExpertMetaData] = {}
        for e in range(self.number_of_experts):
            self.experts_metadata[e] = ExpertMetaData([], 0, None, None, 0, SegmentQueue())
        for b in range(self.number_of_expert_blocks):
            for e in self.expert_blocks[b]:
                self.experts_metadata[e].block_indexes.append(b)
                self.experts_metadata[e].expert_shared_rate += 1

    # ------------------------------------------------------------------ fault tolerance
    async def _abort_all_dispatched_to(self, experts_block_index: int) -> None:
        async with self.async_lock:
            names = self.expert_block_tasks.get(experts_block_index, [])
            self.expert_block_tasks[experts_block_index] = []
            for name in names:
                task = self.pipeline_tasks.get(name)
                if task is not None:
                    task.abort()
                    if task.dispatch_done:
                        self.transferred_activations[0] -= task.used_activations
                        if not task.combine_done:
                            self.active_pipeline_tasks[0] -= 1
                for tasks in (self.dispatch_tasks, self.combine_tasks):
                    t = tasks.pop(name, None)
                    if t is not None:
                        t.cancel()
                self.pipeline_tasks.pop(name, None)
            if names:
                self.combining.set()

    async def _expert_block_health_checker(self, experts_block_index: int, remote_name: str) -> None:
        try:
            while self.monitoring_flag:
                try:
                    await asyncio.sleep(0.02)
                    if experts_block_index in self.disabled_expert_blocks:
                        continue
                    pair = self.health_check_p2p_pairs.get(remote_name)
                    if not pair:
                        continue
                    try:
                        await pair.pusher.send(self.tensor_transfer_engine.serialize_p2p_packet(P2PHeaders.Ping.value, []))
                    except Exception as e:
                        self.logger.error(f"health check: ping to EB #{experts_block_index} failed: {e}")
                        continue
                    try:
                        # A pong may take as long as the configured P2P timeout (the sockets'
                        # RCVTIMEO), as in the reference: a block busy in a long GPU call is late,
                        # not dead.
                        packet = await asyncio.wait_for(pair.puller.recv(),
                                                        timeout=max(1.0, self.health_check_timeout / 1000.0))
                        header, _ = self.tensor_transfer_engine.deserialize_p2p_packet(packet)
                        if header != P2PHeaders.Pong.value:
                            raise RuntimeError(f"unexpected health check header {header}")
                        md = self.expert_blocks_pool.expert_blocks_metadata[experts_block_index]
                        if experts_block_index not in self.disabled_expert_blocks and not md.is_alive:
                            self.expert_blocks_pool.mark_alive(experts_block_index)
                    except Exception:
                        if self.expert_blocks_pool.expert_blocks_metadata[experts_block_index].is_alive:
                            self.expert_blocks_pool.mark_dead(experts_block_index)
                            self.logger.warning(f"EB #{experts_block_index} marked as dead (no pong)")
                            await self._abort_all_dispatched_to(experts_block_index)
                    if self.active_pipeline_tasks[0] == 0:
                        self.combining.set()
                except asyncio.CancelledError:
                    break
                except Exception as e:
                    self.expert_blocks_pool.mark_dead(experts_block_index)
                    await self._abort_all_dispatched_to(experts_block_index)
                    self.logger.error(f"health check failure for block {experts_block_index}: {e}")
        except asyncio.CancelledError:
            pass

    async def _expert_block_p2p_handler(self, experts_block_index: int, remote_name: str) -> None:
        try:
            while self.monitoring_flag:
                try:
                    header, metadata = await self.tensor_transfer_engine.async_get_metadata_from(remote_name)
                except asyncio.CancelledError:
                    break
                except Exception:
                    continue
                md = self.expert_blocks_pool.expert_blocks_metadata[experts_block_index]
                if experts_block_index not in self.disabled_expert_blocks and not md.is_alive:
                    self.expert_blocks_pool.mark_alive(experts_block_index)
                if header == P2PHeaders.HostOutputBufferUnlocked.value:
                    name: bytes = metadata[-1][1]
                    task = self.pipeline_tasks.get(name)
                    if task is not None:
                        # Combined in this handler (the reference starts a task per ack,
                        # MoE/DistMoEBlock.py:462): the
                        # combine only enqueues a gather and updates counters.
                        try:
                            await task.combine(self.active_pipeline_tasks, self.output_batch, self.combining)
                        finally:
                            self.dispatch_tasks.pop(name, None)
                            self.pipeline_tasks.pop(name, None)
                    else:
                        self.logger.debug(f"stale combine ack for task {name.hex()[:8]}")
                elif header == P2PHeaders.HostInputBufferUnlocked.value:
                    task = self.pipeline_tasks.get(metadata[-1][1])
                    if task is not None:
                        task.release_input_buffer()
                elif header == P2PHeaders.IOTransferDescriptorsRequest.value:
                    await self.tensor_transfer_engine.async_send_metadata_to(
                        remote_name, P2PHeaders.IOTransferDescriptorsSubmit.value, self._build_io_descriptors_packet())
                elif header == P2PHeaders.Pong.value:
                    self.expert_blocks_pool.mark_alive(experts_block_index)
                else:
                    self.logger.warning(f"P2P handler: unknown header {header}")
        except asyncio.CancelledError:
            pass

    def setup_monitoring(self) -> None:
        for b, remote_name in enumerate(self.tensor_transfer_engine.remote_names):
            self.monitoring_tasks.append(self.event_loop.create_task(self._expert_block_health_checker(b, remote_name)))
            self.monitoring_tasks.append(self.event_loop.create_task(self._expert_block_p2p_handler(b, remote_name)))

    # ------------------------------------------------------------------ forward
    def _route(self, x: torch.Tensor, w_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        cfg = self.config
        mode = N.ROUTER_SOFTMAX if cfg.router_mode == "softmax" else N.ROUTER_SIGMOID_GROUP
        kw = dict(mode=mode, renormalize=cfg.renormalize, scale=cfg.routed_scaling_factor, n_group=cfg.n_group,
                  topk_group=cfg.topk_group, w_dtype=w_dtype or self.dtype,
                  score_bias=None if self.score_bias is None else self.score_bias.float().contiguous())
        g = self.gate
        plain_linear = isinstance(g, nn.Linear) and g.weight.dtype == x.dtype and g.weight.is_contiguous()
        if plain_linear and cfg.router_fp32_logits:
            bias = None if g.bias is None else g.bias.detach().float().contiguous()
            idx, w, _ = N.router(x, g.weight.detach(), self.top_k, logit_bias=bias, **kw)
        else:
            # A replaced gate module, or logits in the model dtype as the reference computes them.
            with torch.no_grad():
                logits = g(x).float().contiguous()
            idx, w, _ = N.router(None, None, self.top_k, logits_in=logits, **kw)
        return idx, w

    def _setup_forward_pass(self, input_batch: torch.Tensor) -> Tuple[List[int], torch.Tensor]:
        assert input_batch.dtype == self.dtype
        assert input_batch.device == self.device
        if input_batch.dim() == 3:
            assert input_batch.shape[2] == self.hidden_features
            input_batch = input_batch.reshape(-1, self.hidden_features)
        elif input_batch.dim() == 2:
            assert input_batch.shape[1] == self.hidden_features
        else:
            raise RuntimeError(f"Wrong input batch shape: {input_batch.shape} with hidden size: {self.hidden_features}")
        x = input_batch.contiguous()
        T, E, k = x.shape[0], self.number_of_experts, self.top_k
        stream = torch.cuda.current_stream(self.device)
        self.output_batch = torch.empty(x.shape, dtype=self.dtype, device=self.device)
        if T == 0:
            self.forward_state = None
            return [], x
        idx, w = self._route(x)
        plan = N.route_plan(idx, w, E)
        self._counts_host.copy_(plan["counts"], non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(stream)
        # The shared expert (if any) goes to the GPU before the host waits for the counts.
        shared_done = self._launch_shared_expert(x) if self.shared_expert is not None else None
        ready.synchronize()  # the only host synchronisation of the forward: E counts
        counts = self._counts_host.tolist()
        experts_hit, offsets, base = [], [0] * (E + 1), 0
        for e in range(E):
            offsets[e] = base
            n = counts[e]
            if n:
                experts_hit.append(e)
                self.experts_metadata[e].bind(plan, base, n)
            base += n
        offsets[E] = base
        arena = torch.empty(T * k, self.hidden_features, dtype=self.dtype, device=self.device)
        self.forward_state = ForwardState(x, plan, offsets, w, ready, arena)
        if shared_done is not None:
            self.forward_state.events.append(shared_done)
        return experts_hit, x

    def _finalize(self) -> None:
        """Weighted combine of the permuted rows on the caller's stream.  After a timeout,
        rows that never came back are zeroed first, so their tokens get a partial sum, as
        the reference's partial output does (``:716-718``)."""
        fs = self.forward_state
        stream = torch.cuda.current_stream(self.device)
        for ev in fs.events:
            stream.wait_event(ev)
        T = fs.x.shape[0]
        if sum(n for _e, _l, n in fs.covered) < T * self.top_k:
            import numpy as np

            covered = np.zeros(T * self.top_k, dtype=bool)
            for e, l, n in fs.covered:
                covered[fs.offsets[e] + l: fs.offsets[e] + l + n] = True
            missing = np.flatnonzero(~covered)
            if missing.size:
                fs.arena[torch.from_numpy(missing).to(self.device)] = 0
        N.combine(fs.arena, fs.plan["inverse"], fs.routing_weights, self.output_batch,
                  accumulate=self.shared_expert is not None)

    def set_shared_expert(self, gate_proj: torch.Tensor, up_proj: torch.Tensor, down_proj: torch.Tensor) -> None:
        """Add an always-on shared expert: act(x W_g^T) * (x W_u^T) W_d^T with weight 1 for
        every token (W_g, W_u [I_s, d]; W_d [d, I_s]).  It runs on the host's GPU on a side
        stream while the routed tokens are dispatched (the shared expert is replicated on
        every GPU, so it never crosses NVLink)."""
        d = self.hidden_features
        if gate_proj.shape != up_proj.shape or gate_proj.dim() != 2 or gate_proj.shape[1] != d \
                or down_proj.shape != (d, gate_proj.shape[0]):
            raise ValueError("shared expert weights must be gate/up [I_s, d] and down [d, I_s]")
        prep = lambda w: w.detach().to(device=self.device, dtype=self.dtype).contiguous().unsqueeze(0)
        self.shared_expert = (prep(gate_proj), prep(up_proj), prep(down_proj))
        if self._shared_stream is None:
            self._shared_stream = torch.cuda.Stream(device=self.device)

    def _launch_shared_expert(self, x: torch.Tensor) -> torch.cuda.Event:
        """Shared expert over all tokens into output_batch on the side stream; the final
        combine waits for the returned event and accumulates the routed sum on top."""
        g, u, dn = self.shared_expert
        cur = torch.cuda.current_stream(self.device)
        side = self._shared_stream
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            N.grouped_gated_mlp(x, g, u, dn, [0], [x.shape[0]], ACTIVATIONS[self.config.activation], self.output_batch,
                                op_name="shared_expert_mlp")
            done = torch.cuda.Event()
            done.record(side)
        if not torch.cuda.is_current_stream_capturing():  # a captured graph owns its buffers
            x.record_stream(side)
            self.output_batch.record_stream(side)
        return done

    def _blocks_with_pending_work(self) -> int:
        hit = set(self.experts_hit)
        n = 0
        for md in self.expert_blocks_pool.expert_blocks_metadata:
            if md.is_alive and any(e in hit and self.experts_metadata[e].expert_offsets.has_rows()
                                   for e in md.expert_indexes):
                n += 1
        return n

    def dispatch(self, input_batch: torch.Tensor, number_of_dispatches: int, using_grouped_gemm: bool = True,
                 using_alignment: bool = False) -> List[asyncio.Task]:
        """Create up to `number_of_dispatches` host tasks (``MoE/DistMoEBlock.py:638-668``);
        returns their dispatch coroutines' tasks."""
        submits = 0
        wave: List[asyncio.Task] = []
        while self.transferred_activations[0] < self.total_activations and submits < number_of_dispatches:
            task = HostPipelineTask(self.tensor_transfer_engine, self.input_buffers_pool, self.output_buffers_pool,
                                    self.experts_hit, self.expert_blocks_pool, self.experts_metadata, self.async_lock,
                                    self.metrics_collector, forward_state=self.forward_state)
            self.pipeline_tasks[task.name] = task
            self.dispatch_tasks[task.name] = asyncio.create_task(task.dispatch(
                input_batch, self.active_pipeline_tasks, self.transferred_activations, self.expert_block_tasks,
                self.activations_batch_size_candidates if using_alignment else None, using_grouped_gemm))
            wave.append(self.dispatch_tasks[task.name])
            submits += 1
        return wave

    async def async_forward(self, input_batch: torch.Tensor, using_grouped_gemm: bool = True,
                            using_alignment: bool = False) -> torch.Tensor:
        if self.metrics_collector is not None:
            self.metrics_collector.start_forward_pass()
        if self.combine_tasks:
            await asyncio.gather(*list(self.combine_tasks.values()), return_exceptions=True)
        self.dispatch_tasks.clear()
        self.combine_tasks.clear()
        self.pipeline_tasks.clear()
        self.expert_block_tasks.clear()

        shape = input_batch.shape
        self.experts_hit, x = self._setup_forward_pass(input_batch)
        if not self.experts_hit:
            self.output_batch.zero_()
            if self.metrics_collector is not None:
                self.metrics_collector.end_setup_phase()
                self.metrics_collector.end_forward_pass()
            return self.output_batch.reshape(shape)

        self.total_activations = self.top_k * x.shape[0]
        self.active_pipeline_tasks[0] = 0
        self.transferred_activations[0] = 0
        if self.metrics_collector is not None:
            self.metrics_collector.end_setup_phase()

        start = timeit.default_timer()
        stalled_waves = 0
        while self.transferred_activations[0] < self.total_activations:
            self.combining.clear()
            before = self.transferred_activations[0]
            n = max(math.ceil((self.total_activations - before) / self.io_buffer_size), 1)
            if self.config.dispatch_all_blocks:
                n = max(n, self._blocks_with_pending_work())
            wave = self.dispatch(x, n, using_grouped_gemm, using_alignment)
            try:
                if wave:
                    await asyncio.wait(wave, timeout=max(self.forward_timeout / 1000 - (timeit.default_timer() - start), 0))
                if self.active_pipeline_tasks[0] == 0 and self.transferred_activations[0] == before:
                    # Every task of the wave drew a block with nothing left to pack (a FIFO
                    # turn can land on such a block): take the next turn at once instead of
                    # waiting for a combine that will not come.
                    stalled_waves += 1
                    if stalled_waves > len(self.expert_blocks) + 1 or \
                            timeit.default_timer() - start > self.forward_timeout / 1000:
                        self.logger.error("dispatch made no progress; returning a partial result")
                        break
                    continue
                stalled_waves = 0
                elapsed = timeit.default_timer() - start
                await asyncio.wait_for(self.combining.wait(), timeout=(self.forward_timeout / 1000 - elapsed))
            except asyncio.TimeoutError:
                break
        # Every dispatched task has been combined unless the SLA expired.
        if self.active_pipeline_tasks[0] > 0:
            try:
                elapsed = timeit.default_timer() - start
                while self.active_pipeline_tasks[0] > 0:
                    self.combining.clear()
                    await asyncio.wait_for(self.combining.wait(), timeout=max(self.forward_timeout / 1000 - elapsed, 0))
            except asyncio.TimeoutError:
                pass
        for name, t in list(self.dispatch_tasks.items()):
            t.cancel()
            task = self.pipeline_tasks.get(name)
            if task is not None and not task.combine_done:
                task.close()
        for name, t in list(self.combine_tasks.items()):
            t.cancel()
        self._finalize()
        if self.metrics_collector is not None:
            self.metrics_collector.end_forward_pass()
        return self.output_batch.reshape(shape)

    def forward(self, input_batch: torch.Tensor, using_grouped_gemm: bool = True, using_alignment: bool = False) -> torch.Tensor:
        if self._ep is not None:
            return self._direct_forward(input_batch)
        return self.event_loop.run_until_complete(self.async_forward(input_batch, using_grouped_gemm, using_alignment))

    # ------------------------------------------------------------------ device-driven data plane
    def setup_direct_plane(self, world: int, rank: int, block_ranks: List[int], local_stack, capacity: int,
                           exchange: Callable[[bytes], List[bytes]], max_tokens: int,
                           wait_timeout_ms: Optional[int] = None, cuda_graphs: bool = False,
                           expert_precision: str = "model") -> None:
        """Switch forward() to the device-driven exchange (``NVLinkDirect`` backend only).

        world, rank: this host's group (one rank per GPU, every rank calls forward once per
        step); block_ranks[b]: the rank holding expert block b; local_stack: this rank's
        (gate [S, I, d], up [S, I, d], down [S, d, I]) for its blocks in index order (S = its
        expert instances); capacity: receive rows per GPU (at least the rows all hosts can
        send it: world * max_tokens * top_k covers any routing); exchange(mine) returns every
        rank's window descriptor in rank order; max_tokens: tokens per forward of this host.
        cuda_graphs: capture the forward once per token count (after one eager forward of
        that count) and replay it; the input is copied into a static buffer and the result
        copied out, so callers see ordinary tensors.  expert_precision: "model" (the layer's
        dtype) or "fp8": the routed experts' gate/up weights are quantised once to e4m3 with
        one scale per output channel, each token row is quantised to e4m3 with one scale
        before the gather (8-bit records cross NVLink: about half the bytes), the gate/up
        GEMM runs on 8-bit tensor cores and the down projection in bf16 (bf16 layers only;
        the reference's benchmark offers "fp8" as a whole-layer 8-bit cast,
        src/python/MoE/benchmarks/bench.py:184-185)."""
        tte = self.tensor_transfer_engine
        if not getattr(tte, "direct", False):
            raise RuntimeError("the device-driven data plane needs the NVLinkDirect backend")
        E, k, d = self.number_of_experts, self.top_k, self.hidden_features
        inst = InstanceTable.from_blocks(self.expert_blocks, block_ranks, world, E)
        n_local = inst.local_count(rank)
        g, u, dn = local_stack
        if g.dim() != 3 or g.shape[0] != n_local or g.shape[2] != d or u.shape != g.shape \
                or dn.shape != (n_local, d, g.shape[1]):
            raise ValueError(f"rank {rank} holds {n_local} expert instances: its stack must be gate/up "
                             f"[{n_local}, I, {d}] and down [{n_local}, {d}, I]")
        if self.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise NotImplementedError("the device-driven data plane computes in bf16, fp16 or fp32")
        if expert_precision not in ("model", "fp8"):
            raise ValueError(f"expert_precision {expert_precision!r}: 'model' or 'fp8'")
        fp8 = expert_precision == "fp8"
        if fp8 and (self.dtype != torch.bfloat16 or d % 16):
            raise ValueError("8-bit experts need a bf16 layer and hidden % 16 == 0")
        dev = self.device
        with torch.cuda.device(dev):
            tte.open_window(capacity, max(max_tokens * k, 1), d, self.dtype, inst.n_inst, dev,
                            record_bytes=N.fp8_record_bytes(d) if fp8 else None)
            descs = exchange(tte.window_descriptor())
            win = tte.attach_windows(descs, rank)
            i32 = dict(dtype=torch.int32, device=dev)
            R = N.EP_MAX_REPLICAS
            policy = N.EP_POLICY_SPLIT if self.config.expert_block_policy == "least_loaded" else N.EP_POLICY_ROTATE
            timeout_ms = wait_timeout_ms if wait_timeout_ms is not None else min(self.forward_timeout, 5000)
            self._ep = {
                "world": world, "rank": rank, "inst": inst, "win": win, "cap": capacity, "policy": policy,
                "n_local": n_local, "stack": (g, u, dn), "max_tokens": max_tokens,
                "fp8": N.Fp8Experts(g, u, dn) if fp8 and n_local > 0 else None, "is_fp8": fp8,
                "records": torch.empty(max(max_tokens, 1), N.fp8_record_bytes(d), dtype=torch.uint8, device=dev)
                if fp8 else None,
                "timeout_ns": int(timeout_ms) * 1_000_000,
                "inst_rank": torch.tensor(inst.inst_rank, **i32),
                "inst_slot": torch.tensor(inst.inst_slot, **i32),
                "inst_first": torch.tensor(inst.inst_first, **i32),
                "alive": torch.zeros(E + E * R, **i32), "alive_key": None,
                "part_n": torch.zeros(E, **i32), "part_inst": torch.zeros(E * R, **i32),
                "part_start": torch.zeros(E * (R + 1), **i32), "dest_off": torch.zeros(inst.n_inst, **i32),
                "seg_expert": torch.zeros(max(n_local, 1), **i32), "seg_end": torch.zeros(max(n_local, 1), **i32),
                "done": torch.zeros(1, **i32), "ret": torch.empty(max(max_tokens * k, 1), **i32),
                "cuda_graphs": cuda_graphs, "graphs": {},
                "x_static": torch.zeros(max_tokens, d, dtype=self.dtype, device=dev) if cuda_graphs else None,
            }
            torch.cuda.synchronize(dev)

    def _direct_alive(self) -> None:
        """Upload the per-expert alive instances when the pool's alive flags changed."""
        ep = self._ep
        key = tuple(md.is_alive for md in self.expert_blocks_pool.expert_blocks_metadata)
        if key != ep["alive_key"]:
            n, inst = ep["inst"].alive_arrays(key)
            ep["alive"].copy_(torch.tensor(n + inst, dtype=torch.int32).pin_memory(), non_blocking=True)
            ep["alive_key"] = key

    def _direct_forward(self, input_batch: torch.Tensor) -> torch.Tensor:
        ep = self._ep
        assert input_batch.dtype == self.dtype and input_batch.device == self.device
        shape = input_batch.shape
        if input_batch.dim() not in (2, 3) or shape[-1] != self.hidden_features:
            raise RuntimeError(f"Wrong input batch shape: {shape} with hidden size: {self.hidden_features}")
        x = input_batch.reshape(-1, self.hidden_features).contiguous()
        T = x.shape[0]
        if T > ep["max_tokens"]:
            raise ValueError(f"{T} tokens exceed the {ep['max_tokens']} this data plane was sized for")
        if not ep["cuda_graphs"]:
            return self._direct_step(x).reshape(shape)
        self._direct_alive()  # any upload of the alive table happens outside the graph
        g = ep["graphs"].get(T)
        if g is None:
            out = self._direct_step(x)  # this step runs eagerly; the capture runs no kernel
            self._direct_capture(T)
            return out.reshape(shape)
        xs, out_static, graph, launches = g
        xs.copy_(x)
        graph.replay()
        N.count_graph_replay(launches)
        return out_static.clone().reshape(shape)

    def _direct_capture(self, T: int) -> None:
        """Capture the forward of T tokens from the static input buffer."""
        ep = self._ep
        xs = ep["x_static"][:T]
        graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(self.device)
        before = N.launch_count()
        with torch.cuda.graph(graph):
            out = self._direct_step(xs)
        ep["graphs"][T] = (xs, out, graph, N.launch_count() - before)

    def _direct_tile_policy(self, T: int) -> int:
        """Tile shape of the grouped MLP from the rows an expert instance can expect (every
        rank sending about T tokens): the segment table is on the device, so the host cannot
        see the actual sizes.  Hundreds of rows per expert or more: 256-row pair tiles; a few
        hundred: pair tiles plus single-SM tiles for remainders of at most 128 rows (a
        segment of 257-384 rows then costs three SM-tiles, not four); fewer: single-SM tiles.
        DMOE_TILE_POLICY (0 auto, 1 pair, 2 single, 3 pair + single remainders) overrides."""
        forced = os.environ.get("DMOE_TILE_POLICY")
        if forced:
            return int(forced)
        ep = self._ep
        expected = ep["world"] * T * self.top_k / max(1, ep["inst"].n_inst)
        if expected >= 768:
            return N.TILES_PAIR
        if expected >= 128:
            return N.TILES_PAIR_SPLIT
        return N.TILES_SINGLE

    def _direct_step(self, x: torch.Tensor) -> torch.Tensor:
        ep = self._ep
        T, E, k = x.shape[0], self.number_of_experts, self.top_k
        capturing = torch.cuda.is_current_stream_capturing()
        if self.metrics_collector is not None and not capturing:
            self.metrics_collector.start_forward_pass()
        dev = self.device
        win, cap, tmo = ep["win"], ep["cap"], ep["timeout_ns"]
        out = torch.empty(x.shape, dtype=self.dtype, device=dev)
        self.output_batch = out
        shared = self.shared_expert is not None and T > 0
        if not capturing:
            self._direct_alive()
        table = (ep["alive"][:E], ep["alive"][E:], ep["inst_rank"], ep["inst_slot"], ep["inst_first"])
        placement = (ep["part_n"], ep["part_inst"], ep["part_start"], ep["dest_off"])
        if T > 0:
            idx, w = self._route(x, w_dtype=torch.float32)
            plan = N.route_plan(idx, None, E, want_slot=True, want_weight=False)
            counts, offsets, perm_token, inverse = plan["counts"], plan["offsets"], plan["perm_token"], plan["inverse"]
            perm_slot = plan["perm_slot"]
        else:
            counts = offsets = perm_token = perm_slot = inverse = w = None
        inst = ep["inst"]
        N.ep_plan(win, counts, E, inst.n_inst, ep["policy"], table, cap, tmo, placement + (ep["seg_expert"], ep["seg_end"]))
        # 8-bit experts: each token row leaves as one record (e4m3 codes + its scale).
        rows_out = N.quantize_records(x, ep["records"][:T]) if ep["is_fp8"] else x
        N.ep_dispatch(win, rows_out, T, k, E, offsets, perm_token, perm_slot, placement, ep["inst_rank"], cap,
                      ep["ret"], ep["done"])
        # The shared expert starts on a side stream once the rows are sent: the routing kernels
        # before it never wait for its SMs, and it overlaps the wait for the other ranks' rows
        # and the routed grouped MLP's last, partly empty wave of tiles.
        shared_done = self._launch_shared_expert(x) if shared else None
        # This GPU's expert instances, once, over every host's rows (the expert blocks' part).
        N.ep_wait(win, N.EP_FLAG_DATA, tmo, dev)
        if ep["n_local"] > 0:
            # The down-projection stores every row straight into its host's return rows.
            g, u, dn = ep["stack"]
            rows = T * k if ep["world"] == 1 else None
            segs = (ep["seg_expert"][:ep["n_local"]], ep["seg_end"][:ep["n_local"]])
            act = ACTIVATIONS[self.config.activation]
            if ep["fp8"] is not None:
                N.ep_expert_mlp_fp8(win, ep["fp8"], *segs, cap, act, self._direct_tile_policy(T), work_rows=rows)
            else:
                N.ep_expert_mlp(win, g, u, dn, *segs, cap, act, self._direct_tile_policy(T), work_rows=rows)
        N.ep_signal(win, N.EP_FLAG_RESULTS, dev)
        N.ep_wait(win, N.EP_FLAG_RESULTS, tmo, dev)
        if T > 0:
            if shared_done is not None:
                torch.cuda.current_stream(dev).wait_event(shared_done)
            N.ep_combine(win, inverse, ep["ret"], w, T, k, out, accumulate=shared)
        if self.metrics_collector is not None and not capturing:
            self.metrics_collector.end_forward_pass()
        return out

    # ------------------------------------------------------------------ shutdown
    def close(self) -> None:
        if self._is_closed:
            return

        async def send_stop_signals():
            for remote_name in self.tensor_transfer_engine.remote_names:
                try:
                    await asyncio.wait_for(self.tensor_transfer_engine.async_send_metadata_to(
                        remote_name, P2PHeaders.ExpertsBlockStop.value, []), timeout=5.0)
                except Exception as e:
                    self.logger.warning(f"stop signal to {remote_name} failed: {e}")

        if not self.event_loop.is_closed():
            try:
                self.event_loop.run_until_complete(send_stop_signals())
            except Exception as e:
                self.logger.error(f"Error sending stop signals: {e}")
            self.monitoring_flag = False
            for t in self.monitoring_tasks:
                if not t.done():
                    t.cancel()
            try:
                self.event_loop.run_until_complete(
                    asyncio.wait_for(asyncio.gather(*self.monitoring_tasks, return_exceptions=True), timeout=2.0))
            except Exception:
                pass
            self.event_loop.close()
        self._loop_stopped.set()
        self.input_buffers_pool.close()
        self.output_buffers_pool.close()
        for pair in self.health_check_p2p_pairs.values():
            try:
                pair.pusher.close(linger=0)
                pair.puller.close(linger=0)
            except Exception:
                pass
        try:
            self.health_check_context.term()
        except Exception:
            pass
        self.tensor_transfer_engine.close()
        self._is_closed = True
