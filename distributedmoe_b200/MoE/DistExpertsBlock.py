"""Expert side of the distributed MoE layer (reference ``MoE/DistExpertsBlock.py``).

Same API and main loop: ``DistExpertsBlock(experts_block_index, config, expert_layers,
tte_config, metrics_collector=None)``, ``main_loop()``, ``close()``; it parses the host's
buffer descriptors, answers health pings, and runs one ``ExpertsBlockPipelineTask`` per
``DispatchSubmit``.  The expert weights are stacked once, contiguous, in ``nn.Linear``
layout (gate/up ``[E_b, I, d]``, down ``[E_b, d, I]``), which is the K-major operand
layout the tcgen05 grouped GEMM reads through TMA.
"""

from __future__ import annotations

import asyncio
import struct
import threading
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import zmq
import zmq.asyncio

from distributedmoe_b200.MoE.DistMoE import P2PHeaders
from distributedmoe_b200.MoE.DistMoEBlock import ACTIVATIONS, DistMoEBlockConfig
from distributedmoe_b200.MoE.PipelineTask import ExpertsBlockPipelineTask
from distributedmoe_b200.MoE.pools.BuffersPool import BuffersPool
from distributedmoe_b200.TensorTransferEngine import create_transfer_engine
from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import TensorTransferEngineConfig
from distributedmoe_b200.TensorTransferEngine.utils import P2PPair, join_host_port
from distributedmoe_b200.utils.logging_config import get_logger


def stack_expert_weights(expert_layers: List[Any], device: torch.device, dtype: torch.dtype):
    """Stack gate/up/down weights of the block's experts (``DistExpertsBlock.py:163-177``)."""
    with torch.no_grad():
        gate = torch.stack([m.gate_proj.weight.detach().to(device=device, dtype=dtype) for m in expert_layers]).contiguous()
        up = torch.stack([m.up_proj.weight.detach().to(device=device, dtype=dtype) for m in expert_layers]).contiguous()
        down = torch.stack([m.down_proj.weight.detach().to(device=device, dtype=dtype) for m in expert_layers]).contiguous()
    return gate, up, down


class DistExpertsBlock(nn.Module):
    def __init__(self, experts_block_index: int, config: DistMoEBlockConfig, expert_layers: List,
                 tte_config: TensorTransferEngineConfig, metrics_collector=None, stacked_weights=None):
        super().__init__()
        self.experts_block_index = experts_block_index
        self.logger = get_logger("dist_moe.moe.expert_block", {"block_index": str(experts_block_index)})
        self._is_closed = False
        self.device = torch.device(config.eb_devices[experts_block_index])
        self.metrics_collector = metrics_collector
        self.event_loop = asyncio.new_event_loop()
        asyncio.set_event_loop(self.event_loop)
        self._loop_stopped = threading.Event()
        self.hidden_features = config.hidden_features
        self.dtype = config.dtype
        if self.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise NotImplementedError("the tcgen05 grouped expert MLP computes in bf16, fp16 or fp32 (tf32 MMAs)")
        self.activation = ACTIVATIONS[config.activation]

        block_experts = config.expert_blocks[experts_block_index]
        self.expert_layers: Dict[int, Any] = {}
        self.expert_streams: Dict[int, torch.cuda.Stream] = {}
        self.initialize_expert_layers(config.expert_blocks, expert_layers, stacked_weights)

        with torch.cuda.device(self.device):
            self.tensor_transfer_engine = create_transfer_engine(config.backend, tte_config)
        self.host_address = self.tensor_transfer_engine.remote_names[0]
        self.health_check_context = zmq.asyncio.Context()
        self.health_check_p2p_pair: Optional[P2PPair] = None
        self.setup_health_check(config, tte_config)
        self.EOR = False
        self.async_lock = asyncio.Lock()
        self.io_buffer_size = config.io_buffer_size
        self.number_of_io_buffers = config.number_of_io_buffers
        self.host_input_buffers_transfer_descs: Dict[bytes, Any] = {}
        self.host_output_buffers_transfer_descs: Dict[bytes, Any] = {}
        self.initialize_io_buffers()
        self.logger.info(f"DistExpertsBlock initialized - Device: {self.device}, Experts: {block_experts}")

    def initialize_expert_layers(self, expert_blocks: List[List[int]], expert_layers: List, stacked_weights=None) -> None:
        experts = expert_blocks[self.experts_block_index]
        if stacked_weights is None:
            assert len(experts) == len(expert_layers)
            for e, layer in zip(experts, expert_layers):
                self.expert_layers[e] = layer
            gate, up, down = stack_expert_weights(expert_layers, self.device, self.dtype)
        else:
            # Weights already stacked on the device ([E_b, I, d], [E_b, I, d], [E_b, d, I]).
            gate, up, down = stacked_weights
        position = {e: i for i, e in enumerate(experts)}
        self.experts_combine_layer = (position, gate, up, down)

    def setup_health_check(self, config: DistMoEBlockConfig, tte_config: TensorTransferEngineConfig) -> None:
        if self.experts_block_index >= len(config.remote_health_check_ports):
            return
        pair = P2PPair(self.health_check_context.socket(zmq.PUSH), self.health_check_context.socket(zmq.PULL))
        pair.puller.connect(join_host_port(tte_config.remote_addresses[0],
                                           config.host_health_check_ports[self.experts_block_index], "tcp"))
        pair.pusher.bind(join_host_port(tte_config.host_address,
                                        config.remote_health_check_ports[self.experts_block_index], "tcp"))
        self.health_check_p2p_pair = pair

    async def _health_check_handler(self) -> None:
        tte = self.tensor_transfer_engine
        while not self.EOR:
            try:
                packet = await asyncio.wait_for(self.health_check_p2p_pair.puller.recv(), timeout=2.0)
                header, _ = tte.deserialize_p2p_packet(packet)
                if header == P2PHeaders.Ping.value:
                    await self.health_check_p2p_pair.pusher.send(tte.serialize_p2p_packet(P2PHeaders.Pong.value, []))
            except asyncio.TimeoutError:
                continue
            except asyncio.CancelledError:
                break
            except Exception as e:
                if not self.EOR:
                    self.logger.warning(f"health check handler error: {e}")
                break

    def initialize_io_buffers(self) -> None:
        args = (self.tensor_transfer_engine, self.io_buffer_size, self.hidden_features, self.dtype, self.device)
        self.input_buffers_pool = BuffersPool(self.number_of_io_buffers, *args)
        self.output_buffers_pool = BuffersPool(self.number_of_io_buffers, *args)
        if not self.tensor_transfer_engine.handshake():
            raise RuntimeError(f"expert block {self.experts_block_index}: hand-shake with its host failed (see the log)")

    def parse_host_io_buffer_descriptors(self, metadata: List[Tuple[int, bytes]]) -> None:
        n = struct.unpack("!H", metadata[0][1])[0]
        assert len(metadata) == 1 + 2 * 2 * n
        off = 1
        for i in range(2 * n):
            bid: bytes = metadata[off][1]
            descs = self.tensor_transfer_engine.deserialize_descs(metadata[off + 1])
            (self.host_input_buffers_transfer_descs if i < n else self.host_output_buffers_transfer_descs)[bid] = descs
            off += 2

    async def async_main_loop(self) -> None:
        tte = self.tensor_transfer_engine
        tasks: List[asyncio.Task] = []
        if self.health_check_p2p_pair is not None:
            tasks.append(asyncio.create_task(self._health_check_handler()))
        torch.cuda.set_device(self.device)
        while not self.EOR:
            try:
                header, metadata = await tte.async_get_metadata_from(self.host_address)
            except asyncio.TimeoutError:
                continue
            except Exception as e:
                if self.EOR:
                    break
                self.logger.error(f"main loop receive error: {e}")
                continue
            if header == P2PHeaders.ExpertsBlockStop.value:
                self.EOR = True
                break
            if header == P2PHeaders.IOTransferDescriptorsSubmit.value:
                self.parse_host_io_buffer_descriptors(metadata)
            elif header == P2PHeaders.DispatchSubmit.value:
                task = ExpertsBlockPipelineTask(tte, self.input_buffers_pool, self.output_buffers_pool, self.expert_layers,
                                                self.experts_combine_layer, self.expert_streams, self.host_address,
                                                metadata, self.async_lock, self.metrics_collector, self.activation)
                # Run the task here rather than as a new asyncio task (the reference's
                # MoE/DistExpertsBlock.py:271-276): with stream-ordered transfers it only
                # enqueues GPU work and never waits for it, so it ends quickly, and the
                # extra event-loop turn would delay the expert MLP's launch.
                await task.run(self.experts_block_index, self.host_input_buffers_transfer_descs,
                               self.host_output_buffers_transfer_descs)
            else:
                self.logger.warning(f"Unknown header received: {header}")
        pending = [t for t in tasks if not t.done()]
        if pending:
            for t in pending:
                t.cancel()
            await asyncio.gather(*pending, return_exceptions=True)

    def main_loop(self) -> None:
        try:
            self.event_loop.run_until_complete(self.async_main_loop())
        except asyncio.CancelledError:
            pass
        finally:
            self.close()

    def forward(self, input_batch: torch.Tensor) -> torch.Tensor:  # the reference leaves this unimplemented too
        raise NotImplementedError

    def close(self) -> None:
        if self._is_closed:
            return
        self.EOR = True
        if not self.event_loop.is_closed() and not self.event_loop.is_running():
            self.event_loop.close()
        self._loop_stopped.set()
        try:
            self.input_buffers_pool.close()
            self.output_buffers_pool.close()
        except Exception as e:
            self.logger.warning(f"Error closing buffer pools: {e}")
        if self.health_check_p2p_pair is not None:
            try:
                self.health_check_p2p_pair.pusher.close(linger=0)
                self.health_check_p2p_pair.puller.close(linger=0)
            except Exception:
                pass
        try:
            self.health_check_context.term()
        except Exception:
            pass
        try:
            self.tensor_transfer_engine.close()
        except Exception as e:
            self.logger.warning(f"Error closing tensor transfer engine: {e}")
        self._is_closed = True
