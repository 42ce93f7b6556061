"""Host- and expert-side pipeline tasks (reference ``MoE/PipelineTask.py``).

Control flow, packet format and counters follow the reference: a host task takes an expert
block (round robin over alive blocks), packs that block's pending expert segments into one
input buffer in the block's expert order (optionally padded to an alignment candidate),
and sends ``DispatchSubmit``; the expert block reads the buffer, runs the grouped expert
MLP, writes the host's output buffer and acknowledges with ``HostOutputBufferUnlocked``;
the host then combines.

The data path is different: every GPU step is a library kernel issued on the buffer's
stream and ordered by the transfer engine's region events, so neither side blocks on the
GPU.  The host gather is one segmented-gather launch per task (the reference issues a
gather and one copy per expert and then synchronises the stream, ``:231-252``).  The expert
side runs the tcgen05 grouped MLP directly on the stacked weights (the reference copies the
active experts' weights every run, ``:511-513``).  The host combine moves the task's rows
into the forward's permuted-order arena; the weighted sum over the top-k rows of each token
happens once, after the last task, in ``DistMoEBlock``.
"""

from __future__ import annotations

import asyncio
import bisect
import struct
from typing import Any, Dict, List, Optional, Tuple

import torch

from distributedmoe_b200 import _native as N
from distributedmoe_b200.MoE.DistMoE import ExpertMetaData, P2PHeaders
from distributedmoe_b200.MoE.pools.BuffersPool import Buffer, BuffersPool
from distributedmoe_b200.MoE.pools.ExpertBlocksPool import ExpertBlocksPool
from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import TensorTransferEngine
from distributedmoe_b200.TensorTransferEngine.utils import _next_random_name
from distributedmoe_b200.utils.logging_config import get_logger


class ForwardState:
    """Device-side state of one host forward pass shared by its tasks."""

    def __init__(self, x: torch.Tensor, plan: Dict[str, torch.Tensor], offsets: List[int], routing_weights: torch.Tensor,
                 ready: torch.cuda.Event, arena: torch.Tensor):
        self.x = x
        self.plan = plan
        self.offsets = offsets
        self.routing_weights = routing_weights
        self.ready = ready
        self.arena = arena
        self.events: List[torch.cuda.Event] = []
        self.covered: List[Tuple[int, int, int]] = []  # (expert, l, n) moved into the arena


class PipelineTask:
    def __init__(self, tensor_transfer_engine: TensorTransferEngine, input_buffers_pool: BuffersPool,
                 output_buffers_pool: BuffersPool, async_lock: asyncio.Lock) -> None:
        self.name: bytes = _next_random_name()
        self.logger = get_logger("dist_moe.moe.pipeline", {"task_id": self.name.hex()})
        self.tensor_transfer_engine = tensor_transfer_engine
        self.input_buffers_pool = input_buffers_pool
        self.output_buffers_pool = output_buffers_pool
        self.input_buffer: Optional[Buffer] = None
        self.input_buffer_index: int = -1
        self.output_buffer: Optional[Buffer] = None
        self.output_buffer_index: int = -1
        self.async_lock = async_lock

    def release_input_buffer(self) -> None:
        if self.input_buffer_index != -1:
            self.input_buffers_pool.release(self.input_buffer_index)
            self.input_buffer = None
            self.input_buffer_index = -1

    def release_output_buffer(self) -> None:
        if self.output_buffer_index != -1:
            self.output_buffers_pool.release(self.output_buffer_index)
            self.output_buffer = None
            self.output_buffer_index = -1

    def close(self) -> None:
        self.release_input_buffer()
        self.release_output_buffer()


class HostPipelineTask(PipelineTask):
    def __init__(self, tensor_transfer_engine: TensorTransferEngine, input_buffers_pool: BuffersPool,
                 output_buffers_pool: BuffersPool, experts_hit: List[int], experts_block_pool: ExpertBlocksPool,
                 experts_metadata: Dict[int, ExpertMetaData], async_lock: asyncio.Lock, metrics_collector=None,
                 forward_state: Optional[ForwardState] = None) -> None:
        super().__init__(tensor_transfer_engine, input_buffers_pool, output_buffers_pool, async_lock)
        self.experts_block_pool = experts_block_pool
        self.experts_block_index: int = -1
        self.dispatched_block: int = -1
        self.experts_hit = experts_hit
        self.experts_metadata = experts_metadata
        self.used_activations: int = 0
        # (expert_index, expert_offset, padded_size, actual_size), as in the reference
        self.experts_metadata_snapshot: List[Tuple[int, int, int, int]] = []
        self.dispatch_done = False
        self.combine_done = False
        self.metrics_collector = metrics_collector
        self.forward_state = forward_state

    def _pending_blocks(self) -> List[int]:
        hit = self.experts_hit_set
        out = []
        for md in self.experts_block_pool.expert_blocks_metadata:
            for e in md.expert_indexes:
                if e in hit and self.experts_metadata[e].expert_offsets.has_rows():
                    out.append(md.experts_block_index)
                    break
        return out

    async def dispatch(self, input_batch: torch.Tensor, active_pipeline_tasks: List[int],
                       transferred_activations: List[int], experts_block_tasks: Dict[int, List[bytes]],
                       activations_batch_size_candidates: Optional[List[int]], using_grouped_gemm: bool = True) -> None:
        task_id = self.name.hex()
        if self.metrics_collector is not None:
            self.metrics_collector.start_dispatch(task_id)
        fs = self.forward_state
        try:
            sizeof_ul = 2
            packet: List[Tuple[int, bytes]] = []
            num_experts = 0
            self.experts_hit_set = set(self.experts_hit)
            candidates = self._pending_blocks() if self.experts_block_pool.policy == "least_loaded" else None
            self.experts_block_index, block_md = await self.experts_block_pool.aquire(candidates)
            experts_block_tasks.setdefault(self.experts_block_index, []).append(self.name)
            self.dispatched_block = self.experts_block_index
            self.experts_block_pool.release(self.experts_block_index)
            self.experts_block_index = -1

            packet.append((len(self.name), self.name))
            packet.append((1, struct.pack("!B", int(using_grouped_gemm))))
            packet.append((sizeof_ul, b""))

            seg_src: List[int] = []
            seg_dst: List[int] = []
            seg_len: List[int] = []
            used_padded = 0
            capacity = self.input_buffers_pool.buffer_size
            hit = self.experts_hit_set
            for expert_index in block_md.expert_indexes:
                if expert_index not in hit:
                    continue
                if used_padded >= capacity:
                    break
                md = self.experts_metadata[expert_index]
                if md.expert_offsets.empty():
                    continue
                l, r = md.expert_offsets.get_nowait()
                remaining = capacity - used_padded
                actual = min(r - l, remaining)
                size = actual
                if size <= 0:
                    md.expert_offsets.put_nowait((l, r))
                    continue
                if activations_batch_size_candidates:
                    i = bisect.bisect_left(activations_batch_size_candidates, actual)
                    if i < len(activations_batch_size_candidates):
                        opt = activations_batch_size_candidates[i]
                        if opt > remaining:
                            md.expert_offsets.put_nowait((l, r))
                            continue
                        size = opt
                    else:
                        md.expert_offsets.put_nowait((l, r))
                        continue
                self.experts_metadata_snapshot.append((expert_index, l, size, actual))
                seg_src.append(md.expert_base + l)
                seg_dst.append(used_padded)
                seg_len.append(actual)
                packet.append((sizeof_ul, struct.pack("!H", expert_index)))
                packet.append((sizeof_ul, struct.pack("!H", used_padded)))
                packet.append((sizeof_ul, struct.pack("!H", size)))
                self.used_activations += actual
                used_padded += size
                num_experts += 1
                md.expert_offsets.put_nowait((l + actual, r))

            if num_experts > 0:
                packet[2] = (sizeof_ul, struct.pack("!H", num_experts))
                if self.input_buffer_index == -1:
                    self.input_buffer_index, self.input_buffer = await self.input_buffers_pool.acquire()
                if self.input_buffer is None:
                    raise RuntimeError(f"While dispatching {self.name}, input buffer acquisition error has been occured.")

                # Gather the packed rows into the input buffer on its stream, after the routing
                # plan and after the buffer's previous user; no host synchronisation.
                buf = self.input_buffer
                s = buf.cuda_stream
                s.wait_event(fs.ready)
                buf.begin_use(s)
                N.permute_rows(fs.x, buf.data, seg_src, seg_dst, seg_len, row_map=fs.plan["perm_token"],
                               stream=s.cuda_stream)
                buf.end_use(s)
                ev = torch.cuda.Event()
                ev.record(s)
                fs.events.append(ev)

                if self.output_buffer_index == -1:
                    self.output_buffer_index, self.output_buffer = await self.output_buffers_pool.acquire()
                if self.output_buffer is None:
                    raise RuntimeError(f"While dispatching {self.name}, output buffer acquisition error has been occured.")

                packet.append((len(self.input_buffer.id), self.input_buffer.id))
                packet.append((len(self.output_buffer.id), self.output_buffer.id))

                await self.tensor_transfer_engine.async_send_metadata_to(
                    self.tensor_transfer_engine.remote_names[block_md.experts_block_index],
                    header=P2PHeaders.DispatchSubmit.value, body=packet)

                async with self.async_lock:
                    transferred_activations[0] += self.used_activations
                    active_pipeline_tasks[0] += 1
                self.experts_block_pool.add_load(self.dispatched_block, self.used_activations)
            else:
                self.logger.debug("dispatch skipped: nothing to pack for this block")
        except (asyncio.TimeoutError, RuntimeError, KeyError) as e:
            self.logger.error(f"dispatch {type(e).__name__}: {e}")
            self.close()
        except Exception as e:
            self.logger.error(f"dispatch unknown error: {e}")
            self.close()
        finally:
            if self.experts_block_index != -1:
                self.experts_block_pool.release(self.experts_block_index)
                self.experts_block_index = -1
            self.dispatch_done = True
            if self.metrics_collector is not None:
                self.metrics_collector.end_dispatch(task_id)

    async def combine(self, active_pipeline_tasks: List[int], output_batch: torch.Tensor, combining: asyncio.Event) -> None:
        """Move this task's expert outputs into the forward's permuted-order arena (rows
        ``offsets[e] + l ...``); the weighted per-token sum happens after the last task."""
        task_id = self.name.hex()
        if self.metrics_collector is not None:
            self.metrics_collector.start_combine(task_id)
        fs = self.forward_state
        try:
            if self.output_buffer is None:
                raise RuntimeError(f"While combining {self.name}, there is no acquired output buffer.")
            buf = self.output_buffer
            s = buf.cuda_stream
            seg_src, seg_dst, seg_len = [], [], []
            o = 0
            for e, l, padded, actual in self.experts_metadata_snapshot:
                seg_src.append(o)
                seg_dst.append(fs.offsets[e] + l)
                seg_len.append(actual)
                o += padded
            buf.begin_use(s)
            N.permute_rows(buf.data, fs.arena, seg_src, seg_dst, seg_len, stream=s.cuda_stream)
            buf.end_use(s)
            ev = torch.cuda.Event()
            ev.record(s)
            fs.events.append(ev)
            fs.covered.extend((e, l, actual) for e, l, _p, actual in self.experts_metadata_snapshot)
        except Exception as e:
            self.close()
            self.logger.error(f"Combine failed for task {self.name.hex()[:8]}: {e}")
        finally:
            async with self.async_lock:
                active_pipeline_tasks[0] -= 1
                should_signal = active_pipeline_tasks[0] <= 0
            self.release_input_buffer()
            self.release_output_buffer()
            self.experts_block_pool.sub_load(self.dispatched_block, self.used_activations)
            if should_signal:
                combining.set()
            self.combine_done = True
            if self.metrics_collector is not None:
                self.metrics_collector.end_combine(task_id)

    def abort(self) -> None:
        """Return this task's segments to the experts' queues for re-dispatch (``:372-375``)."""
        for e, l, _size, actual in self.experts_metadata_snapshot:
            self.experts_metadata[e].expert_offsets.put((l, l + actual))
        if self.dispatched_block != -1 and not self.combine_done:
            self.experts_block_pool.sub_load(self.dispatched_block, self.used_activations)
        self.close()

    def close(self) -> None:
        if self.experts_block_index != -1:
            self.experts_block_pool.release(self.experts_block_index)
            self.experts_block_index = -1
        super().close()


class ExpertsBlockPipelineTask(PipelineTask):
    def __init__(self, tensor_transfer_engine: TensorTransferEngine, input_buffers_pool: BuffersPool,
                 output_buffers_pool: BuffersPool, expert_layers: Dict[int, Any], experts_combine_layer: Optional[Any],
                 expert_streams: Dict[int, torch.cuda.Stream], host_address: str, metadata: List[Tuple[int, bytes]],
                 async_lock: asyncio.Lock, metrics_collector=None, activation: int = N.ACT_RELU) -> None:
        super().__init__(tensor_transfer_engine, input_buffers_pool, output_buffers_pool, async_lock)
        self.host_address = host_address
        self.metadata = metadata
        self.expert_layers = expert_layers
        self.expert_streams = expert_streams
        # (expert index -> stack position, gate [E,I,d], up [E,I,d], down [E,d,I])
        self.experts_combine_layer = experts_combine_layer
        self.metrics_collector = metrics_collector
        self.activation = activation

    async def run(self, experts_block_index: int, host_input_buffers_transfer_descs: Dict[bytes, Any],
                  host_output_buffers_transfer_descs: Dict[bytes, Any]) -> None:
        task_id = self.name.hex()
        if self.metrics_collector is not None:
            self.metrics_collector.start_expert_run(task_id, experts_block_index)
        try:
            host_task_name: bytes = self.metadata[0][1]
            number_of_experts = struct.unpack("!H", self.metadata[2][1])[0]
            if len(self.metadata) != 3 + number_of_experts * 3 + 2:
                raise RuntimeError(f"While running {self.name}, metadata packet structure is broken.")
            host_in_id: bytes = self.metadata[-2][1]
            host_out_id: bytes = self.metadata[-1][1]

            position, gate_w, up_w, down_w = self.experts_combine_layer
            seg_pos: List[int] = []
            seg_end: List[int] = []
            for i in range(number_of_experts):
                e = struct.unpack("!H", self.metadata[3 + 3 * i][1])[0]
                off = struct.unpack("!H", self.metadata[4 + 3 * i][1])[0]
                size = struct.unpack("!H", self.metadata[5 + 3 * i][1])[0]
                seg_pos.append(position[e])
                seg_end.append(off + size)
            rows = seg_end[-1] if seg_end else 0

            if self.input_buffer_index == -1:
                self.input_buffer_index, self.input_buffer = await self.input_buffers_pool.acquire()
            in_buf = self.input_buffer
            tte = self.tensor_transfer_engine
            host_in = host_input_buffers_transfer_descs[host_in_id]
            host_out = host_output_buffers_transfer_descs[host_out_id]
            dev = in_buf.device.index
            if hasattr(tte, "region_is_local") and tte.region_is_local(host_in[0], dev) \
                    and tte.region_is_local(host_out[0], dev):
                # The host's buffers live on this GPU: compute straight from its input buffer
                # into its output buffer (no READ/WRITE copies), ordered by their region events.
                s = in_buf.cuda_stream
                with torch.cuda.stream(s):
                    tte.wait_region(host_in + host_out, s)
                    N.grouped_gated_mlp_ptrs(tte.region_ptr(host_in[0]), tte.region_ptr(host_out[0]), max(rows, 1),
                                             gate_w, up_w, down_w, seg_pos, seg_end, self.activation)
                    tte.signal_region(host_in + host_out, s)
                self.input_buffers_pool.release(self.input_buffer_index)
                self.input_buffer = None
                self.input_buffer_index = -1
                await tte.async_send_metadata_to(
                    self.host_address, P2PHeaders.HostOutputBufferUnlocked.value, [(len(host_task_name), host_task_name)])
                return

            # READ: only the rows this task packed.
            if self.metrics_collector is not None:
                self.metrics_collector.record_transfer_start(task_id, "read", rows * in_buf.row_bytes)
            await in_buf.read_from(self.host_address, host_input_buffers_transfer_descs[host_in_id],
                                   nbytes=rows * in_buf.row_bytes)
            if self.metrics_collector is not None:
                self.metrics_collector.record_transfer_end(task_id, "read")

            # COMPUTE: grouped gated MLP on the input buffer's stream.
            if self.output_buffer_index == -1:
                self.output_buffer_index, self.output_buffer = await self.output_buffers_pool.acquire()
            out_buf = self.output_buffer
            s = in_buf.cuda_stream
            with torch.cuda.stream(s):
                in_buf.begin_use(s)
                out_buf.begin_use(s)
                N.grouped_gated_mlp(in_buf.data, gate_w, up_w, down_w, seg_pos, seg_end, self.activation,
                                    out_buf.data, m_rows=max(rows, 1))
                in_buf.end_use(s)
                out_buf.end_use(s)
            self.input_buffers_pool.release(self.input_buffer_index)
            self.input_buffer = None
            self.input_buffer_index = -1

            # WRITE into the host's output buffer, then acknowledge.
            if self.metrics_collector is not None:
                self.metrics_collector.record_transfer_start(task_id, "write", rows * out_buf.row_bytes)
            await out_buf.write_to(self.host_address, host_output_buffers_transfer_descs[host_out_id],
                                   nbytes=rows * out_buf.row_bytes)
            if self.metrics_collector is not None:
                self.metrics_collector.record_transfer_end(task_id, "write")
            await self.tensor_transfer_engine.async_send_metadata_to(
                self.host_address, P2PHeaders.HostOutputBufferUnlocked.value, [(len(host_task_name), host_task_name)])
        except Exception as e:
            self.logger.error(f"Experts block runtime error: {type(e).__name__}: {e}")
        finally:
            if self.metrics_collector is not None:
                self.metrics_collector.end_expert_run(task_id)
            self.close()
