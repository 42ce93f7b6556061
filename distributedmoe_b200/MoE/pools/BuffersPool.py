"""Registered I/O buffers and their pool (reference ``MoE/pools/BuffersPool.py``).

A ``Buffer`` is a ``[size, hidden]`` tensor registered with the transfer engine plus a
CUDA stream.  The buffers of one pool share one stream (the reference gives each buffer its
own ``torch.cuda.Stream``, ``BuffersPool.py:45-46``; torch hands out 32 distinct streams
per device and priority, so with the many buffers of an expert-parallel process unrelated
buffers ended up sharing streams anyway).  The work on a pool's buffers is sequential:
one task's gather, copy or expert MLP after another.  With a stream-ordered engine (the NVLink backend) ``read_from`` and
``write_to`` enqueue the copy on the buffer's stream and return: work issued later on that
stream, or ordered after the region's completion event, sees the data.  Other engines are
waited for on the host with a 1000 ms limit, as the reference does (``BuffersPool.py:55-90``).
``begin_use``/``end_use`` bracket every GPU access: the buffer's last access is a CUDA event
(the engine's region event, visible to peers), so a new user on any stream, in any
process, is ordered after the previous one.
"""

from __future__ import annotations

import asyncio
from typing import List, Optional, Tuple

import torch

from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import TensorTransferEngine
from distributedmoe_b200.TensorTransferEngine.utils import _next_random_name
from distributedmoe_b200.utils.logging_config import get_logger


class Buffer:
    def __init__(self, tensor_transfer_engine: TensorTransferEngine, size: int, hidden_features: int,
                 dtype: torch.dtype, device: torch.device, cuda_stream: Optional[torch.cuda.Stream] = None) -> None:
        assert tensor_transfer_engine is not None
        self.id: bytes = b""
        self.logger = get_logger("dist_moe.buffer")
        self._tensor_transfer_engine = tensor_transfer_engine
        self.size = size
        self.hidden_features = hidden_features
        self.dtype = dtype
        self.row_bytes = hidden_features * dtype.itemsize
        self.size_in_bytes = size * self.row_bytes
        self.device = device
        self.data = torch.empty(size, hidden_features, dtype=dtype, device=device)
        self.cuda_stream = cuda_stream if cuda_stream is not None else torch.cuda.Stream(device=device)
        self.last_use = torch.cuda.Event()
        self.transfer_descs, self.register_descs = tensor_transfer_engine.register_batch(
            [self.data], "VRAM" if device.type == "cuda" else "DRAM", device.index)
        self.serialized_transfer_descs = tensor_transfer_engine.serialize_descs(self.transfer_descs)

    def begin_use(self, stream: torch.cuda.Stream) -> None:
        """Order `stream` after the buffer's last access (any process, any stream)."""
        tte = self._tensor_transfer_engine
        if hasattr(tte, "wait_region"):
            tte.wait_region(self.transfer_descs, stream)
        else:
            stream.wait_event(self.last_use)

    def end_use(self, stream: torch.cuda.Stream) -> None:
        """Record the work issued so far on `stream` as the buffer's last access."""
        tte = self._tensor_transfer_engine
        if hasattr(tte, "signal_region"):
            tte.signal_region(self.transfer_descs, stream)
        else:
            self.last_use.record(stream)

    async def _transfer(self, kind: str, remote_name: str, descs, nbytes: Optional[int]) -> None:
        tte = self._tensor_transfer_engine
        name = _next_random_name()
        n = self.size_in_bytes if nbytes is None else int(nbytes)
        with torch.cuda.stream(self.cuda_stream):
            if kind == "read":
                tte.read_batch_transfer(remote_name, name, descs, self.transfer_descs, [n])
            else:
                tte.write_batch_transfer(remote_name, name, self.transfer_descs, descs, [n])
        if getattr(tte, "stream_ordered", False):
            return
        timeout = 1000  # ms
        done = await asyncio.to_thread(tte.wait_for_transfer_efficient, name, timeout)
        if not done:
            self.logger.error(f"{kind} transfer {name.hex()} timed out after {timeout} ms")
            raise TimeoutError(f"{kind.capitalize()} transfer timed out")

    async def read_from(self, remote_name: str, src_buffer_transfer_descs, nbytes: Optional[int] = None) -> None:
        """Copy the remote buffer into this one (``nbytes`` defaults to the whole buffer)."""
        await self._transfer("read", remote_name, src_buffer_transfer_descs, nbytes)

    async def write_to(self, remote_name: str, dst_buffer_transfer_descs, nbytes: Optional[int] = None) -> None:
        """Copy this buffer into the remote one (``nbytes`` defaults to the whole buffer)."""
        await self._transfer("write", remote_name, dst_buffer_transfer_descs, nbytes)

    def close(self) -> None:
        try:
            self._tensor_transfer_engine.deregister_batch(self.register_descs)
        except Exception as e:
            self.logger.error(f"Failed to deregister buffer memory: {e}")


class BuffersPool:
    def __init__(self, pool_size: int, tensor_transfer_engine: TensorTransferEngine, buffer_size: int,
                 hidden_features: int, dtype: torch.dtype, device: torch.device) -> None:
        self.logger = get_logger("dist_moe.buffer_pool", {"pool_size": str(pool_size)})
        self.pool_size = pool_size
        self.buffer_size = buffer_size
        self.hidden_features = hidden_features
        self.dtype = dtype
        self.device = device
        self.buffers: List[Buffer] = []
        self.buffer_index_pool: asyncio.Queue = asyncio.Queue()
        self.cuda_stream = torch.cuda.Stream(device=device) if device.type == "cuda" else None
        for i in range(pool_size):
            self.buffers.append(Buffer(tensor_transfer_engine, buffer_size, hidden_features, dtype, device,
                                       cuda_stream=self.cuda_stream))
            self.buffer_index_pool.put_nowait(i)

    async def acquire(self) -> Tuple[int, Buffer]:
        try:
            i: int = await self.buffer_index_pool.get()
            return i, self.buffers[i]
        except (asyncio.QueueEmpty, AttributeError):
            raise RuntimeError("Buffer pool queue is shut down.")

    def release(self, buffer_index: int) -> None:
        self.buffer_index_pool.put_nowait(buffer_index)

    def close(self) -> None:
        failed = 0
        for i, b in enumerate(self.buffers):
            try:
                b.close()
            except Exception as e:
                failed += 1
                self.logger.error(f"Failed to close buffer {i}: {e}")
        if failed:
            self.logger.warning(f"BuffersPool cleanup: {failed} of {len(self.buffers)} buffers failed")

