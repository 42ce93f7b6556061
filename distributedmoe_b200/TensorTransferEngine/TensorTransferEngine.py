"""Transfer-engine abstraction with the reference's interface
(``TensorTransferEngine/TensorTransferEngine.py:21-370``).

What stays the same: the configuration dataclass, the ZeroMQ PUSH/PULL metadata channel
per remote, the 2-byte framed packet format, the synchronous/asynchronous metadata calls,
``wait_for_transfer_efficient`` and the abstract backend methods.

What changes: the backend enum gains ``NVLinkIPC`` (CUDA IPC peer buffers over NVLink /
NVSwitch) and ``NVLinkDirect`` (the same plus a kernel-driven exchange window), and the
base class no longer imports a transfer library.  The completion monitor
sleeps while nothing is in flight instead of polling every millisecond, and waiters poll
their own transfer, so a finished copy is seen within microseconds.
"""

from __future__ import annotations

import asyncio
import struct
import threading
import time
import timeit
from abc import ABC, abstractmethod
from dataclasses import dataclass
from enum import Enum
from typing import Any, Dict, List, Optional, Tuple

import zmq
import zmq.asyncio

from distributedmoe_b200.TensorTransferEngine.utils import (
    HandshakeType,
    P2PPair,
    Transfer,
    TransferProtocol,
    TransferStatus,
    join_host_port,
)
from distributedmoe_b200.utils.logging_config import get_logger


class TensorTransferEngineBackend(Enum):
    MoonCake = "MoonCake"
    NIXL = "NIXL"
    NVLinkIPC = "NVLinkIPC"
    # NVLinkIPC plus the device-driven exchange: senders' kernels write rows into the
    # receivers' buffers over NVLink and epoch flags replace the per-task messages.
    NVLinkDirect = "NVLinkDirect"


@dataclass
class TensorTransferEngineConfig:
    # This engine's own endpoint: the address and port that name it, and one local port per
    # remote on which it pushes metadata packets to that remote.
    host_address: str
    host_port: int
    host_p2p_ports: List[int]

    # The peers, one entry per remote engine: their addresses, the ports that name them, and
    # the ports on which they push metadata to this engine.
    remote_addresses: List[str]
    remote_ports: List[int]
    remote_p2p_ports: List[int]

    # How long (ms) a metadata send or receive may block before it fails.
    p2p_timeout_duration: int

    # Which side speaks first in the start-up exchange of identities.
    handshake_type: HandshakeType

    # Link family the backend moves data over (RDMA or NVLink).
    transfer_protocol: TransferProtocol

    # InfiniBand adapters for RDMA backends; the NVLink backend ignores it.
    ib_device_names: str

    # Settings of MoonCake's metadata service; the NVLink backend ignores them.
    metadata_schema: Optional[str] = None
    metadata_host: Optional[str] = None
    metadata_port: Optional[int] = None
    metadata_dir: Optional[str] = None


class TensorTransferEngine(ABC):
    def __init__(self, config: TensorTransferEngineConfig) -> None:
        self.logger = get_logger("dist_moe.tte.engine")

        assert len(config.remote_addresses) == len(config.remote_p2p_ports)
        assert len(config.remote_addresses) == len(config.remote_ports)
        assert len(config.host_p2p_ports) == len(config.remote_p2p_ports)

        self.transfer_protocol = config.transfer_protocol
        self.ib_device_names = config.ib_device_names

        self.host_name = join_host_port(config.host_address, config.host_port)
        self.remote_names = [join_host_port(h, p) for h, p in zip(config.remote_addresses, config.remote_ports)]

        self.handshake_type = config.handshake_type
        self.p2p_timeout_duration = config.p2p_timeout_duration
        self.metadata_p2p_pairs: Dict[str, P2PPair] = {}
        self.setup_p2p_connections(config)

        self.transfer_engine: Any = None
        self.done_transfers: Dict[bytes, Transfer] = {}

        self._stop_event = threading.Event()
        self._transfers: List[Transfer] = []
        self._transfers_lock = threading.Lock()
        self._transfer_condition = threading.Condition(self._transfers_lock)
        self._transfers_thread = threading.Thread(target=self._monitor_transfers, daemon=True)
        self._transfers_thread.start()

        self._serialized_size = 2
        self.is_closed = False
        self.logger.info(f"TensorTransferEngine initialized - Host: {self.host_name}, Remotes: {len(self.remote_names)}")

    # ------------------------------------------------------------------ P2P channel
    def setup_p2p_connections(self, config: TensorTransferEngineConfig) -> None:
        self.context = zmq.asyncio.Context()
        for i, remote_name in enumerate(self.remote_names):
            pair = P2PPair(self.context.socket(zmq.PUSH), self.context.socket(zmq.PULL))
            pair.pusher.bind(join_host_port(config.host_address, config.host_p2p_ports[i], "tcp"))
            pair.pusher.setsockopt(zmq.RCVTIMEO, self.p2p_timeout_duration)
            pair.puller.connect(join_host_port(config.remote_addresses[i], config.remote_p2p_ports[i], "tcp"))
            pair.puller.setsockopt(zmq.RCVTIMEO, self.p2p_timeout_duration)
            self.metadata_p2p_pairs[remote_name] = pair

    @abstractmethod
    def _init_transfer_engine(self) -> None:
        ...

    @abstractmethod
    def handshake_with_remote(self, remote_name: str) -> bool:
        ...

    def handshake(self) -> bool:
        if self.handshake_type == HandshakeType.NONE:
            return True
        try:
            for remote_name in self.remote_names:
                assert self.handshake_with_remote(remote_name)
        except Exception as e:
            self.logger.error(f"handshake failed: {e}")
            return False
        return True

    # ------------------------------------------------------------------ backend data plane
    @abstractmethod
    def register_batch(self, data_ptrs: List[Any], data_location: Optional[str], device_id: int,
                       data_sizes: Optional[List[int]] = None) -> Tuple[Any, Any]:
        ...

    @abstractmethod
    def deregister_batch(self, data_registration_descs: Any, data_sizes: Optional[List[int]] = None) -> None:
        ...

    @abstractmethod
    def write_batch_transfer(self, remote_name: str, transfer_name: bytes, src_data_transfer_descs: Any,
                             dst_data_transfer_descs: Any, src_data_sizes: Optional[List[int]] = None) -> None:
        ...

    @abstractmethod
    def read_batch_transfer(self, remote_name: str, transfer_name: bytes, src_data_transfer_descs: Any,
                            dst_data_transfer_descs: Any, src_data_sizes: Optional[List[int]] = None) -> None:
        ...

    @abstractmethod
    def serialize_descs(self, data_descs: Any) -> Tuple[int, bytes]:
        ...

    @abstractmethod
    def deserialize_descs(self, data_serialized_descs: Tuple[int, bytes]) -> Any:
        ...

    @abstractmethod
    def _check_handler_status(self, transfer: Transfer) -> bool:
        ...

    # ------------------------------------------------------------------ packets
    def serialize_p2p_packet(self, header: int, body) -> bytes:
        """``!H header, !H count, [!H size, bytes] * count`` (``TensorTransferEngine.py:194-207``)."""
        parts = [struct.pack("!H", header)]
        if isinstance(body, list):
            parts.append(struct.pack("!H", len(body)))
            for size, meta in body:
                parts.append(struct.pack("!H", size))
                parts.append(meta)
        else:
            parts.append(struct.pack("!H", 1))
            parts.append(struct.pack("!H", body[0]))
            parts.append(body[1])
        return b"".join(parts)

    def deserialize_p2p_packet(self, packet: bytes) -> Tuple[int, List[Tuple[int, bytes]]]:
        n = self._serialized_size
        header = struct.unpack("!H", packet[0:n])[0]
        count = struct.unpack("!H", packet[n:2 * n])[0]
        off = 2 * n
        body = []
        for _ in range(count):
            size = struct.unpack("!H", packet[off:off + n])[0]
            off += n
            body.append((size, packet[off:off + size]))
            off += size
        return header, body

    async def async_send_metadata_to(self, remote_name: str, header: int, body) -> None:
        await self.async_send_packet_to(remote_name, self.serialize_p2p_packet(header, body))

    async def async_send_packet_to(self, remote_name: str, packet: bytes) -> None:
        try:
            await asyncio.wait_for(self.metadata_p2p_pairs[remote_name].pusher.send(packet),
                                   self.p2p_timeout_duration / 1000.0)
        except zmq.Again:
            raise asyncio.TimeoutError()

    async def async_get_metadata_from(self, remote_name: str) -> Tuple[int, List[Tuple[int, bytes]]]:
        try:
            packet = await asyncio.wait_for(self.metadata_p2p_pairs[remote_name].puller.recv(),
                                            self.p2p_timeout_duration / 1000.0)
        except zmq.Again:
            raise asyncio.TimeoutError()
        return self.deserialize_p2p_packet(packet)

    def _run_blocking(self, coro_fn):
        try:
            loop = asyncio.get_running_loop()
        except RuntimeError:
            loop = None
        if loop is None:
            return asyncio.run(coro_fn())
        return asyncio.run_coroutine_threadsafe(coro_fn(), loop).result()

    def send_metadata_to(self, remote_name: str, header: int, body, deadline_s: Optional[float] = None) -> None:
        """Blocking send; retries on timeout (``TensorTransferEngine.py:258-275``), for at most
        deadline_s seconds when given (then TimeoutError)."""
        t0 = timeit.default_timer()
        while True:
            try:
                return self._run_blocking(lambda: self.async_send_metadata_to(remote_name, header, body))
            except (asyncio.TimeoutError, zmq.Again):
                if deadline_s is not None and timeit.default_timer() - t0 > deadline_s:
                    raise TimeoutError(f"no metadata could be sent to {remote_name} in {deadline_s:.0f} s") from None
                self.logger.warning(f"Waiting to send metadata to {remote_name}, retrying...")

    def get_metadata_from(self, remote_name: str,
                          deadline_s: Optional[float] = None) -> Tuple[int, List[Tuple[int, bytes]]]:
        """Blocking receive; retries on timeout (``TensorTransferEngine.py:281-295``), for at
        most deadline_s seconds when given (then TimeoutError)."""
        t0 = timeit.default_timer()
        while True:
            try:
                return self._run_blocking(lambda: self.async_get_metadata_from(remote_name))
            except (asyncio.TimeoutError, zmq.Again):
                if deadline_s is not None and timeit.default_timer() - t0 > deadline_s:
                    raise TimeoutError(f"no metadata from {remote_name} in {deadline_s:.0f} s") from None
                self.logger.warning(f"Waiting for metadata from {remote_name}, retrying...")

    # ------------------------------------------------------------------ completion
    def _track_transfer(self, transfer: Transfer) -> None:
        with self._transfer_condition:
            self._transfers.append(transfer)
            self._transfer_condition.notify_all()

    def _finish(self, transfer: Transfer) -> None:
        transfer.status = TransferStatus.FINISHED
        transfer.duration = (timeit.default_timer() - transfer.duration) * 1000
        self.done_transfers[transfer.name] = transfer

    def wait_for_transfer(self, transfer_name: bytes) -> Optional[Transfer]:
        return self.wait_for_transfer_efficient(transfer_name, None)

    def wait_for_transfer_efficient(self, transfer_name: bytes, timeout: Optional[int] = None) -> Optional[Transfer]:
        """Block until the named transfer finished; None after ``timeout`` ms
        (``TensorTransferEngine.py:305-314``).  The waiter checks its own transfer, so it does
        not depend on the monitor's polling period."""
        deadline = time.monotonic() + timeout / 1000 if timeout is not None else None
        while True:
            with self._transfer_condition:
                done = self.done_transfers.get(transfer_name)
                if done is not None or len(transfer_name) == 0:
                    return done
                mine = next((t for t in self._transfers if t.name == transfer_name), None)
                if mine is not None and self._check_handler_status(mine):
                    self._transfers.remove(mine)
                    self._finish(mine)
                    self._transfer_condition.notify_all()
                    return mine
            if deadline is not None and time.monotonic() >= deadline:
                return None
            time.sleep(20e-6)

    def _monitor_transfers(self) -> None:
        while not self._stop_event.is_set():
            with self._transfer_condition:
                if not self._transfers:
                    self._transfer_condition.wait(0.05)
                    continue
                finished = [t for t in self._transfers if self._check_handler_status(t)]
                for t in finished:
                    self._transfers.remove(t)
                    self._finish(t)
                if finished:
                    self._transfer_condition.notify_all()
            time.sleep(100e-6)

    def close(self) -> None:
        if self.is_closed:
            return
        self._stop_event.set()
        with self._transfer_condition:
            self._transfer_condition.notify_all()
        self._transfers_thread.join(timeout=5.0)
        for remote_name, pair in self.metadata_p2p_pairs.items():
            try:
                pair.pusher.close(linger=0)
                pair.puller.close(linger=0)
            except Exception as e:
                self.logger.warning(f"Error closing P2P pair for {remote_name}: {e}")
        try:
            self.context.term()
        except Exception as e:
            self.logger.warning(f"Error terminating ZMQ context: {e}")
        self.is_closed = True
