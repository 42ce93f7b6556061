"""NVLink / CUDA-IPC transfer engine: the B200 data plane replacing NIXL/UCX and MoonCake
(``TensorTransferEngine/NIXLTensorTransferEngine.py``, ``MCTETensorTransferEngine.py``).

A registered region is described by (pid, device, pointer, size, CUDA-IPC memory handle +
offset, completion-event token).  A peer in the same process uses the pointer directly
(UVA + peer access over NVLink); a peer in another process maps the IPC handle once and
caches the mapping.  READ and WRITE are stream-ordered copies issued on the caller's current
CUDA stream: they wait for the last-access events of both regions, copy over NVLink /
NVSwitch (or within HBM when both regions are on one GPU), and record both events again.
Consumers order themselves after a region with :meth:`wait_region` instead of a host round
trip; :meth:`wait_for_transfer_efficient` still works for callers that want a host wait.

Completion events are raw CUDA events of the library (``dmoe_event_*``), shared through a
process-local registry or as CUDA IPC event handles across processes.  Only the owner of a
region records its event.  A process that touched another process's region records an
interprocess event of its own on that stream and sends the owner a completion notice ahead
of its next message; the owner then orders the region's event after it.  An interprocess
event is only waited on by streams of the GPU it belongs to: other GPUs go through a helper
stream on that GPU.  No kernel spins on a flag here, so host and expert block may share one
GPU.
"""

from __future__ import annotations

import asyncio
import itertools
import os
import socket
import struct
import threading
import time
import timeit
from collections import OrderedDict, deque
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import torch

from distributedmoe_b200 import _native as N
from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import (
    TensorTransferEngine,
    TensorTransferEngineConfig,
)
from distributedmoe_b200.TensorTransferEngine.utils import HandshakeType, Transfer, TransferStatus
from distributedmoe_b200.utils.logging_config import get_logger

# Engines of this process by their own name ("address:port"), for the in-process metadata channel.
_ENGINES: Dict[str, "NVLinkTensorTransferEngine"] = {}
_ENGINES_LOCK = threading.Lock()


class _Inbox:
    """Thread-safe FIFO of metadata packets from one in-process peer; the receiving coroutine
    sleeps on a future of its own event loop and is woken with call_soon_threadsafe."""

    def __init__(self) -> None:
        self.lock = threading.Lock()
        self.items: deque = deque()
        self.waiter: Optional[asyncio.Future] = None

    def put(self, packet: bytes) -> None:
        with self.lock:
            self.items.append(packet)
            w, self.waiter = self.waiter, None
        if w is not None:
            w.get_loop().call_soon_threadsafe(_wake, w)

    async def get(self, timeout_s: float) -> bytes:
        while True:
            with self.lock:
                if self.items:
                    return self.items.popleft()
                fut = asyncio.get_running_loop().create_future()
                self.waiter = fut
            try:
                await asyncio.wait_for(fut, timeout_s)
            except asyncio.TimeoutError:
                with self.lock:
                    if self.waiter is fut:
                        self.waiter = None
                raise


def _wake(fut: asyncio.Future) -> None:
    if not fut.done():
        fut.set_result(None)


# Process-local registry of region events (raw interprocess CUDA events), addressed by
# 8-byte tokens in descriptors.
_EVENTS: Dict[int, int] = {}
_EVENTS_LOCK = threading.Lock()
_TOKENS = itertools.count(1)

_DESC = struct.Struct("!IhQQ64sQQ64s")  # pid, device, ptr, size, mem handle, offset, event token, event handle

# Copy handles kept for wait_for_transfer_efficient.
_KEPT_TRANSFERS = 4096

# Metadata header of a completion notice (outside the pipeline's 1000-1999 range).
NOTICE_HEADER = 4738


@dataclass
class NVLinkRegion:
    pid: int
    device: int
    ptr: int
    size: int
    mem_handle: bytes
    mem_offset: int
    event_token: int
    event_handle: bytes


class NVLinkTensorTransferEngine(TensorTransferEngine):
    """``TensorTransferEngine`` over CUDA IPC + NVLink (backend ``NVLinkIPC``)."""

    stream_ordered = True

    def __init__(self, config: TensorTransferEngineConfig) -> None:
        super().__init__(config)
        self.nv_logger = get_logger("dist_moe.tte.nvlink")
        self.pid = os.getpid()
        self.remote_info: Dict[str, Tuple[int, int, str]] = {}
        self._opened_mem: Dict[bytes, int] = {}       # mem handle -> mapped base (other processes)
        self._opened_events: Dict[Tuple[bytes, int], int] = {}  # (IPC event handle, device) -> event
        self._local_regions: Dict[int, NVLinkRegion] = {}
        self._helpers: Dict[Tuple[int, Any], torch.cuda.Stream] = {}
        self._lock = threading.Lock()
        # Local (not interprocess) events of each GPU for hand-offs between streams; one is
        # recorded and waited on as one step under _tmp_lock.
        self._tmp_events: Dict[int, int] = {}
        self._tmp_lock = threading.Lock()
        # Notice events: one interprocess event per stream that touched another process's
        # region, with its exported handle.  Re-recording it on the same stream only makes a
        # late waiter wait longer.
        self._notice_events: Dict[int, Tuple[int, int, bytes]] = {}  # stream -> (device, event, handle)
        self._pending_notice: Dict[str, Dict[int, set]] = {}  # owner -> stream -> region tokens
        self._region_owner: Dict[int, str] = {}
        self._notice_outbox: Dict[str, deque] = {}
        self._xfers: "OrderedDict[bytes, Transfer]" = OrderedDict()
        self._xfer_lock = threading.Lock()
        # Peers in this process exchange metadata through in-memory inboxes instead of ZeroMQ
        # once the handshake has shown that they share the process.
        self._inproc: Dict[str, bool] = {}
        self._inboxes: Dict[str, _Inbox] = {name: _Inbox() for name in self.remote_names}
        with _ENGINES_LOCK:
            _ENGINES[self.host_name] = self
        self._init_transfer_engine()
        if not self.handshake():
            raise RuntimeError(f"{self.host_name}: transfer-engine hand-shake failed (see the log)")

    def _init_transfer_engine(self) -> None:
        self.transfer_engine = "cuda-ipc"

    # ------------------------------------------------------------------ handshake
    def _identity(self) -> bytes:
        dev = torch.cuda.current_device() if torch.cuda.is_available() else -1
        return struct.pack("!Ih", self.pid, dev) + socket.gethostname().encode()[:200]

    HANDSHAKE_DEADLINE_S = 120.0

    def handshake_with_remote(self, remote_name: str) -> bool:
        """Exchange (pid, device, hostname); CLIENT speaks first, as the NIXL agents do
        (``NIXLTensorTransferEngine.py:87-108``)."""
        # A peer that never answers (its process or listener failed during set-up) ends the
        # hand-shake with an error after HANDSHAKE_DEADLINE_S instead of a retry loop forever.
        dl = self.HANDSHAKE_DEADLINE_S
        try:
            if self.handshake_type == HandshakeType.CLIENT:
                ident = self._identity()
                self.send_metadata_to(remote_name, 0, (len(ident), ident), deadline_s=dl)
                header, body = self.get_metadata_from(remote_name, deadline_s=dl)
            elif self.handshake_type == HandshakeType.SERVER:
                header, body = self.get_metadata_from(remote_name, deadline_s=dl)
                ident = self._identity()
                self.send_metadata_to(remote_name, 0, (len(ident), ident), deadline_s=dl)
            else:
                return True
            assert header == 0
            raw = body[-1][1]
            pid, dev = struct.unpack("!Ih", raw[:6])
            self.remote_info[remote_name] = (pid, dev, raw[6:].decode(errors="replace"))
            if pid == self.pid:
                with _ENGINES_LOCK:
                    peer = _ENGINES.get(remote_name)
                if peer is not None and self.host_name in peer._inboxes:
                    self._inproc[remote_name] = True
            if pid == self.pid and dev >= 0 and torch.cuda.is_available():
                here = torch.cuda.current_device()
                if dev != here:
                    N.enable_peer_access(here, dev)
                    N.enable_peer_access(dev, here)
            return True
        except Exception as e:
            self.nv_logger.error(f"handshake with {remote_name} failed: {e}")
            return False

    # ------------------------------------------------------------------ metadata channel
    async def async_send_metadata_to(self, remote_name: str, header: int, body) -> None:
        # Notices go first and stay queued until sent, so a send that times out and is
        # retried still delivers them ahead of the message.
        outbox = self._notice_outbox.setdefault(remote_name, deque())
        outbox.extend(self._take_notices(remote_name))
        while outbox:
            await self._send_packet(remote_name, outbox[0])
            outbox.popleft()
        await self._send_packet(remote_name, self.serialize_p2p_packet(header, body))

    async def _send_packet(self, remote_name: str, packet: bytes) -> None:
        if self._inproc.get(remote_name):
            with _ENGINES_LOCK:
                peer = _ENGINES.get(remote_name)
            if peer is not None and not peer.is_closed:
                peer._inboxes[self.host_name].put(packet)
                return
        await self.async_send_packet_to(remote_name, packet)

    async def async_get_metadata_from(self, remote_name: str):
        while True:
            if self._inproc.get(remote_name):
                packet = await self._inboxes[remote_name].get(self.p2p_timeout_duration / 1000.0)
                header, body = self.deserialize_p2p_packet(packet)
            else:
                header, body = await super().async_get_metadata_from(remote_name)
            if header != NOTICE_HEADER:
                return header, body
            self._apply_notice(body)

    # ------------------------------------------------------------------ registration
    def register_batch(self, data_ptrs: List[Any], data_location: Optional[str], device_id: int,
                       data_sizes: Optional[List[int]] = None) -> Tuple[List[NVLinkRegion], List[NVLinkRegion]]:
        regions = []
        for i, item in enumerate(data_ptrs):
            if isinstance(item, torch.Tensor):
                if not item.is_cuda:
                    raise ValueError("the NVLink transfer engine registers GPU memory only")
                ptr, size, dev = item.data_ptr(), item.numel() * item.element_size(), item.device.index
            else:
                ptr, size, dev = int(item), int(data_sizes[i]), int(device_id)
            if data_sizes is not None:
                size = int(data_sizes[i])
            with torch.cuda.device(dev):
                mem_handle, mem_offset = N.ipc_export(ptr)
            ev = N.event_create(dev, interprocess=True)  # not recorded yet: waits on it return at once
            ev_handle = N.ipc_event_export(ev)
            token = next(_TOKENS)
            with _EVENTS_LOCK:
                _EVENTS[token] = ev
            r = NVLinkRegion(self.pid, dev, ptr, size, mem_handle, mem_offset, token, ev_handle)
            self._local_regions[token] = r
            regions.append(r)
        return regions, regions

    def deregister_batch(self, data_registration_descs: List[NVLinkRegion], data_sizes: Optional[List[int]] = None) -> None:
        for r in data_registration_descs:
            self._local_regions.pop(r.event_token, None)
            with _EVENTS_LOCK:
                ev = _EVENTS.pop(r.event_token, None)
            if ev is not None:
                try:
                    N.event_destroy(ev)
                except Exception as e:  # pragma: no cover - best effort at shutdown
                    self.nv_logger.warning(f"destroying a region event failed: {e}")

    def serialize_descs(self, data_descs: List[NVLinkRegion]) -> Tuple[int, bytes]:
        blob = struct.pack("!H", len(data_descs)) + b"".join(
            _DESC.pack(r.pid, r.device, r.ptr, r.size, r.mem_handle, r.mem_offset, r.event_token, r.event_handle)
            for r in data_descs)
        return len(blob), blob

    def deserialize_descs(self, data_serialized_descs: Tuple[int, bytes]) -> List[NVLinkRegion]:
        _, blob = data_serialized_descs
        (n,) = struct.unpack("!H", blob[:2])
        out = []
        for i in range(n):
            f = _DESC.unpack_from(blob, 2 + i * _DESC.size)
            out.append(NVLinkRegion(f[0], f[1], f[2], f[3], f[4], f[5], f[6], f[7]))
        # Map another process's buffers, open their events and set up the helper stream on
        # their GPU now (set-up time), not inside the first transfer.
        if torch.cuda.is_available():
            for r in out:
                if r.pid != self.pid:
                    self.region_ptr(r)
                    self.region_event(r)
                    self._tmp_event(r.device)  # also brings up this process's context on that GPU
        return out

    # ------------------------------------------------------------------ addressing
    def region_ptr(self, r: NVLinkRegion) -> int:
        """A pointer to the region usable from this process (peer pointer or IPC mapping)."""
        if r.pid == self.pid:
            return r.ptr
        with self._lock:
            base = self._opened_mem.get(r.mem_handle)
            if base is None:
                base = N.ipc_open(r.mem_handle, torch.cuda.current_device())
                self._opened_mem[r.mem_handle] = base
        return base + r.mem_offset

    def region_is_local(self, r: NVLinkRegion, device: int) -> bool:
        """True when the region is memory of `device` mapped in this process (kernels on that
        GPU can use it directly, with no transfer)."""
        return r.pid == self.pid and r.device == device

    def region_event(self, r: NVLinkRegion) -> int:
        """The region's last-access event: the registry entry for this process's regions, the
        owner's event opened once (on the owner's GPU) for another process's."""
        if r.pid == self.pid:
            with _EVENTS_LOCK:
                return _EVENTS[r.event_token]
        return self._open_event(r.event_handle, r.device)

    def _open_event(self, handle: bytes, device: int) -> int:
        key = (bytes(handle), device)
        with self._lock:
            ev = self._opened_events.get(key)
            if ev is None:
                ev = N.ipc_event_open(handle, device)
                self._opened_events[key] = ev
        return ev

    def wait_region(self, regions: List[NVLinkRegion], stream: Optional[torch.cuda.Stream] = None) -> None:
        """Order `stream` after the last completion recorded for each region."""
        stream = stream or torch.cuda.current_stream()
        for r in regions:
            self._wait_event_of(stream, self.region_event(r), r.device)

    def _wait_event_of(self, stream: torch.cuda.Stream, ev: int, ev_device: int) -> None:
        """Order `stream` after interprocess event `ev` of GPU `ev_device`.  Such an event is
        waited on only by a stream of its own GPU: for a stream elsewhere a helper stream on
        that GPU waits for it and hands over through a local event."""
        if stream.device.index == ev_device:
            N.stream_wait_event(stream.cuda_stream, ev)
            return
        h = self._helper_stream(ev_device, stream.cuda_stream)
        with self._tmp_lock:
            tmp = self._tmp_event(ev_device)
            N.stream_wait_event(h.cuda_stream, ev)
            N.event_record(tmp, h.cuda_stream)
            N.stream_wait_event(stream.cuda_stream, tmp)

    def _helper_stream(self, device: int, user: Any) -> torch.cuda.Stream:
        """A dedicated stream on `device` for one user (a stream, or a notice source).  A
        helper only waits and records; one per user keeps a late event of one user from
        holding up the others queued behind it."""
        key = (device, user)
        with self._lock:
            h = self._helpers.get(key)
            if h is None:
                # torch's high-priority pool: apart from the buffer pools' streams, which come
                # from the default-priority pool.
                h = torch.cuda.Stream(device=device, priority=-1)
                self._helpers[key] = h
        return h

    def _tmp_event(self, device: int) -> int:
        with self._lock:
            ev = self._tmp_events.get(device)
            if ev is None:
                ev = N.event_create(device)
                self._tmp_events[device] = ev
        return ev

    def signal_region(self, regions: List[NVLinkRegion], stream: Optional[torch.cuda.Stream] = None) -> None:
        """Record the work issued so far on `stream` as the regions' last access.  An event is
        recorded on a stream of its own GPU, so a region of another GPU is signalled through
        a helper stream there that waits for `stream`.  Regions of other processes get a
        completion notice instead."""
        stream = stream or torch.cuda.current_stream()
        here = stream.device.index
        foreign = [r for r in regions if r.pid != self.pid]
        if foreign:
            self._note_foreign(foreign, stream)
        for r in regions:
            if r.pid != self.pid:
                continue
            ev = self.region_event(r)
            if r.device == here:
                N.event_record(ev, stream.cuda_stream)
                continue
            h = self._helper_stream(r.device, stream.cuda_stream)
            with self._tmp_lock:
                tmp = self._tmp_event(here)
                N.event_record(tmp, stream.cuda_stream)
                N.stream_wait_event(h.cuda_stream, tmp)
            N.event_record(ev, h.cuda_stream)

    # ------------------------------------------------------------------ cross-process ordering
    def _note_foreign(self, regions: List[NVLinkRegion], stream: torch.cuda.Stream) -> None:
        """Record this stream's notice event after its work so far and remember, per owner,
        which of the owner's regions the work touched; the notice goes out ahead of the next
        message to that owner."""
        key = stream.cuda_stream
        with self._lock:
            entry = self._notice_events.get(key)
            if entry is None:
                dev = stream.device.index
                ev = N.event_create(dev, interprocess=True)
                entry = (dev, ev, N.ipc_event_export(ev))
                self._notice_events[key] = entry
            N.event_record(entry[1], key)
            for r in regions:
                owner = self._owner_name(r)
                if owner is None:
                    raise RuntimeError(f"no peer of this engine owns the region of pid {r.pid}")
                self._pending_notice.setdefault(owner, {}).setdefault(key, set()).add(r.event_token)

    def _owner_name(self, r: NVLinkRegion) -> Optional[str]:
        name = self._region_owner.get(r.event_token)
        if name is not None:
            return name
        for remote, (pid, _dev, _host) in self.remote_info.items():
            if pid == r.pid:
                self._region_owner[r.event_token] = remote
                return remote
        return None

    def _take_notices(self, remote_name: str) -> List[bytes]:
        with self._lock:
            pending = self._pending_notice.pop(remote_name, None)
            if not pending:
                return []
            out = []
            for key, tokens in pending.items():
                dev, _ev, handle = self._notice_events[key]
                body = [(2, struct.pack("!h", dev)), (len(handle), handle)] + \
                       [(8, struct.pack("!Q", t)) for t in sorted(tokens)]
                out.append(self.serialize_p2p_packet(NOTICE_HEADER, body))
        return out

    def _apply_notice(self, body) -> None:
        """Order the named regions' next users after the sender's work: a helper stream on
        each region's GPU waits for the sender's event, then records the region's event."""
        (dev,) = struct.unpack("!h", body[0][1])
        ev = self._open_event(body[1][1], dev)
        for _, raw in body[2:]:
            (token,) = struct.unpack("!Q", raw)
            r = self._local_regions.get(token)
            if r is None:
                continue
            # One helper per sending GPU: its notices come from the one block there that
            # serves this host, in that block's order.
            h = self._helper_stream(r.device, ("notice", dev))
            self._wait_event_of(h, ev, dev)
            N.event_record(self.region_event(r), h.cuda_stream)

    # ------------------------------------------------------------------ transfers
    def _transfer(self, remote_name: str, transfer_name: bytes, src: List[NVLinkRegion], dst: List[NVLinkRegion],
                  sizes: Optional[List[int]]) -> None:
        stream = torch.cuda.current_stream()
        total = 0
        # A region's event marks its last access: wait for both ends, then record both.
        self.wait_region(list(src) + list(dst), stream)
        for i, (s, d) in enumerate(zip(src, dst)):
            n = min(s.size, d.size) if sizes is None else int(sizes[i])
            if n > min(s.size, d.size):
                raise ValueError(f"transfer of {n} bytes exceeds the registered regions")
            N.copy_bytes(self.region_ptr(d), self.region_ptr(s), n, stream.cuda_stream)
            total += n
        self.signal_region(list(src) + list(dst), stream)
        done = torch.cuda.Event()
        done.record(stream)
        self._track_transfer(Transfer(transfer_name, TransferStatus.CREATED, remote_name, done, total,
                                      timeit.default_timer()))

    def read_batch_transfer(self, remote_name: str, transfer_name: bytes, src_data_transfer_descs: List[NVLinkRegion],
                            dst_data_transfer_descs: List[NVLinkRegion], src_data_sizes: Optional[List[int]] = None) -> None:
        """Remote -> local, on the current stream (``NIXLTensorTransferEngine.py:205-249``)."""
        self._transfer(remote_name, transfer_name, src_data_transfer_descs, dst_data_transfer_descs, src_data_sizes)

    def write_batch_transfer(self, remote_name: str, transfer_name: bytes, src_data_transfer_descs: List[NVLinkRegion],
                             dst_data_transfer_descs: List[NVLinkRegion], src_data_sizes: Optional[List[int]] = None) -> None:
        """Local -> remote, on the current stream (``NIXLTensorTransferEngine.py:159-203``)."""
        self._transfer(remote_name, transfer_name, src_data_transfer_descs, dst_data_transfer_descs, src_data_sizes)

    def _check_handler_status(self, transfer: Transfer) -> bool:
        return bool(transfer.handler.query())  # a local torch event of the copy stream

    # ------------------------------------------------------------------ completion
    def _track_transfer(self, transfer: Transfer) -> None:
        """Copies are stream-ordered, so the pipeline never waits for them on the host.  The
        handle is kept (the most recent _KEPT_TRANSFERS) for callers of
        wait_for_transfer_efficient, which polls it itself; the monitor thread stays idle."""
        with self._xfer_lock:
            self._xfers[transfer.name] = transfer
            while len(self._xfers) > _KEPT_TRANSFERS:
                self._xfers.popitem(last=False)

    def wait_for_transfer_efficient(self, transfer_name: bytes, timeout: Optional[int] = None) -> Optional[Transfer]:
        """Block until the named copy finished; None after ``timeout`` ms or for an unknown
        name (``TensorTransferEngine.py:305-314``)."""
        with self._xfer_lock:
            t = self._xfers.get(transfer_name)
        if t is None:
            return None
        deadline = time.monotonic() + timeout / 1000 if timeout is not None else None
        while not self._check_handler_status(t):
            if deadline is not None and time.monotonic() >= deadline:
                return None
            time.sleep(20e-6)
        if t.status != TransferStatus.FINISHED:
            t.status = TransferStatus.FINISHED
            t.duration = (timeit.default_timer() - t.duration) * 1000
        return t

    def close(self) -> None:
        if self.is_closed:
            return
        for base in self._opened_mem.values():
            try:
                N.ipc_close(base)
            except Exception as e:  # pragma: no cover - best effort at shutdown
                self.nv_logger.warning(f"closing an IPC mapping failed: {e}")
        self._opened_mem.clear()
        events = list(self._opened_events.values()) + list(self._tmp_events.values()) + \
            [e[1] for e in self._notice_events.values()]
        for ev in events:
            try:
                N.event_destroy(ev)
            except Exception:  # pragma: no cover - best effort at shutdown
                pass
        self._opened_events.clear()
        self._tmp_events.clear()
        self._notice_events.clear()
        self._helpers.clear()
        self.deregister_batch(list(self._local_regions.values()))
        with _ENGINES_LOCK:
            if _ENGINES.get(self.host_name) is self:
                del _ENGINES[self.host_name]
        super().close()
