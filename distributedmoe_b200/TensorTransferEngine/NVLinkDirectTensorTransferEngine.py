"""NVLinkDirect: the NVLink / CUDA-IPC engine plus a receive window for the device-driven
expert-parallel exchange (backend ``NVLinkDirect``).

Everything the NVLinkIPC engine does (registration, IPC mappings, metadata channel, region
events) stays available.  On top, each engine owns one window in its GPU's memory:

* ``recv``   [capacity, d]  the rows every host dispatches to this GPU's expert instances
             (the input buffer of the GPU's expert blocks, written by the senders' gather
             kernel through peer pointers); with 8-bit experts, uint8 records of d e4m3
             codes and the row's fp32 scale (d + 16 bytes);
* ``back``   [capacity] int32  each receive row's return address (host rank, token * k +
             slot), written by the senders' gather beside the row;
* ``rows``   [max_tokens * k, d]  this host's expert outputs in (token, slot) order, written
             by the owners' down-projection epilogues through peer pointers (the host's
             output buffer), read by its own combine;
* ``flags``  epoch flags [kind][sender] that senders and receivers raise on each other;
* ``counts`` the per-instance row counts every sender writes before dispatching.

The regions are registered like any buffer (``register_batch``), their descriptors go to
every rank once, and :meth:`attach_windows` maps the peers' regions and returns the table
the exchange kernels take.  Replaces the NIXL/MoonCake registration and transfer calls of
``TensorTransferEngine/NIXLTensorTransferEngine.py:113-249`` for this path: no READ/WRITE
copies and no per-task metadata messages remain on the data path.
"""

from __future__ import annotations

import struct
from typing import List, Optional

import torch

from distributedmoe_b200 import _native as N
from distributedmoe_b200.TensorTransferEngine.NVLinkTensorTransferEngine import NVLinkTensorTransferEngine


class NVLinkDirectTensorTransferEngine(NVLinkTensorTransferEngine):
    """``TensorTransferEngine`` for the device-driven exchange (backend ``NVLinkDirect``)."""

    direct = True

    def __init__(self, config) -> None:
        super().__init__(config)
        self.recv: Optional[torch.Tensor] = None
        self.back: Optional[torch.Tensor] = None
        self.rows: Optional[torch.Tensor] = None
        self.flags: Optional[torch.Tensor] = None
        self.counts: Optional[torch.Tensor] = None
        self.capacity = 0
        self._window_regions = None
        self._peer_regions: List[list] = []
        self.window: Optional[N.EpWindow] = None

    def open_window(self, capacity: int, return_rows: int, hidden: int, dtype: torch.dtype, n_inst: int,
                    device: torch.device, record_bytes: Optional[int] = None) -> None:
        """Allocate and register this GPU's window (flags and counts zeroed).  capacity:
        receive rows; return_rows: this host's max_tokens * top_k; record_bytes: bytes of one
        receive row when it is not `hidden` elements of `dtype` (8-bit records)."""
        if self.recv is not None:
            raise RuntimeError("the window is already open")
        if capacity < 1 or return_rows < 1:
            raise ValueError("the window needs at least one receive row and one return row")
        device = torch.device(device)
        with torch.cuda.device(device):
            if record_bytes is None:
                self.recv = torch.empty(capacity, hidden, dtype=dtype, device=device)
            else:
                self.recv = torch.empty(capacity, record_bytes, dtype=torch.uint8, device=device)
            self.back = torch.full((capacity,), -1, dtype=torch.int32, device=device)
            self.rows = torch.empty(return_rows, hidden, dtype=dtype, device=device)
            self.flags = torch.zeros(N.ep_flags_bytes() // 8, dtype=torch.int64, device=device)
            self.counts = torch.zeros(max(N.ep_counts_bytes(n_inst) // 4, 1), dtype=torch.int32, device=device)
            torch.cuda.synchronize(device)  # zeros are in place before any peer can see the window
        self.capacity = capacity
        regions, _ = self.register_batch([self.flags, self.counts, self.recv, self.back, self.rows], "VRAM",
                                         device.index)
        self._window_regions = regions

    def window_descriptor(self) -> bytes:
        """Serialized descriptors of this window's regions (flags, counts, recv, back, rows)."""
        if self._window_regions is None:
            raise RuntimeError("open_window first")
        _, blob = self.serialize_descs(self._window_regions)
        return struct.pack("!Q", self.capacity) + blob

    def attach_windows(self, descriptors: List[bytes], rank: int) -> N.EpWindow:
        """Map every rank's window (descriptors in rank order, this rank's included) and
        build the table the exchange kernels read."""
        world = len(descriptors)
        if not 1 <= world <= N.EP_MAX_RANKS:
            raise ValueError(f"{world} ranks; 1..{N.EP_MAX_RANKS} supported")
        flags, counts, recv, back, rows = [], [], [], [], []
        self._peer_regions = []
        for g, blob in enumerate(descriptors):
            (cap,) = struct.unpack("!Q", blob[:8])
            if cap != self.capacity:
                raise ValueError(f"rank {g} opened a window of {cap} rows, this rank {self.capacity}")
            regions = self.deserialize_descs((len(blob) - 8, blob[8:]))
            if len(regions) != 5:
                raise ValueError("a window descriptor holds five regions")
            if g != rank and regions[0].device == self.recv.device.index and regions[0].pid != self.pid:
                raise ValueError("two ranks share one GPU: the exchange needs a GPU per rank")
            self._peer_regions.append(regions)
            ptrs = [self.region_ptr(r) for r in regions]
            flags.append(ptrs[0])
            counts.append(ptrs[1])
            recv.append(ptrs[2])
            back.append(ptrs[3])
            rows.append(ptrs[4])
        self.window = N.ep_window(world, rank, flags, counts, recv, back, rows)
        return self.window

    def close(self) -> None:
        self.window = None
        super().close()
