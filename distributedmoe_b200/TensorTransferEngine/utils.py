"""Transfer-engine value types, kept identical in meaning to the reference
(``TensorTransferEngine/utils.py:12-66``) so callers keep working: protocol and handshake
enums, the transfer record, the ZeroMQ socket pair and the name helpers."""

from __future__ import annotations

import uuid
from dataclasses import dataclass
from enum import Enum
from typing import Any

import zmq.asyncio


class TransferProtocol(Enum):
    RDMA = "rdma"
    NVLINK = "nvlink"


class HandshakeType(Enum):
    NONE = 0
    SERVER = 1
    CLIENT = 2


class TransferStatus(Enum):
    CREATED = 0
    FINISHED = 1
    RELEASED = 2


@dataclass
class Transfer:
    name: bytes
    status: TransferStatus
    remote_name: str
    handler: Any      # backend handle (a CUDA event for the NVLink backend)
    size: int         # bytes
    duration: float   # ms (start timestamp while in flight)


@dataclass
class P2PPair:
    pusher: zmq.asyncio.Socket
    puller: zmq.asyncio.Socket


def join_host_port(host: str, port: int, scheme: str = "", dir: str = "") -> str:
    if scheme:
        return f"{scheme}://{host}:{port}/{dir}" if dir else f"{scheme}://{host}:{port}"
    return f"{host}:{port}"


def _next_random_name() -> bytes:
    """8 random bytes naming a task or transfer (``utils.py:432-436``)."""
    return uuid.uuid4().bytes[-8:]
