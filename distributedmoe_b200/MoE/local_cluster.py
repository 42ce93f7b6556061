"""Start a host ``DistMoEBlock`` and its ``DistExpertsBlock``s inside one process.

This mirrors the reference test fixture (``MoE/tests/dist_moe_test.py:55-169``): every
expert block is a thread with its own event loop, transfer engine and ZeroMQ ports on
localhost; the host block is built last (its handshake waits for the blocks).  Blocks may
sit on any local GPUs (NVLink peers) or share the host's GPU.
"""

from __future__ import annotations

import os
import random
import socket
import threading
import time
from typing import List, Optional, Sequence, Tuple

import torch

from distributedmoe_b200.MoE.DistExpertsBlock import DistExpertsBlock
from distributedmoe_b200.MoE.DistMoEBlock import DistMoEBlock, DistMoEBlockConfig
from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import (
    TensorTransferEngineBackend,
    TensorTransferEngineConfig,
)
from distributedmoe_b200.TensorTransferEngine.utils import HandshakeType, TransferProtocol


def _ephemeral_range() -> Tuple[int, int]:
    try:
        with open("/proc/sys/net/ipv4/ip_local_port_range") as f:
            lo, hi = (int(v) for v in f.read().split()[:2])
        return lo, hi
    except (OSError, ValueError):
        return 32768, 60999


def free_ports(n: int) -> List[int]:
    """n distinct ports that are free now, to be bound as listeners soon after.  They are
    taken below the kernel's ephemeral range when it leaves room: a port from that range can
    be handed to an outgoing connection (the engines' own ZeroMQ connects, the process
    group's sockets) between this pick and the bind, and a listener that then fails to bind
    leaves its peers waiting for a hand-shake."""
    lo, _ = _ephemeral_range()
    base, top = 20000, min(lo, 32000)
    socks, ports = [], []
    try:
        if top - base >= 8 * n:
            rng = random.Random(os.getpid() ^ int(time.time_ns()))
            tried = 0
            while len(ports) < n and tried < 64 * n:
                tried += 1
                port = rng.randrange(base, top)
                if port in ports:
                    continue
                s = socket.socket()
                try:
                    s.bind(("127.0.0.1", port))
                except OSError:
                    s.close()
                    continue
                socks.append(s)
                ports.append(port)
        while len(ports) < n:  # no room below the ephemeral range: let the kernel choose
            s = socket.socket()
            s.bind(("127.0.0.1", 0))
            socks.append(s)
            ports.append(s.getsockname()[1])
    finally:
        for s in socks:
            s.close()
    return ports


class LocalCluster:
    """``with LocalCluster(...) as moe: y = moe(x)``.

    expert_layers: one list per block of modules with gate_proj/up_proj/down_proj, or
    ``stacked`` = one (gate, up, down) tuple per block of already stacked device tensors."""

    def __init__(self, number_of_experts: int, expert_blocks: List[List[int]], top_k: int, hidden_features: int,
                 dtype: torch.dtype, moe_device: torch.device, eb_devices: Sequence[torch.device],
                 expert_layers: Optional[List[list]] = None, stacked: Optional[list] = None,
                 io_buffer_size: int = 8192, number_of_io_buffers: int = 4, forward_timeout: int = 60000,
                 p2p_timeout_ms: int = 3000, backend: TensorTransferEngineBackend = TensorTransferEngineBackend.NVLinkIPC,
                 max_tokens: Optional[int] = None, cuda_graphs: bool = False, expert_precision: str = "model",
                 **options):
        """backend NVLinkDirect runs forward() as the device-driven exchange with world 1: every
        block must sit on the host's GPU; the blocks' stacks are concatenated (block order)
        into the one weight stack the grouped MLP reads; max_tokens (default io_buffer_size *
        number_of_io_buffers // top_k) sizes the receive window; cuda_graphs replays each
        token count's forward from a captured CUDA graph; expert_precision "fp8" runs the
        routed experts on 8-bit records (DistMoEBlock.setup_direct_plane)."""
        nb = len(expert_blocks)
        ports = free_ports(1 + 5 * nb)
        host_port, rest = ports[0], ports[1:]
        host_p2p = rest[0:nb]
        eb_ports = rest[nb:2 * nb]
        eb_p2p = rest[2 * nb:3 * nb]
        host_hc = rest[3 * nb:4 * nb]
        eb_hc = rest[4 * nb:5 * nb]
        direct = backend == TensorTransferEngineBackend.NVLinkDirect
        if direct and any(torch.device(d) != torch.device(moe_device) for d in eb_devices):
            raise ValueError("the single-process device-driven plane needs every block on the host's GPU")
        self.config = DistMoEBlockConfig(
            backend=backend, number_of_experts=number_of_experts,
            expert_blocks=expert_blocks, number_of_io_buffers=number_of_io_buffers, io_buffer_size=io_buffer_size,
            top_k=top_k, hidden_features=hidden_features, dtype=dtype, moe_device=torch.device(moe_device),
            eb_devices=[torch.device(d) for d in eb_devices], forward_timeout=forward_timeout,
            host_health_check_ports=host_hc, remote_health_check_ports=eb_hc, **options)
        self.threads: List[threading.Thread] = []
        self.expert_blocks_objs: List[Optional[DistExpertsBlock]] = [None] * nb
        self.errors: List[BaseException] = []
        for b in range(nb):
            eb_cfg = TensorTransferEngineConfig(
                host_address="127.0.0.1", host_port=eb_ports[b], host_p2p_ports=[eb_p2p[b]],
                remote_addresses=["127.0.0.1"], remote_ports=[host_port], remote_p2p_ports=[host_p2p[b]],
                p2p_timeout_duration=p2p_timeout_ms, handshake_type=HandshakeType.CLIENT,
                transfer_protocol=TransferProtocol.NVLINK, ib_device_names="")
            layers = expert_layers[b] if expert_layers is not None else []
            st = stacked[b] if stacked is not None else None

            def job(b=b, eb_cfg=eb_cfg, layers=layers, st=st):
                try:
                    torch.cuda.set_device(self.config.eb_devices[b])
                    blk = DistExpertsBlock(b, self.config, layers, eb_cfg, None, stacked_weights=st)
                    self.expert_blocks_objs[b] = blk
                    blk.main_loop()
                except BaseException as e:  # surfaced by close()
                    self.errors.append(e)

            t = threading.Thread(target=job, daemon=True, name=f"experts-block-{b}")
            t.start()
            self.threads.append(t)
        host_cfg = TensorTransferEngineConfig(
            host_address="127.0.0.1", host_port=host_port, host_p2p_ports=host_p2p,
            remote_addresses=["127.0.0.1"] * nb, remote_ports=eb_ports, remote_p2p_ports=eb_p2p,
            p2p_timeout_duration=p2p_timeout_ms, handshake_type=HandshakeType.SERVER,
            transfer_protocol=TransferProtocol.NVLINK, ib_device_names="")
        with torch.cuda.device(self.config.moe_device):
            self.moe = DistMoEBlock(self.config, host_cfg)
            if direct:
                if stacked is not None:
                    stacks = stacked
                else:
                    from distributedmoe_b200.MoE.DistExpertsBlock import stack_expert_weights
                    stacks = [stack_expert_weights(expert_layers[b], self.config.moe_device, dtype) for b in range(nb)]
                local = stacks[0] if nb == 1 else tuple(torch.cat([st[i] for st in stacks]).contiguous()
                                                        for i in range(3))
                mt = max_tokens if max_tokens is not None else max(1, io_buffer_size * number_of_io_buffers // top_k)
                self.moe.setup_direct_plane(1, 0, [0] * nb, local, mt * top_k, lambda mine: [mine], mt,
                                            cuda_graphs=cuda_graphs, expert_precision=expert_precision)

    def __enter__(self) -> DistMoEBlock:
        return self.moe

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        self.moe.close()
        for t in self.threads:
            t.join(timeout=15.0)
        if self.errors:
            raise RuntimeError(f"an expert block failed: {self.errors[0]!r}") from self.errors[0]
