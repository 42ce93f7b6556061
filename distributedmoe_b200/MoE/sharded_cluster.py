"""Expert-parallel MoE layer over the GPUs of one node, one process per GPU.

Every rank g owns the experts ``[g*E/G, (g+1)*E/G)`` (its stacked weights) and runs:

* one host ``DistMoEBlock`` for its own tokens, whose ``expert_blocks`` list has one block
  per rank (block b = the experts of rank b), and
* G ``DistExpertsBlock`` threads, block g of every rank's host, all sharing this rank's
  weights.

So there are G x G expert-block objects in total, and no single host GPU funnels all
traffic (a star with one host would be bound by that GPU's NVLink egress).

Two data planes:

* ``NVLinkDirect`` (default): every rank's forward is device-driven.  The hosts exchange
  per-expert row counts, their gather kernels store rows straight into the owning GPU's
  receive window over NVLink (each expert's rows from all hosts contiguous), each GPU runs
  ONE grouped MLP over everything it received, and each host's combine reads its results
  back through peer pointers; epoch flags order the steps.  The expert blocks keep answering
  health checks; no per-task message is sent.  Every rank must call forward once per step.
* ``NVLinkIPC``: the reference's task protocol, metadata over ZeroMQ between processes and
  activations copied over NVLink between CUDA-IPC buffers (completion notices order the
  accesses); one grouped MLP per host task.

``torch.distributed`` (any backend) is used at set-up only: to exchange the engines' ports
and window descriptors, plus barriers at set-up and shut-down; the data path has no
collective.
"""

from __future__ import annotations

import threading
from typing import List, Optional

import torch
import torch.distributed as dist

from distributedmoe_b200 import _native as N
from distributedmoe_b200.MoE.DistExpertsBlock import DistExpertsBlock
from distributedmoe_b200.MoE.DistMoEBlock import DistMoEBlock, DistMoEBlockConfig
from distributedmoe_b200.MoE.local_cluster import free_ports
from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import (
    TensorTransferEngineBackend,
    TensorTransferEngineConfig,
)
from distributedmoe_b200.TensorTransferEngine.utils import HandshakeType, TransferProtocol
from distributedmoe_b200.utils.logging_config import get_logger


def _ports_collide(table: List[dict]) -> bool:
    seen = set()
    for row in table:
        ports = [row["host_port"], *row["host_p2p"], *row["host_hc"], *row["eb_port"], *row["eb_p2p"], *row["eb_hc"]]
        for port in ports:
            if (row["address"], port) in seen:
                return True
            seen.add((row["address"], port))
    return False


def exchange_engine_ports(address: str, device_index: int, group: Optional[dist.ProcessGroup] = None) -> List[dict]:
    """Pick this rank's engine ports (1 host port, then G each of host P2P, host health-check,
    block port, block P2P, block health-check) and gather every rank's choice; all ranks get
    the same table.  The first collective sets up the process group's own sockets (NCCL binds
    its listeners lazily), so it runs before any port is picked; a table with a port used
    twice on one address is picked again."""
    G = dist.get_world_size(group)
    dist.barrier(group=group)
    for _attempt in range(5):
        p = free_ports(1 + 5 * G)
        mine = {"host_port": p[0], "host_p2p": p[1:1 + G], "host_hc": p[1 + G:1 + 2 * G],
                "eb_port": p[1 + 2 * G:1 + 3 * G], "eb_p2p": p[1 + 3 * G:1 + 4 * G],
                "eb_hc": p[1 + 4 * G:1 + 5 * G], "address": address, "device": device_index}
        table: List[dict] = [None] * G  # type: ignore[list-item]
        dist.all_gather_object(table, mine, group=group)
        if not _ports_collide(table):  # every rank sees the same table and decides alike
            return table
    raise RuntimeError("could not pick distinct engine ports on all ranks")


def gather_window_descriptors(mine: bytes, group: Optional[dist.ProcessGroup] = None) -> List[bytes]:
    """Every rank's NVLinkDirect window descriptor, in rank order (one all-gather at set-up)."""
    out: List[bytes] = [b""] * dist.get_world_size(group)
    dist.all_gather_object(out, mine, group=group)
    return out


def experts_of_rank(number_of_experts: int, world: int, rank: int) -> List[int]:
    per = number_of_experts // world
    return list(range(rank * per, (rank + 1) * per))


class ShardedCluster:
    """``with ShardedCluster(...) as moe: y = moe(x_local)`` on every rank.

    stacked: this rank's (gate [E_g, I, d], up [E_g, I, d], down [E_g, d, I]) on its GPU.
    gemm_sm_reserve: SMs the grouped-MLP launches of this process leave free (process-wide)."""

    def __init__(self, number_of_experts: int, top_k: int, hidden_features: int, dtype: torch.dtype,
                 device: torch.device, stacked, group: Optional[dist.ProcessGroup] = None,
                 io_buffer_size: Optional[int] = None, number_of_io_buffers: Optional[int] = None,
                 forward_timeout: int = 60000, p2p_timeout_ms: int = 3000, address: str = "127.0.0.1",
                 gemm_sm_reserve: Optional[int] = None,
                 backend: TensorTransferEngineBackend = TensorTransferEngineBackend.NVLinkDirect,
                 max_tokens: int = 8192, blocks: Optional[List[List[int]]] = None, cuda_graphs: bool = False,
                 expert_precision: str = "model", **options):
        """stacked: this rank's weight stack for the experts of its block, in block order.
        blocks[g]: the experts of rank g's block (default: the contiguous E/G of rank g); an
        expert listed by two ranks is replicated.  max_tokens: tokens per forward of one host
        (sizes the NVLinkDirect receive windows: G * max_tokens * top_k rows per GPU).
        cuda_graphs: replay each token count's forward from a captured CUDA graph (every rank
        captures at the same step; capturing runs no kernel, so the ranks stay in step).
        expert_precision: "fp8" sends 8-bit records and runs the gate/up GEMM on e4m3 tensor
        cores (DistMoEBlock.setup_direct_plane)."""
        direct = backend == TensorTransferEngineBackend.NVLinkDirect
        if direct:
            # The task buffers only serve the metadata hand-shake: keep them small.
            io_buffer_size = io_buffer_size or 256
            number_of_io_buffers = number_of_io_buffers or 1
            gemm_sm_reserve = 0 if gemm_sm_reserve is None else gemm_sm_reserve
        else:
            io_buffer_size = io_buffer_size or 8192
            number_of_io_buffers = number_of_io_buffers or 2
            options.setdefault("dispatch_all_blocks", True)  # one task per GPU's block at once
            # Each GPU computes other hosts' experts while its own host gathers and combines:
            # keep a few SMs out of the persistent grouped-MLP launches for those short kernels.
            gemm_sm_reserve = 8 if gemm_sm_reserve is None else gemm_sm_reserve
        N.set_gemm_sm_reserve(gemm_sm_reserve)
        G = dist.get_world_size(group)
        r = dist.get_rank(group)
        if blocks is None:
            if number_of_experts % G:
                raise ValueError("number_of_experts must divide evenly over the ranks")
            blocks = [experts_of_rank(number_of_experts, G, g) for g in range(G)]
        if len(blocks) != G:
            raise ValueError("one expert block per rank")
        self.group = group
        self.rank, self.world = r, G
        device = torch.device(device)
        table = exchange_engine_ports(address, device.index, group)
        mine = table[r]
        eb_devices = [torch.device("cuda", table[g]["device"]) for g in range(G)]
        if direct and len({(row["address"], row["device"]) for row in table}) != G:
            raise ValueError("the device-driven exchange needs one GPU per rank")

        def config_of_host(h: int) -> DistMoEBlockConfig:
            # host h's view: block g lives on rank g and uses the ports rank g opened for host h
            return DistMoEBlockConfig(
                backend=backend, number_of_experts=number_of_experts,
                expert_blocks=blocks, number_of_io_buffers=number_of_io_buffers, io_buffer_size=io_buffer_size,
                top_k=top_k, hidden_features=hidden_features, dtype=dtype, moe_device=eb_devices[h],
                eb_devices=eb_devices, forward_timeout=forward_timeout,
                host_health_check_ports=list(table[h]["host_hc"]),
                remote_health_check_ports=[table[g]["eb_hc"][h] for g in range(G)], **options)

        self.logger = get_logger("dist_moe.sharded_cluster")
        self.errors: List[BaseException] = []
        self.threads: List[threading.Thread] = []
        for h in range(G):
            cfg = config_of_host(h)
            eb_tte = TensorTransferEngineConfig(
                host_address=address, host_port=mine["eb_port"][h], host_p2p_ports=[mine["eb_p2p"][h]],
                remote_addresses=[table[h]["address"]], remote_ports=[table[h]["host_port"]],
                remote_p2p_ports=[table[h]["host_p2p"][r]], p2p_timeout_duration=p2p_timeout_ms,
                handshake_type=HandshakeType.CLIENT, transfer_protocol=TransferProtocol.NVLINK, ib_device_names="")

            def job(cfg=cfg, eb_tte=eb_tte, h=h):
                try:
                    torch.cuda.set_device(device)
                    blk = DistExpertsBlock(r, cfg, [], eb_tte, None, stacked_weights=stacked)
                    blk.main_loop()
                except BaseException as e:  # logged now (a host may be waiting for it), raised by close()
                    self.logger.error(f"expert block {r} for host {h} failed: {e!r}")
                    self.errors.append(e)

            t = threading.Thread(target=job, daemon=True, name=f"experts-block-{r}-for-host-{h}")
            t.start()
            self.threads.append(t)

        host_tte = TensorTransferEngineConfig(
            host_address=address, host_port=mine["host_port"], host_p2p_ports=list(mine["host_p2p"]),
            remote_addresses=[table[g]["address"] for g in range(G)],
            remote_ports=[table[g]["eb_port"][r] for g in range(G)],
            remote_p2p_ports=[table[g]["eb_p2p"][r] for g in range(G)], p2p_timeout_duration=p2p_timeout_ms,
            handshake_type=HandshakeType.SERVER, transfer_protocol=TransferProtocol.NVLINK, ib_device_names="")
        with torch.cuda.device(device):
            self.moe = DistMoEBlock(config_of_host(r), host_tte)
            # Load the grouped-MLP kernels once here rather than inside a block's first task,
            # where the first launches would delay its health-check replies.
            g, u, dn = stacked
            rows = torch.zeros(256, hidden_features, dtype=dtype, device=device)
            N.grouped_gated_mlp(rows, g, u, dn, [0], [256], N.ACT_SILU, torch.empty_like(rows))
            torch.cuda.synchronize(device)
            if direct:
                self.moe.setup_direct_plane(G, r, list(range(G)), stacked, G * max_tokens * top_k,
                                            lambda mine: gather_window_descriptors(mine, group), max_tokens,
                                            cuda_graphs=cuda_graphs, expert_precision=expert_precision)
        self.direct = direct
        self.device = device
        dist.barrier(group=group)  # every host and block of every rank is up before the first forward

    def __enter__(self) -> DistMoEBlock:
        return self.moe

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        # With the device-driven plane a peer's combine may still read this rank's window:
        # every rank's GPU work ends before any rank releases its window.
        if self.direct:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        # Stop this rank's host (which stops its G blocks on all ranks), then wait until every
        # host has done the same before joining this rank's blocks.
        self.moe.close()
        dist.barrier(group=self.group)
        for t in self.threads:
            t.join(timeout=30.0)
        if self.errors:
            raise RuntimeError(f"an expert block failed: {self.errors[0]!r}") from self.errors[0]
