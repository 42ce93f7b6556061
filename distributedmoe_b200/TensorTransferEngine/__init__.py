"""Transfer engines: the reference's abstract interface and the NVLink / CUDA-IPC backend."""

from distributedmoe_b200.TensorTransferEngine.TensorTransferEngine import (  # noqa: F401
    TensorTransferEngine,
    TensorTransferEngineBackend,
    TensorTransferEngineConfig,
)
from distributedmoe_b200.TensorTransferEngine.utils import (  # noqa: F401
    HandshakeType,
    P2PPair,
    Transfer,
    TransferProtocol,
    TransferStatus,
    join_host_port,
)


def create_transfer_engine(backend, config):
    """Instantiate the engine of `backend`.  NIXL and MoonCake are not part of this build
    (their libraries are replaced by the NVLink backend)."""
    if backend == TensorTransferEngineBackend.NVLinkIPC:
        from distributedmoe_b200.TensorTransferEngine.NVLinkTensorTransferEngine import NVLinkTensorTransferEngine

        return NVLinkTensorTransferEngine(config)
    if backend == TensorTransferEngineBackend.NVLinkDirect:
        from distributedmoe_b200.TensorTransferEngine.NVLinkDirectTensorTransferEngine import (
            NVLinkDirectTensorTransferEngine,
        )

        return NVLinkDirectTensorTransferEngine(config)
    raise NotImplementedError(f"transfer backend {backend} is not available in this build; use NVLinkIPC "
                              "or NVLinkDirect")
