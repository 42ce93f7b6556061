"""B200-native (sm_100a) MoE-layer hot path of DistributedMoE.

Subpackages mirror the reference's module layout:
  ``distributedmoe_b200.MoE``                   DistMoEBlock, DistExpertsBlock, pipeline tasks, pools
  ``distributedmoe_b200.TensorTransferEngine``  transfer-engine ABC and the NVLink/CUDA-IPC backend
The compute path is ``libdmoe_b200.so`` (C ABI in ``include/dmoe_b200.h``), reached through
``distributedmoe_b200._native``.
"""

__version__ = "0.1.0"
