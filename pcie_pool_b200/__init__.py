"""pcie_pool_b200: PCIe bandwidth pooling across the GPUs of a B200 node.

A per-node daemon schedules idle GPUs as relays; every host<->device transfer
is split over the target's direct PCIe lane plus relay lanes whose staged
chunks a fused sm_100a landing kernel pulls over NVLink.  The public names
below match the reference client package (turbobus/__init__.py) so existing
applications switch by changing the import.
"""

from .api import DaemonIntentClient, TurboBusClient
from .client import CudaIpcDeviceBuffer, SharedPinnedCpuBuffer, SharedPinnedCpuBufferAllocator
from .schema import (BufferHandle, BufferKind, ExecutionTicket, JobIdentity, SchedulingDecision,
                     SchedulingDecisionState, TopologySnapshot, TransferIntent, TransferReceipt,
                     TransferStatusState, WorkloadKind)

__version__ = "0.1.0"

__all__ = ["BufferHandle", "BufferKind", "CudaIpcDeviceBuffer", "DaemonIntentClient", "ExecutionTicket",
           "JobIdentity", "SchedulingDecision", "SchedulingDecisionState", "SharedPinnedCpuBuffer",
           "SharedPinnedCpuBufferAllocator", "TopologySnapshot", "TransferIntent", "TransferReceipt",
           "TransferStatusState", "TurboBusClient", "WorkloadKind"]
