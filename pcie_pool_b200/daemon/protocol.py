"""Names used on the daemon wire (contract objects + topology records)."""

from ..schema import (BufferRegistration, CleanupRequest, DaemonRequest, DaemonResponse, JobIdentity,
                      LeaseToken, PeerIdentity, RelayQuota, RequestType, Session, TransferReservation,
                      TransferStatus, TransferStatusState, WorkerBufferHandle, WorkerDataPlaneCompletion,
                      WorkerDataPlaneRequest, WorkerStagingBufferRequirement, WorkerTransferAuthorization,
                      WorkerTransferAuthorizationRequest)
from ..topology import DaemonResourceInventory, FabricLinkRecord, GpuInventoryRecord, PciePathRecord

__all__ = ["BufferRegistration", "CleanupRequest", "DaemonRequest", "DaemonResourceInventory", "DaemonResponse",
           "FabricLinkRecord", "GpuInventoryRecord", "JobIdentity", "LeaseToken", "PeerIdentity", "PciePathRecord",
           "RelayQuota", "RequestType", "Session", "TransferReservation", "TransferStatus", "TransferStatusState",
           "WorkerBufferHandle", "WorkerDataPlaneCompletion", "WorkerDataPlaneRequest",
           "WorkerStagingBufferRequirement", "WorkerTransferAuthorization", "WorkerTransferAuthorizationRequest"]
