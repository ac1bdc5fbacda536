"""Worker helper: the process that executes daemon-authorized transfers on
client-shared buffers (public names as turbobus/worker/__init__.py)."""

from .codec import (WorkerMessageCodecError, decode_worker_request_envelope, decode_worker_response_envelope,
                    encode_worker_request_envelope, encode_worker_response_envelope, handle_worker_service_message)
from .cuda_executor import CudaWorkerExecutor
from .endpoint import WorkerServiceEndpoint
from .helper import (WorkerAuthorizationError, WorkerCleanupError, WorkerDataPlaneCompletion,
                     WorkerDataPlaneCompletionEnvelope, WorkerDataPlaneRequest, WorkerServiceRequestEnvelope,
                     WorkerServiceResponseEnvelope, WorkerStatusReportError, WorkerTransferAuthorizer,
                     WorkerTransferCleanupCoordinator, WorkerTransferClient, WorkerTransferLifecycleRecord,
                     WorkerTransferRequest, WorkerTransferResult, WorkerTransferService, WorkerTransferState,
                     WorkerTransferStatusReporter, parse_worker_authorization_request_payload)
from .process import build_worker_helper_transport, run_worker_helper_process
from .process import main as worker_process_main
from .resources import (WorkerDataPlaneResourceBinder, WorkerDataPlaneResourceBinding, WorkerDataPlaneResourceError,
                        WorkerDataPlaneResources)
from .socket_client import WorkerServiceSocketClient
from .staging_pool import WorkerStagingPool, WorkerStagingPoolError, WorkerStagingSlot
from .transport import WorkerServiceUnixSocketTransport

__all__ = [
    "CudaWorkerExecutor", "WorkerAuthorizationError", "WorkerCleanupError", "WorkerDataPlaneCompletion",
    "WorkerDataPlaneCompletionEnvelope", "WorkerDataPlaneRequest", "WorkerDataPlaneResourceBinder",
    "WorkerDataPlaneResourceBinding", "WorkerDataPlaneResourceError", "WorkerDataPlaneResources",
    "WorkerMessageCodecError", "WorkerServiceEndpoint", "WorkerServiceRequestEnvelope",
    "WorkerServiceResponseEnvelope", "WorkerServiceSocketClient", "WorkerServiceUnixSocketTransport",
    "WorkerStagingPool", "WorkerStagingPoolError", "WorkerStagingSlot", "WorkerStatusReportError",
    "WorkerTransferAuthorizer", "WorkerTransferCleanupCoordinator", "WorkerTransferClient",
    "WorkerTransferLifecycleRecord", "WorkerTransferRequest", "WorkerTransferResult", "WorkerTransferService",
    "WorkerTransferState", "WorkerTransferStatusReporter", "build_worker_helper_transport",
    "decode_worker_request_envelope", "decode_worker_response_envelope", "encode_worker_request_envelope",
    "encode_worker_response_envelope", "handle_worker_service_message", "parse_worker_authorization_request_payload",
    "run_worker_helper_process", "worker_process_main",
]
