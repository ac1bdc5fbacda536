"""Worker wire codec: one JSON object per message, keys sorted, compact
separators, newline-terminated on the socket.  The byte format matches
turbobus/worker/codec.py:74-78 so either side can talk to the other."""

from __future__ import annotations

import json
from collections.abc import Mapping

from .helper import WorkerServiceRequestEnvelope, WorkerServiceResponseEnvelope


class WorkerMessageCodecError(ValueError):
    pass


def _dump(obj: Mapping[str, object]) -> str:
    try:
        return json.dumps(dict(obj), sort_keys=True, separators=(",", ":"))
    except (TypeError, ValueError) as exc:
        raise WorkerMessageCodecError(str(exc)) from exc


def _load(message: str | bytes) -> Mapping[str, object]:
    if isinstance(message, (bytes, bytearray)):
        message = bytes(message).decode("utf-8")
    if not isinstance(message, str):
        raise TypeError("message must be str or bytes")
    try:
        obj = json.loads(message)
    except json.JSONDecodeError as exc:
        raise WorkerMessageCodecError(str(exc)) from exc
    if not isinstance(obj, Mapping):
        raise WorkerMessageCodecError("worker message must decode to a mapping")
    return obj


def _mapping(obj: Mapping[str, object], name: str, required: bool) -> Mapping[str, object] | None:
    v = obj.get(name)
    if v is None and not required:
        return None
    if not isinstance(v, Mapping):
        raise WorkerMessageCodecError(f"{name} must be a mapping")
    return v


def encode_worker_request_envelope(envelope: WorkerServiceRequestEnvelope) -> str:
    if not isinstance(envelope, WorkerServiceRequestEnvelope):
        raise TypeError("envelope must be a WorkerServiceRequestEnvelope")
    return _dump(envelope.as_dict())


def decode_worker_request_envelope(message: str | bytes) -> WorkerServiceRequestEnvelope:
    obj = _load(message)
    try:
        return WorkerServiceRequestEnvelope(payload=_mapping(obj, "payload", True),
                                            cleanup_target_kind=str(obj.get("cleanup_target_kind", "reservation")))
    except (TypeError, ValueError) as exc:
        raise WorkerMessageCodecError(str(exc)) from exc


def encode_worker_response_envelope(envelope: WorkerServiceResponseEnvelope) -> str:
    if not isinstance(envelope, WorkerServiceResponseEnvelope):
        raise TypeError("envelope must be a WorkerServiceResponseEnvelope")
    return _dump(envelope.as_dict())


def decode_worker_response_envelope(message: str | bytes) -> WorkerServiceResponseEnvelope:
    obj = _load(message)
    try:
        return WorkerServiceResponseEnvelope(ok=bool(obj["ok"]), completion=_mapping(obj, "completion", False),
                                             error=obj.get("error"), final_state=obj.get("final_state"))
    except (KeyError, TypeError, ValueError) as exc:
        raise WorkerMessageCodecError(str(exc)) from exc


def handle_worker_service_message(service, message: str | bytes) -> str:
    try:
        req = decode_worker_request_envelope(message)
    except WorkerMessageCodecError as exc:
        return encode_worker_response_envelope(WorkerServiceResponseEnvelope.from_error(str(exc)))
    return encode_worker_response_envelope(service.handle_envelope(req))


__all__ = ["WorkerMessageCodecError", "decode_worker_request_envelope", "decode_worker_response_envelope",
           "encode_worker_request_envelope", "encode_worker_response_envelope", "handle_worker_service_message"]
