"""AdamW whose fp32 state lives in host memory and streams through the GPU.

Training offload keeps the fp32 master weights and both Adam moments on the
host: 12 bytes per parameter, six times the bf16 parameters themselves.
``StreamedAdamW.step`` runs the whole optimizer step as ONE pooled round
trip: chunks of the host state go host -> staging slot over the direct PCIe
lane and the relay lanes, the landing kernel on the training GPU applies
AdamW to each 24 KiB state tile with the local bf16 gradients (written by
backward) and writes the new bf16 parameters in place, and the updated tile
returns slot -> host on the same lane's device-to-host copy engine while the
next chunk streams in (``PoolEngine`` op ``OP_ADAMW``).  No fp32 copy of the
state is ever resident on the GPU, no separate optimizer kernel runs, and
the CPU does no arithmetic.

The reference moves only gradient and parameter buckets
(turbobus/adapters/training_offload.py:15-131,
benchmarks/training_offload.py:167-201); its optimizer step is the
application's.

Host layout: tile t holds parameters [2048 t, 2048 t + 2048) as
``[master | exp_avg | exp_avg_sq]`` fp32 (the last tile zero-padded).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

TILE_PARAMS = 2048
TILE_BYTES = 3 * 4 * TILE_PARAMS


@dataclass
class StepStats:
    step: int
    bytes: int          # state bytes streamed each way
    cuda_ms: float
    lanes: list

    @property
    def gb_per_s(self) -> float:
        """State bytes per second in each direction."""
        return self.bytes / 1e9 / (self.cuda_ms / 1e3) if self.cuda_ms > 0 else 0.0


class StreamedAdamW:
    """AdamW over a flat bf16 CUDA parameter vector with host-resident fp32
    state.  Drive it with a ``PoolEngine`` (``engine=``, lanes = the target
    plus ``relays``) or through the node daemon (``client=`` and
    ``daemon_client=`` with a session and job), where each step is one intent
    whose relays come from the daemon's leases."""

    def __init__(self, params, *, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, engine=None, relays: Sequence[int] = (),
                 chunk_bytes: int = 16 << 20, client=None, daemon_client=None, session_id: str | None = None,
                 job_id: str | None = None, prefix: str = "adamw", host_state=None) -> None:
        import torch

        if (engine is None) == (client is None):
            raise ValueError("give exactly one of engine= or client=")
        if params.dtype != torch.bfloat16 or not params.is_contiguous() or (engine is not None and not params.is_cuda):
            raise ValueError("params must be a contiguous bf16 CUDA tensor")
        self.params = params.view(-1)
        self.nparams = self.params.numel()
        self.target = int(params.device.index or 0)
        self.relays = [int(r) for r in relays if int(r) != self.target]
        self.lr, self.betas, self.eps, self.weight_decay = float(lr), tuple(betas), float(eps), float(weight_decay)
        self.tiles = -(-self.nparams // TILE_PARAMS)
        self.tiles_per_chunk = max(1, int(chunk_bytes) // TILE_BYTES)
        self.engine = engine
        self.client, self.dc = client, daemon_client
        self.session_id, self.job_id, self.prefix = session_id, job_id, prefix
        self.t = 0
        if host_state is None:
            host_state = torch.zeros(self.tiles * TILE_BYTES, dtype=torch.uint8,
                                     pin_memory=torch.cuda.is_available())
        if host_state.numel() * host_state.element_size() < self.tiles * TILE_BYTES:
            raise ValueError("host state is smaller than the tiled optimizer state")
        self.host = host_state
        st = self._tiled()
        st.zero_()
        flat = torch.zeros(self.tiles * TILE_PARAMS, dtype=torch.float32)
        flat[:self.nparams] = self.params.float().cpu()
        st[:, 0, :] = flat.view(self.tiles, TILE_PARAMS)
        self._ids = None

    # ---- state views ----------------------------------------------------------------
    def _tiled(self):
        import torch

        return self.host.view(torch.uint8)[:self.tiles * TILE_BYTES].view(torch.float32).view(self.tiles, 3,
                                                                                              TILE_PARAMS)

    def state(self) -> dict:
        """fp32 master / exp_avg / exp_avg_sq as flat host tensors (copies)."""
        st = self._tiled()
        return {k: st[:, i, :].reshape(-1)[:self.nparams].clone()
                for i, k in enumerate(("master", "exp_avg", "exp_avg_sq"))}

    def hyper(self) -> dict:
        return {"lr": self.lr, "beta1": self.betas[0], "beta2": self.betas[1], "eps": self.eps,
                "weight_decay": self.weight_decay, "grad_scale": 1.0, "step": self.t}

    # ---- the step ---------------------------------------------------------------------
    def lanes(self):
        """Contiguous tile spans per lane (direct first), chunked."""
        from ..parallel.engine import Lane

        devs = [self.target, *self.relays]
        per = -(-self.tiles // len(devs))
        out = []
        for i, dev in enumerate(devs):
            t0, t1 = i * per, min(self.tiles, (i + 1) * per)
            if t0 >= t1:
                continue
            starts = np.arange(t0, t1, self.tiles_per_chunk, dtype=np.uint64)
            ntiles = np.minimum(self.tiles_per_chunk, t1 - starts).astype(np.uint64)
            off = starts * np.uint64(TILE_BYTES)
            out.append(Lane(dev, off.copy(), off.copy(), ntiles * np.uint64(TILE_BYTES),
                            unit0=starts.astype(np.uint32)))
        return out

    def step(self, grads) -> StepStats:
        """One AdamW step with ``grads`` (bf16, same shape as the params)."""
        import torch

        g = grads.view(-1)
        if g.dtype != torch.bfloat16 or g.numel() != self.nparams or g.device != self.params.device:
            raise ValueError("grads must be bf16 on the params' device with one value per parameter")
        if not g.is_contiguous():
            raise ValueError("grads must be contiguous")
        self.t += 1
        if g.is_cuda:
            # the engine's streams do not wait for the caller's stream (backward)
            torch.cuda.current_stream(self.params.device).synchronize()
        if self.engine is not None:
            return self._step_engine(g)
        return self._step_daemon(g)

    def _step_engine(self, g) -> StepStats:
        from .._native import native
        from ..parallel.engine import H2D

        C = native()
        adam = {**self.hyper(), "grads": g.data_ptr(), "params": self.params.data_ptr(), "nparams": self.nparams}
        host_bytes = self.tiles * TILE_BYTES
        r = self.engine.run(H2D, self.target, self.host.data_ptr(), host_bytes, self.params.data_ptr(),
                            self.nparams * 2, self.lanes(), op=C.OP_ADAMW, adam=adam)
        if not r.ok:
            raise RuntimeError(f"streamed AdamW step {self.t} failed: {r.error} (the host state of the lanes "
                               "after the failure point is undefined; restore it from a checkpoint)")
        return StepStats(self.t, host_bytes, r.cuda_ms, [(l.device, l.bytes, round(l.cuda_ms, 3)) for l in r.lanes])

    def _register(self, g) -> tuple[str, str, str]:
        from ..daemon.client import InProcessDaemonClient

        ids = (f"{self.prefix}-state", f"{self.prefix}-params", f"{self.prefix}-grads")
        if self._ids is None:
            if not isinstance(self.dc, InProcessDaemonClient):
                raise ValueError("the streamed optimizer through a daemon process needs shared buffers; "
                                 "use an in-process daemon or the engine")
            host_bytes = self.tiles * TILE_BYTES
            for bid, kind, size, addr, dev in ((ids[0], "cpu_pinned", host_bytes, self.host.data_ptr(), None),
                                               (ids[1], "gpu", self.nparams * 2, self.params.data_ptr(), self.target),
                                               (ids[2], "gpu", self.nparams * 2, g.data_ptr(), self.target)):
                r = self.dc.register_buffer(bid, self.job_id, kind, size, device_index=dev, address=addr,
                                            pinned=kind == "cpu_pinned")
                if not r.ok:
                    raise RuntimeError(r.error)
            self._ids = ids
            self._grads_ptr = g.data_ptr()
        elif g.data_ptr() != self._grads_ptr:
            raise ValueError("daemon steps reuse the gradient buffer registered by the first step")
        return self._ids

    def _step_daemon(self, g) -> StepStats:
        from .. import TransferIntent, TransferStatusState
        from ..schema import WorkloadKind

        sid, pid, gid = self._register(g)
        n = self.tiles * TILE_BYTES
        landing = {"op": "adamw", "adam": {**self.hyper(), "grads_buffer": gid, "nparams": self.nparams}}
        it = TransferIntent(f"{self.prefix}-step{self.t}", self.job_id, self.session_id, sid, pid, "h2d", n,
                            ({"src_offset": 0, "dst_offset": 0, "bytes": n},), workload_kind=WorkloadKind.OPTIMIZER_STATE,
                            metadata={"chunk_bytes": self.tiles_per_chunk * TILE_BYTES, "landing": landing})
        r = self.client.transfer(it, timeout_seconds=600)
        if r.state is not TransferStatusState.COMPLETE:
            raise RuntimeError(f"streamed AdamW step {self.t} failed: {r.error}")
        meas = (r.metadata or {}).get("measured", {}) or {}
        return StepStats(self.t, n, float(meas.get("cuda_ms", 0.0) or 0.0),
                         [(p.get("relay_device"), p.get("bytes"), round(float(p.get("cuda_ms", 0.0)), 3))
                          for p in (r.path_stats or ())])


__all__ = ["StepStats", "StreamedAdamW", "TILE_BYTES", "TILE_PARAMS"]
