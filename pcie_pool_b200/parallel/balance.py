"""Adaptive lane weights.

Lanes that share host resources (memory controllers, the socket link, a
PCIe switch) do not deliver their solo bandwidth when all run together.  On
the 8xB200 nodes of this pool, for example, GPUs 4-7 sustain ~23 GB/s each
while GPUs 0-3 sustain ~36 GB/s once all eight pull from host memory at once.
A split proportional to solo bandwidth therefore finishes when the slow lanes
do.  ``LaneBalancer`` keeps an exponentially weighted estimate of each lane's
rate *under the concurrency it actually ran with* (bytes / lane time of every
completed transfer) and the planner splits the next transfer in proportion
to it, which converges to all lanes finishing together.  This implements the
reference's declared but unused ``enable_dynamic_weights`` /
``dynamic_weight_alpha`` options (cpp/include/turbobus/types.h:115-116).
"""

from __future__ import annotations

import threading
from typing import Sequence


class LaneBalancer:
    def __init__(self, alpha: float = 0.5) -> None:
        if not 0.0 < alpha <= 1.0:
            raise ValueError("alpha must be in (0, 1]")
        self.alpha = float(alpha)
        self._rates: dict[tuple[int, str], dict[int, float]] = {}
        self._lock = threading.Lock()

    def observe(self, target: int, direction: str, result) -> None:
        """Fold one completed transfer's per-lane rates into the estimates."""
        key = (int(target), str(direction))
        with self._lock:
            est = self._rates.setdefault(key, {})
            for lane in getattr(result, "lanes", []):
                if lane.cuda_ms <= 0 or lane.bytes <= 0:
                    continue
                rate = (lane.bytes / float(1 << 30)) / (lane.cuda_ms / 1e3)
                prev = est.get(lane.device)
                est[lane.device] = rate if prev is None else (1 - self.alpha) * prev + self.alpha * rate

    def observe_rates(self, target: int, direction: str, rates: dict[int, float]) -> None:
        """Fold measured per-lane rates (GiB/s by device) into the estimates."""
        key = (int(target), str(direction))
        with self._lock:
            est = self._rates.setdefault(key, {})
            for dev, rate in rates.items():
                if rate > 0.0:
                    prev = est.get(int(dev))
                    est[int(dev)] = rate if prev is None else (1 - self.alpha) * prev + self.alpha * rate

    def seed(self, target: int, direction: str, rates: dict[int, float]) -> None:
        with self._lock:
            self._rates[(int(target), str(direction))] = {int(k): float(v) for k, v in rates.items()}

    def rates(self, target: int, direction: str) -> dict[int, float]:
        with self._lock:
            return dict(self._rates.get((int(target), str(direction)), {}))

    def weights(self, target: int, direction: str, devices: Sequence[int]) -> list[float] | None:
        """Per-device rate estimates in ``devices`` order, or None until every
        device has been observed."""
        r = self.rates(target, direction)
        if not all(int(d) in r for d in devices):
            return None
        return [max(r[int(d)], 1e-6) for d in devices]
