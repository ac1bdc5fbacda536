"""Scheduling: turn session, bandwidth profile, quotas and load into plans."""

from ..schema import SchedulingDecision
from .daemon import DaemonScheduler, scheduling_decision_leases, scheduling_decision_stats
from .fairness import LoadView, charge_bytes, load_view

__all__ = ["DaemonScheduler", "LoadView", "SchedulingDecision", "charge_bytes", "load_view",
           "scheduling_decision_leases", "scheduling_decision_stats"]
