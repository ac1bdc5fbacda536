"""``python -m pcie_pool_b200.daemon``: start the node daemon (or print its
state when no socket path is given)."""

from __future__ import annotations

import argparse
import json
import sys

from .startup import DaemonStartupConfig, DaemonStartupError, create_production_daemon


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="pcie_pool_b200 node daemon")
    p.add_argument("--topology-provider", default="cuda-nvml")
    p.add_argument("--target-gpu", type=int, required=True)
    p.add_argument("--min-relays", type=int, default=1)
    p.add_argument("--allow-missing-fabric", action="store_true",
                   help="start even when no GPU fabric links are reported")
    p.add_argument("--allow-missing-pcie", action="store_true",
                   help="start even when no PCIe paths are reported")
    p.add_argument("--max-sessions-per-relay", type=int, default=1)
    p.add_argument("--max-inflight-chunks-per-relay", type=int, default=8)
    p.add_argument("--session-timeout-seconds", type=float, default=0.0)
    p.add_argument("--profile-max-age-seconds", type=float, default=0.0)
    p.add_argument("--execute", action="store_true",
                   help="run admitted intents on this node's GPUs (data plane in the daemon)")
    p.add_argument("--profile-on-start", action="store_true",
                   help="measure link bandwidth at startup and cache the profiles")
    p.add_argument("--profile-store", default=None, help="persist the profile cache in this JSON file")
    p.add_argument("--gpus", default=None,
                   help="comma-separated GPU indices the daemon may use (default: every GPU of the node)")
    p.add_argument("--executor-workers", type=int, default=4,
                   help="intents executed at once (a session's next intent queues behind its current one)")
    p.add_argument("--socket-path", default=None,
                   help="serve on this Unix socket instead of printing the daemon state")
    return p


def startup_config_from_args(args) -> DaemonStartupConfig:
    return DaemonStartupConfig(
        topology_provider=args.topology_provider, target_gpu=args.target_gpu,
        min_relay_count=args.min_relays, require_fabric=not args.allow_missing_fabric,
        require_pcie=not args.allow_missing_pcie, max_sessions_per_relay=args.max_sessions_per_relay,
        max_inflight_chunks_per_relay=args.max_inflight_chunks_per_relay,
        session_timeout_seconds=args.session_timeout_seconds,
        profile_max_age_seconds=args.profile_max_age_seconds, execute=args.execute,
        profile_on_start=args.profile_on_start, profile_store_path=args.profile_store,
        devices=None if not args.gpus else tuple(int(x) for x in str(args.gpus).split(",") if x.strip()),
        executor_workers=args.executor_workers)


def main(argv=None) -> None:
    from ..utils.log import configure_from_env

    configure_from_env()
    parser = build_parser()
    args = parser.parse_args(argv)
    try:
        daemon = create_production_daemon(startup_config_from_args(args))
    except DaemonStartupError as exc:
        parser.exit(2, f"pcie_pool_b200 daemon startup failed: {exc}\n")
    if args.socket_path:
        daemon.serve_forever(args.socket_path)
        return
    json.dump(daemon.describe().payload, sys.stdout, indent=2, default=str)
    print()


if __name__ == "__main__":
    main()
