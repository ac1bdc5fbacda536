"""``python -m pcie_pool_b200.benchmarks.phase7_server_run ...`` = ``phase7 server-run``
(see pcie_pool_b200.benchmarks.phase7)."""

import sys

from .phase7 import main

if __name__ == "__main__":
    raise SystemExit(main(["server-run", *sys.argv[1:]]))
