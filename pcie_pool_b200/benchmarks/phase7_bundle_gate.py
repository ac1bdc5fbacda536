"""``python -m pcie_pool_b200.benchmarks.phase7_bundle_gate ...`` = ``phase7 gate``
(see pcie_pool_b200.benchmarks.phase7)."""

import sys

from .phase7 import main

if __name__ == "__main__":
    raise SystemExit(main(["gate", *sys.argv[1:]]))
