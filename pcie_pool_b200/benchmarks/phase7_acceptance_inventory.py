"""``python -m pcie_pool_b200.benchmarks.phase7_acceptance_inventory ...`` = ``phase7 inventory``
(see pcie_pool_b200.benchmarks.phase7)."""

import sys

from .phase7 import main

if __name__ == "__main__":
    raise SystemExit(main(["inventory", *sys.argv[1:]]))
