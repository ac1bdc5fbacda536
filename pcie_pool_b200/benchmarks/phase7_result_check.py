"""``python -m pcie_pool_b200.benchmarks.phase7_result_check ...`` = ``phase7 check``
(see pcie_pool_b200.benchmarks.phase7)."""

import sys

from .phase7 import main

if __name__ == "__main__":
    raise SystemExit(main(["check", *sys.argv[1:]]))
