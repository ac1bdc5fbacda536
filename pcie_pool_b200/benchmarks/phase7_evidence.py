"""``python -m pcie_pool_b200.benchmarks.phase7_evidence ...`` = ``phase7 evidence``
(see pcie_pool_b200.benchmarks.phase7)."""

import sys

from .phase7 import main

if __name__ == "__main__":
    raise SystemExit(main(["evidence", *sys.argv[1:]]))
