"""``python -m pcie_pool_b200.benchmarks.phase7_ingest_artifacts ...`` = ``phase7 ingest``
(see pcie_pool_b200.benchmarks.phase7)."""

import sys

from .phase7 import main

if __name__ == "__main__":
    raise SystemExit(main(["ingest", *sys.argv[1:]]))
