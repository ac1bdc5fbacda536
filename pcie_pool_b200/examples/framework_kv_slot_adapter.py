"""Entry point for framework integrations: a framework describes its KV
blocks as slots over one CPU backing and one GPU backing and drives
save/restore through ``FrameworkKVSlotAdapter`` (see
``pcie_pool_b200.inference``).  ``make_contiguous_slots`` builds a slot table
for a contiguous layout."""

from ..inference import (FrameworkKVSlot, FrameworkKVSlotAdapter, InferenceKVSlot,  # noqa: F401
                         InferenceKVSlotAdapter, make_contiguous_kv_slots)


def make_contiguous_slots(prefix: str, count: int, block_bytes: int) -> list[FrameworkKVSlot]:
    return make_contiguous_kv_slots(prefix, count, block_bytes)


if __name__ == "__main__":
    for s in make_contiguous_slots("demo", 4, 32 << 10):
        print(s)
