"""The footprint chunk planner against plans made by the reference's own
planner (tests/golden/make_planner_golden.py)."""

import json
from pathlib import Path

import pytest

from gofish_b200.footprint_chunk_planner import plan_footprint_chunks

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "planner_golden.json").read_text())


@pytest.mark.parametrize("entry", GOLDEN, ids=[str(i) for i in range(len(GOLDEN))])
def test_plan_matches_reference(entry):
    count, free, total, reserved, allocated = entry["case"]
    kwargs = dict(driver_free_bytes=free, device_total_bytes=total, allocator_reserved_bytes=reserved,
                  allocator_allocated_bytes=allocated)
    if "error" in entry:
        with pytest.raises({"MemoryError": MemoryError, "ValueError": ValueError}[entry["error"]]):
            plan_footprint_chunks(count, **kwargs)
    else:
        assert plan_footprint_chunks(count, **kwargs).record() == entry["plan"]


def test_rejects_inconsistent_accounting():
    with pytest.raises(ValueError):
        plan_footprint_chunks(10, driver_free_bytes=1, device_total_bytes=1, allocator_reserved_bytes=1,
                              allocator_allocated_bytes=2)
    with pytest.raises(ValueError):
        plan_footprint_chunks(-1, driver_free_bytes=1, device_total_bytes=1, allocator_reserved_bytes=0,
                              allocator_allocated_bytes=0)
