"""Generates tests/golden/planner_golden.json from the reference's own
threedgut_tracer/footprint_chunk_planner.py (standard library only), run in a
container where the reference checkout is present.

    python tests/golden/make_planner_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

GIB = 1 << 30
CASES = [
    (0, 10 * GIB, 180 * GIB, 0, 0),
    (1_000_000, 170 * GIB, 180 * GIB, 2 * GIB, 1 * GIB),
    (6_000_000, 4 * GIB, 180 * GIB, 3 * GIB, 1 * GIB),
    (6_000_000, 6 * GIB + 123, 180 * GIB, 0, 0),
    (10_000, 6 * GIB, 180 * GIB, 0, 0),
    (16_384, 5_700_000_000, 180 * GIB, 0, 0),
    (50_000_000, 40 * GIB, 80 * GIB, 5 * GIB, 5 * GIB),
    (3, 70 << 20, 1 << 30, 0, 0),
    (100_000, 100 << 20, 1 << 30, 0, 0),
    (1, 0, 1 << 30, 0, 0),
    (6_000_000, 10 * GIB, 180 * GIB, 0, 0),
    (20_000_000, 20 * GIB, 180 * GIB, 4 * GIB, 1 * GIB),
    (30_000, 5_820_000_000, 180 * GIB, 0, 0),
    (200_000, 64 << 20, 1 << 30, 512 << 20, 0),
]


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference")
    root = Path(sys.argv[1])
    spec = importlib.util.spec_from_file_location("ref_planner", root / "threedgut_tracer" /
                                                  "footprint_chunk_planner.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_planner"] = mod
    spec.loader.exec_module(mod)
    out = []
    for count, free, total, reserved, allocated in CASES:
        try:
            plan = mod.plan_footprint_chunks(count, driver_free_bytes=free, device_total_bytes=total,
                                             allocator_reserved_bytes=reserved,
                                             allocator_allocated_bytes=allocated)
            out.append({"case": [count, free, total, reserved, allocated], "plan": plan.record()})
        except (MemoryError, ValueError) as e:
            out.append({"case": [count, free, total, reserved, allocated], "error": type(e).__name__})
    path = Path(__file__).resolve().parent / "planner_golden.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", path)


if __name__ == "__main__":
    main()
