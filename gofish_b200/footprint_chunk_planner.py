# Interface and decision logic follow tuallen/GOFish (threedgut_tracer), which carries:
# Copyright Amazon.com, Inc. or its affiliates. All Rights Reserved.
# SPDX-License-Identifier: CC-BY-NC-4.0

"""Memory plan for the per-view full-shape operator over N Gaussians
(threedgut_tracer/footprint_chunk_planner.py:13-124, the same inputs,
constants, decisions and FootprintChunkPlan record, so a caller's plan is
unchanged when it switches library).

The constants are the reference operator's accounting (a 16,384-row solver
batch, 320 retained bytes and 1 KiB peak per row, 1/32 of the device as
library headroom); this library's fused operator needs far less than that
(``gofish_b200.full_shape``: 128 B of packed output and no solver work space
per row), so the plan is conservative for it.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass

SOLVER_BATCH_ROWS = 16384
CUDA_THREADS = 256
CUDA_SIGNED_BLOCK_LIMIT = (1 << 31) - 1
CUDA_INDEX_ROW_LIMIT = CUDA_THREADS * CUDA_SIGNED_BLOCK_LIMIT
CHUNKED_RETAINED_AND_CONCAT_BYTES_PER_ROW = 320
NATIVE_PEAK_BYTES_PER_CHUNK_ROW = 1024
MIN_LIBRARY_HEADROOM_BYTES = 64 << 20
DEVICE_HEADROOM_DIVISOR = 32


@dataclass(frozen=True)
class FootprintChunkPlan:
    mode: str
    particle_count: int
    chunk_rows: int
    chunk_count: int
    driver_free_bytes: int
    reusable_reserved_bytes: int
    effective_available_bytes: int
    device_total_bytes: int
    library_headroom_bytes: int
    retained_and_concat_reservation_bytes: int
    transient_budget_bytes: int
    native_peak_bytes_per_chunk_row: int
    solver_batch_rows: int
    decision: str

    def record(self) -> dict[str, object]:
        return asdict(self)


def _chunk_rows(budget_rows: int, count: int) -> int:
    """Largest usable chunk: every row when the count fits one solver batch,
    else a whole number of solver batches (0 when not even one fits)."""
    rows = min(int(budget_rows), int(count), CUDA_INDEX_ROW_LIMIT)
    if count <= SOLVER_BATCH_ROWS:
        return count if rows >= count else 0
    return 0 if rows < SOLVER_BATCH_ROWS else rows - rows % SOLVER_BATCH_ROWS


def plan_footprint_chunks(particle_count: int, *, driver_free_bytes: int, device_total_bytes: int,
                          allocator_reserved_bytes: int, allocator_allocated_bytes: int) -> FootprintChunkPlan:
    count, free, total, reserved, allocated = (int(particle_count), int(driver_free_bytes),
                                               int(device_total_bytes), int(allocator_reserved_bytes),
                                               int(allocator_allocated_bytes))
    if min(count, free, total, reserved, allocated) < 0 or total <= 0:
        raise ValueError("footprint memory-accounting values must be nonnegative")
    if allocated > reserved:
        raise ValueError("allocated CUDA bytes exceed reserved bytes")
    reusable = reserved - allocated
    available = free + reusable
    headroom = max(MIN_LIBRARY_HEADROOM_BYTES, total // DEVICE_HEADROOM_DIVISOR)
    retained = count * CHUNKED_RETAINED_AND_CONCAT_BYTES_PER_ROW
    if count == 0:
        rows, mode, decision = 0, "single_call", "empty_identity"
    elif count <= CUDA_INDEX_ROW_LIMIT and available >= headroom + count * NATIVE_PEAK_BYTES_PER_CHUNK_ROW:
        rows, mode, decision = count, "single_call", "one_call_fits_accounted_peak"
    else:
        rows = _chunk_rows((available - headroom - retained) // NATIVE_PEAK_BYTES_PER_CHUNK_ROW, count)
        if rows <= 0:
            raise MemoryError("footprint retained outputs plus device-derived library headroom "
                              "do not fit current CUDA memory")
        mode, decision = "contiguous_chunks", "full_call_exceeds_accounted_peak_or_cuda_index_limit"
    return FootprintChunkPlan(
        mode=mode, particle_count=count, chunk_rows=rows,
        chunk_count=0 if count == 0 else math.ceil(count / max(1, rows)),
        driver_free_bytes=free, reusable_reserved_bytes=reusable, effective_available_bytes=available,
        device_total_bytes=total, library_headroom_bytes=headroom,
        retained_and_concat_reservation_bytes=retained,
        transient_budget_bytes=max(0, available - headroom - retained),
        native_peak_bytes_per_chunk_row=NATIVE_PEAK_BYTES_PER_CHUNK_ROW, solver_batch_rows=SOLVER_BATCH_ROWS,
        decision=decision)


__all__ = ["CHUNKED_RETAINED_AND_CONCAT_BYTES_PER_ROW", "CUDA_INDEX_ROW_LIMIT", "FootprintChunkPlan",
           "NATIVE_PEAK_BYTES_PER_CHUNK_ROW", "SOLVER_BATCH_ROWS", "plan_footprint_chunks"]
