"""Autograd boundary of the per-view full-shape operator
(threedgut_tracer/footprint_shape_operator.py:51-351).

For each Gaussian and view: C = Sigma + Q_v, the factor B = C^{1/2} R and
B^-1, the mass-preserving factor m and the density m * o, with the VJP back
to the intrinsic scale, rotation quaternion (w, x, y, z) and opacity.  Both
directions are single sm_100a float64 kernels (gf_full_shape,
gf_full_shape_bwd); rows are independent and are processed in the contiguous
chunks the footprint planner gives.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _native
from .footprint_chunk_planner import plan_footprint_chunks
from .view_observation_filter import FILTER_VARIANCE_PIXELS

MODES = {"exact": 0, "cholesky": 1}
_STATUS_TEXT = {1: "covariance not positive definite", 2: "degenerate projected covariance",
                4: "non-finite output"}


class FootprintNumericalError(RuntimeError):
    """Numerical failure of the operator, with the offending global row."""

    def __init__(self, message: str, *, global_row: int | None, completed_native_chunks: int):
        super().__init__(message)
        self.global_row = global_row
        self.completed_native_chunks = int(completed_native_chunks)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


# Chunk plans by device: (rows, allocator reserved bytes, plan, calls since the
# device's free memory was last read).
_PLANS: dict = {}
PLAN_REFRESH_CALLS = 64


def _chunk_plan(n: int, device: torch.device):
    """plan_footprint_chunks for n rows on ``device``, fed as the reference
    feeds it (threedgut_tracer/footprint_shape_operator.py:305-315): the
    driver's free and total memory and the caching allocator's reserved and
    allocated bytes.  The free-memory query (cudaMemGetInfo) costs tens of
    microseconds to milliseconds of host time per call, so a plan is kept while
    the row count and the allocator's reserved bytes stay the same (the free
    memory this process sees changes only with them, unless another process
    allocates on the device) and is re-derived at least every
    PLAN_REFRESH_CALLS calls."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    stats = torch.cuda.memory_stats_as_nested_dict(index)
    reserved = int(stats.get("reserved_bytes", {}).get("all", {}).get("current", 0))
    allocated = int(stats.get("allocated_bytes", {}).get("all", {}).get("current", 0))
    cached = _PLANS.get(index)
    if cached is not None and cached[0] == n and cached[1] == reserved and cached[3] < PLAN_REFRESH_CALLS:
        _PLANS[index] = (n, reserved, cached[2], cached[3] + 1)
        return cached[2]
    free, total = torch.cuda.mem_get_info(index)
    plan = plan_footprint_chunks(n, driver_free_bytes=int(free), device_total_bytes=int(total),
                                 allocator_reserved_bytes=reserved, allocator_allocated_bytes=allocated)
    _PLANS[index] = (n, reserved, plan, 1)
    return plan


def _forward(scales, quaternion, density, q6, jacobian, observed, mass_preserving, gamma, mode, pending, start):
    n = scales.shape[0]
    dev = scales.device
    cov = torch.empty((n, 3, 3), dtype=torch.float32, device=dev)
    factor = torch.empty_like(cov)
    inverse = torch.empty_like(cov)
    comp = torch.empty(n, dtype=torch.float32, device=dev)
    dens = torch.empty_like(density)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    lib = _native.load()
    _native.check(lib.gf_full_shape(scales.data_ptr(), quaternion.data_ptr(), density.data_ptr(), q6.data_ptr(),
                                    jacobian.data_ptr(), observed.data_ptr(), n, float(gamma), int(mass_preserving),
                                    MODES[mode], cov.data_ptr(), factor.data_ptr(), inverse.data_ptr(),
                                    comp.data_ptr(), dens.data_ptr(), status.data_ptr(), _stream(scales)),
                  "full shape")
    # the status words reach pinned host memory without a host synchronization;
    # FullShape.check() reads them once the copy's event has completed
    _status_copy(dev, status, start, pending)
    return cov, factor, inverse, comp, dens


# Pinned host words and events for the status copies, per device: allocated
# once and reused round-robin, so a call allocates no pinned memory and
# creates no event (a fresh pinned block costs a cudaHostAlloc, up to
# milliseconds, whenever more calls are in flight than the caching host
# allocator has blocks for).  A slot comes round again STATUS_SLOTS calls
# later: its last copy is waited for and, if its FullShape has not been
# checked yet, the words are moved into ordinary host memory first.
STATUS_SLOTS = 64
_SLOTS: dict = {}


def _status_copy(device: torch.device, status: torch.Tensor, start: int, pending: list) -> None:
    index = device.index if device.index is not None else torch.cuda.current_device()
    ring = _SLOTS.get(index)
    if ring is None:
        ring = {"host": torch.zeros((STATUS_SLOTS, 4), dtype=torch.int32, pin_memory=True),
                "events": [torch.cuda.Event() for _ in range(STATUS_SLOTS)], "owner": [None] * STATUS_SLOTS,
                "next": 0}
        _SLOTS[index] = ring
    i = ring["next"]
    ring["next"] = (i + 1) % STATUS_SLOTS
    host, done = ring["host"][i], ring["events"][i]
    owner = ring["owner"][i]
    if owner is not None:
        done.synchronize()
        lst, at = owner
        if at < len(lst) and lst[at][0].data_ptr() == host.data_ptr():
            lst[at] = (host.clone(),) + tuple(lst[at][1:])
    host.copy_(status, non_blocking=True)
    done.record(torch.cuda.current_stream(device))
    pending.append((host, done, start, status))
    ring["owner"][i] = (pending, len(pending) - 1)


def _raise_failures(pending) -> None:
    for index, (host, done, start, _status) in enumerate(pending):
        done.synchronize()
        flags = host
        if int(flags[0]) != 0:
            local = int(flags[2:].view(torch.int64)[0])
            row = start + local
            text = ", ".join(v for k, v in _STATUS_TEXT.items() if int(flags[0]) & k)
            raise FootprintNumericalError(f"footprint full-shape failure ({text}) local_row={local} global_row={row}",
                                          global_row=row, completed_native_chunks=index)


class _FullShape(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scales, quaternion, density, q6, jacobian, observed, mass_preserving, gamma, mode, pending, start):
        s, q, d = scales.detach().float().contiguous(), quaternion.detach().float().contiguous(), \
            density.detach().float().contiguous()
        ob = observed.detach().to(torch.uint8).contiguous()
        q6c, jc = q6.detach().contiguous(), jacobian.detach().contiguous()
        outs = _forward(s, q, d, q6c, jc, ob, mass_preserving, gamma, mode, pending, start)
        ctx.save_for_backward(s, q, d, q6c, jc, ob)
        ctx.mass_preserving, ctx.gamma, ctx.mode = bool(mass_preserving), float(gamma), mode
        ctx.set_materialize_grads(False)
        return outs

    @staticmethod
    def backward(ctx, g_cov, g_factor, g_inverse, g_comp, g_dens):
        if ctx.mode != "exact":
            raise RuntimeError("the Cholesky full shape is forward only (inference)")
        s, q, d, q6, jac, ob = ctx.saved_tensors
        n = s.shape[0]
        gs = torch.empty_like(s)
        gq = torch.empty_like(q)
        gd = torch.empty_like(d)

        # float32 contiguous copies, held until the kernel has been enqueued
        keep = [None if t is None else t.float().contiguous() for t in (g_cov, g_factor, g_inverse, g_comp, g_dens)]

        def ptr(t):
            return None if t is None else t.data_ptr()

        lib = _native.load()
        _native.check(lib.gf_full_shape_bwd(s.data_ptr(), q.data_ptr(), d.data_ptr(), q6.data_ptr(), jac.data_ptr(),
                                            ob.data_ptr(), n, ctx.gamma, int(ctx.mass_preserving),
                                            *(ptr(t) for t in keep), gs.data_ptr(), gq.data_ptr(), gd.data_ptr(),
                                            _stream(s)), "full shape backward")
        return gs, gq, gd, None, None, None, None, None, None, None, None


@dataclass(frozen=True)
class FullShape:
    covariance: torch.Tensor
    factor: torch.Tensor
    inverse_factor: torch.Tensor
    compensation: torch.Tensor
    density: torch.Tensor
    observed: torch.Tensor
    pending: list = field(default_factory=list)  # (host words, event, first row, device words) per launch

    def check(self) -> None:
        """Raises FootprintNumericalError for the first failed row (waits for
        the status words of the operator's launches)."""
        _raise_failures(self.pending)

    def ready(self) -> bool:
        """Whether the status words of every launch are on the host (check() will not wait)."""
        return all(done.query() for _host, done, _start, _status in self.pending)


def build_full_shape(scales, quaternion, density, q6, jacobian, observed, *, mass_preserving: bool = True,
                     pixel_variance: float = FILTER_VARIANCE_PIXELS, mode: str = "exact",
                     defer_check: bool = False) -> FullShape:
    """Full-shape factors for detached Q (float64 [N,6]) and Jacobian (float32 [N,2,3]).

    A numerical failure raises FootprintNumericalError with the global row.
    With ``defer_check`` the call does not wait for the device: the caller
    runs ``FullShape.check()`` later (the training renderer does so once the
    trace has synchronised its stream)."""
    n = scales.shape[0]
    if q6.requires_grad or q6.dtype != torch.float64 or tuple(q6.shape) != (n, 6):
        raise ValueError("q6 must be detached float64 with shape [N,6]")
    if jacobian.requires_grad or jacobian.dtype != torch.float32 or tuple(jacobian.shape) != (n, 2, 3):
        raise ValueError("jacobian must be detached float32 with shape [N,2,3]")
    if observed.requires_grad or observed.dtype != torch.bool:
        raise ValueError("observed must be a detached bool tensor")
    if mode not in MODES:
        raise ValueError(f"unknown full-shape mode {mode!r}")
    rows = _chunk_plan(n, scales.device).chunk_rows if n else 0
    parts = []
    pending: list = []
    for start in range(0, n, max(1, rows)) if n else []:
        stop = min(n, start + rows)
        parts.append(_FullShape.apply(scales[start:stop], quaternion[start:stop], density[start:stop],
                                      q6[start:stop], jacobian[start:stop], observed[start:stop],
                                      bool(mass_preserving), float(pixel_variance), mode, pending, start))
    if not defer_check:
        _raise_failures(pending)
    if not parts:
        empty = scales.new_zeros((0, 3, 3))
        return FullShape(empty, empty, empty, scales.new_zeros(0), density[:0], observed)
    outs = parts[0] if len(parts) == 1 else tuple(torch.cat([p[i] for p in parts], 0) for i in range(5))
    return FullShape(*outs, observed=observed, pending=pending)


__all__ = ["FootprintNumericalError", "FullShape", "build_full_shape"]
