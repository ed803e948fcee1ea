"""GPU-memory-aware task former for B200 workspaces.

The capacity logic restates shear-core/src/algorithm/pipnn/d0_capacity.rs
(P/d0_capacity.rs): thresholds c_high / c_target / c_low from the largest
admissible subtree (:201-223), the root-leader plan (:225-257), the split
count of an oversized child (:259-264), nearest-rank percentiles and the child
size telemetry (:266-296), and find_max_admissible_rows (:55-103, doubling then
binary search of the largest subtree an admission predicate accepts).

The admission predicate is resized for this library (the reference's counts
its persistent kernel's device queues, compute_backend.rs:909-929 and
:1309-1521).  A resident subtree of R rows needs, with fanout amplification
f = min(max_fanout, 4) (each row lands in up to f leaves, as the reference
bounds it) and M = R * f leaf rows:

* resident payload: SQ8 codes R * padded_dim + scale, norm, global id
  (12 bytes per row), plus R * dim * 4 of f32 rows when the assignment reads
  raw vectors;
* leaf batch: member ids M * 4, leaf-ordered code scratch M * padded_dim when
  members are not contiguous, lists M * k * 8, the exact-fallback row list
  M * 8 + 16, leaf layout and tile table (16 bytes per leaf, 8 per 128-row
  tile, leaves of at least leaf_min rows), and for padded_dim <= 1024 the
  column-split kernel's per-row zone dump M * (8 * D + 128 + 2) with
  D = min(k + 7, 48) rounded down to even (38 at k = 32);
* assignment: member / leader ids 4 * (R + leaders), outputs R * r_h * 8.

``library_scratch_bytes`` reports what a context actually holds, and the GPU
tests check the model bounds it from above.
"""
from __future__ import annotations

import dataclasses
import math

GPU_PERSISTENT_LEAF_MIN = 64  # smallest leaf the planner counts (compute_backend.rs:385-391)


@dataclasses.dataclass(frozen=True)
class D0CapacityConfig:
    """P/d0_capacity.rs:11-35 (defaults as the reference's)."""
    enabled: bool = False
    high_ratio: float = 0.60
    target_ratio: float = 0.50
    low_ratio: float = 0.15
    min_efficient_rows: int = 32 * 1024
    quality_min_root_leaders: int = 64
    root_leader_cap: int = 10_000
    split_recursion_limit: int = 8


@dataclasses.dataclass(frozen=True)
class D0CapacityThresholds:
    c_gpu: int
    c_high: int
    c_target: int
    c_low: int


@dataclasses.dataclass(frozen=True)
class D0LeaderPlan:
    k_capacity: int = 0
    k_initial: int = 0
    root_leader_cap: int = 0
    root_leader_source: str = ""


@dataclasses.dataclass
class D0CapacityTelemetry:
    actual_child_max_unique_rows: int = 0
    actual_child_p50_unique_rows: int = 0
    actual_child_p95_unique_rows: int = 0
    actual_child_p99_unique_rows: int = 0
    oversized_child_count: int = 0
    small_child_count: int = 0
    small_child_rows: int = 0


def _clamp(v, lo, hi):
    return max(lo, min(hi, v))


def compute_thresholds(c_gpu: int, cfg: D0CapacityConfig) -> D0CapacityThresholds:
    """P/d0_capacity.rs:201-223."""
    if c_gpu == 0:
        return D0CapacityThresholds(0, 0, 0, 0)
    high = _clamp(cfg.high_ratio, 0.01, 1.0)
    target = _clamp(cfg.target_ratio, 0.01, high)
    low = _clamp(cfg.low_ratio, 0.0, target)
    c_high = max(math.floor(c_gpu * high), 1)
    c_target = max(math.floor(c_gpu * target), 1)
    ratio_low = max(math.floor(c_gpu * low), 1)
    c_low = min(max(ratio_low, cfg.min_efficient_rows), c_target)
    return D0CapacityThresholds(c_gpu, c_high, c_target, c_low)


def plan_root_leaders(total_points: int, root_fanout: int, thr: D0CapacityThresholds,
                      cfg: D0CapacityConfig) -> D0LeaderPlan:
    """P/d0_capacity.rs:225-257."""
    if total_points == 0 or root_fanout == 0:
        return D0LeaderPlan()
    assignments = total_points * root_fanout
    k_capacity = 0 if thr.c_target == 0 else max(-(-assignments // thr.c_target), 1)
    cap = min(max(cfg.root_leader_cap, 1), max(total_points, 1))
    capacity_target = max(k_capacity, 1)
    floor = min(max(cfg.quality_min_root_leaders, 1), max(total_points, 1))
    desired = max(capacity_target, floor)
    if desired > cap:
        source = "root_leader_cap"
    elif floor > capacity_target:
        source = "quality_floor"
    else:
        source = "capacity"
    return D0LeaderPlan(k_capacity, _clamp(desired, 1, cap), cap, source)


def split_leader_count(rows: int, thr: D0CapacityThresholds) -> int:
    """P/d0_capacity.rs:259-264."""
    if rows <= thr.c_high or thr.c_target == 0:
        return 1
    return max(-(-rows // thr.c_target), 2)


def percentile_nearest_rank(sorted_values, pct: int) -> int:
    """P/d0_capacity.rs:266-272."""
    if not sorted_values:
        return 0
    rank = -(-(len(sorted_values) * pct) // 100)
    return sorted_values[min(max(rank - 1, 0), len(sorted_values) - 1)]


def observe_child_unique_sizes(tel: D0CapacityTelemetry, thr: D0CapacityThresholds, sizes: list) -> None:
    """P/d0_capacity.rs:274-296 (sorts `sizes` in place, as the reference does)."""
    sizes.sort()
    tel.actual_child_max_unique_rows = sizes[-1] if sizes else 0
    tel.actual_child_p50_unique_rows = percentile_nearest_rank(sizes, 50)
    tel.actual_child_p95_unique_rows = percentile_nearest_rank(sizes, 95)
    tel.actual_child_p99_unique_rows = percentile_nearest_rank(sizes, 99)
    tel.oversized_child_count = sum(1 for s in sizes if s > thr.c_high)
    small = [s for s in sizes if s < thr.c_low]
    tel.small_child_count = len(small)
    tel.small_child_rows = sum(small)


# ------------------------------------------------------------ B200 admission

def padded_dim(dim: int, k_align: int = 16) -> int:
    return -(-dim // k_align) * k_align


@dataclasses.dataclass(frozen=True)
class SubtreePlan:
    supported: bool
    resident_bytes: int
    leaf_bytes: int
    assignment_bytes: int
    required_bytes: int
    budget_bytes: int | None


def plan_subtree_admission(rows: int, dim: int, leaf_k: int, max_fanout: int, budget_bytes: int | None,
                           leaders: int = 128, r_h: int = 2, raw_assignment: bool = False,
                           leaf_ordered: bool = False) -> SubtreePlan:
    """Device bytes this library needs to process a resident subtree of `rows`
    rows (the model in the module docstring) and whether they fit."""
    pd = padded_dim(dim)
    f = max(1, min(max_fanout, 4))
    m = rows * f
    resident = rows * (pd + 12) + (rows * dim * 4 if raw_assignment else 0)
    leaves = -(-m // GPU_PERSISTENT_LEAF_MIN) if m else 0
    tiles = leaves + -(-m // 128)
    kk = min(leaf_k, 32)
    zone = min(kk + 7, 48) & ~1
    dump = m * (8 * zone + 128 + 2) + 16 if pd <= 1024 else 0
    leaf = (m * 4 + (0 if leaf_ordered else m * pd) + m * kk * 8 + m * 8 + 16
            + leaves * 16 + tiles * 8 + dump)
    assign = 4 * (rows + leaders) + rows * r_h * 8
    required = resident + leaf + assign
    ok = leaf_k <= 32 and (budget_bytes is None or rows == 0 or required <= budget_bytes)
    return SubtreePlan(ok, resident, leaf, assign, required, budget_bytes)


def find_max_admissible_rows(dim: int, leaf_k: int, max_fanout: int, budget_bytes: int | None, **kw) -> int:
    """P/d0_capacity.rs:55-103: the largest row count the admission accepts
    (doubling, then binary search), 0 if not even one row fits."""
    if dim == 0:
        return 0

    def supported(r):
        return plan_subtree_admission(r, dim, leaf_k, max_fanout, budget_bytes, **kw).supported

    if not supported(1):
        return 0
    lo, hi = 1, 2
    while supported(hi) and hi < (1 << 31):
        lo, hi = hi, hi * 2
    while lo + 1 < hi:
        mid = lo + (hi - lo) // 2
        if supported(mid):
            lo = mid
        else:
            hi = mid
    return lo


def b200_workspace_budget(total_device_bytes: int, reserve_fraction: float = 0.10) -> int:
    """Workspace for subtree tasks on one device: its memory less a reserve
    for the context, the CUDA runtime and the caller's own buffers."""
    return int(total_device_bytes * (1.0 - reserve_fraction))


def library_scratch_bytes(ctx=None, device: int = 0) -> int:
    """Device bytes the library context currently holds (tessa_ctx_device_bytes)."""
    import ctypes

    from . import _capi as C, ops
    ctx = ctx or ops.context(device)
    n = ctypes.c_uint64()
    C.check(C.load().tessa_ctx_device_bytes(ctx.handle, ctypes.byref(n)))
    return int(n.value)
