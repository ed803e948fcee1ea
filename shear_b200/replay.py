"""TESSA operator replay on B200: the host side of ``tessa_operator_replay run``.

Mirrors shear-core/src/algorithm/pipnn/tessa_replay.rs (names, argument
meaning, validation and error behaviour) with the CUDA backend swapped for
libtessa_sm100.so:

* ``TessaReplayMode`` -- P/tessa_replay.rs:18-86;
* ``prepare_tessa_replay`` -- :1252-1429 (union of member rows, raw norms,
  SQ8 codes, per-task layouts, contiguous outputs);
* ``TessaCudaReplaySession`` -- CB:34597-35305 (``new`` uploads once,
  ``run_mode`` clears outputs, runs assignment then leaf between CUDA events and
  downloads the results);
* ``run_tessa_operator_replay`` -- :333-456 (warm-up and measured sweeps in
  rotated mode order, cross-sweep determinism and the SQ8 A2 == A3 bit gate).

The pair / payload formulas (:1070-1118) and the nearest-rank percentile
(:1120-1140) are restated exactly; their unit tests are ported in
tests/test_replay_host.py.
"""
from __future__ import annotations

import ctypes
import enum
import math
from dataclasses import dataclass, field

import numpy as np

from . import _capi as C


class ReplayError(ValueError):
    """TESSA replay validation failure (reference: ``replay_error``)."""

    def __init__(self, message: str):
        super().__init__(f"TESSA replay: {message}")


class TessaReplayMode(enum.IntEnum):
    A0Fp32Simt = 0
    A1Tf32Wmma = 1
    A2Sq8Dp4aBatch1 = 2
    A3Sq8WmmaBatch8 = 3
    Sq8Dp4aBatch8 = 4
    Sq8WmmaBatch1 = 5

    def as_str(self) -> str:
        return ["a0-fp32-simt", "a1-tf32-wmma", "a2-sq8-dp4a-batch1", "a3-sq8-wmma-batch8",
                "sq8-dp4a-batch8", "sq8-wmma-batch1"][int(self)]

    def uses_sq8(self) -> bool:
        return self not in (TessaReplayMode.A0Fp32Simt, TessaReplayMode.A1Tf32Wmma)

    def replays_leaf_tasks(self) -> bool:
        return int(self) <= 3

    def assignment_ticket_batch(self) -> int:
        return 8 if self in (TessaReplayMode.A3Sq8WmmaBatch8, TessaReplayMode.Sq8Dp4aBatch8) else 1

    def assignment_executor_code(self) -> int:
        return {0: 0, 1: 1, 2: 2, 4: 2, 3: 3, 5: 3}[int(self)]

    def leaf_executor_code(self):
        return {0: 0, 1: 0, 2: 1, 3: 2}.get(int(self))

    @classmethod
    def ALL(cls):
        return [cls(i) for i in range(6)]


SQ8_MODES = [TessaReplayMode.A2Sq8Dp4aBatch1, TessaReplayMode.A3Sq8WmmaBatch8,
             TessaReplayMode.Sq8Dp4aBatch8, TessaReplayMode.Sq8WmmaBatch1]


def tessa_rotated_mode_order(sweep: int, modes=None):
    """P/tessa_replay.rs:1245-1250 (rotation of the mode list by sweep)."""
    modes = list(modes if modes is not None else TessaReplayMode.ALL())
    r = sweep % len(modes)
    return modes[r:] + modes[:r]


# ------------------------------------------------------------ task formats

@dataclass
class TessaAssignmentTask:
    """P/tessa_capture.rs:26-36."""
    task_hash: int
    priority: int
    depth: int
    retry: int
    r_h: int
    padded_dim: int
    member_ids: list
    leader_ids: list


@dataclass
class TessaLeafTask:
    """P/tessa_capture.rs:38-45."""
    task_hash: int
    priority: int
    k: int
    padded_dim: int
    member_ids: list


@dataclass
class TessaAssignmentLayout:
    member_offset: int
    member_count: int
    leader_offset: int
    leader_count: int
    r_h: int
    output_offset: int


@dataclass
class TessaLeafLayout:
    member_offset: int
    member_count: int
    k: int
    output_offset: int


@dataclass
class TessaCandidateBlock:
    output_offset: int
    rows: int
    width: int
    pair_weight: int


@dataclass
class TessaPreparedReplay:
    """P/tessa_replay.rs:1052-1074."""
    dim: int
    padded_dim: int
    global_ids: np.ndarray
    vectors_row_major: np.ndarray
    raw_norms: np.ndarray
    sq8_codes: np.ndarray
    sq8_scales: np.ndarray
    sq8_norms: np.ndarray
    assignment_members: np.ndarray
    assignment_leaders: np.ndarray
    assignment_layouts: list
    leaf_members: np.ndarray
    leaf_layouts: list
    leaf_k: int
    assignment_blocks: list
    leaf_blocks: list
    assignment_pairs: int
    leaf_pairs: int
    assignment_unique_rows: int
    leaf_unique_rows: int


# ------------------------------------------------------------ formulas

def tessa_assignment_pairs(tasks) -> int:
    return sum(len(t.member_ids) * len(t.leader_ids) for t in tasks)


def tessa_leaf_pairs(tasks) -> int:
    return sum(len(t.member_ids) * max(len(t.member_ids) - 1, 0) for t in tasks)


def _logical_payload_bytes(unique_rows: int, dimensions: int, bytes_per_dimension: int,
                           metadata_bytes: int) -> int:
    return unique_rows * (dimensions * bytes_per_dimension + metadata_bytes)


def tessa_fp32_logical_payload_bytes(unique_rows: int, dim: int) -> int:
    return _logical_payload_bytes(unique_rows, dim, 4, 4)


def tessa_sq8_logical_payload_bytes(unique_rows: int, padded_dim: int) -> int:
    return _logical_payload_bytes(unique_rows, padded_dim, 1, 8)


def tessa_nearest_rank_percentile(values, percentile: float) -> float:
    """Nearest-rank percentile (P/tessa_replay.rs:1120-1140)."""
    if len(values) == 0:
        raise ReplayError("percentile requires at least one value")
    if not math.isfinite(percentile) or not 0.0 <= percentile <= 1.0:
        raise ReplayError("percentile must be finite and in [0, 1]")
    if any(not math.isfinite(v) for v in values):
        raise ReplayError("percentile input contains a non-finite value")
    s = sorted(values)
    rank = max(1, math.ceil(percentile * len(s)))
    return float(s[min(rank, len(s)) - 1])


# ------------------------------------------------------------ preparation

def prepare_tessa_replay(vectors_by_global_id, dim: int, assignment_tasks, leaf_tasks,
                         padded_dim: int | None = None, device: int = 0) -> TessaPreparedReplay:
    """P/tessa_replay.rs:1252-1429.

    ``vectors_by_global_id(ids) -> float32 [len(ids), dim]`` reads base rows
    (the reference reads the fbin through DirectPointStore).  SQ8 codes are
    produced by the GPU quantizer, which is bit-exact with the CPU quantizer the
    reference calls here.
    """
    from .ops import padded_dim as _pd, quantize_sq8_host

    a_ids = set()
    for t in assignment_tasks:
        a_ids.update(int(v) for v in t.member_ids)
        a_ids.update(int(v) for v in t.leader_ids)
    l_ids = set()
    for t in leaf_tasks:
        l_ids.update(int(v) for v in t.member_ids)
    global_ids = np.array(sorted(a_ids | l_ids), dtype=np.uint32)
    if global_ids.size == 0:
        raise ReplayError("capture contains no replay rows")
    vectors = np.ascontiguousarray(vectors_by_global_id(global_ids), dtype=np.float32)
    if vectors.shape != (global_ids.size, dim):
        raise ReplayError(f"base shape mismatch: got {vectors.shape}, expected ({global_ids.size}, {dim})")
    codes, scales, norms = quantize_sq8_host(vectors, 16, 8, device)
    pd = _pd(dim, 16)
    raw_norms = norms.copy()  # same sequential f32 sum (P/tessa_replay.rs:1287-1290)
    local = {int(g): i for i, g in enumerate(global_ids)}

    def map_ids(ids):
        try:
            return [local[int(v)] for v in ids]
        except KeyError as e:  # pragma: no cover - ids come from the union
            raise ReplayError(f"captured global row {e.args[0]} is missing from replay union")

    a_members, a_leaders, a_layouts, a_blocks = [], [], [], []
    out = 0
    for t in assignment_tasks:
        if t.padded_dim != pd:
            raise ReplayError(f"assignment task padded_dim mismatch: captured={t.padded_dim} prepared={pd}")
        if t.r_h == 0 or t.r_h > 4 or t.r_h > len(t.leader_ids):
            raise ReplayError(f"assignment task {t.task_hash} has invalid r_h={t.r_h} for "
                              f"{len(t.leader_ids)} leaders")
        moff, loff = len(a_members), len(a_leaders)
        a_members += map_ids(t.member_ids)
        a_leaders += map_ids(t.leader_ids)
        a_blocks.append(TessaCandidateBlock(out, len(t.member_ids), t.r_h,
                                            len(t.member_ids) * len(t.leader_ids)))
        a_layouts.append(TessaAssignmentLayout(moff, len(t.member_ids), loff, len(t.leader_ids), t.r_h, out))
        out += len(t.member_ids) * t.r_h

    l_members, l_layouts, l_blocks = [], [], []
    out = 0
    leaf_k = None
    for t in leaf_tasks:
        if t.padded_dim != pd:
            raise ReplayError(f"leaf task padded_dim mismatch: captured={t.padded_dim} prepared={pd}")
        if t.k == 0 or t.k >= len(t.member_ids):
            raise ReplayError(f"leaf task {t.task_hash} has invalid k={t.k} for {len(t.member_ids)} rows")
        if leaf_k is not None and leaf_k != t.k:
            raise ReplayError(f"captured leaf tasks must use one k, found {leaf_k} and {t.k}")
        leaf_k = t.k
        moff = len(l_members)
        l_members += map_ids(t.member_ids)
        n = len(t.member_ids)
        l_blocks.append(TessaCandidateBlock(out, n, t.k, n * (n - 1)))
        l_layouts.append(TessaLeafLayout(moff, n, t.k, out))
        out += n * t.k
    if leaf_k is None:
        raise ReplayError("capture contains no leaf tasks")
    if not a_layouts:
        raise ReplayError("capture contains no assignment tasks")
    return TessaPreparedReplay(
        dim=dim, padded_dim=pd, global_ids=global_ids, vectors_row_major=vectors, raw_norms=raw_norms,
        sq8_codes=codes, sq8_scales=scales, sq8_norms=norms,
        assignment_members=np.array(a_members, dtype=np.uint32),
        assignment_leaders=np.array(a_leaders, dtype=np.uint32), assignment_layouts=a_layouts,
        leaf_members=np.array(l_members, dtype=np.uint32), leaf_layouts=l_layouts, leaf_k=leaf_k,
        assignment_blocks=a_blocks, leaf_blocks=l_blocks,
        assignment_pairs=tessa_assignment_pairs(assignment_tasks), leaf_pairs=tessa_leaf_pairs(leaf_tasks),
        assignment_unique_rows=len(a_ids), leaf_unique_rows=len(l_ids))


# ------------------------------------------------------------ session

@dataclass
class TessaCudaModeResult:
    """P/tessa_replay.rs:190-200 (counters replaced by the device error word)."""
    assignment_event_ms: float
    leaf_event_ms: float | None
    total_event_ms: float
    assignment_ids: np.ndarray
    assignment_dists: np.ndarray
    leaf_ids: np.ndarray
    leaf_dists: np.ndarray
    device_error_bits: int = 0


class TessaCudaReplaySession:
    """CB:34597-35305 on libtessa_sm100.so."""

    def __init__(self, device: int, prepared: TessaPreparedReplay):
        p = prepared
        if p.global_ids.size == 0 or not p.assignment_layouts or not p.leaf_layouts:
            raise ReplayError("prepared replay tasks must be non-empty")
        self.prepared = p
        a = p.assignment_layouts
        self._keep = dict(
            gids=np.ascontiguousarray(p.global_ids, np.uint32),
            x=np.ascontiguousarray(p.vectors_row_major, np.float32),
            raw=np.ascontiguousarray(p.raw_norms, np.float32),
            codes=np.ascontiguousarray(p.sq8_codes, np.int8),
            scales=np.ascontiguousarray(p.sq8_scales, np.float32),
            norms=np.ascontiguousarray(p.sq8_norms, np.float32),
            am=np.ascontiguousarray(p.assignment_members, np.uint32),
            al=np.ascontiguousarray(p.assignment_leaders, np.uint32),
            moff=np.array([l.member_offset for l in a], np.uint32),
            mcnt=np.array([l.member_count for l in a], np.uint32),
            loff=np.array([l.leader_offset for l in a], np.uint32),
            lcnt=np.array([l.leader_count for l in a], np.uint32),
            rh=np.array([l.r_h for l in a], np.uint32),
            out=np.array([l.output_offset for l in a], np.uint64),
            lm=np.ascontiguousarray(p.leaf_members, np.uint32),
            ls=np.array([l.member_offset for l in p.leaf_layouts], np.uint64),
            lz=np.array([l.member_count for l in p.leaf_layouts], np.uint64),
        )
        for l in p.leaf_layouts:
            if l.output_offset != l.member_offset * l.k:
                raise ReplayError("leaf output layout is not contiguous")
        k = self._keep
        self.assignment_output_len = max(b.output_offset + b.rows * b.width for b in p.assignment_blocks)
        self.leaf_output_len = max(b.output_offset + b.rows * b.width for b in p.leaf_blocks)
        pr = C.PreparedReplay(
            dim=p.dim, padded_dim=p.padded_dim, resident_rows=k["gids"].size, global_ids=k["gids"].ctypes.data,
            vectors=k["x"].ctypes.data, raw_norms=k["raw"].ctypes.data, sq8_codes=k["codes"].ctypes.data,
            sq8_scales=k["scales"].ctypes.data, sq8_norms=k["norms"].ctypes.data,
            assignment_members=k["am"].ctypes.data, assignment_member_rows=k["am"].size,
            assignment_leaders=k["al"].ctypes.data, assignment_leader_rows=k["al"].size,
            task_member_offsets=k["moff"].ctypes.data, task_member_counts=k["mcnt"].ctypes.data,
            task_leader_offsets=k["loff"].ctypes.data, task_leader_counts=k["lcnt"].ctypes.data,
            task_rh=k["rh"].ctypes.data, task_output_offsets=k["out"].ctypes.data, task_count=len(a),
            assignment_output_len=self.assignment_output_len, leaf_members=k["lm"].ctypes.data,
            leaf_rows=k["lm"].size, leaf_starts=k["ls"].ctypes.data, leaf_sizes=k["lz"].ctypes.data,
            leaf_count=k["ls"].size, leaf_k=p.leaf_k)
        h = ctypes.c_void_p()
        C.check(C.load().tessa_replay_session_create(int(device), ctypes.byref(pr), ctypes.byref(h)))
        self.handle = h

    def run_mode(self, mode: TessaReplayMode) -> TessaCudaModeResult:
        mode = TessaReplayMode(mode)
        aids = np.empty(self.assignment_output_len, np.uint32)
        adists = np.empty(self.assignment_output_len, np.float32)
        leaf = mode.replays_leaf_tasks()
        lids = np.empty(self.leaf_output_len if leaf else 0, np.uint32)
        ldists = np.empty(self.leaf_output_len if leaf else 0, np.float32)
        r = C.ModeResult(assignment_ids=aids.ctypes.data, assignment_dists=adists.ctypes.data,
                         leaf_ids=lids.ctypes.data if leaf else None,
                         leaf_dists=ldists.ctypes.data if leaf else None)
        C.check(C.load().tessa_replay_run_mode(self.handle, int(mode), ctypes.byref(r)))
        return TessaCudaModeResult(r.assignment_event_ms, r.leaf_event_ms if r.leaf_event_ms >= 0 else None,
                                   r.total_event_ms, aids, adists, lids, ldists, r.device_error_bits)

    def close(self):
        if getattr(self, "handle", None):
            C.load().tessa_replay_session_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def validate_deterministic_mode_output(mode, expected: TessaCudaModeResult, actual: TessaCudaModeResult):
    """P/tessa_replay.rs:571-586: every measured sweep reproduces the first."""
    same = (np.array_equal(expected.assignment_ids, actual.assignment_ids)
            and np.array_equal(_bits(expected.assignment_dists), _bits(actual.assignment_dists))
            and np.array_equal(expected.leaf_ids, actual.leaf_ids)
            and np.array_equal(_bits(expected.leaf_dists), _bits(actual.leaf_dists)))
    if not same:
        raise ReplayError(f"mode {TessaReplayMode(mode).as_str()} output differs across measured sweeps")


def run_tessa_operator_replay(prepared: TessaPreparedReplay, warmup_sweeps: int = 5, measured_sweeps: int = 20,
                              device: int = 0, modes=None, formal: bool = False):
    """P/tessa_replay.rs:333-456 on the B200 backend.

    Returns (samples, canonical results).  ``formal`` enforces the reference's
    5 warm-up / 20 measured sweeps (:221-237).
    """
    if formal and (warmup_sweeps != 5 or measured_sweeps != 20):
        raise ReplayError(f"formal replay requires exactly 5 warmup and 20 measured sweeps, got "
                          f"{warmup_sweeps}/{measured_sweeps}")
    if warmup_sweeps == 0 or measured_sweeps == 0:
        raise ReplayError("warmup_sweeps and measured_sweeps must both be positive")
    modes = list(modes if modes is not None else SQ8_MODES)
    session = TessaCudaReplaySession(device, prepared)
    samples, canonical = [], {}
    try:
        for phase, count in (("warmup", warmup_sweeps), ("measured", measured_sweeps)):
            for sweep in range(count):
                results = {}
                for order, mode in enumerate(tessa_rotated_mode_order(sweep, modes)):
                    res = session.run_mode(mode)
                    samples.append(dict(phase=phase, sweep=sweep, order=order, mode=mode.as_str(),
                                        assignment_ms=res.assignment_event_ms, leaf_ms=res.leaf_event_ms,
                                        total_ms=res.total_event_ms))
                    if phase == "measured":
                        if mode in canonical:
                            validate_deterministic_mode_output(mode, canonical[mode], res)
                        else:
                            canonical[mode] = res
                    results[mode] = res
                a2 = results.get(TessaReplayMode.A2Sq8Dp4aBatch1)
                a3 = results.get(TessaReplayMode.A3Sq8WmmaBatch8)
                if a2 is not None and a3 is not None:
                    kinds = []
                    if not (np.array_equal(a2.assignment_ids, a3.assignment_ids)
                            and np.array_equal(_bits(a2.assignment_dists), _bits(a3.assignment_dists))):
                        kinds.append("assignment")
                    if not (np.array_equal(a2.leaf_ids, a3.leaf_ids)
                            and np.array_equal(_bits(a2.leaf_dists), _bits(a3.leaf_dists))):
                        kinds.append("leaf")
                    if kinds:
                        raise ReplayError(f"A2 SQ8-DP4A and A3 SQ8-WMMA {' and '.join(kinds)} candidate "
                                          f"output differs")
    finally:
        session.close()
    return samples, canonical
