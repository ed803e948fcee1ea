"""ctypes access to the reference's own CUDA kernels (test infrastructure only).

``oracle/_ref/libref_leaf.so`` and ``libref_assign.so`` are built by
``make -C oracle ref REF_ROOT=<reference root>`` from the reference's kernel
source (see ``ref_harness.cu``).  They run ``gpu_persistent_subtree_topk_only``
and ``gpu_tessa_assignment_replay`` exactly as the reference's replay session
launches them (shear-core/src/algorithm/pipnn/compute_backend.rs:34841-35230),
from host buffers, and return their outputs, counters and the mean kernel time.

Used by tests/ as a second checker beside the C restatement and by bench.py's
``reference_gpu`` leg; nothing in the product loads these libraries.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
COUNTER_WORDS = 159

# Counter words read by tessa_replay_counters (CB:35232-35257).
P_OVERFLOW_FLAGS = 7
P_WATCHDOG_TRIPS = 41
P_LEAF_EXACT_FALLBACK_ROWS = 91
P_LEAF_SURVIVOR_OVERFLOW_ROWS = 92
P_ASSIGNMENT_TICKET_CLAIMS = 144
P_ASSIGNMENT_DP4A_TILES = 146
P_ASSIGNMENT_WMMA_TILES = 147
P_LEAF_DP4A_TILES = 157
P_LEAF_WMMA_TILES = 158

_libs: dict = {}


class RefKernelError(RuntimeError):
    pass


def _path(name: str) -> str:
    return os.path.join(REF_DIR, name)


def available() -> bool:
    return os.path.exists(_path("libref_leaf.so")) and os.path.exists(_path("libref_assign.so"))


def _lib(name: str):
    if name not in _libs:
        L = ctypes.CDLL(_path(name))
        L.ref_last_error.restype = ctypes.c_char_p
        _libs[name] = L
    return _libs[name]


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


def leaf_replay(codes, scales, norms, global_ids, leaf_members, leaf_starts, leaf_sizes, k, executor,
                *, staged=True, repeats=1, x=None, raw_norms=None, dim=None):
    """Leaf lists from the reference kernel: ids (u32) and dists (f32), rows x k at
    member_offset * k, plus the counter words and the mean kernel milliseconds.

    executor 1 = SQ8 DP4A scalar filter (mode A2), 2 = s8 WMMA filter (mode A3).
    """
    codes = _c(codes, np.int8)
    rows, padded = codes.shape
    dim = padded if dim is None else int(dim)
    scales, norms = _c(scales, np.float32), _c(norms, np.float32)
    gids = _c(global_ids, np.uint32)
    members = _c(leaf_members, np.uint32)
    starts, sizes = _c(leaf_starts, np.uint64), _c(leaf_sizes, np.uint64)
    xx = _c(np.zeros((rows, dim), np.float32) if x is None else x, np.float32)
    rn = _c(np.zeros(rows, np.float32) if raw_norms is None else raw_norms, np.float32)
    n = members.size
    ids = np.empty(n * k, np.uint32)
    dists = np.empty(n * k, np.float32)
    counters = np.zeros(COUNTER_WORDS, np.uint64)
    ms = ctypes.c_float(0.0)
    L = _lib("libref_leaf.so")
    rc = L.ref_leaf_replay(_ptr(xx), _ptr(gids), _ptr(rn), _ptr(codes), _ptr(scales), _ptr(norms),
                           ctypes.c_uint32(rows), ctypes.c_uint32(dim), ctypes.c_uint32(padded),
                           _ptr(members), ctypes.c_uint32(n), _ptr(starts), _ptr(sizes),
                           ctypes.c_uint32(starts.size), ctypes.c_uint32(k), ctypes.c_uint32(executor),
                           ctypes.c_int(1 if staged else 0), ctypes.c_int(repeats), _ptr(ids), _ptr(dists),
                           _ptr(counters), ctypes.byref(ms))
    if rc != 0:
        raise RefKernelError(f"reference leaf replay failed ({rc}): {L.ref_last_error().decode()}")
    return ids, dists, counters, float(ms.value)


def assign_replay(x, raw_norms, codes, scales, norms, global_ids, members, leaders, task_member_offsets,
                  task_member_counts, task_leader_offsets, task_leader_counts, task_rh, task_output_offsets,
                  output_len, executor, *, ticket_batch=1, repeats=1):
    """Assignment outputs from the reference kernel (ids u32, dists f32, counters, mean ms).

    executor 0 = FP32 SIMT (A0), 1 = TF32 WMMA (A1), 2 = SQ8 DP4A (A2), 3 = SQ8 WMMA (A3).
    """
    codes = _c(codes, np.int8)
    rows, padded = codes.shape
    x = _c(x, np.float32)
    dim = x.shape[1]
    arrs = [_c(a, np.float32) for a in (raw_norms, scales, norms)]
    gids = _c(global_ids, np.uint32)
    mem, lead = _c(members, np.uint32), _c(leaders, np.uint32)
    mo, mc, lo, lc, rh = (_c(a, np.uint32) for a in (task_member_offsets, task_member_counts,
                                                     task_leader_offsets, task_leader_counts, task_rh))
    to = _c(task_output_offsets, np.uint64)
    ids = np.empty(int(output_len), np.uint32)
    dists = np.empty(int(output_len), np.float32)
    counters = np.zeros(COUNTER_WORDS, np.uint64)
    ms = ctypes.c_float(0.0)
    L = _lib("libref_assign.so")
    rc = L.ref_assign_replay(_ptr(x), _ptr(gids), _ptr(arrs[0]), _ptr(codes), _ptr(arrs[1]), _ptr(arrs[2]),
                             ctypes.c_uint32(rows), ctypes.c_uint32(dim), ctypes.c_uint32(padded),
                             _ptr(mem), ctypes.c_uint32(mem.size), _ptr(lead), ctypes.c_uint32(lead.size),
                             _ptr(mo), _ptr(mc), _ptr(lo), _ptr(lc), _ptr(rh), _ptr(to),
                             ctypes.c_uint32(mo.size), ctypes.c_uint64(int(output_len)),
                             ctypes.c_uint32(executor), ctypes.c_uint32(ticket_batch), ctypes.c_int(repeats),
                             _ptr(ids), _ptr(dists), _ptr(counters), ctypes.byref(ms))
    if rc != 0:
        raise RefKernelError(f"reference assignment replay failed ({rc}): {L.ref_last_error().decode()}")
    return ids, dists, counters, float(ms.value)


def leaf_safety_gate(counters, executor):
    """tessa_validate_mode_counters for the leaf half (CB:35271-35305): no overflow,
    no watchdog trip, no exact-fallback or survivor-overflow rows, and only the
    requested executor's tiles."""
    c = [int(v) for v in counters]
    problems = []
    if c[P_OVERFLOW_FLAGS]:
        problems.append(f"overflow flags 0x{c[P_OVERFLOW_FLAGS]:x}")
    if c[P_WATCHDOG_TRIPS]:
        problems.append(f"watchdog trips {c[P_WATCHDOG_TRIPS]}")
    if c[P_LEAF_EXACT_FALLBACK_ROWS] or c[P_LEAF_SURVIVOR_OVERFLOW_ROWS]:
        problems.append(f"fallback rows {c[P_LEAF_EXACT_FALLBACK_ROWS]}/{c[P_LEAF_SURVIVOR_OVERFLOW_ROWS]}")
    if executor == 1 and not (c[P_LEAF_DP4A_TILES] > 0 and c[P_LEAF_WMMA_TILES] == 0):
        problems.append(f"executor tiles dp4a={c[P_LEAF_DP4A_TILES]} wmma={c[P_LEAF_WMMA_TILES]}")
    if executor == 2 and not (c[P_LEAF_WMMA_TILES] > 0 and c[P_LEAF_DP4A_TILES] == 0):
        problems.append(f"executor tiles dp4a={c[P_LEAF_DP4A_TILES]} wmma={c[P_LEAF_WMMA_TILES]}")
    return problems


def assign_safety_gate(counters, executor):
    """The assignment half of tessa_validate_mode_counters (CB:35271-35305)."""
    c = [int(v) for v in counters]
    problems = []
    if c[P_OVERFLOW_FLAGS]:
        problems.append(f"overflow flags 0x{c[P_OVERFLOW_FLAGS]:x}")
    if c[P_WATCHDOG_TRIPS]:
        problems.append(f"watchdog trips {c[P_WATCHDOG_TRIPS]}")
    dp4a, wmma = c[P_ASSIGNMENT_DP4A_TILES], c[P_ASSIGNMENT_WMMA_TILES]
    ok = {0: dp4a == 0 and wmma == 0, 1: dp4a == 0 and wmma == 0,
          2: dp4a > 0 and wmma == 0, 3: wmma > 0 and dp4a == 0}[executor]
    if not ok or c[P_ASSIGNMENT_TICKET_CLAIMS] == 0:
        problems.append(f"executor counters dp4a={dp4a} wmma={wmma} claims={c[P_ASSIGNMENT_TICKET_CLAIMS]}")
    return problems
