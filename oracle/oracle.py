"""ctypes front end of the CPU checker library (``oracle/tessa_oracle.c``).

Test infrastructure only: tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg import this module to check or time the CUDA path.  The
shipped package never imports it.

Each wrapper restates one reference function; the C file cites the
reference file:line for each.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libtessa_oracle.so")
_lib = None

EMPTY_ID = 0xFFFFFFFF
EMPTY_DIST = np.float32(3.402823466e38)


def build() -> str:
    """Compile the checker library with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _p(dtype):
    return np.ctypeslib.ndpointer(dtype=dtype, flags="C_CONTIGUOUS")


def _declare(L):
    u32, u64, i64, f32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float
    L.oracle_padded_dim.restype = u32
    L.oracle_padded_dim.argtypes = [u32, u32]
    L.oracle_quantize_sq8.restype = i64
    L.oracle_quantize_sq8.argtypes = [_p(np.float32), u64, u32, u32, u32, _p(np.int8),
                                      _p(np.float32), _p(np.float32)]
    L.oracle_raw_norms.restype = None
    L.oracle_raw_norms.argtypes = [_p(np.float32), u64, u32, _p(np.float32)]
    L.oracle_sq8_dot.restype = ctypes.c_int32
    L.oracle_sq8_dot.argtypes = [_p(np.int8), _p(np.int8), u32]
    L.oracle_sq8_l2_from_dot.restype = f32
    L.oracle_sq8_l2_from_dot.argtypes = [ctypes.c_int32, f32, f32, f32, f32]
    L.oracle_leaf_topk_sq8.restype = ctypes.c_int
    L.oracle_leaf_topk_sq8.argtypes = [_p(np.int8), _p(np.float32), _p(np.float32), _p(np.uint32),
                                       u64, u32, _p(np.uint32), _p(np.uint64), _p(np.uint64), u64,
                                       u32, u32, u32, _p(np.uint32), _p(np.float32)]
    L.oracle_hash64.restype = u64
    L.oracle_d0_assign_sq8.restype = ctypes.c_int
    L.oracle_d0_assign_sq8.argtypes = [_p(np.int8), _p(np.float32), _p(np.float32), u64, u32, _p(np.int8),
                                       _p(np.float32), _p(np.float32), _p(np.uint32), u32, u32,
                                       _p(np.uint32), _p(np.float32)]
    L.oracle_sketch_rows.restype = None
    L.oracle_sketch_rows.argtypes = [_p(np.float32), u64, u32, _p(np.float32), u32, _p(np.float32)]
    L.oracle_compute_hash.restype = u32
    L.oracle_compute_hash.argtypes = [_p(np.float32), _p(np.float32), u32]
    L.oracle_flush_edges.restype = u64
    L.oracle_flush_edges.argtypes = [_p(np.uint32), _p(np.uint32), _p(np.float32), u64, u32, _p(np.float32), u32, u32,
                                     _p(np.uint32), _p(np.uint32), _p(np.uint16), _p(np.float32), u64]
    L.oracle_hash64.argtypes = [u64]
    L.oracle_assignment_tie_key.restype = u64
    L.oracle_assignment_tie_key.argtypes = [u32, u32]
    L.oracle_assign.restype = ctypes.c_int
    L.oracle_assign.argtypes = [u32, _p(np.float32), _p(np.float32), _p(np.int8), _p(np.float32),
                                _p(np.uint32), u64, u32, u32, _p(np.uint32), _p(np.uint32),
                                _p(np.uint32), _p(np.uint32), _p(np.uint32), _p(np.uint32),
                                _p(np.uint32), _p(np.uint64), u32, _p(np.uint32), _p(np.float32)]
    L.oracle_num_threads.restype = ctypes.c_int
    L.oracle_set_num_threads.argtypes = [ctypes.c_int]
    L.oracle_slot_hashes.restype = None
    L.oracle_slot_hashes.argtypes = [_p(np.uint32), _p(np.uint32), u64, u32, _p(np.float32), u32, u32,
                                     _p(np.uint16), _p(np.uint16)]
    L.oracle_adaptive_psamp.restype = f32
    L.oracle_adaptive_psamp.argtypes = [f32, u32, u32]
    L.oracle_subtree_partition.restype = i64
    L.oracle_subtree_partition.argtypes = [_p(np.int8), _p(np.float32), _p(np.float32), u32, _p(np.uint32),
                                           _p(np.uint64), _p(np.uint32), _p(np.uint64), u32, _p(np.uint32), f32,
                                           _p(np.uint32), u64, _p(np.uint64), _p(np.uint32), _p(np.uint32), u64,
                                           _p(np.uint64)]


def padded_dim(dim: int, k_align: int = 16) -> int:
    return int(lib().oracle_padded_dim(dim, k_align))


def quantize_sq8(x: np.ndarray, k_align: int = 16, bits: int = 8):
    """P/dco_sq_int8.rs:1331-1375 -> (codes [rows, padded_dim] i8, scales, norms)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, dim = x.shape
    pd = padded_dim(dim, k_align)
    codes = np.zeros((rows, pd), dtype=np.int8)
    scales = np.zeros(rows, dtype=np.float32)
    norms = np.zeros(rows, dtype=np.float32)
    rc = lib().oracle_quantize_sq8(x.reshape(-1), rows, dim, k_align, bits, codes.reshape(-1),
                                   scales, norms)
    if rc < 0:
        raise ValueError(f"SQ-int8 quantization failed (code {rc})")
    return codes, scales, norms


def raw_norms(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape[0], dtype=np.float32)
    lib().oracle_raw_norms(x.reshape(-1), x.shape[0], x.shape[1], out)
    return out


def sq8_dot(a: np.ndarray, b: np.ndarray) -> int:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    return int(lib().oracle_sq8_dot(a, b, a.shape[0]))


def sq8_l2_from_dot(dot, rs, rn, cs, cn) -> np.float32:
    return np.float32(lib().oracle_sq8_l2_from_dot(int(dot), float(rs), float(rn), float(cs),
                                                   float(cn)))


def leaf_topk_sq8(codes, scales, norms, global_ids, leaf_members, leaf_offsets, leaf_counts, k,
                  col_task_width: int = 0, staged_min_rows: int = 512):
    """Leaf top-k over a batch of leaves; returns (ids, dists) of len(leaf_members)*k."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    leaf_members = np.ascontiguousarray(leaf_members, dtype=np.uint32)
    offs = np.ascontiguousarray(leaf_offsets, dtype=np.uint64)
    cnts = np.ascontiguousarray(leaf_counts, dtype=np.uint64)
    n_out = int(leaf_members.shape[0]) * k
    ids = np.full(n_out, EMPTY_ID, dtype=np.uint32)
    dists = np.full(n_out, EMPTY_DIST, dtype=np.float32)
    rc = lib().oracle_leaf_topk_sq8(codes.reshape(-1), np.ascontiguousarray(scales, np.float32),
                                    np.ascontiguousarray(norms, np.float32),
                                    np.ascontiguousarray(global_ids, np.uint32), codes.shape[0],
                                    codes.shape[1], leaf_members, offs, cnts, offs.shape[0], k,
                                    col_task_width, staged_min_rows, ids, dists)
    if rc != 0:
        raise ValueError(f"oracle leaf top-k failed (code {rc})")
    return ids, dists


def d0_assign(raw_vectors, global_ids, leader_ids, leader_vectors, fanout_top, leader_payload=None):
    """P/dco_sq_int8.rs:1929-2070 quantize_sq8_and_assign_global_d0_reference.

    Returns dict(codes, scales, norms, child_ids [rows, fanout] (leader
    indices, best first), point_ids [rows, fanout], dists [rows, fanout]).
    leader_payload = (codes, scales, norms) replaces quantizing leader_vectors.
    Raises ValueError with the reference's messages on invalid requests.
    """
    raw = np.ascontiguousarray(raw_vectors, dtype=np.float32)
    gids = np.ascontiguousarray(global_ids, dtype=np.uint32)
    lids = np.ascontiguousarray(leader_ids, dtype=np.uint32)
    rows, leaders = gids.shape[0], lids.shape[0]
    if rows == 0:
        raise ValueError("SQ GPU-D0 staging requires at least one input row")
    dim = raw.shape[1] if raw.ndim == 2 else (raw.size // rows if rows else 0)
    if dim == 0:
        raise ValueError("SQ GPU-D0 staging requires dim > 0")
    if leaders == 0:
        raise ValueError("SQ GPU-D0 staging requires at least one global D0 leader")
    if fanout_top == 0 or fanout_top > leaders or fanout_top > 32:
        raise ValueError(f"SQ GPU-D0 staging fanout must be in 1..=min(32, leaders), got fanout={fanout_top} "
                         f"leaders={leaders}")
    raw = raw.reshape(rows, dim)
    codes, scales, norms = quantize_sq8(raw)
    if leader_payload is None:
        lcodes, lscales, lnorms = quantize_sq8(np.ascontiguousarray(leader_vectors, np.float32).reshape(leaders, dim))
    else:
        lcodes, lscales, lnorms = (np.ascontiguousarray(leader_payload[0], np.int8),
                                   np.ascontiguousarray(leader_payload[1], np.float32),
                                   np.ascontiguousarray(leader_payload[2], np.float32))
        if lcodes.shape != (leaders, codes.shape[1]):
            raise ValueError("SQ GPU-D0 staging leader payload shape mismatch")
    child = np.zeros(rows * fanout_top, dtype=np.uint32)
    dists = np.zeros(rows * fanout_top, dtype=np.float32)
    rc = lib().oracle_d0_assign_sq8(codes.reshape(-1), scales, norms, rows, codes.shape[1], lcodes.reshape(-1),
                                    lscales, lnorms, lids, leaders, fanout_top, child, dists)
    if rc != 0:
        raise ValueError(f"oracle D0 assignment failed (code {rc})")
    return dict(codes=codes, scales=scales, norms=norms, child_ids=child.reshape(rows, fanout_top),
                point_ids=np.repeat(gids, fanout_top).reshape(rows, fanout_top),
                dists=dists.reshape(rows, fanout_top))


def sketch_rows(x, planes):
    """P/hash_prune.rs:2208-2232 fill_sketch_row for every row -> [rows, m] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    planes = np.ascontiguousarray(planes, dtype=np.float32)
    rows, dim = x.shape
    m = planes.shape[0]
    out = np.zeros((rows, m), np.float32)
    lib().oracle_sketch_rows(x.reshape(-1), rows, dim, planes.reshape(-1), m, out.reshape(-1))
    return out


def compute_hash(sketch_p, sketch_c, m_bits: int) -> int:
    """P/hash_prune.rs:2239-2251."""
    return int(lib().oracle_compute_hash(np.ascontiguousarray(sketch_p, np.float32),
                                         np.ascontiguousarray(sketch_c, np.float32), m_bits))


def flush_edges(point_ids, topk_ids, topk_dists, k, sketches, m_bits):
    """P/leaf_build.rs:1749-1808: (p, c, hash, dist) edge arrays in the reference's order."""
    pid = np.ascontiguousarray(point_ids, np.uint32)
    ids = np.ascontiguousarray(topk_ids, np.uint32).reshape(-1)
    ds = np.ascontiguousarray(topk_dists, np.float32).reshape(-1)
    sk = np.ascontiguousarray(sketches, np.float32)
    rows = pid.shape[0]
    z = np.zeros(0, np.uint32)
    n = int(lib().oracle_flush_edges(pid, ids, ds, rows, k, sk.reshape(-1), sk.shape[1], m_bits, z, z,
                                     np.zeros(0, np.uint16), np.zeros(0, np.float32), 0))
    p, c = np.zeros(n, np.uint32), np.zeros(n, np.uint32)
    h, d = np.zeros(n, np.uint16), np.zeros(n, np.float32)
    lib().oracle_flush_edges(pid, ids, ds, rows, k, sk.reshape(-1), sk.shape[1], m_bits, p, c, h, d, n)
    return p, c, h, d


def assign(mode, x, norms, codes, scales, global_ids, members, leaders, task_member_offsets,
           task_member_counts, task_leader_offsets, task_leader_counts, task_rh,
           task_output_offsets, output_len):
    """Assignment replay semantics (CB:15729-15943); mode 0 FP32, 2 SQ8 plain, 3 SQ8 fused."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    ids = np.full(output_len, EMPTY_ID, dtype=np.uint32)
    dists = np.full(output_len, EMPTY_DIST, dtype=np.float32)
    u32 = lambda a: np.ascontiguousarray(a, dtype=np.uint32)
    rc = lib().oracle_assign(mode, x.reshape(-1), np.ascontiguousarray(norms, np.float32),
                             codes.reshape(-1), np.ascontiguousarray(scales, np.float32),
                             u32(global_ids), x.shape[0], x.shape[1], codes.shape[1], u32(members),
                             u32(leaders), u32(task_member_offsets), u32(task_member_counts),
                             u32(task_leader_offsets), u32(task_leader_counts), u32(task_rh),
                             np.ascontiguousarray(task_output_offsets, np.uint64),
                             len(task_rh), ids, dists)
    if rc != 0:
        raise ValueError(f"oracle assignment failed (code {rc})")
    return ids, dists


def hash64(v: int) -> int:
    return int(lib().oracle_hash64(v))


def tie_key(point: int, leader: int) -> int:
    return int(lib().oracle_assignment_tie_key(point, leader))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


# ------------------------------------------------------------ subtree partition

SUBTREE_ERRORS = {-10: "oversized terminal node", -11: "leader overflow", -12: "fanout over 4",
                  -13: "node row overflow", -14: "output capacity", -15: "out of memory", -1: "bad argument"}


def subtree_params(leaf_max=2048, leaf_min=64, max_depth=10, max_leaders=1000, fanout_second=3, root_depth=1,
                   small_node_limit=4096):
    """Persistent-subtree plan values (CB:1309-1340 with PiPNNParams defaults, P/params.rs:3342-3368):
    leaf_max = max(256, c_max), leaf_min 64, small_node_limit 4096, max_leaders capped at 128."""
    return np.array([leaf_max, leaf_min, max_depth, max_leaders, fanout_second, root_depth, small_node_limit],
                    np.uint32)


def subtree_partition(codes, scales, norms, members, task_offsets, task_counts, task_seeds, params=None,
                      psamp=0.001):
    """Recursive leader partition of subtree tasks into leaves (CB:16336-17381, sequential
    canonical order).  Returns (leaf_rows u32 resident ids, leaf_starts u64, leaf_sizes u32,
    leaf_tasks u32, stats {rounds, large_assignments, retries, balanced, small_nodes})."""
    codes = np.ascontiguousarray(codes, np.int8)
    members = np.ascontiguousarray(members, np.uint32)
    toff = np.ascontiguousarray(task_offsets, np.uint64)
    tcnt = np.ascontiguousarray(task_counts, np.uint32)
    tseed = np.ascontiguousarray(task_seeds, np.uint64)
    prm = subtree_params() if params is None else np.ascontiguousarray(params, np.uint32)
    total = int(tcnt.sum())
    cap_rows = 4 * total + 16
    rows = np.zeros(cap_rows, np.uint32)
    starts = np.zeros(cap_rows, np.uint64)
    sizes = np.zeros(cap_rows, np.uint32)
    tasks = np.zeros(cap_rows, np.uint32)
    stats = np.zeros(5, np.uint64)
    n = lib().oracle_subtree_partition(codes.reshape(-1), np.ascontiguousarray(scales, np.float32),
                                       np.ascontiguousarray(norms, np.float32), codes.shape[1], members, toff, tcnt,
                                       tseed, tcnt.size, prm, psamp, rows, cap_rows, starts, sizes, tasks,
                                       cap_rows, stats)
    if n < 0:
        raise ValueError(f"oracle subtree partition failed: {SUBTREE_ERRORS.get(int(n), n)}")
    n = int(n)
    used = int(starts[n - 1] + sizes[n - 1]) if n else 0
    keys = ["rounds", "large_assignments", "retries", "balanced", "small_nodes"]
    return rows[:used].copy(), starts[:n].copy(), sizes[:n].copy(), tasks[:n].copy(), \
        dict(zip(keys, (int(v) for v in stats)))


def slot_hashes(point_ids, topk_ids, k, sketches, m_bits):
    """(hash_fwd, hash_rev) uint16 of every leaf slot (P/leaf_build.rs:1749-1808)."""
    pid = np.ascontiguousarray(point_ids, np.uint32)
    ids = np.ascontiguousarray(topk_ids).view(np.uint32).reshape(-1)
    sk = np.ascontiguousarray(sketches, np.float32)
    hf = np.zeros(ids.size, np.uint16)
    hr = np.zeros(ids.size, np.uint16)
    lib().oracle_slot_hashes(pid, ids, pid.size, k, sk.reshape(-1), sk.shape[1], m_bits, hf, hr)
    return hf, hr
