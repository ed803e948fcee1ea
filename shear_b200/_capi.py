"""ctypes binding of libtessa_sm100.so (declarations mirror include/tessa_sm100.h).

The shared library is the product; this module only loads it and declares the
entry points.  Loading fails loudly: there is no CPU fallback anywhere in this
package.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtessa_sm100.so")

TESSA_OK = 0
ERRORS = {
    -1: "TESSA_ERR_INVALID_ARG",
    -2: "TESSA_ERR_CUDA",
    -3: "TESSA_ERR_OOM",
    -4: "TESSA_ERR_TIMEOUT",
    -5: "TESSA_ERR_BAD_ROW",
    -6: "TESSA_ERR_UNSUPPORTED",
    -7: "TESSA_ERR_NONFINITE",
    -8: "TESSA_ERR_NO_DEVICE",
    -9: "TESSA_ERR_BAD_TASK",
    -10: "TESSA_ERR_PARTITION",
    -11: "TESSA_ERR_AGAIN",
}
MAX_LEAF_K = 32
MAX_RH = 4
MAX_PADDED_DIM = 1024
MAX_HASH_BITS = 16
NOALLOC_SCRATCH_BYTES = 64 << 20
ASSIGN_FP32 = 0
ASSIGN_SQ8 = 2

c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_u64p = ctypes.POINTER(ctypes.c_uint64)
c_f32p = ctypes.POINTER(ctypes.c_float)
c_i8p = ctypes.POINTER(ctypes.c_int8)
c_vp = ctypes.c_void_p


class TessaError(RuntimeError):
    """A TESSA_ERR_* code returned across the C ABI."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


class LeafArgs(ctypes.Structure):
    _fields_ = [
        ("codes", c_vp), ("scales", c_vp), ("norms", c_vp), ("global_ids", c_vp),
        ("resident_rows", ctypes.c_uint64), ("padded_dim", ctypes.c_uint32), ("k", ctypes.c_uint32),
        ("leaf_members", c_vp), ("leaf_starts", c_vp), ("leaf_sizes", c_vp),
        ("leaf_count", ctypes.c_uint64), ("leaf_rows", ctypes.c_uint64),
        ("topk_ids", c_vp), ("topk_dists", c_vp), ("leaf_ordered_codes", c_vp),
    ]


class AssignArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_vp), ("raw_norms", c_vp), ("codes", c_vp), ("scales", c_vp), ("sq8_norms", c_vp),
        ("global_ids", c_vp), ("resident_rows", ctypes.c_uint64), ("dim", ctypes.c_uint32),
        ("padded_dim", ctypes.c_uint32), ("members", c_vp), ("leaders", c_vp),
        ("task_member_offsets", c_vp), ("task_member_counts", c_vp), ("task_leader_offsets", c_vp),
        ("task_leader_counts", c_vp), ("task_rh", c_vp), ("task_output_offsets", c_vp),
        ("task_count", ctypes.c_uint32), ("member_rows", ctypes.c_uint64), ("out_ids", c_vp),
        ("out_dists", c_vp),
    ]


class D0Args(ctypes.Structure):
    _fields_ = [
        ("raw_vectors", c_vp), ("global_ids", c_vp), ("rows", ctypes.c_uint64), ("dim", ctypes.c_uint32),
        ("fanout_top", ctypes.c_uint32), ("leader_ids", c_vp), ("leader_vectors", c_vp),
        ("leader_codes", c_vp), ("leader_scales", c_vp), ("leader_norms", c_vp),
        ("leader_count", ctypes.c_uint32), ("codes", c_vp), ("scales", c_vp), ("norms", c_vp),
        ("child_ids", c_vp), ("point_ids", c_vp), ("dists", c_vp),
    ]


class D0Profile(ctypes.Structure):
    _fields_ = [
        ("leader_quantize_ms", ctypes.c_double), ("quantize_ms", ctypes.c_double), ("assign_ms", ctypes.c_double),
        ("fragment_ms", ctypes.c_double), ("rows", ctypes.c_uint64), ("fallback_rows", ctypes.c_uint64),
        ("leaders", ctypes.c_uint32), ("fanout", ctypes.c_uint32), ("padded_dim", ctypes.c_uint32),
    ]


class PreparedReplay(ctypes.Structure):
    _fields_ = [
        ("dim", ctypes.c_uint32), ("padded_dim", ctypes.c_uint32), ("resident_rows", ctypes.c_uint64),
        ("global_ids", c_vp), ("vectors", c_vp), ("raw_norms", c_vp), ("sq8_codes", c_vp),
        ("sq8_scales", c_vp), ("sq8_norms", c_vp), ("assignment_members", c_vp),
        ("assignment_member_rows", ctypes.c_uint64), ("assignment_leaders", c_vp),
        ("assignment_leader_rows", ctypes.c_uint64), ("task_member_offsets", c_vp),
        ("task_member_counts", c_vp), ("task_leader_offsets", c_vp), ("task_leader_counts", c_vp),
        ("task_rh", c_vp), ("task_output_offsets", c_vp), ("task_count", ctypes.c_uint32),
        ("assignment_output_len", ctypes.c_uint64), ("leaf_members", c_vp),
        ("leaf_rows", ctypes.c_uint64), ("leaf_starts", c_vp), ("leaf_sizes", c_vp),
        ("leaf_count", ctypes.c_uint64), ("leaf_k", ctypes.c_uint32),
    ]


class ModeResult(ctypes.Structure):
    _fields_ = [
        ("assignment_event_ms", ctypes.c_double), ("leaf_event_ms", ctypes.c_double),
        ("total_event_ms", ctypes.c_double), ("assignment_ids", c_vp), ("assignment_dists", c_vp),
        ("leaf_ids", c_vp), ("leaf_dists", c_vp), ("device_error_bits", ctypes.c_uint64),
    ]


class SubtreeArgs(ctypes.Structure):
    _fields_ = [
        ("codes", c_vp), ("scales", c_vp), ("sq8_norms", c_vp), ("resident_rows", ctypes.c_uint64),
        ("padded_dim", ctypes.c_uint32), ("task_members", c_vp), ("member_rows", ctypes.c_uint64),
        ("task_offsets", c_vp), ("task_counts", c_vp), ("task_seeds", c_vp), ("task_count", ctypes.c_uint32),
        ("leaf_max", ctypes.c_uint32), ("leaf_min", ctypes.c_uint32), ("max_depth", ctypes.c_uint32),
        ("max_leaders", ctypes.c_uint32), ("fanout_second", ctypes.c_uint32), ("root_depth", ctypes.c_uint32),
        ("small_node_limit", ctypes.c_uint32), ("psamp_fraction", ctypes.c_float),
        ("leaf_rows", c_vp), ("leaf_rows_capacity", ctypes.c_uint64), ("leaf_starts", c_vp),
        ("leaf_sizes", c_vp), ("leaf_tasks", c_vp), ("leaf_capacity", ctypes.c_uint64), ("leaf_codes", c_vp),
    ]


class SubtreeResult(ctypes.Structure):
    _fields_ = [
        ("leaf_count", ctypes.c_uint64), ("leaf_rows_used", ctypes.c_uint64), ("rounds", ctypes.c_uint32),
        ("large_assignments", ctypes.c_uint32), ("retries", ctypes.c_uint32), ("balanced", ctypes.c_uint32),
        ("small_nodes", ctypes.c_uint32), ("kernel_launches", ctypes.c_uint32),
        ("assign_ms", ctypes.c_float), ("scatter_ms", ctypes.c_float), ("small_ms", ctypes.c_float),
        ("wall_ms", ctypes.c_float), ("host_prep_ms", ctypes.c_float), ("host_decide_ms", ctypes.c_float),
        ("sync_wait_ms", ctypes.c_float),
    ]


class SubtreeRequest(ctypes.Structure):
    _fields_ = [("partition", SubtreeArgs), ("global_ids", c_vp), ("k", ctypes.c_uint32)]


class CompactView(ctypes.Structure):
    _fields_ = [
        ("ticket", ctypes.c_uint64), ("rows", ctypes.c_uint64), ("k", ctypes.c_uint32),
        ("leaf_count", ctypes.c_uint64), ("leaf_starts", c_vp), ("leaf_sizes", c_vp), ("leaf_tasks", c_vp),
        ("point_ids", c_vp), ("topk_ids", c_vp), ("topk_dists", c_vp), ("partition", SubtreeResult),
        ("fallback_rows", ctypes.c_uint64),
    ]


# (name, restype, argtypes) for every entry point of include/tessa_sm100.h
SIGNATURES = [
    ("tessa_abi_version", ctypes.c_int, []),
    ("tessa_strerror", ctypes.c_char_p, [ctypes.c_int]),
    ("tessa_last_error_message", ctypes.c_char_p, []),
    ("tessa_create", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(c_vp)]),
    ("tessa_destroy", None, [c_vp]),
    ("tessa_ctx_device", ctypes.c_int, [c_vp]),
    ("tessa_ctx_device_bytes", ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    ("tessa_quantize_sq8", ctypes.c_int,
     [c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp,
      c_vp]),
    ("tessa_quantize_sq8_host", ctypes.c_int,
     [c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp]),
    ("tessa_leaf_topk_sq8", ctypes.c_int, [c_vp, ctypes.POINTER(LeafArgs), c_vp]),
    ("tessa_leaf_topk_sq8_host", ctypes.c_int, [c_vp, ctypes.POINTER(LeafArgs)]),
    ("tessa_leaf_topk_sq8_noalloc", ctypes.c_int, [ctypes.POINTER(LeafArgs), c_vp]),
    ("tessa_leaf_last_fallback_rows", ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    ("tessa_set_host_batch_bytes", ctypes.c_int, [c_vp, ctypes.c_uint64]),
    ("tessa_assign", ctypes.c_int, [c_vp, ctypes.c_uint32, ctypes.POINTER(AssignArgs), c_vp]),
    ("tessa_quantize_sq8_assign_d0", ctypes.c_int, [c_vp, ctypes.POINTER(D0Args), c_vp]),
    ("tessa_quantize_sq8_assign_d0_host", ctypes.c_int, [c_vp, ctypes.POINTER(D0Args)]),
    ("tessa_d0_last_profile", ctypes.c_int, [c_vp, ctypes.POINTER(D0Profile)]),
    ("tessa_sketch_rows", ctypes.c_int,
     [c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, c_vp, ctypes.c_uint32, c_vp, c_vp]),
    ("tessa_edge_hashes", ctypes.c_int,
     [c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint64, c_vp, ctypes.c_uint64,
      ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp]),
    ("tessa_membership_digests", ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint64, c_vp, c_vp, c_vp]),
    ("tessa_graph_search", ctypes.c_int,
     [c_vp, ctypes.c_uint64, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint64, ctypes.c_uint32,
      ctypes.c_uint32, ctypes.c_uint32, c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    ("tessa_expand_edges", ctypes.c_int,
     [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp,
      ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    ("tessa_replay_session_create", ctypes.c_int,
     [ctypes.c_int, ctypes.POINTER(PreparedReplay), ctypes.POINTER(c_vp)]),
    ("tessa_replay_run_mode", ctypes.c_int, [c_vp, ctypes.c_uint32, ctypes.POINTER(ModeResult)]),
    ("tessa_replay_session_destroy", None, [c_vp]),
    ("tessa_subtree_partition", ctypes.c_int,
     [c_vp, ctypes.POINTER(SubtreeArgs), ctypes.POINTER(SubtreeResult), c_vp]),
    ("tessa_set_wait_timeout_ns", ctypes.c_int, [c_vp, ctypes.c_uint64]),
    ("tessa_set_leaf_kernel", ctypes.c_int, [c_vp, ctypes.c_uint32]),
    ("tessa_check_bounded_wait", ctypes.c_int, [c_vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64), c_vp]),
    ("tessa_reducer_create", ctypes.c_int, [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(c_vp)]),
    ("tessa_reducer_add", ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32]),
    ("tessa_reducer_finish", ctypes.c_int, [c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    ("tessa_reducer_edges", ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    ("tessa_reducer_add_grouped", ctypes.c_int, [c_vp, c_vp, c_vp]),
    ("tessa_group_edges", ctypes.c_int,
     [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, c_vp, c_vp,
      ctypes.c_uint64, c_vp]),
    ("tessa_reducer_destroy", None, [c_vp]),
    ("tessa_subtree_submit", ctypes.c_int,
     [c_vp, ctypes.POINTER(SubtreeRequest), ctypes.POINTER(ctypes.c_uint64), c_vp]),
    ("tessa_subtree_poll", ctypes.c_int, [c_vp, ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(CompactView)]),
    ("tessa_subtree_release", ctypes.c_int, [c_vp, ctypes.c_uint64]),
    ("tessa_reduce_records", ctypes.c_int,
     [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32,
      c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64), c_vp]),
    ("tessa_reduce_grouped", ctypes.c_int,
     [c_vp, ctypes.c_uint32, c_vp, c_vp, c_vp, ctypes.c_uint64, ctypes.c_uint32, c_vp, c_vp, c_vp,
      ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64), c_vp]),
]

_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing; build it with `python -m shear_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(code: int) -> None:
    if code != TESSA_OK:
        msg = load().tessa_last_error_message()
        raise TessaError(code, msg.decode() if msg else "")
