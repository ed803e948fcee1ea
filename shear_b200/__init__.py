"""shear_b200 -- B200-native (sm_100a) TESSA hot path of SHEAR's GPU graph build.

The product is ``libtessa_sm100.so`` (C ABI, ``include/tessa_sm100.h``): SQ8
quantization, TESSA leader assignment and the fused SQ8 leaf top-k
(tcgen05 int8 GEMM + per-row bounded selection).  This package is the Python
host side above that ABI, mirroring the reference's replay interface
(``shear-core/src/algorithm/pipnn/tessa_replay.rs``):

* :mod:`shear_b200.ops` -- device-tensor entry points (``leaf_topk_sq8``,
  ``quantize_sq8``, ``assign``) and their host-buffer forms;
* :mod:`shear_b200.replay` -- ``TessaReplayMode``, ``TessaPreparedReplay``,
  ``prepare_tessa_replay``, ``TessaCudaReplaySession`` and
  ``run_tessa_operator_replay``;
* :mod:`shear_b200.sharding` -- the host work queue that spreads independent
  leaf / subtree tasks over the GPUs of one box (no collective).

Nothing here falls back to the CPU: if the library or a GPU is missing the
calls raise.
"""
from ._capi import TessaError, load as load_library, LIB_PATH  # noqa: F401

__all__ = ["TessaError", "load_library", "LIB_PATH"]
