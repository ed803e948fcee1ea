"""Host-side replay logic (no GPU): formulas, mode table, validation.

Ports shear-core/src/algorithm/pipnn/tessa_replay.rs unit tests.
"""
import math

import pytest

from shear_b200 import replay as R


def _a(task_hash, r_h, members, leaders):
    return R.TessaAssignmentTask(42, task_hash, 0, 0, r_h, 16, members, leaders)


def _l(k, members):
    return R.TessaLeafTask(42, 2, k, 16, members)


def test_tessa_replay_pair_and_payload_formulas_are_exact():
    # tessa_replay.rs:1474-1488
    assignments = [_a(1, 2, [0, 1, 2], [3, 4]), _a(2, 1, [5, 6], [7, 8, 9])]
    leaves = [_l(2, [0, 1, 2, 3]), _l(2, [4, 5, 6])]
    assert R.tessa_assignment_pairs(assignments) == 12
    assert R.tessa_leaf_pairs(leaves) == 18
    assert R.tessa_fp32_logical_payload_bytes(7, 16) == 476
    assert R.tessa_sq8_logical_payload_bytes(7, 16) == 168


def test_nearest_rank_percentile():
    assert R.tessa_nearest_rank_percentile([0.5, 0.5, 1.0, 1.0], 0.05) == 0.5
    assert R.tessa_nearest_rank_percentile([0.5, 0.5, 1.0, 1.0], 0.5) == 0.5
    assert R.tessa_nearest_rank_percentile([0.5, 0.5, 1.0, 1.0], 0.95) == 1.0
    with pytest.raises(R.ReplayError):
        R.tessa_nearest_rank_percentile([], 0.5)
    with pytest.raises(R.ReplayError):
        R.tessa_nearest_rank_percentile([1.0], 1.5)
    with pytest.raises(R.ReplayError):
        R.tessa_nearest_rank_percentile([math.inf], 0.5)


def test_mode_table_matches_reference():
    M = R.TessaReplayMode
    assert [m.as_str() for m in M.ALL()] == ["a0-fp32-simt", "a1-tf32-wmma", "a2-sq8-dp4a-batch1",
                                             "a3-sq8-wmma-batch8", "sq8-dp4a-batch8", "sq8-wmma-batch1"]
    assert [m.uses_sq8() for m in M.ALL()] == [False, False, True, True, True, True]
    assert [m.replays_leaf_tasks() for m in M.ALL()] == [True, True, True, True, False, False]
    assert [m.assignment_ticket_batch() for m in M.ALL()] == [1, 1, 1, 8, 8, 1]
    assert [m.assignment_executor_code() for m in M.ALL()] == [0, 1, 2, 3, 2, 3]
    assert [m.leaf_executor_code() for m in M.ALL()] == [0, 0, 1, 2, None, None]


def test_rotated_mode_order():
    order = R.tessa_rotated_mode_order(2)
    assert order[0] == R.TessaReplayMode.A2Sq8Dp4aBatch1
    assert len(order) == 6 and set(order) == set(R.TessaReplayMode.ALL())
    assert R.tessa_rotated_mode_order(6) == R.TessaReplayMode.ALL()


def test_formal_replay_requires_5_and_20_sweeps():
    with pytest.raises(R.ReplayError, match="formal replay requires"):
        R.run_tessa_operator_replay(None, 4, 20, formal=True)
    with pytest.raises(R.ReplayError, match="must both be positive"):
        R.run_tessa_operator_replay(None, 0, 20)
