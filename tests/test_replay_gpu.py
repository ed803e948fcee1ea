"""TessaCudaReplaySession on the B200 with the reference's replay fixtures."""
import numpy as np
import pytest

from shear_b200 import replay as R

pytestmark = pytest.mark.gpu


def _fixture_607():
    rows, dim = 607, 1024
    r = np.arange(rows)[:, None]
    a = np.arange(dim)[None, :]
    src = np.where(r == 7, 6, r)
    base = (((src * 17 + a * 13) % 97).astype(np.float32) * np.float32(0.03125) - np.float32(1.0))
    assign = [R.TessaAssignmentTask(1, 1, 0, 0, 2, 1024, list(range(rows)), list(range(16)))]
    leaf = [R.TessaLeafTask(2, 1, 2, 1024, list(range(rows)))]
    return base, assign, leaf


def _prepare(base, assign, leaf):
    return R.prepare_tessa_replay(lambda ids: base[ids.astype(np.int64)], base.shape[1], assign, leaf)


def test_replay_sq8_modes_bit_exact_and_match_oracle(oracle):
    base, assign, leaf = _fixture_607()
    p = _prepare(base, assign, leaf)
    s = R.TessaCudaReplaySession(0, p)
    try:
        a2 = s.run_mode(R.TessaReplayMode.A2Sq8Dp4aBatch1)
        a3 = s.run_mode(R.TessaReplayMode.A3Sq8WmmaBatch8)
        assert np.array_equal(a2.assignment_ids, a3.assignment_ids)
        assert np.array_equal(a2.leaf_ids, a3.leaf_ids)
        assert np.array_equal(a2.leaf_dists.view(np.uint32), a3.leaf_dists.view(np.uint32))
        b4 = s.run_mode(R.TessaReplayMode.Sq8Dp4aBatch8)
        assert b4.leaf_event_ms is None and b4.leaf_ids.size == 0
        with pytest.raises(Exception, match="UNSUPPORTED"):
            s.run_mode(R.TessaReplayMode.A0Fp32Simt)
    finally:
        s.close()
    lo = p.leaf_layouts[0]
    wi, wd = oracle.leaf_topk_sq8(p.sq8_codes, p.sq8_scales, p.sq8_norms, p.global_ids, p.leaf_members,
                                  [lo.member_offset], [lo.member_count], p.leaf_k)
    assert np.array_equal(a2.leaf_ids, wi)
    assert np.array_equal(a2.leaf_dists.view(np.uint32), wd.view(np.uint32))
    al = p.assignment_layouts[0]
    ai, ad = oracle.assign(3, p.vectors_row_major, p.sq8_norms, p.sq8_codes, p.sq8_scales, p.global_ids,
                           p.assignment_members, p.assignment_leaders, [al.member_offset], [al.member_count],
                           [al.leader_offset], [al.leader_count], [al.r_h], [al.output_offset],
                           al.member_count * al.r_h)
    assert np.array_equal(a2.assignment_ids, ai)
    assert np.array_equal(a2.assignment_dists.view(np.uint32), ad.view(np.uint32))


def test_run_tessa_operator_replay_is_deterministic():
    base, assign, leaf = _fixture_607()
    p = _prepare(base, assign, leaf)
    samples, canonical = R.run_tessa_operator_replay(p, 1, 3)
    assert len(canonical) == 4
    assert all(s["total_ms"] > 0 for s in samples)


def test_prepare_validates_tasks():
    base, assign, leaf = _fixture_607()
    bad_leaf = [R.TessaLeafTask(2, 1, 700, 1024, list(range(607)))]
    with pytest.raises(R.ReplayError, match="invalid k"):
        _prepare(base, assign, bad_leaf)
    bad_rh = [R.TessaAssignmentTask(1, 1, 0, 0, 5, 1024, [0, 1], [2, 3, 4, 5, 6])]
    with pytest.raises(R.ReplayError, match="invalid r_h"):
        _prepare(base, bad_rh, leaf)
