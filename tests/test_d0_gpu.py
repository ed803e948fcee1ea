"""Global-D0 SQ8 staging on the B200 (quantizer + rectangular tcgen05 top-k
through the C ABI) vs the oracle restatement of
quantize_sq8_and_assign_global_d0_reference (P/dco_sq_int8.rs:1929-2070).

Bit-exact: codes, scales, norms, child ids, point ids and distance bits.
"""
import numpy as np
import pytest

from d0cases import random_case, reference_fixture_43857

pytestmark = pytest.mark.gpu


def _same(got, want):
    from shear_b200 import ops
    assert np.array_equal(got.codes, want["codes"])
    assert np.array_equal(got.scales.view(np.uint32), want["scales"].view(np.uint32))
    assert np.array_equal(got.norms.view(np.uint32), want["norms"].view(np.uint32))
    bad = np.argwhere(got.child_ids != want["child_ids"])
    assert bad.size == 0, f"{len(bad)} child mismatches, first {bad[:4].tolist()}: got " \
                          f"{[got.child_ids[tuple(b)] for b in bad[:4]]} want {[want['child_ids'][tuple(b)] for b in bad[:4]]}"
    assert np.array_equal(got.point_ids, want["point_ids"])
    assert np.array_equal(got.dists.view(np.uint32), want["dists"].view(np.uint32))
    assert isinstance(ops.leaf_last_fallback_rows(), int)


def test_d0_reference_golden_stable_ties(oracle):
    # P/dco_sq_int8.rs:3422-3453
    from shear_b200 import ops
    leaders = np.array([[1.0, 0.0], [-1.0, 0.0]], np.float32)
    payload = oracle.quantize_sq8(leaders)
    got = ops.quantize_sq8_and_assign_global_d0(np.array([[0.0, 0.0], [1.0, 0.0]], np.float32), [0, 1], [5, 3],
                                                leaders, 1, leader_payload=payload)
    assert got.fragments() == [(1, 0), (0, 1)]
    assert got.rows == 2 and got.padded_dim == 16


@pytest.mark.parametrize("fanout", [1, 6, 17, 32])
def test_d0_compute_backend_fixture(oracle, fanout):
    # compute_backend.rs:43857-43940 (the reference's GPU-vs-reference test inputs)
    from shear_b200 import ops
    raw, gids, lids, lv = reference_fixture_43857()
    want = oracle.d0_assign(raw, gids, lids, lv, fanout)
    _same(ops.quantize_sq8_and_assign_global_d0(raw, gids, lids, lv, fanout), want)


CASES = [
    # rows, dim, leaders, fanout, near-duplicate leaders
    (1, 8, 1, 1, 0),
    (129, 100, 37, 3, 0),
    (300, 768, 128, 6, 0),
    (257, 768, 129, 32, 0),
    (1000, 128, 700, 8, 0),
    (2000, 768, 1000, 6, 0),
    (513, 256, 300, 16, 40),
    (400, 64, 64, 32, 64),
    (300, 64, 32, 32, 0),     # fanout equal to the leader count
]


@pytest.mark.parametrize("rows,dim,leaders,fanout,near", CASES)
def test_d0_host_matches_oracle(oracle, rows, dim, leaders, fanout, near):
    from shear_b200 import ops
    raw, gids, lids, lv = random_case(rows, dim, leaders, seed=rows + dim + leaders + fanout, near_dup_leaders=near)
    want = oracle.d0_assign(raw, gids, lids, lv, fanout)
    _same(ops.quantize_sq8_and_assign_global_d0(raw, gids, lids, lv, fanout), want)


def test_d0_device_form_and_leader_payload(oracle):
    import torch
    from shear_b200 import ops
    raw, gids, lids, lv = random_case(700, 384, 200, seed=9)
    want = oracle.d0_assign(raw, gids, lids, lv, 5)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    got = ops.quantize_sq8_assign_d0(t(raw), t(gids.view(np.int32)), t(lids.view(np.int32)), 5,
                                     leader_vectors=t(lv))
    torch.cuda.synchronize()

    class H:
        pass
    h = H()
    h.codes = got.codes.cpu().numpy()
    h.scales = got.scales.cpu().numpy()
    h.norms = got.norms.cpu().numpy()
    h.child_ids = ops.as_u32(got.child_ids)
    h.point_ids = ops.as_u32(got.point_ids)
    h.dists = got.dists.cpu().numpy()
    _same(h, want)
    # a precomputed leader payload (host leader ids) gives the same fragments
    lc, ls, ln = oracle.quantize_sq8(lv)
    got2 = ops.quantize_sq8_assign_d0(t(raw), t(gids.view(np.int32)), torch.from_numpy(lids.view(np.int32)), 5,
                                      leader_payload=(t(lc), t(ls), t(ln)))
    torch.cuda.synchronize()
    assert np.array_equal(ops.as_u32(got2.child_ids), want["child_ids"])


def test_d0_duplicate_leader_ids_keep_the_earlier_index(oracle):
    from shear_b200 import ops
    raw, gids, lids, lv = random_case(300, 64, 50, seed=4)
    lids[10] = lids[20] = lids[30] = 7
    lv[20] = lv[10]
    lv[30] = lv[10]
    want = oracle.d0_assign(raw, gids, lids, lv, 4)
    got = ops.quantize_sq8_and_assign_global_d0(raw, gids, lids, lv, 4)
    _same(got, want)


def test_d0_rejects_invalid_requests():
    from shear_b200 import ops, TessaError
    lv = np.ones((2, 4), np.float32)
    with pytest.raises(TessaError, match="at least one input row"):
        ops.quantize_sq8_and_assign_global_d0(np.zeros((0, 4), np.float32), [], [1, 2], lv, 1)
    for f in (0, 3, 33):
        with pytest.raises(TessaError, match="fanout must be in"):
            ops.quantize_sq8_and_assign_global_d0(np.ones((1, 4), np.float32), [0], [1, 2], lv, f)
    bad = np.ones((3, 4), np.float32)
    bad[1, 2] = np.nan
    with pytest.raises(TessaError, match="NONFINITE"):
        ops.quantize_sq8_and_assign_global_d0(bad, [0, 1, 2], [1, 2], lv, 1)
    # the context stays usable after an error
    got = ops.quantize_sq8_and_assign_global_d0(np.ones((1, 4), np.float32), [9], [1, 2], lv, 2)
    assert got.fragments() == [(0, 9), (1, 9)]


def test_d0_host_pipeline_batches(oracle):
    # ~256 rows of f32 per batch: the host call uploads, assigns and downloads
    # in a dozen overlapping batches; results equal the single-call oracle.
    from shear_b200 import ops, TessaError
    raw, gids, lids, lv = random_case(3000, 64, 150, seed=21, near_dup_leaders=20)
    want = oracle.d0_assign(raw, gids, lids, lv, 7)
    try:
        ops.set_host_batch_bytes(256 * 64 * 4)
        got = ops.quantize_sq8_and_assign_global_d0(raw, gids, lids, lv, 7)
        _same(got, want)
        bad = raw.copy()
        bad[1700, 5] = np.inf
        with pytest.raises(TessaError, match="NONFINITE"):
            ops.quantize_sq8_and_assign_global_d0(bad, gids, lids, lv, 7)
        _same(ops.quantize_sq8_and_assign_global_d0(raw, gids, lids, lv, 7), want)
    finally:
        ops.set_host_batch_bytes(0)
