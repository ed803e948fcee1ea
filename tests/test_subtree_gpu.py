"""Subtree partition (tessa_subtree_partition) on the B200 vs the oracle.

The leaves must match the C restatement of the reference's recursion
(CB:16336-17381) exactly: same leaves in the same (round) order, same task,
same resident rows in the same order.
"""
import numpy as np
import pytest

from subtreecases import clustered_rows, oracle_leaves, seeds_for

pytestmark = pytest.mark.gpu


def _gpu_leaves(codes, scales, norms, members, offsets, counts, seeds, params):
    import torch
    from shear_b200 import ops
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    rows, starts, sizes, tasks, stats = ops.subtree_partition(t(codes), t(scales), t(norms),
                                                              t(members.view(np.int32)), offsets, counts, seeds,
                                                              params)
    torch.cuda.synchronize()
    rows = ops.as_u32(rows)
    leaves = [rows[int(s):int(s) + int(z)] for s, z in zip(starts, sizes)]
    return leaves, tasks, stats


def _assert_same(oracle, codes, scales, norms, members, offsets, counts, seeds, params):
    got, gtasks, gstats = _gpu_leaves(codes, scales, norms, members, offsets, counts, seeds, params)
    want, wtasks, wstats = oracle_leaves(oracle, codes, scales, norms, members, offsets, counts, seeds,
                                         params.as_array(), params.psamp_fraction)
    assert len(got) == len(want), (len(got), len(want), gstats, wstats)
    assert np.array_equal(gtasks, wtasks)
    for i, (g, w) in enumerate(zip(got, want)):
        assert np.array_equal(g, w), f"leaf {i}: {g[:8]} vs {w[:8]} (sizes {g.size} {w.size})"
    for key in ("rounds", "large_assignments", "retries", "balanced", "small_nodes"):
        assert gstats[key] == wstats[key], (key, gstats, wstats)
    return gstats


def test_partition_matches_oracle_clustered_tasks(oracle):
    from shear_b200 import ops
    x = clustered_rows(60000, 128, 64, seed=0)
    codes, scales, norms = oracle.quantize_sq8(x)
    # a large, a small-path (1000 x 3 <= 4096) and a probe-overflow (1500 x 3 > 4096) root
    sizes = [30000, 1000, 1500, 27500]
    members = np.arange(60000, dtype=np.uint32)
    offsets = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    st = _assert_same(oracle, codes, scales, norms, members, offsets, np.array(sizes, np.uint32),
                      seeds_for(sizes), ops.SubtreeParams(c_max=1024, max_depth=20))
    assert st["small_nodes"] == 1 and st["rounds"] >= 3


def test_partition_matches_oracle_overlapping_768d_tasks(oracle):
    # D0-style child runs: each row in two tasks, 768-d unit rows, leaf_max 2048
    from shear_b200 import ops
    rng = np.random.default_rng(4)
    x = clustered_rows(40000, 768, 32, seed=4, unit=True)
    codes, scales, norms = oracle.quantize_sq8(x)
    tasks = []
    for t in range(5):
        m = np.sort(rng.choice(40000, size=int(rng.integers(3000, 16000)), replace=False)).astype(np.uint32)
        tasks.append(m)
    members = np.concatenate(tasks)
    counts = np.array([m.size for m in tasks], np.uint32)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint64)
    _assert_same(oracle, codes, scales, norms, members, offsets, counts, seeds_for(counts),
                 ops.SubtreeParams(c_max=2048))


def test_partition_duplicate_rows_retry(oracle):
    # four distinct rows repeated 2500 times: distances tie exactly, the hash
    # tie keys decide, and some splits are not meaningful, so the large path
    # resamples its leaders (retry rounds)
    from shear_b200 import ops
    rng = np.random.default_rng(9)
    base = rng.standard_normal((4, 64)).astype(np.float32)
    x = np.repeat(base, 2500, axis=0)
    codes, scales, norms = oracle.quantize_sq8(x)
    members = np.arange(10000, dtype=np.uint32)
    counts = np.array([10000], np.uint32)
    st = _assert_same(oracle, codes, scales, norms, members, np.array([0], np.uint64), counts, seeds_for(counts),
                      ops.SubtreeParams(c_max=256, fanout_second=2, max_depth=30))
    assert st["retries"] > 0


def test_partition_tiny_tasks_and_fanout_one(oracle):
    from shear_b200 import ops
    x = clustered_rows(3000, 32, 8, seed=2)
    codes, scales, norms = oracle.quantize_sq8(x)
    sizes = [1, 2, 5, 64, 300, 2000, 628]
    members = np.arange(3000, dtype=np.uint32)
    offsets = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    counts = np.array(sizes, np.uint32)
    for fs in (1, 2, 4):
        _assert_same(oracle, codes, scales, norms, members, offsets, counts, seeds_for(counts),
                     ops.SubtreeParams(c_max=256, fanout_second=fs, max_depth=30))


def test_partition_depth_limit_is_an_error(oracle):
    from shear_b200 import ops, TessaError
    x = clustered_rows(20000, 32, 4, seed=5)
    codes, scales, norms = oracle.quantize_sq8(x)
    members = np.arange(20000, dtype=np.uint32)
    counts = np.array([20000], np.uint32)
    prm = ops.SubtreeParams(c_max=256, max_depth=2)
    with pytest.raises(ValueError, match="oversized"):
        oracle_leaves(oracle, codes, scales, norms, members, np.array([0], np.uint64), counts, seeds_for(counts),
                      prm.as_array(), prm.psamp_fraction)
    with pytest.raises(TessaError, match="PARTITION"):
        _gpu_leaves(codes, scales, norms, members, np.array([0], np.uint64), counts, seeds_for(counts), prm)
