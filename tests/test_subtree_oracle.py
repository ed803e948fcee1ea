"""CPU checks of the oracle's restatement of the reference's subtree recursion
(CB:16336-17381): structural invariants the reference's own plan relies on,
and the helper formulas against the reference's definitions."""
import numpy as np
import pytest

from subtreecases import clustered_rows, oracle_leaves, seeds_for


def _run(oracle, x, sizes, **kw):
    from shear_b200 import ops
    codes, scales, norms = oracle.quantize_sq8(x)
    members = np.arange(x.shape[0], dtype=np.uint32)[:sum(sizes)]
    offsets = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    counts = np.array(sizes, np.uint32)
    prm = ops.SubtreeParams(**kw)
    leaves, tasks, stats = oracle_leaves(oracle, codes, scales, norms, members, offsets, counts, seeds_for(counts),
                                         prm.as_array(), prm.psamp_fraction)
    return leaves, tasks, stats, prm, members, offsets, counts


def test_every_row_lands_in_fanout_leaves_of_its_task(oracle):
    x = clustered_rows(40000, 64, 32, seed=1)
    sizes = [25000, 15000]
    # leaves of 512 rows need more levels than the default max_depth 10 gives
    leaves, tasks, stats, prm, members, offsets, counts = _run(oracle, x, sizes, c_max=512, fanout_second=3,
                                                               max_depth=20)
    assert stats["rounds"] >= 2
    for t in range(2):
        rows = np.concatenate([l for l, tk in zip(leaves, tasks) if tk == t])
        _, c = np.unique(rows, return_counts=True)
        # large root: each row goes to fanout_second children, deeper levels partition
        assert c.min() == 3 and c.max() == 3
        lo, hi = int(offsets[t]), int(offsets[t]) + int(counts[t])
        assert set(rows.tolist()) == set(range(lo, hi))
    assert all(l.size <= prm.leaf_max for l in leaves)
    assert all(np.all(np.diff(l.astype(np.int64)) > 0) for l in leaves)  # ascending, distinct


def test_partition_is_deterministic(oracle):
    x = clustered_rows(20000, 64, 16, seed=3)
    a = _run(oracle, x, [20000], c_max=256, max_depth=30)
    b = _run(oracle, x, [20000], c_max=256, max_depth=30)
    assert len(a[0]) == len(b[0]) and all(np.array_equal(p, q) for p, q in zip(a[0], b[0]))


def test_small_root_merges_children_below_leaf_min(oracle):
    # a 1000-row root takes the small path (1000 * 3 <= 4096)
    x = clustered_rows(1000, 32, 4, seed=6)
    leaves, tasks, stats, prm, *_ = _run(oracle, x, [1000], c_max=1024)
    assert stats["small_nodes"] == 1 and stats["large_assignments"] == 0
    assert all(l.size >= prm.leaf_min or len(leaves) == 1 for l in leaves)


def test_duplicates_force_retries(oracle):
    base = np.random.default_rng(2).standard_normal((2, 16)).astype(np.float32)
    x = np.repeat(base, 3000, axis=0)
    leaves, tasks, stats, prm, *_ = _run(oracle, x, [6000], c_max=256, fanout_second=2, max_depth=30)
    assert stats["retries"] > 0
    assert all(l.size <= prm.leaf_max for l in leaves)


@pytest.mark.parametrize("n,depth,want", [(50, 0, 0.001), (100000, 0, 0.0007), (100000, 1, 0.00056),
                                          (5_000_000, 3, 0.0001), (30_000_000, 6, 0.00005), (10, 0, 0.001)])
def test_adaptive_psamp_fraction(oracle, n, depth, want):
    # CB:7044-7075 with base 0.001
    got = float(oracle.lib().oracle_adaptive_psamp(np.float32(0.001), n, depth))
    assert abs(got - want) <= 1e-9 + 1e-6 * want


def test_root_seed_formula():
    # CB:1597-1603: random_seed ^ depth*phi ^ rotl(len,17) ^ rotl(parent,7) ^ rotl(min_recurse,29)
    from shear_b200.ops import subtree_root_seed
    rotl = lambda v, r: ((v << r) | (v >> (64 - r))) & (2 ** 64 - 1)
    want = 42 ^ ((1 * 0x9E3779B97F4A7C15) % 2 ** 64) ^ rotl(1000, 17) ^ rotl(5000, 7) ^ rotl(4096, 29)
    assert subtree_root_seed(42, 1, 1000, 5000, 4096) == want
