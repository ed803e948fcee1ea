"""Task former: the capacity logic against the reference's own tests
(P/d0_capacity.rs:298-479), and the B200 admission model."""
import pytest

from shear_b200 import task_former as tf


def test_config_default_uses_strict_ratios():
    cfg = tf.D0CapacityConfig()
    assert (cfg.high_ratio, cfg.target_ratio, cfg.low_ratio) == (0.60, 0.50, 0.15)


def test_thresholds_keep_target_below_high_and_low_below_target():
    cfg = tf.D0CapacityConfig(high_ratio=0.85, target_ratio=0.75, low_ratio=0.20, min_efficient_rows=32)
    t = tf.compute_thresholds(1_000, cfg)
    assert (t.c_gpu, t.c_high, t.c_target, t.c_low) == (1_000, 850, 750, 200)


def test_thresholds_clamp_target_when_config_exceeds_high():
    cfg = tf.D0CapacityConfig(high_ratio=0.60, target_ratio=0.90, low_ratio=0.20, min_efficient_rows=1)
    t = tf.compute_thresholds(1_000, cfg)
    assert (t.c_high, t.c_target, t.c_low) == (600, 600, 200)


def test_root_leader_plan_lifts_configured_leaders_to_capacity_target():
    cfg = tf.D0CapacityConfig(quality_min_root_leaders=64, root_leader_cap=10_000)
    t = tf.D0CapacityThresholds(400_000, 340_000, 300_000, 64_000)
    p = tf.plan_root_leaders(10_000_000, 6, t, cfg)
    assert (p.k_capacity, p.k_initial, p.root_leader_cap, p.root_leader_source) == (200, 200, 10_000, "capacity")


def test_root_leader_plan_preserves_quality_floor_when_capacity_target_is_lower():
    t = tf.D0CapacityThresholds(1_000_000, 850_000, 750_000, 64_000)
    p = tf.plan_root_leaders(1_000_000, 6, t, tf.D0CapacityConfig(quality_min_root_leaders=128, root_leader_cap=10_000))
    assert (p.k_capacity, p.k_initial, p.root_leader_source) == (8, 128, "quality_floor")
    c = tf.plan_root_leaders(20_000_000, 6, t, tf.D0CapacityConfig(quality_min_root_leaders=160, root_leader_cap=100))
    assert (c.k_capacity, c.k_initial, c.root_leader_cap, c.root_leader_source) == (160, 100, 100, "root_leader_cap")


def test_split_leader_count_is_minimum_capacity_cut():
    t = tf.D0CapacityThresholds(400_000, 340_000, 300_000, 64_000)
    assert [tf.split_leader_count(r, t) for r in (300_000, 341_000, 900_001)] == [1, 2, 4]


def test_child_size_observation_records_tail_and_small_counts():
    t = tf.D0CapacityThresholds(400_000, 340_000, 300_000, 64)
    tel = tf.D0CapacityTelemetry()
    tf.observe_child_unique_sizes(tel, t, [10, 100, 200, 300, 400_000])
    assert (tel.actual_child_max_unique_rows, tel.actual_child_p50_unique_rows, tel.actual_child_p95_unique_rows,
            tel.actual_child_p99_unique_rows) == (400_000, 200, 400_000, 400_000)
    assert (tel.oversized_child_count, tel.small_child_count, tel.small_child_rows) == (1, 1, 10)


def test_admission_binary_search_finds_the_boundary():
    budget = 24 * (1 << 30)  # the 35M config's per-GPU workspace cap
    r = tf.find_max_admissible_rows(768, 32, 3, budget)
    assert tf.plan_subtree_admission(r, 768, 32, 3, budget).supported
    assert not tf.plan_subtree_admission(r + 1, 768, 32, 3, budget).supported
    # leaf-ordered members skip the gather scratch: more rows fit
    assert tf.find_max_admissible_rows(768, 32, 3, budget, leaf_ordered=True) > r
    # raw f32 rows for the assignment: fewer rows fit
    assert tf.find_max_admissible_rows(768, 32, 3, budget, raw_assignment=True) < r
    assert tf.find_max_admissible_rows(0, 32, 3, budget) == 0
    assert tf.find_max_admissible_rows(768, 33, 3, budget) == 0  # k above the leaf kernel's 32


def test_b200_root_plan_for_the_35m_config():
    # The reference's resident-budget test (P/d0_capacity.rs:383-431) finds
    # capacity pressure for Wiki35M under its persistent-kernel queue model.
    # This library's footprint is about 3.8 KB per row at fanout 3 and leaf
    # k = 2 (codes, leaf batch with the column-split kernel's zone dump,
    # assignment): the 35M config's 24 GiB workspace admits ~6.8M-row subtrees,
    # where the quality floor (64 root leaders) binds; a 16 GiB workspace
    # admits ~4.6M rows and capacity binds (93 root leaders).
    cfg = tf.D0CapacityConfig()
    c_gpu = tf.find_max_admissible_rows(768, 2, 3, 24 * (1 << 30))
    p = tf.plan_root_leaders(35_000_000, 6, tf.compute_thresholds(c_gpu, cfg), cfg)
    assert 6_000_000 < c_gpu < 7_500_000
    assert p.k_capacity < cfg.quality_min_root_leaders
    assert (p.k_initial, p.root_leader_source) == (64, "quality_floor")
    small = tf.find_max_admissible_rows(768, 2, 3, 16 * (1 << 30))
    q = tf.plan_root_leaders(35_000_000, 6, tf.compute_thresholds(small, cfg), cfg)
    assert 4_000_000 < small < 5_000_000
    assert q.k_capacity > cfg.quality_min_root_leaders and q.root_leader_source == "capacity"


@pytest.mark.gpu
def test_admission_model_bounds_the_library_footprint():
    # run the leaf operator through the host-buffer call (the largest staging
    # user) on one subtree's worth of leaves and compare the context's device
    # bytes with the model
    import numpy as np
    from shear_b200 import ops
    rows, dim, k = 40_000, 256, 16
    rng = np.random.default_rng(0)
    codes = rng.integers(-127, 128, (rows, dim), dtype=np.int8)
    scales = np.full(rows, 0.01, np.float32)
    norms = np.ones(rows, np.float32)
    gids = np.arange(rows, dtype=np.uint32)
    members = rng.permutation(rows).astype(np.uint32)  # not leaf-ordered: the gather scratch is used
    sizes = np.full(rows // 1000, 1000, np.uint64)
    starts = (np.arange(sizes.size, dtype=np.uint64) * 1000).astype(np.uint64)
    ctx = ops.Context(0)
    try:
        before = tf.library_scratch_bytes(ctx)
        a = ops.C.LeafArgs
        ids = np.empty(rows * k, np.uint32)
        dists = np.empty(rows * k, np.float32)
        import ctypes
        args = a(codes=codes.ctypes.data, scales=scales.ctypes.data, norms=norms.ctypes.data,
                 global_ids=gids.ctypes.data, resident_rows=rows, padded_dim=dim, k=k,
                 leaf_members=members.ctypes.data, leaf_starts=starts.ctypes.data, leaf_sizes=sizes.ctypes.data,
                 leaf_count=sizes.size, leaf_rows=rows, topk_ids=ids.ctypes.data, topk_dists=dists.ctypes.data,
                 leaf_ordered_codes=None)
        ops.C.check(ops.C.load().tessa_leaf_topk_sq8_host(ctx.handle, ctypes.byref(args)))
        used = tf.library_scratch_bytes(ctx) - before
        model = tf.plan_subtree_admission(rows, dim, k, 1, None)
        assert 0 < used <= model.required_bytes, (used, model)
    finally:
        ctx.close()
