"""Subtree submissions (tessa_subtree_submit / poll / release) on the B200.

A submission is the reference's submit_owned_quantized_subtree_l2_compact_topk
with its two-slot persistent async D2H ring (P/persistent_async_d2h.rs): the
CompactTopKBatch it hands back must equal the synchronous path --
tessa_subtree_partition, then tessa_leaf_topk_sq8 over the same leaves, with
point ids mapped through the global ids -- and the leaves equal the oracle's
recursion.  The ring's contract: two slots, TESSA_ERR_AGAIN when both are
leased, views valid until release, stale tickets rejected, a failed
submission reports its error and frees its slot, the caller's context stays
usable meanwhile.
"""
import numpy as np
import pytest

from subtreecases import clustered_rows, oracle_leaves, seeds_for

pytestmark = pytest.mark.gpu


def _case(oracle, n, dim, sizes, seed):
    x = clustered_rows(n, dim, 32, seed=seed, unit=dim >= 256)
    codes, scales, norms = oracle.quantize_sq8(x)
    rng = np.random.default_rng(seed)
    members = np.concatenate([np.sort(rng.choice(n, size=s, replace=False)) for s in sizes]).astype(np.uint32)
    counts = np.array(sizes, np.uint32)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint64)
    gids = (np.arange(n, dtype=np.uint64) * 7 + 3).astype(np.uint32)  # ids distinct from row numbers
    return dict(codes=codes, scales=scales, norms=norms, members=members, counts=counts, offsets=offsets,
                seeds=seeds_for(counts), gids=gids)


def _dev(c):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dict(codes=t(c["codes"]), scales=t(c["scales"]), norms=t(c["norms"]),
                members=t(c["members"].view(np.int32)), gids=t(c["gids"].view(np.int32)))


def _sync_path(c, d, k, prm):
    from shear_b200 import ops
    rows, starts, sizes, tasks, _ = ops.subtree_partition(d["codes"], d["scales"], d["norms"], d["members"],
                                                          c["offsets"], c["counts"], c["seeds"], prm)
    ids, dists = ops.leaf_topk_sq8(d["codes"], d["scales"], d["norms"], d["gids"], rows, starts, sizes, k)
    r = ops.as_u32(rows)
    return r, starts, sizes, tasks, ops.as_u32(ids), dists.cpu().numpy()


def _check_view(v, c, sync, k):
    rows, starts, sizes, tasks, ids, dists = sync
    assert np.array_equal(v["leaf_starts"], starts) and np.array_equal(v["leaf_sizes"], sizes)
    assert np.array_equal(v["leaf_tasks"], tasks)
    for s, z in zip(starts, sizes):
        s, z = int(s), int(z)
        assert np.array_equal(v["point_ids"][s:s + z], c["gids"][rows[s:s + z]])
        assert np.array_equal(v["topk_ids"][s * k:(s + z) * k], ids[s * k:(s + z) * k])
        assert np.array_equal(v["topk_dists"][s * k:(s + z) * k].view(np.uint32),
                              dists[s * k:(s + z) * k].view(np.uint32))


def test_submissions_equal_the_synchronous_path_and_the_oracle(oracle):
    from shear_b200 import ops
    prm = ops.SubtreeParams(c_max=1024, max_depth=20)
    cases = [_case(oracle, 30000, 128, [9000, 1200, 14000], 1), _case(oracle, 12000, 768, [5000, 7000], 2)]
    devs = [_dev(c) for c in cases]
    k = 4
    tickets = [ops.subtree_submit(d["codes"], d["scales"], d["norms"], d["gids"], d["members"], c["offsets"],
                                  c["counts"], c["seeds"], k, prm) for c, d in zip(cases, devs)]
    assert tickets[1] == tickets[0] + 1
    for c, d, t in zip(cases, devs, tickets):
        v = ops.subtree_poll(t, wait=True)
        sync = _sync_path(c, d, k, prm)  # the caller's context runs while the slot is held
        _check_view(v, c, sync, k)
        want, wtasks, _ = oracle_leaves(oracle, c["codes"], c["scales"], c["norms"], c["members"], c["offsets"],
                                        c["counts"], c["seeds"], prm.as_array(), prm.psamp_fraction)
        got = [sync[0][int(s):int(s) + int(z)] for s, z in zip(v["leaf_starts"], v["leaf_sizes"])]
        assert len(got) == len(want) and all(np.array_equal(g, w) for g, w in zip(got, want))
        ops.subtree_release(t)


def test_ring_contract(oracle):
    from shear_b200 import ops, TessaError
    prm = ops.SubtreeParams(c_max=512, max_depth=20)
    c = _case(oracle, 8000, 64, [3000, 2500], 5)
    d = _dev(c)
    sub = lambda p=prm: ops.subtree_submit(d["codes"], d["scales"], d["norms"], d["gids"], d["members"],
                                           c["offsets"], c["counts"], c["seeds"], 2, p)
    t1, t2 = sub(), sub()
    with pytest.raises(TessaError, match="AGAIN"):
        sub()  # both slots leased
    v1 = ops.subtree_poll(t1)
    first = v1["topk_ids"].copy()
    v2 = ops.subtree_poll(t2)
    assert np.array_equal(v2["topk_ids"], first)  # same request, same batch
    ops.subtree_release(t1)
    with pytest.raises(TessaError, match="INVALID_ARG"):
        ops.subtree_release(t1)  # stale
    with pytest.raises(TessaError, match="INVALID_ARG"):
        ops.subtree_poll(t1)
    t3 = sub()  # a slot is free again
    assert np.array_equal(v2["topk_ids"], first)  # the held view is untouched by the next batch
    ops.subtree_release(t2)
    v3 = ops.subtree_poll(t3)
    assert np.array_equal(v3["topk_ids"], first)
    ops.subtree_release(t3)
    # a submission that cannot finish reports its error at poll and frees its slot
    bad = ops.SubtreeParams(c_max=512, max_depth=1)
    t4 = sub(bad)
    with pytest.raises(TessaError, match="PARTITION"):
        ops.subtree_poll(t4)
    t5, t6 = sub(), sub()
    for t in (t5, t6):
        assert ops.subtree_poll(t)["rows"] == v3["rows"]
        ops.subtree_release(t)
