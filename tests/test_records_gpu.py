"""tessa_group_edges on the B200: every reservoir's group holds exactly the
distinct edges flush_compact_topk_batch_into_edges forms (P/leaf_build.rs:
1749-1808), ascending by target, and the reducer fed with the groups equals
the reducer fed with the records (repeated edges included)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_group_edges_matches_host_grouping_and_reducer():
    import torch
    from shear_b200 import ops
    from test_reducer import _batches, _group_on_host
    rng = np.random.default_rng(3)
    points, k = 5000, 3
    (batch,) = _batches(rng, points, 40000, k, 1, 12, dup_dist=True)
    pid, ids, ds, hf, hr, _ = batch
    # repeat some records exactly (overlapping leaves do) so the grouping drops copies
    rep = rng.integers(0, pid.size, 8000)
    pid, ids, ds = np.concatenate([pid, pid[rep]]), np.concatenate([ids, ids[rep]]), np.concatenate([ds, ds[rep]])
    hf, hr = np.concatenate([hf, hf[rep]]), np.concatenate([hr, hr[rep]])
    batch = (pid, ids, ds, hf, hr, k)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    offsets, edges = ops.group_edges(t(pid.view(np.int32)), t(ids.view(np.int32).reshape(-1)), t(ds.reshape(-1)),
                                     t(hf.view(np.int16).reshape(-1)), t(hr.view(np.int16).reshape(-1)), k, points)
    torch.cuda.synchronize()
    off = offsets.cpu().numpy().view(np.uint64)
    e = edges.cpu().numpy()[:int(off[-1]) * 12].view(ops.EDGE_DTYPE)
    want_off, want_e = _group_on_host(batch, points)
    assert int(off[-1]) < int(want_off[-1])  # the batch repeats edges; repeats are dropped
    for p in range(points):
        a = e[int(off[p]):int(off[p + 1])]
        b = np.unique(want_e[int(want_off[p]):int(want_off[p + 1])])
        assert np.array_equal(np.sort(a, order=["target", "hash", "dist"]), np.sort(b, order=["target", "hash",
                                                                                                "dist"])), p
        assert np.all(np.diff(a["target"].astype(np.int64)) >= 0), p
    r1 = ops.Reducer(points, 32, 4)
    r1.add(*batch)
    r2 = ops.Reducer(points, 32, 4)
    r2.add_grouped(off, e)
    a, b = r1.finish(), r2.finish()
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_group_edges_rejects_out_of_range_ids():
    import torch
    from shear_b200 import ops, TessaError
    dev = torch.device("cuda:0")
    pid = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    ids = torch.tensor([1, 7], dtype=torch.int32, device=dev)
    ds = torch.tensor([0.5, 0.25], device=dev)
    h = torch.zeros(2, dtype=torch.int16, device=dev)
    with pytest.raises(TessaError, match="BAD_ROW"):
        ops.group_edges(pid, ids, ds, h, h, 1, 4)
