"""Host HashPrune reducer (tessa_reducer_*) against the Python restatement of
the reference's reservoir (oracle/hashprune.py, P/hash_prune.rs:1326-1452).
Host code: runs without a GPU."""
import numpy as np
import pytest

from oracle import hashprune as HP


def _batches(rng, points, rows_per, k, nb, m_bits, dup_dist=False):
    out = []
    for _ in range(nb):
        pid = rng.integers(0, points, rows_per).astype(np.uint32)
        ids = rng.integers(0, points, (rows_per, k)).astype(np.uint32)
        ids[rng.random((rows_per, k)) < 0.05] = 0xFFFFFFFF
        ds = rng.random((rows_per, k)).astype(np.float32)
        if dup_dist:
            ds = np.round(ds * 8).astype(np.float32) / np.float32(8)  # many exact distance ties
        ds[rng.random((rows_per, k)) < 0.02] = np.inf
        hf = rng.integers(0, 1 << m_bits, (rows_per, k)).astype(np.uint16)
        hr = rng.integers(0, 1 << m_bits, (rows_per, k)).astype(np.uint16)
        out.append((pid, ids, ds, hf, hr, k))
    return out


@pytest.mark.parametrize("points,l_max,m_bits,dup", [(50, 8, 4, False), (200, 16, 6, True), (30, 64, 12, False),
                                                     (120, 5, 3, True)])
@pytest.mark.parametrize("threads", [1, 3])
def test_reducer_matches_reservoir_restatement(points, l_max, m_bits, dup, threads):
    from shear_b200 import ops
    rng = np.random.default_rng(points + l_max + m_bits)
    batches = _batches(rng, points, 300, 3, 4, m_bits, dup)
    want = HP.reduce_leaf_batches(points, l_max, batches)
    red = ops.Reducer(points, l_max, threads)
    for b in batches:
        red.add(*b)
    offsets, nb = red.finish()
    red.close()
    got = [nb[int(offsets[p]):int(offsets[p + 1])].tolist() for p in range(points)]
    assert got == want


def test_reducer_result_does_not_depend_on_batch_order():
    from shear_b200 import ops
    rng = np.random.default_rng(5)
    batches = _batches(rng, 500, 2000, 2, 6, 8)
    res = []
    for order in (batches, batches[::-1]):
        red = ops.Reducer(500, 32, 4)
        for b in order:
            red.add(*b)
        res.append(red.finish())
        red.close()
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])


def test_reducer_rejects_out_of_range_ids():
    from shear_b200 import ops, TessaError
    red = ops.Reducer(10, 4, 1)
    with pytest.raises(TessaError, match="BAD_ROW"):
        red.add(np.array([3], np.uint32), np.array([[11]], np.uint32), np.array([[0.5]], np.float32),
                np.array([[1]], np.uint16), np.array([[2]], np.uint16), 1)
    red.close()


def _group_on_host(batch, points):
    """Edges of one record batch grouped by reservoir (numpy), as tessa_group_edges lays them out."""
    from shear_b200.ops import EDGE_DTYPE
    pid, ids, ds, hf, hr, k = batch
    ids = ids.reshape(-1)
    ds = ds.reshape(-1)
    src = np.repeat(pid, k)
    ok = (ids != 0xFFFFFFFF) & np.isfinite(ds)
    s1, t1, h1, d1 = src[ok], ids[ok], hf.reshape(-1)[ok], ds[ok]
    s2, t2, h2 = t1, s1, hr.reshape(-1)[ok]
    s = np.concatenate([s1, s2])
    e = np.zeros(s.size, EDGE_DTYPE)
    e["target"] = np.concatenate([t1, t2])
    e["dist"] = np.concatenate([d1, d1])
    e["hash"] = np.concatenate([h1, h2])
    order = np.argsort(s, kind="stable")
    offsets = np.concatenate([[0], np.cumsum(np.bincount(s, minlength=points))]).astype(np.uint64)
    return offsets, e[order]


@pytest.mark.parametrize("threads", [1, 4])
def test_grouped_add_equals_record_add(threads):
    from shear_b200 import ops
    rng = np.random.default_rng(12)
    batches = _batches(rng, 400, 3000, 2, 3, 8, dup_dist=True)
    a = ops.Reducer(400, 24, threads)
    b = ops.Reducer(400, 24, threads)
    for bt in batches:
        a.add(*bt)
        b.add_grouped(*_group_on_host(bt, 400))
    ra, rb = a.finish(), b.finish()
    a.close()
    b.close()
    assert np.array_equal(ra[0], rb[0]) and np.array_equal(ra[1], rb[1])
