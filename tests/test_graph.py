"""Index graph file format (pipnn_oom_writer.rs:22-79), greedy search
(apps/search_shear_index/src/main.rs:1007-1085) and Recall@k (:388-413)."""
import heapq
import struct

import numpy as np
import pytest


def test_mem_graph_layout_and_round_trip(tmp_path):
    from shear_b200 import graph
    p = str(tmp_path / "g.index")
    size = graph.write_mem_graph(p, [[1, 2], [0], []], start=0, num_frozen_pts=0)
    want = struct.pack("<QIIQ", 48, 2, 0, 0) + struct.pack("<III", 2, 1, 2) + struct.pack("<II", 1, 0) + \
        struct.pack("<I", 0)
    assert size == 48 and open(p, "rb").read() == want
    off, nb, start, max_deg, frozen = graph.read_mem_graph(p)
    assert off.tolist() == [0, 2, 3, 3] and nb.tolist() == [1, 2, 0] and (start, max_deg, frozen) == (0, 2, 0)


def _l2(a, b):
    s = np.float32(0)
    for x, y in zip(a, b):
        d = np.float32(x - y)
        s = np.float32(s + np.float32(d * d))
    return s


def _py_search(q, data, adj, start, k, l):
    # transliteration of search_one_with_stats with (distance, id) heaps
    l_eff = max(l, k + 1)
    visited = {start}
    d0 = _l2(q, data[start])
    cand = [(d0, start)]
    best = [(-d0, -start)]
    while cand:
        cd, cid = heapq.heappop(cand)
        if len(best) >= l_eff and cd > -best[0][0]:
            break
        for nb in adj[cid]:
            if nb in visited:
                continue
            visited.add(nb)
            d = _l2(q, data[nb])
            heapq.heappush(cand, (d, nb))
            heapq.heappush(best, (-d, -nb))
            while len(best) > l_eff:
                heapq.heappop(best)
    res = sorted((-d, -i) for d, i in best)
    return [i for _, i in res[:k]] + [0xFFFFFFFF] * max(0, k - len(res))


def _knn_graph(data, r):
    d = ((data[:, None, :] - data[None, :, :]) ** 2).sum(-1)
    np.fill_diagonal(d, np.inf)
    return [list(np.argsort(row, kind="stable")[:r]) for row in d]


def test_search_matches_transliteration_and_recall():
    from shear_b200 import graph
    rng = np.random.default_rng(0)
    data = rng.standard_normal((400, 16)).astype(np.float32)
    queries = rng.standard_normal((25, 16)).astype(np.float32)
    adj = _knn_graph(data, 8)
    offsets = np.concatenate([[0], np.cumsum([len(a) for a in adj])]).astype(np.uint64)
    nbrs = np.concatenate(adj).astype(np.uint32)
    for k, l in ((10, 10), (5, 40), (1, 2)):
        got, comps = graph.search(data, offsets, nbrs, 7, queries, k, l, threads=3)
        for qi in range(len(queries)):
            assert got[qi].tolist() == _py_search(queries[qi], data, adj, 7, k, l)
        assert comps > 0
    gt = np.argsort(((queries[:, None, :] - data[None, :, :]) ** 2).sum(-1), axis=1)[:, :10]
    got, _ = graph.search(data, offsets, nbrs, 7, queries, 10, 200)
    assert graph.recall_at(got, gt, 10) >= 0.95


def test_recall_at_counts_ground_truth_hits():
    from shear_b200 import graph
    assert graph.recall_at([[1, 2, 3], [4, 5, 6]], [[3, 2, 9, 9], [7, 8, 9, 4]], 3) == pytest.approx((2 / 3 + 0) / 2)


def test_graph_search_rejects_bad_start():
    from shear_b200 import graph, TessaError
    data = np.zeros((3, 2), np.float32)
    with pytest.raises(TessaError, match="INVALID_ARG"):
        graph.search(data, np.array([0, 0, 0, 0], np.uint64), np.zeros(0, np.uint32), 5, data, 1, 2)


@pytest.mark.gpu
def test_exact_knn_matches_numpy():
    import torch
    from shear_b200 import graph
    rng = np.random.default_rng(5)
    base = rng.standard_normal((20000, 96)).astype(np.float32)
    q = rng.standard_normal((300, 96)).astype(np.float32)
    ids, d = graph.exact_knn(torch.from_numpy(base).cuda(), torch.from_numpy(q).cuda(), 10, block=128)
    want = np.argsort(((q.astype(np.float64)[:, None, :] - base[None, :, :]) ** 2).sum(-1), axis=1)[:, :10]
    # the product form rounds differently from the direct sum: compare as sets, allow a rare boundary swap
    agree = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ids.cpu().numpy(), want)])
    assert agree > 0.999
