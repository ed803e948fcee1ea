"""End to end on the B200: SQ8 quantize -> leaf top-k -> sketches and edge
hashes -> host edge expansion -> graph file -> greedy search -> Recall@10
against GPU brute force.  The reducer here is a stand-in (each node keeps its
R nearest candidate edges); the reference's HashPrune / TierLift reducer is
host code outside this library.  The test checks that the pieces compose and
that the leaf lists carry the neighbourhoods the search needs."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_leaf_lists_to_graph_search_recall(tmp_path):
    import torch
    from shear_b200 import graph, ops
    rng = np.random.default_rng(0)
    dev = torch.device("cuda:0")
    # unclustered rows: a nearest-R stand-in reducer keeps such a graph connected
    # (exact float distances through the same steps give Recall@10 0.959 here)
    n, dim, k, R = 12000, 32, 16, 24
    x = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((200, dim)).astype(np.float32)
    xt = torch.from_numpy(x).to(dev)
    codes, scales, norms = ops.quantize_sq8(xt)
    gids = torch.arange(n, dtype=torch.int32, device=dev)
    # four overlapping partitions into leaves of 512 rows: sort by random projections
    layouts = []
    for s in range(4):
        proj = x @ rng.standard_normal(dim).astype(np.float32)
        layouts.append(np.argsort(proj, kind="stable").astype(np.uint32))
    planes = torch.from_numpy(rng.uniform(-1, 1, (12, dim)).astype(np.float32)).to(dev)
    sk = ops.sketch_rows(xt, planes)
    cand = [[] for _ in range(n)]
    for order in layouts:
        size = 512
        starts = np.arange(0, n, size, dtype=np.uint64)
        sizes = np.minimum(size, n - starts).astype(np.uint64)
        members = torch.from_numpy(order.view(np.int32)).to(dev)
        ids, dists = ops.leaf_topk_sq8(codes, scales, norms, gids, members, starts, sizes, k)
        point_ids = members  # global id = local id here
        hf, hr = ops.edge_hashes(point_ids, ids, k, sk, 12, starts, sizes)
        p, c, h, d = ops.expand_edges(order, ops.as_u32(ids), dists.cpu().numpy(), hf.cpu().numpy(),
                                      hr.cpu().numpy(), k)
        assert p.shape[0] == 2 * n * k
        for a, b, dd in zip(p.tolist(), c.tolist(), d.tolist()):
            cand[a].append((dd, b))
    adj = []
    for lst in cand:
        seen, keep = set(), []
        for dd, b in sorted(lst):
            if b not in seen:
                seen.add(b)
                keep.append(b)
            if len(keep) == R:
                break
        adj.append(keep)
    path = str(tmp_path / "g.index")
    graph.write_mem_graph(path, adj, start=0)
    off, nb, start, max_deg, _ = graph.read_mem_graph(path)
    assert max_deg <= R
    gt, _ = graph.exact_knn(xt, torch.from_numpy(q).to(dev), 10)
    res, _ = graph.search(x, off, nb, start, q, 10, 200)
    assert graph.recall_at(res, gt.cpu().numpy(), 10) > 0.9
