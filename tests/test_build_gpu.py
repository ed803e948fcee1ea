"""End-to-end GPU-subtree build (shear_b200.index.build_index) on the B200.

The GPU build and the CPU restatement (oracle/cpu_build.py) take the same
seeded inputs; every stage between them is restated exactly, so the graphs --
and therefore recall -- must be identical, not merely close.
"""
import numpy as np
import pytest

from subtreecases import clustered_rows

pytestmark = pytest.mark.gpu


def _recall(x, offsets, nb, entry, queries, l=100):
    import torch
    from shear_b200 import graph as G
    xd = torch.from_numpy(x).cuda()
    qd = torch.from_numpy(queries).cuda()
    gt, _ = G.exact_knn(xd, qd, 10)
    ids, _ = G.search(x, offsets, nb, entry, queries, 10, l)
    return G.recall_at(ids, gt.cpu().numpy(), 10)


@pytest.mark.parametrize("reduction", ["device", "host"])
@pytest.mark.parametrize("n,dim,c_max,fanout_top", [(20000, 128, 1024, 10), (12000, 768, 2048, 4)])
def test_gpu_build_graph_equals_cpu_restatement(oracle, n, dim, c_max, fanout_top, reduction):
    # device: HashPrune reservoirs on the GPU; host: grouped records reduced by
    # the host reducer.  The CPU restatement inserts every record on the host.
    from oracle.cpu_build import build_index_cpu
    from shear_b200.index import BuildParams, build_index
    x = clustered_rows(n, dim, 64, seed=n + dim, unit=dim == 768)
    p = BuildParams(c_max=c_max, fanout_top=fanout_top, reduction=reduction)
    r = build_index(x, p)
    offs, nb, entry, _, st = build_index_cpu(x, p, r.stats["root_leaders"])
    assert r.stats["leaves"] == st["leaves"] and r.stats["leaf_rows"] == st["leaf_rows"]
    assert r.entry_point == entry
    assert np.array_equal(r.offsets, offs)
    assert np.array_equal(r.neighbors, nb)
    deg = r.degree_stats()
    assert 1 <= deg["mean"] <= p.l_max and deg["max"] <= p.l_max


def test_gpu_build_recall_on_clustered_data(oracle):
    from shear_b200.index import BuildParams, build_index
    xq = clustered_rows(30300, 128, 64, seed=11)  # base rows and queries from one mixture
    x, q = np.ascontiguousarray(xq[:30000]), np.ascontiguousarray(xq[30000:])
    r = build_index(x, BuildParams(c_max=1024))
    rec = _recall(x, r.offsets, r.neighbors, r.entry_point, q)
    assert rec > 0.8, rec


def test_gpu_build_from_device_tensor_equals_host_input(oracle):
    import torch
    from shear_b200.index import BuildParams, build_index
    x = clustered_rows(8000, 64, 16, seed=3)
    p = BuildParams(c_max=512, max_depth=20)
    a = build_index(x, p)
    b = build_index(torch.from_numpy(x).cuda(), p)
    assert np.array_equal(a.offsets, b.offsets) and np.array_equal(a.neighbors, b.neighbors)


@pytest.mark.parametrize("batch_rows,call_rows", [(30000, None), (70000, None), (70000, 6000)])
def test_gpu_build_in_record_batches_equals_one_pass(oracle, batch_rows, call_rows):
    # The child runs split into record batches (partition, leaves and partial
    # reservoirs per batch, merged at the end; optionally each batch's leaves
    # in several leaf calls) give the one-pass graph.
    from shear_b200.index import BuildParams, build_index
    x = clustered_rows(20000, 128, 64, seed=7)
    one = build_index(x, BuildParams(c_max=1024))
    p = BuildParams(c_max=1024, record_batch_rows=batch_rows, leaf_call_rows=call_rows)
    r = build_index(x, p)
    assert r.stats["record_batches"] > 1
    assert r.stats["leaves"] == one.stats["leaves"] and r.stats["leaf_rows"] == one.stats["leaf_rows"]
    assert r.entry_point == one.entry_point
    assert np.array_equal(r.offsets, one.offsets)
    assert np.array_equal(r.neighbors, one.neighbors)
