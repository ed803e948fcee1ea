"""Candidate-edge support on the B200: per-point sketches (fill_sketch_row,
P/hash_prune.rs:2208-2232) and the forward / reverse hashes of every leaf slot
(P/leaf_build.rs:1749-1808, compute_hash P/hash_prune.rs:2239-2251), checked
bit for bit against the oracle restatement."""
import numpy as np
import pytest

from leafcases import make_leaf_batch, oracle_leaf

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,dim,m", [(5000, 768, 12), (333, 100, 16), (64, 37, 1), (1, 8, 12)])
def test_sketch_rows_match_oracle(oracle, rows, dim, m):
    import torch
    from shear_b200 import ops
    rng = np.random.default_rng(rows + dim + m)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    planes = rng.uniform(-1, 1, (m, dim)).astype(np.float32)
    got = ops.sketch_rows(torch.from_numpy(x).cuda(), torch.from_numpy(planes).cuda()).cpu().numpy()
    want = oracle.sketch_rows(x, planes)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("sizes,k,m_bits,width", [([700, 300], 32, 12, 12), ([129, 2048], 8, 16, 16),
                                                  ([40], 2, 1, 16), ([300, 200], 5, 12, 13)])
def test_leaf_edges_match_oracle_flush(oracle, sizes, k, m_bits, width):
    import torch
    from shear_b200 import ops
    dev = torch.device("cuda:0")
    c = make_leaf_batch(oracle, sizes, 128, seed=sum(sizes) + k, dup=True, permute=True)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    ids, dists = ops.leaf_topk_sq8(t(c["codes"]), t(c["scales"]), t(c["norms"]), t(c["gids"].view(np.int32)),
                                   t(c["members"].view(np.int32)), c["starts"], c["sizes"], k)
    # sketch store over every global id the batch can reference
    n_points = int(c["gids"].max()) + 1
    rng = np.random.default_rng(k)
    pts = rng.standard_normal((n_points, 64)).astype(np.float32)
    planes = rng.uniform(-1, 1, (width, 64)).astype(np.float32)  # width 13: the scalar-load path
    sk_dev = ops.sketch_rows(t(pts), t(planes))
    point_ids = c["gids"][c["members"]]  # global id of each leaf row, leaf order
    want_ids, want_d = oracle_leaf(oracle, c, k)
    want = oracle.flush_edges(point_ids, want_ids, want_d, k, oracle.sketch_rows(pts, planes), m_bits)
    for layout in ((c["starts"], c["sizes"]), (None, None)):  # staged per leaf, and direct gathers
        hf, hr = ops.edge_hashes(t(point_ids.view(np.int32)), ids, k, sk_dev, m_bits, *layout)
        torch.cuda.synchronize()
        got = ops.expand_edges(point_ids, ops.as_u32(ids), dists.cpu().numpy(), hf.cpu().numpy(), hr.cpu().numpy(), k)
        for g, w in zip(got, want):
            assert np.array_equal(g.view(np.uint8), w.view(np.uint8))
        assert got[0].shape[0] == 2 * int(np.sum(want_ids != 0xFFFFFFFF))


def test_edge_hashes_reject_bad_arguments():
    import torch
    from shear_b200 import ops, TessaError
    sk = torch.zeros((10, 12), device="cuda")
    pid = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    ids = torch.tensor([2, 1, 1, 50], dtype=torch.int32, device="cuda")
    with pytest.raises(TessaError, match="INVALID_ARG"):
        ops.edge_hashes(pid, ids, 2, sk, 13)
    with pytest.raises(TessaError, match="BAD_ROW"):
        ops.edge_hashes(pid, ids, 2, sk, 12)
    with pytest.raises(TessaError, match="BAD_TASK"):  # candidate 7 is not a member of the leaf {1, 2}
        ops.edge_hashes(pid, torch.tensor([2, 1, 1, 7], dtype=torch.int32, device="cuda"), 2, sk, 12, [0], [2])
    hf, hr = ops.edge_hashes(pid, ids.clone().fill_(1), 2, sk, 12)  # the context stays usable
    # equal sketches: sketch_c - sketch_p = 0 >= 0 sets every bit in both directions
    assert (hf.to(torch.int32) & 0xFFFF).tolist() == [0xFFF] * 4 and (hr.to(torch.int32) & 0xFFFF).tolist() == [0xFFF] * 4
