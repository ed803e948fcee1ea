"""Seeded leaf-batch generators shared by the GPU parity tests."""
import numpy as np


def make_leaf_batch(oracle, sizes, dim, seed, *, dup=False, permute=False, normalize=True, formula=None):
    rng = np.random.default_rng(seed)
    rows = int(sum(sizes))
    if formula is not None:
        x = formula(rows, dim)
    else:
        x = rng.standard_normal((rows, dim)).astype(np.float32)
        if normalize:
            x /= np.linalg.norm(x, axis=1, keepdims=True)
    if dup and rows > 6:
        x[2] = x[1]
        x[5] = x[4]
    codes, scales, norms = oracle.quantize_sq8(x)
    gids = rng.permutation(rows * 3)[:rows].astype(np.uint32)
    members = np.arange(rows, dtype=np.uint32)
    if permute:
        members = rng.permutation(rows).astype(np.uint32)
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    return dict(x=x, codes=codes, scales=scales, norms=norms, gids=gids, members=members,
                starts=starts, sizes=np.asarray(sizes, np.uint64))


def oracle_leaf(oracle, c, k):
    return oracle.leaf_topk_sq8(c["codes"], c["scales"], c["norms"], c["gids"], c["members"], c["starts"],
                                c["sizes"], k)
