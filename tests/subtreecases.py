"""Seeded inputs for the subtree partition tests (shared by CPU and GPU tests)."""
import numpy as np


def clustered_rows(n, dim, comps, seed, sigma=0.3, unit=False):
    """Gaussian-mixture rows (centres ~N(0,1), isotropic sigma), as BASELINE's
    config 1 describes its data; optionally L2-normalised."""
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((comps, dim)).astype(np.float32)
    x = cent[rng.integers(0, comps, n)] + np.float32(sigma) * rng.standard_normal((n, dim)).astype(np.float32)
    if unit:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x, np.float32)


def seeds_for(counts, random_seed=42, parent_points=1_000_000, min_recurse_size=4096):
    """Per-task root seeds as gpu_queue_root_seed (CB:1597-1603) forms them."""
    from shear_b200.ops import subtree_root_seed
    return np.array([subtree_root_seed(random_seed, 1, int(c), parent_points, min_recurse_size) for c in counts],
                    np.uint64)


def oracle_leaves(oracle, codes, scales, norms, members, offsets, counts, seeds, params, psamp):
    rows, starts, sizes, tasks, stats = oracle.subtree_partition(codes, scales, norms, members, offsets, counts,
                                                                 seeds, params, psamp)
    leaves = [rows[int(s):int(s) + int(z)] for s, z in zip(starts, sizes)]
    return leaves, tasks, stats
