"""CPU restatement of the GPU-subtree build (test infrastructure and the
bench's CPU baseline; never part of the shipped path).

The same stages as shear_b200.index.build_index, each on the host through
the C restatement in tessa_oracle.c (OpenMP): D0 quantize + root assignment
(P/dco_sq_int8.rs:1929-2070), child runs, the recursive subtree partition
(compute_backend.rs:16336-17381), leaf top-k (CB:8987-9002, CB:7229-7259),
sketches and slot hashes (hash_prune.rs:2208-2251), and the host HashPrune
reducer -- the reservoir stage, which SHEAR runs on the CPU in every build,
shared with the GPU build.  With the same inputs both builds produce the same
graph.
"""
from __future__ import annotations

import time

import numpy as np

from . import oracle as O


def build_index_cpu(x, p, root_leaders: int, threads: int = 0):
    """x: f32 [n, dim] host rows; p: shear_b200.index.BuildParams;
    root_leaders: the D0 leader count (the GPU build's capacity plan).
    Returns (offsets, neighbors, entry_point, timings, stats)."""
    from shear_b200 import index as IX
    from shear_b200 import ops

    timings = {}
    t_all = time.perf_counter()
    x = np.ascontiguousarray(x, np.float32)
    n, dim = x.shape
    k0 = int(root_leaders)
    fanout = min(p.fanout_top, k0)
    leaders = IX.sample_root_leaders(n, k0, p.random_seed)
    t = time.perf_counter()
    d0 = O.d0_assign(x, np.arange(n, dtype=np.uint32), leaders, x[leaders.astype(np.int64)], fanout)
    child = d0["child_ids"].astype(np.int64)
    keys = child.reshape(-1)
    order = np.argsort(keys, kind="stable")
    members = (order // fanout).astype(np.uint32)
    counts = np.bincount(keys, minlength=k0).astype(np.uint32)
    offsets = np.concatenate([[0], np.cumsum(counts, dtype=np.uint64)[:-1]]).astype(np.uint64)
    timings["d0_s"] = time.perf_counter() - t
    t = time.perf_counter()
    depth, parent, min_rec = IX.child_seed_args(p, n)
    seeds = np.array([ops.subtree_root_seed(p.random_seed, depth, int(c), parent, min_rec) for c in counts],
                     np.uint64)
    sp = ops.SubtreeParams(c_max=p.adaptive_c_max(n), max_depth=p.max_depth, max_leaders=p.max_leaders,
                           fanout_second=p.fanout_second, root_depth=depth, psamp_fraction=p.psamp_fraction)
    rows, starts, sizes, tasks, pst = O.subtree_partition(d0["codes"], d0["scales"], d0["norms"], members, offsets,
                                                          counts, seeds, sp.as_array(), sp.psamp_fraction)
    timings["partition_s"] = time.perf_counter() - t
    t = time.perf_counter()
    k = max(1, min(p.leaf_knn, 32))
    ids, dists = O.leaf_topk_sq8(d0["codes"], d0["scales"], d0["norms"], np.arange(n, dtype=np.uint32), rows,
                                 starts, sizes.astype(np.uint64), k)
    planes = IX.hyperplanes(p.m_hash_bits, dim, p.random_seed)
    sketches = O.sketch_rows(x, planes)
    hf, hr = O.slot_hashes(rows, ids, k, sketches, p.m_hash_bits)
    timings["leaf_s"] = time.perf_counter() - t
    t = time.perf_counter()
    red = ops.Reducer(n, p.l_max, threads)
    red.add(rows, ids, dists, hf, hr, k)
    offs, nb = red.finish()
    red.close()
    timings["reduce_s"] = time.perf_counter() - t
    timings["total_s"] = time.perf_counter() - t_all
    big = int(len(counts) - 1 - np.argmax(counts[::-1]))
    entry = int(members[int(offsets[big])]) if counts[big] else 0
    stats = dict(leaves=int(sizes.size), leaf_rows=int(sizes.sum()), partition=pst)
    return offs, nb, entry, timings, stats
