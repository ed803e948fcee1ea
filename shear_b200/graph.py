"""Index graph files and recall runs.

* ``write_mem_graph`` / ``read_mem_graph`` — the in-memory graph file that
  DirectMemGraphWriter writes (shear-core/src/index/inmem_index/
  pipnn_oom_writer.rs:22-79): header u64 file size, u32 max degree, u32 start,
  u64 frozen points (24 bytes, little endian), then per node a u32 degree and
  that many u32 neighbour ids.
* ``search`` — the greedy search of apps/search_shear_index/src/main.rs
  (:1007-1085) through the library's host implementation (``tessa_graph_search``).
* ``recall_at`` — Recall@k as main.rs:388-413 computes it (hits of the returned
  ids in the query's ground-truth set, averaged).
* ``exact_knn`` — brute-force ground truth on the GPU (squared L2 through one
  matrix product per block and a top-k), for the recall runs' ground-truth
  files.
"""
from __future__ import annotations

import ctypes
import os
import struct

import numpy as np

from . import _capi as C


def write_mem_graph(path: str, neighbors, start: int, num_frozen_pts: int = 0) -> int:
    """Write neighbour lists (a sequence of id arrays) in node order; returns the file size."""
    max_deg = 0
    size = 24
    with open(path, "wb") as f:
        f.write(struct.pack("<QIIQ", 0, 0, start, num_frozen_pts))
        for nb in neighbors:
            a = np.ascontiguousarray(nb, dtype="<u4")
            f.write(struct.pack("<I", a.size))
            f.write(a.tobytes())
            size += 4 * (a.size + 1)
            max_deg = max(max_deg, int(a.size))
        f.seek(0)
        f.write(struct.pack("<QIIQ", size, max_deg, start, num_frozen_pts))
    return size


def read_mem_graph(path: str):
    """-> (offsets uint64 [n+1], neighbors uint32, start, max_degree, num_frozen_pts)."""
    data = open(path, "rb").read()
    if len(data) < 24:
        raise ValueError(f"graph file {path} is shorter than its header")
    size, max_deg, start, frozen = struct.unpack_from("<QIIQ", data, 0)
    if size != len(data):
        raise ValueError(f"graph file {path}: header size {size} != file size {len(data)}")
    words = np.frombuffer(data, dtype="<u4", offset=24)
    offsets, nbrs, pos = [0], [], 0
    while pos < words.size:
        deg = int(words[pos])
        if deg > max_deg or pos + 1 + deg > words.size:
            raise ValueError(f"graph file {path}: node {len(offsets) - 1} degree {deg} is invalid")
        nbrs.append(words[pos + 1:pos + 1 + deg])
        offsets.append(offsets[-1] + deg)
        pos += 1 + deg
    nb = np.concatenate(nbrs).astype(np.uint32) if nbrs else np.zeros(0, np.uint32)
    return np.asarray(offsets, np.uint64), nb, start, max_deg, frozen


def search(data, offsets, neighbors, start: int, queries, k: int, l: int, threads: int = 0):
    """Greedy search of every query; returns (ids uint32 [nq, k], distance evaluations)."""
    data = np.ascontiguousarray(data, np.float32)
    queries = np.ascontiguousarray(queries, np.float32)
    offsets = np.ascontiguousarray(offsets, np.uint64)
    neighbors = np.ascontiguousarray(neighbors, np.uint32)
    n, dim = data.shape
    nq = queries.shape[0]
    out = np.empty((nq, k), np.uint32)
    comps = ctypes.c_uint64()
    threads = threads or min(32, os.cpu_count() or 1)
    C.check(C.load().tessa_graph_search(data.ctypes.data, n, dim, offsets.ctypes.data, neighbors.ctypes.data, start,
                                        queries.ctypes.data, nq, k, l, threads, out.ctypes.data,
                                        ctypes.byref(comps)))
    return out, int(comps.value)


def recall_at(results, gt, recall_at: int) -> float:
    """apps/search_shear_index/src/main.rs:388-413: mean over queries of
    |returned ids in the first recall_at ground-truth ids| / recall_at."""
    results = np.asarray(results)
    gt = np.asarray(gt)[:, :recall_at]
    total = 0.0
    for r, g in zip(results, gt):
        s = set(int(v) for v in g)
        total += sum(1 for v in r if int(v) in s) / recall_at
    return total / len(results)


def exact_knn(base, queries, k: int, block: int = 8192):
    """Brute-force k nearest base rows of every query by squared L2 on the GPU
    (CUDA float32 tensors in; ids int64 and distances out, nearest first)."""
    import torch

    bn = (base * base).sum(1)
    ids, dists = [], []
    for q0 in range(0, queries.shape[0], block):
        q = queries[q0:q0 + block]
        d = (q * q).sum(1, keepdim=True) + bn[None, :] - 2.0 * (q @ base.t())
        v, i = torch.topk(d, k, dim=1, largest=False, sorted=True)
        ids.append(i)
        dists.append(v)
    return torch.cat(ids), torch.cat(dists)
