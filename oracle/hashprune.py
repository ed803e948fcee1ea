"""Pure-Python restatement of SHEAR's HashPrune reservoir (test infrastructure).

Follows HashPruneReservoir::insert_inner (shear-core/src/algorithm/pipnn/
hash_prune.rs:1326-1452) step for step -- slots sorted by hash, binary search
for a hash hit, insert while there is room, replace-and-rotate of the farthest
slot when full -- with the candidate total order of :2094-2130 (distance by
f32 total order, then target, then hash).  Edges of a leaf batch are formed as
flush_compact_topk_batch_into_edges forms them (P/leaf_build.rs:1749-1808).
Small inputs only: this is the checker for the host reducer, never shipped.
"""
from __future__ import annotations

import struct

import numpy as np

EMPTY_ID = 0xFFFFFFFF


def _total_key(d: float) -> int:
    (i,) = struct.unpack("<i", struct.pack("<f", d))
    return i ^ ((i >> 31) & 0x7FFFFFFF)


def order_key(target: int, h: int, d: float):
    """hashprune_candidate_total_order as a sort key."""
    return (_total_key(d), target, h)


class Reservoir:
    def __init__(self, l_max: int):
        self.l_max = l_max
        self.slots = []  # (target, hash, dist), sorted by hash
        self.far = 0

    def _recompute_far(self):
        idx = 0
        for i in range(1, len(self.slots)):
            if order_key(*self.slots[i]) > order_key(*self.slots[idx]):
                idx = i
        self.far = idx

    def insert(self, target: int, h: int, d: float):
        hashes = [s[1] for s in self.slots]
        lo, hi = 0, len(hashes)
        while lo < hi:
            mid = (lo + hi) // 2
            if hashes[mid] < h:
                lo = mid + 1
            else:
                hi = mid
        if lo < len(hashes) and hashes[lo] == h:
            if order_key(target, h, d) < order_key(*self.slots[lo]):
                self.slots[lo] = (target, h, d)
                if lo == self.far:
                    self._recompute_far()
            return
        if len(self.slots) < self.l_max:
            self.slots.insert(lo, (target, h, d))
            if len(self.slots) == 1:
                self.far = 0
            else:
                if lo <= self.far:
                    self.far += 1
                if order_key(*self.slots[lo]) > order_key(*self.slots[self.far]):
                    self.far = lo
            return
        if not order_key(target, h, d) < order_key(*self.slots[self.far]):
            return
        fi = self.far
        self.slots[fi] = (target, h, d)
        if fi > 0 and self.slots[fi - 1][1] > h:
            tp = 0
            while tp < fi and self.slots[tp][1] < h:
                tp += 1
            self.slots[tp:fi + 1] = [self.slots[fi]] + self.slots[tp:fi]
        elif fi + 1 < len(self.slots) and self.slots[fi + 1][1] < h:
            tp = fi + 1
            while tp < len(self.slots) and self.slots[tp][1] < h:
                tp += 1
            self.slots[fi:tp] = self.slots[fi + 1:tp] + [self.slots[fi]]
        self._recompute_far()


def reduce_leaf_batches(num_points: int, l_max: int, batches, slots: bool = False):
    """batches: iterable of (point_ids, topk_ids, topk_dists, hash_fwd, hash_rev, k).
    Returns the per-point neighbour lists (slot targets in hash order), or with
    slots=True the (target, hash, dist) slots themselves."""
    res = [Reservoir(l_max) for _ in range(num_points)]
    for pid, ids, ds, hf, hr, k in batches:
        pid = np.asarray(pid).view(np.uint32)
        ids = np.asarray(ids).view(np.uint32).reshape(-1)
        ds = np.asarray(ds, np.float32).reshape(-1)
        hf = np.asarray(hf).view(np.uint16).reshape(-1)
        hr = np.asarray(hr).view(np.uint16).reshape(-1)
        for i, p in enumerate(pid.tolist()):
            for r in range(k):
                s = i * k + r
                j, d = int(ids[s]), float(ds[s])
                if j == EMPTY_ID or not np.isfinite(d):
                    continue
                res[p].insert(j, int(hf[s]), d)
                res[j].insert(p, int(hr[s]), d)
    if slots:
        return [list(r.slots) for r in res]
    return [[t for t, _, _ in r.slots] for r in res]
