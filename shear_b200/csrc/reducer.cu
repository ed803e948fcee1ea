// Host-side HashPrune reduction of candidate edges (host code only).
//
// SHEAR keeps this stage on the CPU: leaf top-k records are flushed into
// per-point reservoirs (HashPruneReservoir, shear-core/src/algorithm/pipnn/
// hash_prune.rs:269-1420) and each point's final neighbours are the
// reservoir's slots (into_finalized_slots_with_backfill with the default
// backfill off, :1946-1964, emitted by emit_resident_reservoirs_serial,
// mod.rs:2437-2478).  This file restates that reservoir for the build: a
// reservoir holds at most l_max slots (target, hash, dist) sorted by hash;
// a candidate whose hash is present replaces that slot when it is better;
// otherwise it is inserted while there is room, else it replaces the
// farthest slot when better (insert_inner, :1326-1452).  "Better" is the
// total order (dist via total_cmp, target, hash) (:2094-2130).
//
// Edges come from leaf batches exactly as flush_compact_topk_batch_into_edges
// forms them (P/leaf_build.rs:1749-1808): for row i and rank r with a valid id
// j and a finite distance d, (i -> j, hash_fwd, d) then (j -> i, hash_rev, d).
// Batches are distributed over host threads by source point (point % T), so
// every reservoir is owned by one thread; the reservoir's final content does
// not depend on the insertion order, so the result is deterministic.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "kernels.h"

struct tessa_reducer {
  uint64_t points = 0;
  uint32_t l_max = 0;
  uint32_t threads = 1;
  std::vector<uint32_t> target;  // points x l_max
  std::vector<uint16_t> hash;
  std::vector<float> dist;
  std::vector<uint8_t> len;      // slots used (l_max <= 255)
  std::vector<uint8_t> far;      // index of the farthest slot
  uint64_t edges = 0;            // edges inserted so far
};

namespace {

struct Edge {
  uint32_t src, dst;
  float dist;
  uint16_t hash;
};

inline int total_cmp_f32(float a, float b) {
  // f32::total_cmp: order of the sign-flipped bit patterns
  int32_t ia, ib;
  memcpy(&ia, &a, 4);
  memcpy(&ib, &b, 4);
  ia ^= (int32_t)((uint32_t)(ia >> 31) >> 1);
  ib ^= (int32_t)((uint32_t)(ib >> 31) >> 1);
  return ia < ib ? -1 : (ia > ib ? 1 : 0);
}

// hashprune_candidate_total_order (hash_prune.rs:2094-2106): < 0 when (d1, t1, h1) comes first
inline int cand_order(uint32_t t1, uint16_t h1, float d1, uint32_t t2, uint16_t h2, float d2) {
  int c = total_cmp_f32(d1, d2);
  if (c) return c;
  if (t1 != t2) return t1 < t2 ? -1 : 1;
  if (h1 != h2) return h1 < h2 ? -1 : 1;
  return 0;
}

void recompute_far(const uint32_t* t, const uint16_t* h, const float* d, uint32_t n, uint8_t* far) {
  uint32_t idx = 0;
  for (uint32_t i = 1; i < n; ++i)
    if (cand_order(t[i], h[i], d[i], t[idx], h[idx], d[idx]) > 0) idx = i;
  *far = (uint8_t)idx;
}

// insert_inner (hash_prune.rs:1326-1452) on one reservoir.
void insert(tessa_reducer* R, uint64_t p, uint32_t tgt, uint16_t hs, float ds) {
  const uint32_t L = R->l_max;
  uint32_t* t = R->target.data() + p * L;
  uint16_t* h = R->hash.data() + p * L;
  float* d = R->dist.data() + p * L;
  uint32_t n = R->len[p];
  uint8_t* far = &R->far[p];
  // binary search by hash
  uint32_t lo = 0, hi = n;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (h[mid] < hs) lo = mid + 1;
    else hi = mid;
  }
  if (lo < n && h[lo] == hs) {
    if (cand_order(tgt, hs, ds, t[lo], h[lo], d[lo]) < 0) {
      t[lo] = tgt;
      d[lo] = ds;
      if (lo == *far) recompute_far(t, h, d, n, far);
    }
    return;
  }
  if (n < L) {
    for (uint32_t i = n; i > lo; --i) {
      t[i] = t[i - 1];
      h[i] = h[i - 1];
      d[i] = d[i - 1];
    }
    t[lo] = tgt;
    h[lo] = hs;
    d[lo] = ds;
    R->len[p] = (uint8_t)(n + 1);
    if (n == 0) {
      *far = 0;
    } else {
      uint32_t fi = *far;
      if (lo <= fi) fi++;
      if (cand_order(t[lo], h[lo], d[lo], t[fi], h[fi], d[fi]) > 0) fi = lo;
      *far = (uint8_t)fi;
    }
    return;
  }
  const uint32_t fi = *far;
  if (cand_order(tgt, hs, ds, t[fi], h[fi], d[fi]) >= 0) return;
  // replace the farthest slot and move it to its hash position
  uint32_t pos = fi;
  if (fi > 0 && h[fi - 1] > hs) {
    uint32_t tp = 0;
    while (tp < fi && h[tp] < hs) ++tp;
    for (uint32_t i = fi; i > tp; --i) {
      t[i] = t[i - 1];
      h[i] = h[i - 1];
      d[i] = d[i - 1];
    }
    pos = tp;
  } else if (fi + 1 < n && h[fi + 1] < hs) {
    uint32_t tp = fi + 1;
    while (tp < n && h[tp] < hs) ++tp;
    for (uint32_t i = fi; i + 1 < tp; ++i) {
      t[i] = t[i + 1];
      h[i] = h[i + 1];
      d[i] = d[i + 1];
    }
    pos = tp - 1;
  }
  t[pos] = tgt;
  h[pos] = hs;
  d[pos] = ds;
  recompute_far(t, h, d, n, far);
}

template <class F>
void parallel(uint32_t threads, F&& fn) {
  if (threads <= 1) {
    fn(0u);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (uint32_t i = 0; i < threads; ++i) pool.emplace_back(fn, i);
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

TESSA_API int tessa_reducer_create(uint64_t num_points, uint32_t l_max, uint32_t threads, tessa_reducer** out) {
  if (!out) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null output pointer");
  *out = nullptr;
  if (l_max == 0 || l_max > 255)
    return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "reducer l_max must be in 1..255");
  if (num_points == 0 || num_points > 0xffffffffull)
    return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "reducer points must be in 1..2^32");
  tessa_reducer* R = new (std::nothrow) tessa_reducer();
  if (!R) return tessa::set_last_error(TESSA_ERR_OOM, "reducer allocation failed");
  try {
    R->points = num_points;
    R->l_max = l_max;
    R->threads = threads ? threads : 1;
    R->target.resize(num_points * l_max);
    R->hash.resize(num_points * l_max);
    R->dist.resize(num_points * l_max);
    R->len.assign(num_points, 0);
    R->far.assign(num_points, 0);
  } catch (...) {
    delete R;
    return tessa::set_last_error(TESSA_ERR_OOM, "reducer reservoirs do not fit in host memory");
  }
  *out = R;
  return TESSA_OK;
}

TESSA_API int tessa_reducer_add(tessa_reducer* R, const uint32_t* point_ids, const uint32_t* topk_ids,
                                const float* topk_dists, const uint16_t* hash_fwd, const uint16_t* hash_rev,
                                uint64_t rows, uint32_t k) {
  if (!R) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null reducer");
  if (rows == 0) return TESSA_OK;
  if (!point_ids || !topk_ids || !topk_dists || !hash_fwd || !hash_rev || k == 0)
    return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null edge input or k = 0");
  const uint32_t T = R->threads;
  // phase 1: form the edges of a row range per thread, bucketed by owner thread
  std::vector<std::vector<std::vector<Edge>>> buckets(T, std::vector<std::vector<Edge>>(T));
  std::vector<int> bad(T, 0);
  parallel(T, [&](uint32_t w) {
    const uint64_t r0 = rows * w / T, r1 = rows * (w + 1) / T;
    auto& mine = buckets[w];
    for (uint64_t i = r0; i < r1; ++i) {
      const uint32_t p = point_ids[i];
      for (uint32_t r = 0; r < k; ++r) {
        const uint64_t s = i * k + r;
        const uint32_t j = topk_ids[s];
        const float d = topk_dists[s];
        if (j == 0xffffffffu || !std::isfinite(d)) continue;
        if (p >= R->points || j >= R->points) {
          bad[w] = 1;
          continue;
        }
        mine[p % T].push_back(Edge{p, j, d, hash_fwd[s]});
        mine[j % T].push_back(Edge{j, p, d, hash_rev[s]});
      }
    }
  });
  for (int b : bad)
    if (b) return tessa::set_last_error(TESSA_ERR_BAD_ROW, "edge endpoint outside the reducer's points");
  // phase 2: every thread applies the edges of the points it owns
  std::vector<uint64_t> counted(T, 0);
  parallel(T, [&](uint32_t owner) {
    for (uint32_t w = 0; w < T; ++w)
      for (const Edge& e : buckets[w][owner]) insert(R, e.src, e.dst, e.hash, e.dist);
    for (uint32_t w = 0; w < T; ++w) counted[owner] += buckets[w][owner].size();
  });
  for (uint64_t c : counted) R->edges += c;
  return TESSA_OK;
}

// Final neighbour lists (slot targets in hash order) as CSR: offsets has
// num_points + 1 entries; neighbors needs capacity for every slot (at most
// num_points * l_max).  *count = slots written.
TESSA_API int tessa_reducer_finish(const tessa_reducer* R, uint64_t* offsets, uint32_t* neighbors, uint64_t capacity,
                                   uint64_t* count) {
  if (!R || !offsets || !count) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null reducer output");
  uint64_t n = 0;
  for (uint64_t p = 0; p < R->points; ++p) {
    offsets[p] = n;
    n += R->len[p];
  }
  offsets[R->points] = n;
  *count = n;
  if (!neighbors) return TESSA_OK;
  if (capacity < n) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "neighbor capacity below the slot count");
  const uint32_t T = R->threads;
  parallel(T, [&](uint32_t w) {
    const uint64_t p0 = R->points * w / T, p1 = R->points * (w + 1) / T;
    for (uint64_t p = p0; p < p1; ++p)
      memcpy(neighbors + offsets[p], R->target.data() + p * R->l_max, (size_t)R->len[p] * 4);
  });
  return TESSA_OK;
}

TESSA_API int tessa_reducer_edges(const tessa_reducer* R, uint64_t* edges) {
  if (!R || !edges) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null argument");
  *edges = R->edges;
  return TESSA_OK;
}

TESSA_API void tessa_reducer_destroy(tessa_reducer* R) { delete R; }

}  // extern "C"
