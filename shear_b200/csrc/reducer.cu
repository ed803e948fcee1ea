// Host-side HashPrune reduction of candidate edges (host code only).
//
// SHEAR keeps this stage on the CPU: leaf top-k records are flushed into
// per-point reservoirs (HashPruneReservoir, shear-core/src/algorithm/pipnn/
// hash_prune.rs:269-1452) and each point's final neighbours are the
// reservoir's slots (into_finalized_slots_with_backfill with the default
// backfill off, :1946-1964, emitted by emit_resident_reservoirs_serial,
// mod.rs:2437-2478).  A reservoir holds at most l_max slots (target, hash,
// dist) sorted by hash; insert_inner (:1326-1452) replaces a slot whose hash
// matches when the candidate is better, inserts while there is room, and
// otherwise replaces the farthest slot when the candidate is better.  "Better"
// is the total order (dist via total_cmp, target, hash) (:2094-2130).
//
// The slots that sequence of inserts leaves behind do not depend on the
// insertion order: they are the l_max best (in that order) of the per-hash
// minima of every candidate offered.  (A per-hash minimum among the l_max best
// is never rejected -- that needs l_max better slots of other hashes -- and
// never evicted; nothing else can stay.)  The reducer therefore applies a
// batch at once: edges are grouped by source point with counting sorts, and
// each reservoir merges its new candidates in one pass -- per-hash minimum
// through a table indexed by hash, the l_max best by partial selection, the
// survivors sorted by hash -- touching its slots once instead of once per
// candidate.  The result equals the reference's online inserts (tested
// against a line-by-line restatement of insert_inner).
//
// Edges come from leaf batches exactly as flush_compact_topk_batch_into_edges
// forms them (P/leaf_build.rs:1749-1808): for row i and rank r with a valid id
// j and a finite distance d, (i -> j, hash_fwd, d) then (j -> i, hash_rev, d).
// Source point p belongs to host thread p & (T - 1) (T a power of two).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
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
  uint64_t edges = 0;            // edges offered so far
};

namespace {

struct Edge {
  uint32_t src, dst;
  float dist;
  uint32_t hash;
};

inline uint32_t total_key(float d) {
  // f32::total_cmp order as an unsigned key
  uint32_t u;
  memcpy(&u, &d, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// A candidate in hashprune_candidate_total_order (hash_prune.rs:2094-2106):
// (dist by total_cmp, target) packed into one 64-bit key, hash last.
struct Cand {
  uint64_t key;
  uint32_t hash;
  float dist;
};

inline bool cand_less(const Cand& a, const Cand& b) {
  return a.key != b.key ? a.key < b.key : a.hash < b.hash;
}

struct Scratch {
  // per hash value: stamp of the merge that last touched it and the index of
  // its candidate; a bitset of the surviving hashes for hash-ordered output
  std::vector<uint64_t> slot;    // (stamp << 32) | candidate index
  std::vector<uint64_t> bits;
  std::vector<Cand> cand;
  std::vector<uint32_t> count;   // counting sort by local source
  std::unique_ptr<Edge[]> sorted;  // not value-initialised
  uint64_t sorted_cap = 0;
  uint32_t cur = 0;
  Scratch() : slot(1u << 16, 0), bits((1u << 16) / 64, 0) { cand.reserve(512); }
};

inline void offer(Scratch& S, uint32_t target, uint32_t hash, float dist) {
  const Cand c{((uint64_t)total_key(dist) << 32) | target, hash, dist};
  const uint64_t sl = S.slot[hash];
  if ((uint32_t)(sl >> 32) != S.cur) {
    S.slot[hash] = ((uint64_t)S.cur << 32) | (uint32_t)S.cand.size();
    S.cand.push_back(c);
  } else {
    Cand& o = S.cand[(uint32_t)sl];
    if (cand_less(c, o)) o = c;
  }
}

inline uint32_t edge_target(const Edge& e) { return e.dst; }
inline uint32_t edge_target(const tessa_edge& e) { return e.target; }

// Merge the edges of one source into its reservoir: per-hash minimum of the
// old slots and the new edges, the l_max best, written back in hash order.
template <class E>
void merge(tessa_reducer* R, Scratch& S, uint64_t p, const E* e, size_t n) {
  const uint32_t L = R->l_max;
  uint32_t* t = R->target.data() + p * L;
  uint16_t* h = R->hash.data() + p * L;
  float* d = R->dist.data() + p * L;
  if (++S.cur == 0) {  // stamps wrapped: clear them
    std::fill(S.slot.begin(), S.slot.end(), 0ull);
    S.cur = 1;
  }
  S.cand.clear();
  for (uint32_t i = 0; i < R->len[p]; ++i) offer(S, t[i], h[i], d[i]);
  for (size_t i = 0; i < n; ++i) offer(S, edge_target(e[i]), e[i].hash, e[i].dist);
  auto& c = S.cand;
  if (c.size() > L) {
    std::nth_element(c.begin(), c.begin() + L, c.end(), cand_less);
    c.resize(L);
  }
  // emit in hash order through the bitset of surviving hashes
  uint32_t lo_w = 0xffffffffu, hi_w = 0;
  for (uint32_t i = 0; i < c.size(); ++i) {
    const uint32_t hv = c[i].hash;
    S.slot[hv] = ((uint64_t)S.cur << 32) | i;
    S.bits[hv >> 6] |= 1ull << (hv & 63);
    lo_w = std::min(lo_w, hv >> 6);
    hi_w = std::max(hi_w, hv >> 6);
  }
  uint32_t out = 0;
  for (uint32_t w = lo_w; w <= hi_w && out < c.size(); ++w) {
    uint64_t b = S.bits[w];
    S.bits[w] = 0;
    while (b) {
      const uint32_t hv = (w << 6) | (uint32_t)__builtin_ctzll(b);
      b &= b - 1;
      const Cand& x = c[(uint32_t)S.slot[hv]];
      t[out] = (uint32_t)x.key;
      h[out] = (uint16_t)x.hash;
      d[out] = x.dist;
      ++out;
    }
  }
  R->len[p] = (uint8_t)c.size();
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
    uint32_t t = 1;
    while (t * 2 <= (threads ? threads : 1) && t < 256) t *= 2;
    R->threads = t;
    R->target.resize(num_points * l_max);
    R->hash.resize(num_points * l_max);
    R->dist.resize(num_points * l_max);
    R->len.assign(num_points, 0);
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
  const uint32_t T = R->threads, mask = T - 1, shift = (uint32_t)__builtin_ctz(T);
  const uint64_t P = R->points;
  // 1. per (row range w, owner thread o) edge counts
  std::vector<uint64_t> cnt((size_t)T * T, 0);
  std::vector<int> bad(T, 0);
  parallel(T, [&](uint32_t w) {
    const uint64_t r0 = rows * w / T, r1 = rows * (w + 1) / T;
    uint64_t* c = cnt.data() + (size_t)w * T;
    for (uint64_t i = r0; i < r1; ++i) {
      const uint32_t p = point_ids[i];
      for (uint32_t r = 0; r < k; ++r) {
        const uint64_t s = i * k + r;
        const uint32_t j = topk_ids[s];
        if (j == 0xffffffffu || !std::isfinite(topk_dists[s])) continue;
        if (p >= P || j >= P) {
          bad[w] = 1;
          continue;
        }
        c[p & mask]++;
        c[j & mask]++;
      }
    }
  });
  for (int b : bad)
    if (b) return tessa::set_last_error(TESSA_ERR_BAD_ROW, "edge endpoint outside the reducer's points");
  // 2. owner-major layout: owner o's edges are contiguous
  std::vector<uint64_t> off((size_t)T * T), base(T + 1, 0);
  for (uint32_t o = 0; o < T; ++o) {
    uint64_t run = base[o];
    for (uint32_t w = 0; w < T; ++w) {
      off[(size_t)w * T + o] = run;
      run += cnt[(size_t)w * T + o];
    }
    base[o + 1] = run;
  }
  const uint64_t total = base[T];
  std::unique_ptr<Edge[]> edges(new (std::nothrow) Edge[total ? total : 1]);
  if (!edges) return tessa::set_last_error(TESSA_ERR_OOM, "reducer batch does not fit in host memory");
  parallel(T, [&](uint32_t w) {
    const uint64_t r0 = rows * w / T, r1 = rows * (w + 1) / T;
    uint64_t* o = off.data() + (size_t)w * T;
    for (uint64_t i = r0; i < r1; ++i) {
      const uint32_t p = point_ids[i];
      for (uint32_t r = 0; r < k; ++r) {
        const uint64_t s = i * k + r;
        const uint32_t j = topk_ids[s];
        const float d = topk_dists[s];
        if (j == 0xffffffffu || !std::isfinite(d)) continue;
        edges[o[p & mask]++] = Edge{p, j, d, hash_fwd[s]};
        edges[o[j & mask]++] = Edge{j, p, d, hash_rev[s]};
      }
    }
  });
  // 3. every owner sorts its edges by source (counting sort) and merges each
  //    source's edges into its reservoir, sources in ascending order
  std::vector<int> oom(T, 0);
  parallel(T, [&](uint32_t o) {
    static thread_local Scratch S;
    const uint64_t b = base[o], n = base[o + 1] - b;
    if (n == 0) return;
    const uint64_t locals = (P - o + T - 1) >> shift;  // sources p = o + T * li
    try {
      S.count.assign(locals + 1, 0);
      if (S.sorted_cap < n) {
        S.sorted.reset(new Edge[n]);
        S.sorted_cap = n;
      }
    } catch (...) {
      oom[o] = 1;
      return;
    }
    const Edge* e = edges.get() + b;
    uint32_t* cnt_l = S.count.data();
    for (uint64_t i = 0; i < n; ++i) cnt_l[(e[i].src >> shift) + 1]++;
    for (uint64_t li = 0; li < locals; ++li) cnt_l[li + 1] += cnt_l[li];
    Edge* srt = S.sorted.get();
    for (uint64_t i = 0; i < n; ++i) srt[cnt_l[e[i].src >> shift]++] = e[i];
    // count[li] is now the end of source li's edges
    uint64_t lo = 0;
    for (uint64_t li = 0; li < locals; ++li) {
      const uint64_t hi = cnt_l[li];
      if (hi > lo) merge(R, S, o + ((uint64_t)li << shift), srt + lo, hi - lo);
      lo = hi;
    }
  });
  for (int b : oom)
    if (b) return tessa::set_last_error(TESSA_ERR_OOM, "reducer scratch does not fit in host memory");
  R->edges += total;
  return TESSA_OK;
}

TESSA_API int tessa_reducer_add_grouped(tessa_reducer* R, const uint64_t* offsets, const tessa_edge* edges) {
  if (!R || !offsets) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null reducer input");
  const uint64_t P = R->points;
  if (offsets[0] != 0) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "grouped offsets must start at 0");
  for (uint64_t p = 0; p < P; ++p)
    if (offsets[p + 1] < offsets[p]) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "grouped offsets decrease");
  const uint64_t total = offsets[P];
  if (total && !edges) return tessa::set_last_error(TESSA_ERR_INVALID_ARG, "null edges");
  const uint32_t T = R->threads;
  std::vector<int> bad(T, 0);
  // contiguous point ranges of about equal edge counts
  parallel(T, [&](uint32_t w) {
    static thread_local Scratch S;
    const uint64_t e0 = total * w / T, e1 = total * (w + 1) / T;
    uint64_t p = std::upper_bound(offsets, offsets + P + 1, e0) - offsets - 1;
    if (w == 0) p = 0;
    for (; p < P && offsets[p] < e1; ++p) {
      if (w > 0 && offsets[p] < e0) continue;  // owned by the previous range
      const uint64_t a = offsets[p], b = offsets[p + 1];
      if (b == a) continue;
      bool ok = true;
      for (uint64_t i = a; i < b; ++i) ok &= edges[i].target < P;
      if (!ok) {
        bad[w] = 1;
        continue;
      }
      merge(R, S, p, edges + a, b - a);
    }
  });
  for (int b : bad)
    if (b) return tessa::set_last_error(TESSA_ERR_BAD_ROW, "edge target outside the reducer's points");
  R->edges += total;
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
