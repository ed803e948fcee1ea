// Greedy graph search over a built index, for recall runs of graphs written
// in the in-memory graph format (host code; no device work).
//
// Reference (wbh1765091327/SHEAR): apps/search_shear_index/src/main.rs
// search_one_with_stats (:1007-1085): l_eff = max(l, k + 1); start at the
// graph's entry point; a candidate min-heap and a best-l_eff max-heap ordered
// by (distance, id); stop once the closest open candidate is farther than the
// worst kept result of a full list; every unvisited neighbour is scored with
// l2_distance (:1639-1644, sequential f32 sum of (x - y)^2) and pushed to both
// heaps; the result is the kept list sorted by distance, first k ids.  Ties at
// equal distance in that final sort follow the heap's internal order in the
// reference; here they follow (distance, id).
#include <algorithm>
#include <cstdint>
#include <queue>
#include <thread>
#include <utility>
#include <vector>

namespace tessa {

namespace {

float l2_seq(const float* a, const float* b, uint32_t dim) {
  float s = 0.0f;
  for (uint32_t i = 0; i < dim; ++i) {
    const float d = a[i] - b[i];
    const float sq = d * d;
    s = s + sq;
  }
  return s;
}

using Item = std::pair<float, uint32_t>;

uint64_t search_one(const float* q, const float* data, uint64_t n, uint32_t dim, const uint64_t* offsets,
                    const uint32_t* nbrs, uint32_t start, uint32_t k, uint32_t l, std::vector<uint8_t>& visited,
                    std::vector<uint32_t>& touched, uint32_t* out) {
  const uint32_t l_eff = std::max(l, k + 1);
  for (uint32_t v : touched) visited[v] = 0;
  touched.clear();
  std::priority_queue<Item, std::vector<Item>, std::greater<Item>> cand;  // closest first
  std::priority_queue<Item> best;                                          // farthest first
  visited[start] = 1;
  touched.push_back(start);
  const float d0 = l2_seq(q, data + (uint64_t)start * dim, dim);
  cand.push({d0, start});
  best.push({d0, start});
  uint64_t comparisons = 1;
  while (!cand.empty()) {
    const Item c = cand.top();
    cand.pop();
    if (best.size() >= l_eff && c.first > best.top().first) break;
    for (uint64_t e = offsets[c.second]; e < offsets[c.second + 1]; ++e) {
      const uint32_t nb = nbrs[e];
      if (nb >= n || visited[nb]) continue;
      visited[nb] = 1;
      touched.push_back(nb);
      const float d = l2_seq(q, data + (uint64_t)nb * dim, dim);
      ++comparisons;
      cand.push({d, nb});
      best.push({d, nb});
      while (best.size() > l_eff) best.pop();
    }
  }
  std::vector<Item> sorted;
  sorted.reserve(best.size());
  while (!best.empty()) {
    sorted.push_back(best.top());
    best.pop();
  }
  std::sort(sorted.begin(), sorted.end());
  for (uint32_t i = 0; i < k; ++i) out[i] = i < sorted.size() ? sorted[i].second : 0xffffffffu;
  return comparisons;
}

}  // namespace

uint64_t graph_search_host(const float* data, uint64_t n, uint32_t dim, const uint64_t* offsets,
                           const uint32_t* neighbors, uint32_t start, const float* queries, uint64_t nq, uint32_t k,
                           uint32_t l, uint32_t threads, uint32_t* out_ids) {
  if (threads == 0) threads = 1;
  const uint64_t per = (nq + threads - 1) / threads;
  std::vector<uint64_t> comps(threads, 0);
  auto body = [&](uint32_t t) {
    std::vector<uint8_t> visited(n, 0);
    std::vector<uint32_t> touched;
    const uint64_t q0 = t * per, q1 = std::min(nq, q0 + per);
    for (uint64_t qi = q0; qi < q1; ++qi)
      comps[t] += search_one(queries + qi * dim, data, n, dim, offsets, neighbors, start, k, l, visited, touched,
                             out_ids + qi * k);
  };
  std::vector<std::thread> pool;
  for (uint32_t t = 1; t < threads && t * per < nq; ++t) pool.emplace_back(body, t);
  if (nq) body(0);
  for (auto& th : pool) th.join();
  uint64_t total = 0;
  for (uint64_t c : comps) total += c;
  return total;
}

}  // namespace tessa
