// Candidate records grouped by reservoir on the device, for the host reducer.
//
// A leaf batch's records (CompactTopKBatch, shear-core/src/algorithm/pipnn/
// leaf_build.rs:271-290) become two edges per valid slot, as
// flush_compact_topk_batch_into_edges forms them (leaf_build.rs:1749-1808):
// (i -> j, hash_fwd, d) into i's reservoir and (j -> i, hash_rev, d) into j's.
// With overlapping leaves the same directed edge comes from many records (about
// 7 copies per edge in the builds measured here), and every copy is identical:
// the leaf distance is symmetric bit for bit (IEEE addition and multiplication
// commute) and the reverse hash of (j, i) is the forward hash of (i, j).  A
// reservoir ignores a repeated candidate, so the copies are dropped here:
//   keys_kernel     one 64-bit key (source << 32 | target) and one 64-bit
//                   value (hash << 32 | distance bits) per edge; an empty slot
//                   gets the largest key, which sorts last;
//   cub::DeviceRadixSort::SortPairs by value, then stably by key;
//   mark_kernel     an edge is kept unless it equals its predecessor (key and
//                   value), and kept edges are counted per source;
//   cub::DeviceScan over the flags and over the per-source counts;
//   emit_kernel     kept edges -> 12-byte records at their compacted position.
// Result: point p's distinct edges at edges[offsets[p] .. offsets[p+1]),
// ascending by target.  HBM-bound (a few passes over 16 bytes per edge).
#include <cub/cub.cuh>

#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace records {

constexpr unsigned long long kEmpty = ~0ull;

__global__ void keys_kernel(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                            const uint16_t* hash_fwd, const uint16_t* hash_rev, uint64_t rows, uint32_t k,
                            uint64_t num_points, unsigned long long* keys, unsigned long long* vals,
                            uint32_t* err) {
  const uint64_t slots = rows * k;
  for (uint64_t s = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; s < slots;
       s += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = topk_ids[s];
    const float d = topk_dists[s];
    unsigned long long k0 = kEmpty, k1 = kEmpty, v0 = 0, v1 = 0;
    if (j != 0xffffffffu && isfinite(d)) {
      const uint32_t p = point_ids[s / k];
      if (p >= num_points || j >= num_points) {
        atomicOr(err, TESSA_DEVERR_BAD_ROW);
      } else {
        const unsigned long long db = (unsigned long long)__float_as_uint(d);
        k0 = ((unsigned long long)p << 32) | j;
        v0 = ((unsigned long long)hash_fwd[s] << 32) | db;
        k1 = ((unsigned long long)j << 32) | p;
        v1 = ((unsigned long long)hash_rev[s] << 32) | db;
      }
    }
    keys[2 * s] = k0;
    vals[2 * s] = v0;
    keys[2 * s + 1] = k1;
    vals[2 * s + 1] = v1;
  }
}

__global__ void mark_kernel(const unsigned long long* keys, const unsigned long long* vals, uint64_t n,
                            uint32_t* keep, unsigned long long* counts) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const unsigned long long kk = keys[i];
    uint32_t f = 0;
    if (kk != kEmpty && (i == 0 || keys[i - 1] != kk || vals[i - 1] != vals[i])) {
      f = 1;
      atomicAdd(&counts[kk >> 32], 1ull);
    }
    keep[i] = f;
  }
}

__global__ void emit_kernel(const unsigned long long* keys, const unsigned long long* vals, const uint32_t* keep,
                            const uint32_t* pos, uint64_t n, tessa_edge* edges) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    if (!keep[i]) continue;
    const unsigned long long v = vals[i];
    edges[pos[i]] = tessa_edge{(uint32_t)keys[i], __uint_as_float((uint32_t)v), (uint16_t)(v >> 32), 0};
  }
}

}  // namespace records

// Scratch needed for m = 2 * rows * k edges of num_points sources.
size_t group_edges_scratch_bytes(uint64_t m, uint64_t num_points) {
  size_t sort_temp = 0, sort2_temp = 0, scan_temp = 0, scan2_temp = 0;
  cub::DoubleBuffer<unsigned long long> kb(nullptr, nullptr), vb(nullptr, nullptr);
  cub::DeviceRadixSort::SortPairs(nullptr, sort_temp, kb, vb, (int64_t)m, 0, 64);
  cub::DeviceRadixSort::SortPairs(nullptr, sort2_temp, vb, kb, (int64_t)m, 0, 48);
  sort_temp = std::max(sort_temp, sort2_temp);
  cub::DeviceScan::ExclusiveSum(nullptr, scan_temp, (uint32_t*)nullptr, (uint32_t*)nullptr, (int64_t)m);
  cub::DeviceScan::InclusiveSum(nullptr, scan2_temp, (unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                (int64_t)num_points);
  const size_t temp = std::max(sort_temp, std::max(scan_temp, scan2_temp));
  // keys x2, vals x2 (sort double buffers), keep + pos flags, scan temp
  return 4 * m * 8 + 2 * m * 4 + temp + 1024;
}

int group_edges(const GroupEdgesCall& g, cudaStream_t st) {
  using namespace records;
  const uint64_t slots = g.rows * g.k, m = 2 * slots;
  const int grid = g.sm_count * 8;
  if (cudaMemsetAsync(g.offsets, 0, (g.num_points + 1) * 8, st) != cudaSuccess) return TESSA_ERR_CUDA;
  if (m == 0) return TESSA_OK;
  uint8_t* base = reinterpret_cast<uint8_t*>(g.temp);
  auto take = [&](size_t bytes) {
    uint8_t* p = base;
    base += (bytes + 255) & ~size_t(255);
    return p;
  };
  unsigned long long* k0 = reinterpret_cast<unsigned long long*>(take(m * 8));
  unsigned long long* k1 = reinterpret_cast<unsigned long long*>(take(m * 8));
  unsigned long long* v0 = reinterpret_cast<unsigned long long*>(take(m * 8));
  unsigned long long* v1 = reinterpret_cast<unsigned long long*>(take(m * 8));
  uint32_t* keep = reinterpret_cast<uint32_t*>(take(m * 4));
  uint32_t* pos = reinterpret_cast<uint32_t*>(take(m * 4));
  void* temp = base;
  const size_t temp_bytes = g.temp_bytes - (size_t)(base - reinterpret_cast<uint8_t*>(g.temp));
  keys_kernel<<<grid, 256, 0, st>>>(g.point_ids, g.topk_ids, g.topk_dists, g.hash_fwd, g.hash_rev, g.rows, g.k,
                                    g.num_points, k0, v0, g.d_err);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  // (key, value) order: a stable sort by value (hash and distance bits), then
  // a stable sort by key on the bits in use (the target's 32 and enough source
  // bits; the empty key has every bit set and stays last) -- exact repeats end
  // up adjacent
  int src_bits = 1;
  while (src_bits < 32 && (1ull << src_bits) < g.num_points) ++src_bits;
  cub::DoubleBuffer<unsigned long long> kb(k0, k1), vb(v0, v1);
  size_t need = temp_bytes;
  if (cub::DeviceRadixSort::SortPairs(temp, need, vb, kb, (int64_t)m, 0, 48, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  need = temp_bytes;
  if (cub::DeviceRadixSort::SortPairs(temp, need, kb, vb, (int64_t)m, 0, 32 + src_bits + 1, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  if (cudaMemsetAsync(g.offsets, 0, (g.num_points + 1) * 8, st) != cudaSuccess) return TESSA_ERR_CUDA;
  mark_kernel<<<grid, 256, 0, st>>>(kb.Current(), vb.Current(), m, keep,
                                    reinterpret_cast<unsigned long long*>(g.offsets) + 1);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  need = temp_bytes;
  if (cub::DeviceScan::ExclusiveSum(temp, need, keep, pos, (int64_t)m, st) != cudaSuccess) return TESSA_ERR_CUDA;
  need = temp_bytes;
  unsigned long long* off = reinterpret_cast<unsigned long long*>(g.offsets);
  if (cub::DeviceScan::InclusiveSum(temp, need, off + 1, off + 1, (int64_t)g.num_points, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  emit_kernel<<<grid, 256, 0, st>>>(kb.Current(), vb.Current(), keep, pos, m, g.edges);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  return TESSA_OK;
}

}  // namespace tessa
