// Candidate records grouped by reservoir on the device, for the host reducer.
//
// A leaf batch's records (CompactTopKBatch, shear-core/src/algorithm/pipnn/
// leaf_build.rs:271-290) become two edges per valid slot, as
// flush_compact_topk_batch_into_edges forms them (leaf_build.rs:1749-1808):
// (i -> j, hash_fwd, d) into i's reservoir and (j -> i, hash_rev, d) into j's.
// The host reducer merges each reservoir's edges in one pass; grouping them by
// reservoir is a counting sort, done here before the copy to the host:
//   count_kernel   edges per destination point (atomics);
//   exclusive scan of the counts (cub::DeviceScan) -> offsets;
//   scatter_kernel each edge to offsets[p] + atomic cursor.
// The order of a point's edges inside its group is not fixed (atomics); the
// reservoir's content does not depend on it.  HBM-bound: 2 * rows * k edges of
// 12 bytes written, the records read twice.
#include <cub/cub.cuh>

#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace records {

__global__ void count_kernel(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                             uint64_t rows, uint32_t k, uint64_t num_points, unsigned long long* counts,
                             uint32_t* err) {
  const uint64_t slots = rows * k;
  for (uint64_t s = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; s < slots;
       s += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = topk_ids[s];
    if (j == 0xffffffffu || !isfinite(topk_dists[s])) continue;
    const uint32_t p = point_ids[s / k];
    if (p >= num_points || j >= num_points) {
      atomicOr(err, TESSA_DEVERR_BAD_ROW);
      continue;
    }
    atomicAdd(&counts[p], 1ull);
    atomicAdd(&counts[j], 1ull);
  }
}

__global__ void scatter_kernel(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                               const uint16_t* hash_fwd, const uint16_t* hash_rev, uint64_t rows, uint32_t k,
                               uint64_t num_points, unsigned long long* cursor, tessa_edge* edges) {
  const uint64_t slots = rows * k;
  for (uint64_t s = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; s < slots;
       s += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = topk_ids[s];
    const float d = topk_dists[s];
    if (j == 0xffffffffu || !isfinite(d)) continue;
    const uint32_t p = point_ids[s / k];
    if (p >= num_points || j >= num_points) continue;
    const unsigned long long a = atomicAdd(&cursor[p], 1ull);
    edges[a] = tessa_edge{j, d, hash_fwd[s], 0};
    const unsigned long long b = atomicAdd(&cursor[j], 1ull);
    edges[b] = tessa_edge{p, d, hash_rev[s], 0};
  }
}

}  // namespace records

int group_edges(const GroupEdgesCall& g, cudaStream_t st) {
  using namespace records;
  const uint64_t slots = g.rows * g.k;
  const int grid = g.sm_count * 8;
  // counts in offsets[1..n], then an inclusive scan gives every group's start
  if (cudaMemsetAsync(g.offsets, 0, (g.num_points + 1) * 8, st) != cudaSuccess) return TESSA_ERR_CUDA;
  if (slots) {
    count_kernel<<<grid, 256, 0, st>>>(g.point_ids, g.topk_ids, g.topk_dists, g.rows, g.k, g.num_points,
                                       reinterpret_cast<unsigned long long*>(g.offsets) + 1, g.d_err);
    if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  }
  size_t temp = 0;
  unsigned long long* off = reinterpret_cast<unsigned long long*>(g.offsets);
  if (cub::DeviceScan::InclusiveSum(nullptr, temp, off + 1, off + 1, (int64_t)g.num_points, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  if (temp > g.temp_bytes) {
    *g.temp_needed = temp;
    return TESSA_ERR_OOM;
  }
  if (cub::DeviceScan::InclusiveSum(g.temp, temp, off + 1, off + 1, (int64_t)g.num_points, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  if (cudaMemcpyAsync(g.cursor, g.offsets, g.num_points * 8, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  if (slots) {
    scatter_kernel<<<grid, 256, 0, st>>>(g.point_ids, g.topk_ids, g.topk_dists, g.hash_fwd, g.hash_rev, g.rows,
                                         g.k, g.num_points, reinterpret_cast<unsigned long long*>(g.cursor),
                                         g.edges);
    if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  }
  return TESSA_OK;
}

size_t group_edges_temp_bytes(uint64_t num_points) {
  size_t temp = 0;
  cub::DeviceScan::InclusiveSum(nullptr, temp, (unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                (int64_t)num_points);
  return temp;
}

}  // namespace tessa
