// HashPrune reservoirs built on the device.
//
// SHEAR reduces leaf candidate records on the CPU: every edge of
// flush_compact_topk_batch_into_edges (shear-core/src/algorithm/pipnn/
// leaf_build.rs:1749-1808) is inserted into its source's HashPruneReservoir
// with insert_inner (hash_prune.rs:1326-1452), and the final neighbour list is
// the reservoir's slots in hash order (emit_resident_reservoirs_serial,
// mod.rs:2437-2478, backfill off).  The slots a sequence of inserts leaves do
// not depend on its order: they are the l_max best, in the total order (dist
// via total_cmp, target, hash) of hash_prune.rs:2094-2130, of the per-hash
// minima of all candidates offered.  The same result is computed here with
// sorts and one warp per point, so the whole reduction stays in HBM:
//
//   keys        per edge a 64-bit key (source << 16 | hash) and a 64-bit value
//               (total_cmp key of the distance << 32 | target); a missing edge
//               gets the all-ones key, which sorts last;
//   radix sort  by key, over the 17 + log2(points) bits in use: each
//               (source, hash) group becomes one run;
//   runs        the first edge of a run becomes its head and takes the run's
//               smallest value -- the per-hash minimum; heads are counted per
//               source;
//   scans       head positions, per-source head offsets, and output offsets
//               (min(heads, l_max) per source);
//   select      one warp per source: with at most l_max heads all are kept;
//               otherwise a bitwise search over the 64-bit value (and, for
//               equal values, the hash) finds the l_max-th best and the heads
//               up to it are kept.  Heads are already in hash order, so the
//               kept ones are written in order with a ballot prefix.
//
// A run of (source, hash) holds the repeats of one edge (overlapping leaves
// produce about seven copies of each) and the rare distinct targets whose
// sketches collide; the head walks it sequentially.  The pipeline is
// HBM-bound: the sort moves 16 bytes per edge per 8-bit digit pass.
#include <cub/cub.cuh>

#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace reservoirs {

constexpr unsigned long long kEmpty = ~0ull;

// f32::total_cmp order as an unsigned key, and back
__device__ __forceinline__ uint32_t total_key(float d) {
  const uint32_t u = __float_as_uint(d);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_total_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Leaf records -> two edges per valid slot, in the reference's flush form.
__global__ void record_keys_kernel(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                                   const uint16_t* hash_fwd, const uint16_t* hash_rev, uint64_t rows, uint32_t k,
                                   uint64_t num_points, unsigned long long* keys, unsigned long long* vals,
                                   uint32_t* err) {
  const uint64_t slots = rows * k;
  for (uint64_t s = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; s < slots;
       s += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = topk_ids[s];
    const float d = topk_dists[s];
    unsigned long long k0 = kEmpty, k1 = kEmpty, v0 = kEmpty, v1 = kEmpty;
    if (j != 0xffffffffu && isfinite(d)) {
      const uint32_t p = point_ids[s / k];
      if (p >= num_points || j >= num_points) {
        atomicOr(err, TESSA_DEVERR_BAD_ROW);
      } else {
        const unsigned long long dk = (unsigned long long)total_key(d) << 32;
        k0 = ((unsigned long long)p << 16) | hash_fwd[s];
        v0 = dk | j;
        k1 = ((unsigned long long)j << 16) | hash_rev[s];
        v1 = dk | p;
      }
    }
    keys[2 * s] = k0;
    vals[2 * s] = v0;
    keys[2 * s + 1] = k1;
    vals[2 * s + 1] = v1;
  }
}

// Edges grouped by source (CSR over points 0 .. num_points-1; offsets need not
// start at zero) -> keys at base .. base + count.  One warp per source.
__global__ void grouped_keys_kernel(const uint64_t* offsets, const tessa_edge* edges, uint64_t num_points,
                                    uint64_t count, uint64_t base, unsigned long long* keys,
                                    unsigned long long* vals, uint32_t* err) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t off0 = offsets[0];
  for (uint64_t p = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5; p < num_points;
       p += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
    const uint64_t b = offsets[p] - off0, e = offsets[p + 1] - off0;
    if (b > e || e > count) {
      if (lane == 0) atomicOr(err, TESSA_DEVERR_BAD_TASK);
      continue;
    }
    for (uint64_t i = b + lane; i < e; i += 32) {
      const tessa_edge x = edges[i];
      unsigned long long kk = kEmpty, vv = kEmpty;
      if (isfinite(x.dist)) {
        kk = ((unsigned long long)p << 16) | x.hash;
        vv = ((unsigned long long)total_key(x.dist) << 32) | x.target;
      }
      keys[base + i] = kk;
      vals[base + i] = vv;
    }
  }
}

// Heads of (source, hash) runs take the run's smallest value; heads are
// flagged and counted per source.
__global__ void run_kernel(const unsigned long long* keys, unsigned long long* vals, uint64_t m, uint32_t* flag,
                           unsigned long long* heads_per_source) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < m; i += (uint64_t)gridDim.x * blockDim.x) {
    const unsigned long long kk = keys[i];
    uint32_t f = 0;
    if (kk != kEmpty && (i == 0 || keys[i - 1] != kk)) {
      unsigned long long best = vals[i];
      for (uint64_t j = i + 1; j < m && keys[j] == kk; ++j) best = min(best, vals[j]);
      vals[i] = best;
      f = 1;
      atomicAdd(&heads_per_source[kk >> 16], 1ull);
    }
    flag[i] = f;
  }
}

__global__ void compact_kernel(const unsigned long long* keys, const unsigned long long* vals, const uint32_t* flag,
                               const uint32_t* pos, uint64_t m, unsigned long long* head_keys,
                               unsigned long long* head_vals) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < m; i += (uint64_t)gridDim.x * blockDim.x) {
    if (!flag[i]) continue;
    head_keys[pos[i]] = keys[i];
    head_vals[pos[i]] = vals[i];
  }
}

// kept[p + 1] = min(heads[p], l_max); kept[0] = 0 (inclusive-scanned after)
__global__ void kept_kernel(const unsigned long long* heads, uint64_t num_points, uint32_t l_max,
                            unsigned long long* kept) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < num_points;
       p += (uint64_t)gridDim.x * blockDim.x) {
    kept[p + 1] = min(heads[p], (unsigned long long)l_max);
    if (p == 0) kept[0] = 0;
  }
}

__device__ __forceinline__ uint32_t warp_count(bool pred) { return __popc(__ballot_sync(0xffffffffu, pred)); }

__global__ void select_kernel(const unsigned long long* head_keys, const unsigned long long* head_vals,
                              const unsigned long long* head_off, const unsigned long long* out_off,
                              uint64_t num_points, uint32_t l_max, uint32_t* out_neighbors, tessa_edge* out_slots,
                              uint64_t capacity) {
  const uint32_t lane = threadIdx.x & 31;
  for (uint64_t p = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5; p < num_points;
       p += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
    const uint64_t b = head_off[p], c = head_off[p + 1] - b;
    const unsigned long long* kv = head_keys + b;
    const unsigned long long* vv = head_vals + b;
    unsigned long long X = ~0ull;
    uint32_t H = 0xffffu;
    if (c > l_max) {
      // the smallest X with #(value <= X) >= l_max, bit by bit from the top
      X = 0;
      for (int bit = 63; bit >= 0; --bit) {
        const unsigned long long trial = X | ((1ull << bit) - 1ull);
        uint32_t cnt = 0;
        for (uint64_t i = lane; i - lane < c; i += 32) cnt += warp_count(i < c && vv[i] <= trial);
        if (cnt < l_max) X |= 1ull << bit;
      }
      uint32_t less = 0, equal = 0;
      for (uint64_t i = lane; i - lane < c; i += 32) {
        const bool in = i < c;
        less += warp_count(in && vv[i] < X);
        equal += warp_count(in && vv[i] == X);
      }
      const uint32_t need = l_max - less;
      if (equal > need) {
        // equal values (same distance and target) under distinct hashes: the
        // smallest hashes win, as the total order's last field
        H = 0;
        for (int bit = 15; bit >= 0; --bit) {
          const uint32_t trial = H | ((1u << bit) - 1u);
          uint32_t cnt = 0;
          for (uint64_t i = lane; i - lane < c; i += 32)
            cnt += warp_count(i < c && vv[i] == X && (uint32_t)(kv[i] & 0xffffu) <= trial);
          if (cnt < need) H |= 1u << bit;
        }
      }
    }
    uint64_t o = out_off[p];
    for (uint64_t i = lane; i - lane < c; i += 32) {
      bool keep = false;
      unsigned long long key = 0, val = 0;
      if (i < c) {
        key = kv[i];
        val = vv[i];
        keep = val < X || (val == X && (uint32_t)(key & 0xffffu) <= H);
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const uint64_t at = o + __popc(bal & ((1u << lane) - 1u));
        if (at < capacity) {
          const uint32_t target = (uint32_t)val;
          if (out_neighbors) out_neighbors[at] = target;
          if (out_slots)
            out_slots[at] = tessa_edge{target, from_total_key((uint32_t)(val >> 32)), (uint16_t)(key & 0xffffu), 0};
        }
      }
      o += __popc(bal);
    }
  }
}

}  // namespace reservoirs

namespace {

struct Carve {
  uint8_t* base;
  uint8_t* cur;
  template <class T>
  T* take(size_t count) {
    T* p = reinterpret_cast<T*>(cur);
    cur += (count * sizeof(T) + 255) & ~size_t(255);
    return p;
  }
};

size_t cub_temp_bytes(uint64_t m, uint64_t num_points) {
  size_t sort_temp = 0, scan_temp = 0, scan2_temp = 0;
  cub::DoubleBuffer<unsigned long long> kb(nullptr, nullptr), vb(nullptr, nullptr);
  cub::DeviceRadixSort::SortPairs(nullptr, sort_temp, kb, vb, (int64_t)m, 0, 49);
  cub::DeviceScan::ExclusiveSum(nullptr, scan_temp, (uint32_t*)nullptr, (uint32_t*)nullptr, (int64_t)m);
  cub::DeviceScan::InclusiveSum(nullptr, scan2_temp, (unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                (int64_t)num_points + 1);
  return std::max(sort_temp, std::max(scan_temp, scan2_temp));
}

}  // namespace

size_t reservoir_scratch_bytes(uint64_t m, uint64_t num_points) {
  // keys and values double buffers, run flags and positions, per-source head
  // counts and offsets, CUB temp
  return 4 * ((m * 8 + 255) & ~255ull) + 2 * ((m * 4 + 255) & ~255ull) + 2 * (((num_points + 1) * 8 + 255) & ~255ull) +
         cub_temp_bytes(m, num_points) + 1024;
}

int reduce_reservoirs(const ReservoirCall& r, cudaStream_t st) {
  using namespace reservoirs;
  const uint64_t m = r.edges;
  const int grid = r.sm_count * 8;
  Carve cv{reinterpret_cast<uint8_t*>(r.temp), reinterpret_cast<uint8_t*>(r.temp)};
  unsigned long long* k0 = cv.take<unsigned long long>(m);
  unsigned long long* k1 = cv.take<unsigned long long>(m);
  unsigned long long* v0 = cv.take<unsigned long long>(m);
  unsigned long long* v1 = cv.take<unsigned long long>(m);
  uint32_t* flag = cv.take<uint32_t>(m);
  uint32_t* pos = cv.take<uint32_t>(m);
  unsigned long long* heads = cv.take<unsigned long long>(r.num_points + 1);
  unsigned long long* head_off = cv.take<unsigned long long>(r.num_points + 1);
  void* temp = cv.cur;
  const size_t used = (size_t)(cv.cur - cv.base);
  if (used > r.temp_bytes) return TESSA_ERR_INVALID_ARG;
  const size_t temp_bytes = r.temp_bytes - used;
  unsigned long long* out_off = reinterpret_cast<unsigned long long*>(r.out_offsets);

  // ---- keys of every edge
  if (r.groups == 0) {
    record_keys_kernel<<<grid, 256, 0, st>>>(r.point_ids, r.topk_ids, r.topk_dists, r.hash_fwd, r.hash_rev, r.rows,
                                             r.k, r.num_points, k0, v0, r.d_err);
    if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  } else {
    uint64_t base = 0;
    for (uint32_t g = 0; g < r.groups; ++g) {
      if (r.group_counts[g]) {
        grouped_keys_kernel<<<grid, 256, 0, st>>>(r.group_offsets[g], r.group_edges[g], r.num_points,
                                                  r.group_counts[g], base, k0, v0, r.d_err);
        if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
      }
      base += r.group_counts[g];
    }
  }
  if (cudaMemsetAsync(heads, 0, (r.num_points + 1) * 8, st) != cudaSuccess) return TESSA_ERR_CUDA;
  if (m == 0) {
    if (cudaMemsetAsync(out_off, 0, (r.num_points + 1) * 8, st) != cudaSuccess) return TESSA_ERR_CUDA;
    return TESSA_OK;
  }

  // ---- (source, hash) runs: a radix sort over the key bits in use (source
  //      bits, 16 hash bits and one more, set only in the missing-edge key)
  int src_bits = 0;
  while (src_bits < 32 && (1ull << src_bits) < r.num_points) ++src_bits;
  cub::DoubleBuffer<unsigned long long> kb(k0, k1), vb(v0, v1);
  size_t need = temp_bytes;
  if (cub::DeviceRadixSort::SortPairs(temp, need, kb, vb, (int64_t)m, 0, 17 + src_bits, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  run_kernel<<<grid, 256, 0, st>>>(kb.Current(), vb.Current(), m, flag, heads);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  need = temp_bytes;
  if (cub::DeviceScan::ExclusiveSum(temp, need, flag, pos, (int64_t)m, st) != cudaSuccess) return TESSA_ERR_CUDA;
  // heads compacted into the sort's spare buffers, in (source, hash) order
  unsigned long long* hk = kb.Alternate();
  unsigned long long* hv = vb.Alternate();
  compact_kernel<<<grid, 256, 0, st>>>(kb.Current(), vb.Current(), flag, pos, m, hk, hv);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;

  // ---- per-source head offsets and output offsets
  kept_kernel<<<grid, 256, 0, st>>>(heads, r.num_points, r.l_max, out_off);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  need = temp_bytes;
  if (cub::DeviceScan::InclusiveSum(temp, need, out_off + 1, out_off + 1, (int64_t)r.num_points, st) != cudaSuccess)
    return TESSA_ERR_CUDA;
  need = temp_bytes;
  if (cub::DeviceScan::ExclusiveSum(temp, need, heads, head_off, (int64_t)r.num_points + 1, st) != cudaSuccess)
    return TESSA_ERR_CUDA;

  // ---- the l_max best per-hash minima of every source, in hash order
  select_kernel<<<grid, 256, 0, st>>>(hk, hv, head_off, out_off, r.num_points, r.l_max, r.out_neighbors,
                                      r.out_slots, r.capacity);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  return TESSA_OK;
}

}  // namespace tessa
