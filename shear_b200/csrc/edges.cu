// Candidate edges of the leaf lists for the host reducer (HashPrune / TierLift):
// per-point sketches, the two personalised-residual hashes of every leaf slot,
// and the forward / reverse edge expansion in the reference's order.
//
// Reference (wbh1765091327/SHEAR, P = shear-core/src/algorithm/pipnn/):
//   * sketch of point i, hyperplane h = sum over axes in order of x[a] * H[h][a]
//     in f32, one rounding per multiply and per add (`acc += a * b`,
//     P/hash_prune.rs:2208-2232 fill_sketch_row; the hyperplanes come from
//     generate_hyperplanes, :2196-2206, and are an input here);
//   * compute_hash(p, c): bit b = (sketch_c[b] - sketch_p[b] >= 0)
//     (P/hash_prune.rs:2239-2251);
//   * per leaf row i and rank r with j = topk_ids[i*k+r] != u32::MAX and a
//     finite distance d: edge (i -> j, compute_hash(s_i, s_j), d), then
//     (j -> i, compute_hash(s_j, s_i), d)  (P/leaf_build.rs:1749-1808).
//
// B200 split: the GPU computes the sketches (HBM-bound, one pass over the
// rows) and the two 16-bit hashes of every leaf slot right after the leaf
// kernel (4 bytes per slot next to the 8 bytes of ids and distances the host
// receives anyway); the host then expands edges with no sketch gathers.
#include <algorithm>
#include <cmath>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace edges {

constexpr uint32_t kSkWarps = 4;
constexpr uint32_t kSkThreads = kSkWarps * 32;
constexpr uint32_t kMaxPlanes = 16;

// One warp per 32 rows: 32 x 32 slabs of x go through shared memory with
// coalesced loads (lane = column), and the matching 32 columns of the m
// hyperplanes are staged beside them (column-major, 16 floats per column, so
// a lane reads four planes with one broadcast float4 load); then lane r walks
// row r's slab in axis order and advances its m sequential sums (m
// independent chains).
__global__ void __launch_bounds__(kSkThreads)
    sketch_rows_kernel(const float* __restrict__ x, uint64_t rows, uint32_t dim, const float* __restrict__ planes,
                       uint32_t m, float* __restrict__ out) {
  __shared__ float tile[kSkWarps][32][33];
  __shared__ __align__(16) float ptile[kSkWarps][32][kMaxPlanes];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint64_t nblk = (rows + 31) / 32;
  for (uint64_t blk = blockIdx.x * (uint64_t)kSkWarps + warp; blk < nblk; blk += (uint64_t)gridDim.x * kSkWarps) {
    const uint64_t r0 = blk * 32;
    const uint32_t nr = rows - r0 < 32 ? (uint32_t)(rows - r0) : 32u;
    float acc[kMaxPlanes];
#pragma unroll
    for (uint32_t h = 0; h < kMaxPlanes; ++h) acc[h] = 0.0f;
    for (uint32_t c0 = 0; c0 < dim; c0 += 32) {
      const uint32_t nc = dim - c0 < 32 ? dim - c0 : 32u;
      if (lane < nc) {
#pragma unroll 8
        for (uint32_t i = 0; i < 32; ++i) tile[warp][i][lane] = i < nr ? __ldg(x + (r0 + i) * dim + c0 + lane) : 0.0f;
#pragma unroll
        for (uint32_t h = 0; h < kMaxPlanes; ++h)
          ptile[warp][lane][h] = h < m ? __ldg(planes + (uint64_t)h * dim + c0 + lane) : 0.0f;
      }
      __syncwarp();
      for (uint32_t j = 0; j < nc; ++j) {
        const float v = tile[warp][lane][j];
        const float4* pj = reinterpret_cast<const float4*>(&ptile[warp][j][0]);
#pragma unroll
        for (uint32_t q = 0; q < kMaxPlanes / 4; ++q) {
          if (4 * q < m) {
            const float4 w = pj[q];
            acc[4 * q] = __fadd_rn(acc[4 * q], __fmul_rn(v, w.x));
            acc[4 * q + 1] = __fadd_rn(acc[4 * q + 1], __fmul_rn(v, w.y));
            acc[4 * q + 2] = __fadd_rn(acc[4 * q + 2], __fmul_rn(v, w.z));
            acc[4 * q + 3] = __fadd_rn(acc[4 * q + 3], __fmul_rn(v, w.w));
          }
        }
      }
      __syncwarp();
    }
    if (lane < nr) {
      float* o = out + (r0 + lane) * m;
#pragma unroll
      for (uint32_t h = 0; h < kMaxPlanes; ++h)
        if (h < m) o[h] = acc[h];
    }
  }
}

// Both hashes of every (row, rank) slot of a leaf batch.  Slots without a
// candidate (id 0xffffffff) get 0; ids outside the sketch store are flagged.
// Thread = (row, rank) with rank fastest, so a warp covers whole rows and the
// row's sketch comes from L1; sketches with a width that is a multiple of 4
// load as float4.
template <bool VEC>
__global__ void edge_hashes_kernel(const uint32_t* __restrict__ point_ids, const uint32_t* __restrict__ topk_ids,
                                   uint64_t rows, uint32_t k, const float* __restrict__ sketches,
                                   uint64_t sketch_rows, uint32_t width, uint32_t m_bits,
                                   uint16_t* __restrict__ hash_fwd, uint16_t* __restrict__ hash_rev,
                                   uint32_t* __restrict__ err) {
  const uint64_t n = rows * k;
  for (uint64_t s = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; s < n; s += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = n <= 0xffffffffull ? (uint64_t)((uint32_t)s / k) : s / k;
    const uint32_t i = __ldg(point_ids + row);
    const uint32_t j = __ldg(topk_ids + s);
    uint32_t hf = 0, hr = 0;
    if (j != 0xffffffffu) {
      if (i >= sketch_rows || j >= sketch_rows) {
        atomicOr(err, TESSA_DEVERR_BAD_ROW);
      } else {
        float a[16], c[16];
        const float* si = sketches + (uint64_t)i * width;
        const float* sj = sketches + (uint64_t)j * width;
        if constexpr (VEC) {
#pragma unroll
          for (uint32_t q = 0; q < 4; ++q)
            if (4 * q < m_bits) {
              const float4 u = __ldg(reinterpret_cast<const float4*>(si) + q);
              const float4 v = __ldg(reinterpret_cast<const float4*>(sj) + q);
              a[4 * q] = u.x; a[4 * q + 1] = u.y; a[4 * q + 2] = u.z; a[4 * q + 3] = u.w;
              c[4 * q] = v.x; c[4 * q + 1] = v.y; c[4 * q + 2] = v.z; c[4 * q + 3] = v.w;
            }
        } else {
#pragma unroll
          for (uint32_t b = 0; b < 16; ++b)
            if (b < m_bits) {
              a[b] = __ldg(si + b);
              c[b] = __ldg(sj + b);
            }
        }
#pragma unroll
        for (uint32_t b = 0; b < 16; ++b)
          if (b < m_bits) {
            hf |= (__fsub_rn(c[b], a[b]) >= 0.0f ? 1u : 0u) << b;
            hr |= (__fsub_rn(a[b], c[b]) >= 0.0f ? 1u : 0u) << b;
          }
      }
    }
    hash_fwd[s] = (uint16_t)hf;
    hash_rev[s] = (uint16_t)hr;
  }
}

// Per-leaf form (one CTA per leaf, as the reference flushes one leaf batch at
// a time): the leaf's sketches are gathered once into shared memory in leaf
// order and a shared-memory open-addressing table maps global id -> leaf row,
// so each slot reads its two sketches from shared memory instead of gathering
// the candidate's row from the store.  A candidate that is not a member of its
// leaf is an error, as in the reference (P/leaf_build.rs:1771-1777).
constexpr uint32_t kLeafThreads = 512;
constexpr uint32_t kUnroll = 8;  // slots per thread per pass
constexpr uint32_t kEmptyKey = 0xffffffffu;

__device__ __forceinline__ uint32_t table_slot(uint32_t key, uint32_t log2cap) {
  return (key * 0x9E3779B1u) >> (32u - log2cap);
}

__global__ void __launch_bounds__(kLeafThreads)
    leaf_edge_hashes_kernel(const uint32_t* __restrict__ point_ids, const uint32_t* __restrict__ topk_ids,
                            const uint64_t* __restrict__ leaf_starts, const uint32_t* __restrict__ leaf_sizes,
                            uint32_t leaf_count, uint32_t k, const float* __restrict__ sketches,
                            uint64_t sketch_rows, uint32_t width, uint32_t m_bits, uint32_t log2cap,
                            uint16_t* __restrict__ hash_fwd, uint16_t* __restrict__ hash_rev,
                            uint32_t* __restrict__ err) {
  extern __shared__ __align__(16) uint8_t esm[];
  const uint32_t cap = 1u << log2cap;
  uint32_t* keys = reinterpret_cast<uint32_t*>(esm);
  uint32_t* vals = keys + cap;
  float4* sk = reinterpret_cast<float4*>(vals + cap);  // [rows][m4]: m_bits floats, zero padded
  const uint32_t m4 = (m_bits + 3u) / 4u;
  for (uint32_t leaf = blockIdx.x; leaf < leaf_count; leaf += gridDim.x) {
    const uint64_t base = leaf_starts[leaf];
    const uint32_t n = leaf_sizes[leaf];
    for (uint32_t t = threadIdx.x; t < cap; t += blockDim.x) keys[t] = kEmptyKey;
    __syncthreads();
    for (uint32_t r = threadIdx.x; r < n; r += blockDim.x) {
      const uint32_t g = __ldg(point_ids + base + r);
      if (g >= sketch_rows || g == kEmptyKey) {
        atomicOr(err, TESSA_DEVERR_BAD_ROW);
        for (uint32_t q = 0; q < m4; ++q) sk[r * m4 + q] = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      const float* src = sketches + (uint64_t)g * width;
      float v[16];
#pragma unroll
      for (uint32_t b = 0; b < 16; ++b) v[b] = b < m_bits ? __ldg(src + b) : 0.0f;  // all loads before the stores
#pragma unroll
      for (uint32_t q = 0; q < 4; ++q)
        if (q < m4) sk[r * m4 + q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      // First insert of a global id wins; a repeated id has the same sketch.
      // (the table is at most half full, so a free slot lies within cap probes)
      uint32_t t = table_slot(g, log2cap);
      for (uint32_t probe = 0; probe < cap; ++probe) {
        const uint32_t prev = atomicCAS(keys + t, kEmptyKey, g);
        if (prev == kEmptyKey) {
          vals[t] = r;
          break;
        }
        if (prev == g) break;
        t = (t + 1u) & (cap - 1u);
      }
    }
    __syncthreads();
    // The leaf's slots are contiguous (rows base .. base+n, k each): a thread
    // takes kUnroll of them per pass with all id loads issued first, so a pass
    // keeps kUnroll loads per thread in flight.
    const uint32_t nslots = n * k;
    const uint64_t o0 = base * k;
    for (uint32_t s0 = threadIdx.x; s0 < nslots; s0 += blockDim.x * kUnroll) {
      uint32_t jj[kUnroll];
#pragma unroll
      for (uint32_t u = 0; u < kUnroll; ++u) {
        const uint32_t s = s0 + u * blockDim.x;
        jj[u] = s < nslots ? __ldg(topk_ids + o0 + s) : kEmptyKey;
      }
#pragma unroll 1
      for (uint32_t u = 0; u < kUnroll; ++u) {
      const uint32_t s = s0 + u * blockDim.x;
      if (s >= nslots) break;
      const uint32_t r = s / k;
      const uint64_t o = o0 + s;
      const uint32_t j = jj[u];
      uint32_t hf = 0, hr = 0;
      if (j != kEmptyKey) {
        uint32_t t = table_slot(j, log2cap), p = kEmptyKey;
        // at most cap probes: the table is at most half full, so an empty slot ends a miss
        for (uint32_t probe = 0; probe < cap; ++probe) {
          const uint32_t key = keys[t];
          if (key == j) {
            p = vals[t];
            break;
          }
          if (key == kEmptyKey) break;
          t = (t + 1u) & (cap - 1u);
        }
        if (p == kEmptyKey) {
          atomicOr(err, TESSA_DEVERR_BAD_TASK);  // candidate outside its leaf
        } else {
          float a[16], c[16];
#pragma unroll
          for (uint32_t q = 0; q < 4; ++q)
            if (q < m4) {
              const float4 u = sk[r * m4 + q], w = sk[p * m4 + q];
              a[4 * q] = u.x; a[4 * q + 1] = u.y; a[4 * q + 2] = u.z; a[4 * q + 3] = u.w;
              c[4 * q] = w.x; c[4 * q + 1] = w.y; c[4 * q + 2] = w.z; c[4 * q + 3] = w.w;
            }
#pragma unroll
          for (uint32_t b = 0; b < 16; ++b)
            if (b < m_bits) {
              hf |= (__fsub_rn(c[b], a[b]) >= 0.0f ? 1u : 0u) << b;
              hr |= (__fsub_rn(a[b], c[b]) >= 0.0f ? 1u : 0u) << b;
            }
        }
      }
      hash_fwd[o] = (uint16_t)hf;
      hash_rev[o] = (uint16_t)hr;
      }
    }
    __syncthreads();
  }
}

}  // namespace edges

int launch_sketch_rows(const float* x, uint64_t rows, uint32_t dim, const float* planes, uint32_t m, float* out,
                       int sm_count, cudaStream_t stream) {
  if (rows == 0) return TESSA_OK;
  if (m == 0 || m > edges::kMaxPlanes) return TESSA_ERR_INVALID_ARG;
  uint64_t blocks = ((rows + 31) / 32 + edges::kSkWarps - 1) / edges::kSkWarps;
  const uint64_t cap = (uint64_t)sm_count * 16u;
  if (blocks > cap) blocks = cap;
  edges::sketch_rows_kernel<<<(unsigned)blocks, edges::kSkThreads, 0, stream>>>(x, rows, dim, planes, m, out);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

int launch_edge_hashes(const uint32_t* point_ids, const uint32_t* topk_ids, uint64_t rows, uint32_t k,
                       const float* sketches, uint64_t sketch_rows, uint32_t width, uint32_t m_bits,
                       uint16_t* hash_fwd, uint16_t* hash_rev, uint32_t* d_err, int sm_count, cudaStream_t stream) {
  const uint64_t n = rows * k;
  if (n == 0) return TESSA_OK;
  uint64_t blocks = (n + 255) / 256;
  const uint64_t cap = (uint64_t)sm_count * 16u;
  if (blocks > cap) blocks = cap;
  // float4 loads need 16-byte aligned sketch rows; they may read up to 3
  // floats past m_bits, inside the row because width >= round_up(m_bits, 4).
  const bool vec = width % 4u == 0u && (reinterpret_cast<uintptr_t>(sketches) & 15u) == 0u;
  if (vec)
    edges::edge_hashes_kernel<true><<<(unsigned)blocks, 256, 0, stream>>>(point_ids, topk_ids, rows, k, sketches,
                                                                        sketch_rows, width, m_bits, hash_fwd, hash_rev,
                                                                        d_err);
  else
    edges::edge_hashes_kernel<false><<<(unsigned)blocks, 256, 0, stream>>>(point_ids, topk_ids, rows, k, sketches,
                                                                         sketch_rows, width, m_bits, hash_fwd,
                                                                         hash_rev, d_err);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

// Shared memory of the per-leaf form for leaves of up to max_rows rows.
uint32_t leaf_edge_smem(uint32_t max_rows, uint32_t m_bits, uint32_t* log2cap) {
  uint32_t l = 1;
  while ((1u << l) < 2u * max_rows) ++l;
  *log2cap = l;
  return (1u << l) * 8u + max_rows * ((m_bits + 3u) / 4u) * 16u;
}

int launch_leaf_edge_hashes(const uint32_t* point_ids, const uint32_t* topk_ids, const uint64_t* d_leaf_starts,
                            const uint32_t* d_leaf_sizes, uint32_t leaf_count, uint32_t max_rows, uint32_t k,
                            const float* sketches, uint64_t sketch_rows, uint32_t width, uint32_t m_bits,
                            uint16_t* hash_fwd, uint16_t* hash_rev, uint32_t* d_err, int sm_count,
                            cudaStream_t stream) {
  if (leaf_count == 0 || k == 0) return TESSA_OK;
  uint32_t log2cap = 0;
  const uint32_t smem = leaf_edge_smem(max_rows, m_bits, &log2cap);
  if (smem > kLeafEdgeSmemMax) return TESSA_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(edges::leaf_edge_hashes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return TESSA_ERR_CUDA;
  const uint32_t per_sm = std::max<uint32_t>(1u, 220u * 1024u / std::max<uint32_t>(smem, 1u));
  const uint64_t cap = (uint64_t)sm_count * std::min<uint32_t>(per_sm, 4u);
  const uint32_t grid = (uint32_t)std::min<uint64_t>(leaf_count, cap);
  edges::leaf_edge_hashes_kernel<<<grid, edges::kLeafThreads, smem, stream>>>(
      point_ids, topk_ids, d_leaf_starts, d_leaf_sizes, leaf_count, k, sketches, sketch_rows, width, m_bits, log2cap,
      hash_fwd, hash_rev, d_err);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

// Host expansion: rows split into contiguous chunks over `threads` host
// threads; each chunk counts its edges, an exclusive scan places the chunks,
// and each writes its edges in row / rank order, so the output order is the
// reference's sequential one.
uint64_t expand_edges_host(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                           const uint16_t* hash_fwd, const uint16_t* hash_rev, uint64_t rows, uint32_t k,
                           uint32_t* out_p, uint32_t* out_c, uint16_t* out_hash, float* out_dist, uint64_t capacity,
                           uint32_t threads) {
  auto valid = [&](uint64_t s) {
    const uint32_t j = topk_ids[s];
    const float d = topk_dists[s];
    return j != 0xffffffffu && std::isfinite(d);
  };
  if (threads == 0) threads = 1;
  const uint64_t chunk_rows = std::max<uint64_t>(1, (rows + threads - 1) / threads);
  const uint32_t nchunks = (uint32_t)((rows + chunk_rows - 1) / chunk_rows);
  std::vector<uint64_t> count(nchunks + 1, 0);
  auto run = [&](auto&& body) {
    std::vector<std::thread> pool;
    for (uint32_t c = 1; c < nchunks; ++c) pool.emplace_back(body, c);
    if (nchunks > 0) body(0u);
    for (auto& t : pool) t.join();
  };
  run([&](uint32_t c) {
    const uint64_t r0 = c * chunk_rows, r1 = std::min(rows, r0 + chunk_rows);
    uint64_t n = 0;
    for (uint64_t s = r0 * k; s < r1 * k; ++s) n += valid(s) ? 2u : 0u;
    count[c + 1] = n;
  });
  for (uint32_t c = 0; c < nchunks; ++c) count[c + 1] += count[c];
  const uint64_t total = count[nchunks];
  if (total > capacity || !out_p) return total;
  run([&](uint32_t c) {
    const uint64_t r0 = c * chunk_rows, r1 = std::min(rows, r0 + chunk_rows);
    uint64_t e = count[c];
    for (uint64_t i = r0; i < r1; ++i) {
      const uint32_t pi = point_ids[i];
      for (uint32_t r = 0; r < k; ++r) {
        const uint64_t s = i * k + r;
        if (!valid(s)) continue;
        const uint32_t j = topk_ids[s];
        const float d = topk_dists[s];
        out_p[e] = pi;
        out_c[e] = j;
        out_hash[e] = hash_fwd[s];
        out_dist[e] = d;
        ++e;
        out_p[e] = j;
        out_c[e] = pi;
        out_hash[e] = hash_rev[s];
        out_dist[e] = d;
        ++e;
      }
    }
  });
  return total;
}

}  // namespace tessa
