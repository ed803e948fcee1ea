// Membership digests of leaf tasks for the TESSA capture sampler.
//
// Reference (wbh1765091327/SHEAR, P = shear-core/src/algorithm/pipnn/):
// every captured task hash covers its member ids through (count, wrapping sum
// of mix(id), xor of rotl(mix(id), id & 63)) with mix = the splitmix64
// finaliser of id + 0x9e3779b97f4a7c15 (P/tessa_capture.rs:274-293).  Both
// reductions are order-free, so one CTA per leaf reduces its members in any
// order and the result is bit-identical; the host then hashes three words per
// leaf instead of copying and sorting every member list.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace cap {

constexpr uint32_t kThreads = 256;

__device__ __forceinline__ uint64_t mix_membership_id(uint32_t v) {
  uint64_t m = (uint64_t)v + 0x9e3779b97f4a7c15ull;
  m = (m ^ (m >> 30)) * 0xbf58476d1ce4e5b9ull;
  m = (m ^ (m >> 27)) * 0x94d049bb133111ebull;
  return m ^ (m >> 31);
}

__device__ __forceinline__ uint64_t rotl64(uint64_t v, uint32_t r) {
  r &= 63u;
  return r ? (v << r) | (v >> (64u - r)) : v;
}

__global__ void __launch_bounds__(kThreads)
    membership_digest_kernel(const uint32_t* __restrict__ ids, const uint32_t* __restrict__ global_ids,
                             const uint64_t* __restrict__ leaf_starts, const uint64_t* __restrict__ leaf_sizes,
                             uint32_t leaf_count, uint64_t* __restrict__ out_sum, uint64_t* __restrict__ out_xor) {
  __shared__ uint64_t ws[kThreads / 32], wx[kThreads / 32];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  for (uint32_t leaf = blockIdx.x; leaf < leaf_count; leaf += gridDim.x) {
    const uint64_t base = leaf_starts[leaf], n = leaf_sizes[leaf];
    uint64_t s = 0, x = 0;
    for (uint64_t i = threadIdx.x; i < n; i += kThreads) {
      uint32_t id = __ldg(ids + base + i);
      if (global_ids) id = __ldg(global_ids + id);
      const uint64_t m = mix_membership_id(id);
      s += m;
      x ^= rotl64(m, id);
    }
#pragma unroll
    for (uint32_t o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      x ^= __shfl_xor_sync(0xffffffffu, x, o);
    }
    if (lane == 0) {
      ws[warp] = s;
      wx[warp] = x;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint64_t ts = 0, tx = 0;
      for (uint32_t w = 0; w < kThreads / 32; ++w) {
        ts += ws[w];
        tx ^= wx[w];
      }
      out_sum[leaf] = ts;
      out_xor[leaf] = tx;
    }
    __syncthreads();
  }
}

}  // namespace cap

int launch_membership_digests(const uint32_t* ids, const uint32_t* global_ids, const uint64_t* d_leaf_starts,
                              const uint64_t* d_leaf_sizes, uint32_t leaf_count, uint64_t* out_sum,
                              uint64_t* out_xor, int sm_count, cudaStream_t stream) {
  if (leaf_count == 0) return TESSA_OK;
  const uint32_t grid = leaf_count < (uint32_t)sm_count * 8u ? leaf_count : (uint32_t)sm_count * 8u;
  cap::membership_digest_kernel<<<grid, cap::kThreads, 0, stream>>>(ids, global_ids, d_leaf_starts, d_leaf_sizes,
                                                                     leaf_count, out_sum, out_xor);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
