// Per-row symmetric int8 (SQ8) quantization on the GPU, bit-exact with the
// reference CPU quantizer (shear-core/src/algorithm/pipnn/dco_sq_int8.rs:
// 1331-1375 quantize_sq_int8_matrix_with_bits, 1431-1466
// quantize_sq_int8_row_with_max_code), which the reference replay uses
// (P/tessa_replay.rs:1291-1296).  The reference's own GPU quantizer
// (CB:17955-18014) tree-reduces the norm and so differs from the CPU bits; this
// kernel keeps the CPU's sequential order instead: one lane walks one row
// front to back, so norm = (((x0*x0) + x1*x1) + ...) with one rounding per op,
// exactly as Rust evaluates `norm += value * value`.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace quant {

constexpr uint32_t kWarps = 4;
constexpr uint32_t kThreads = kWarps * 32;

// One warp per 32 rows.  Pass 1 stages 32 x 32 slabs of x through shared
// memory with coalesced loads (lane = column), then each lane walks its own
// row's slab front to back (lane = row) -- the reference's sequential order
// for the norm -- and tracks max |x|.  Pass 2 writes the codes with lanes
// over columns (x is read again, mostly from L2).
__global__ void __launch_bounds__(kThreads)
    sq8_quantize_rows_kernel(const float* __restrict__ x, uint64_t rows, uint32_t dim, uint32_t padded,
                             float max_code, int8_t* __restrict__ codes, float* __restrict__ scales,
                             float* __restrict__ norms, uint32_t* err_word) {
  __shared__ float tile[kWarps][32][33];
  __shared__ float wscale[kWarps][32];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint64_t nblk = (rows + 31) / 32;
  for (uint64_t blk = blockIdx.x * (uint64_t)kWarps + warp; blk < nblk; blk += (uint64_t)gridDim.x * kWarps) {
    const uint64_t r0 = blk * 32;
    const uint32_t nr = rows - r0 < 32 ? (uint32_t)(rows - r0) : 32u;
    float max_abs = 0.0f, norm = 0.0f;
    bool bad = false;
    for (uint32_t c0 = 0; c0 < dim; c0 += 32) {
      const uint32_t nc = min(32u, dim - c0);
      if (lane < nc) {
#pragma unroll 8
        for (uint32_t i = 0; i < 32; ++i)
          tile[warp][i][lane] = i < nr ? __ldg(x + (r0 + i) * dim + c0 + lane) : 0.0f;
      }
      __syncwarp();
      for (uint32_t j = 0; j < nc; ++j) {
        const float v = tile[warp][lane][j];
        bad |= !isfinite(v);
        max_abs = fmaxf(max_abs, fabsf(v));
        norm = __fadd_rn(norm, __fmul_rn(v, v));
      }
      __syncwarp();
    }
    const bool zero = max_abs == 0.0f;
    const float scale = zero ? 1.0f : __fdiv_rn(max_abs, max_code);
    if (lane < nr) {
      if (bad) atomicOr(err_word, TESSA_DEVERR_NONFINITE);
      scales[r0 + lane] = scale;
      norms[r0 + lane] = norm;
    }
    wscale[warp][lane] = scale;
    const uint32_t zmask = __ballot_sync(0xffffffffu, zero);
    __syncwarp();
    // Pass 2: lane handles 4 consecutive code bytes of a row per step.
    for (uint32_t i = 0; i < nr; ++i) {
      const float sc = wscale[warp][i];
      const bool z = (zmask >> i) & 1u;
      const float* in = x + (r0 + i) * dim;
      int8_t* orow = codes + (r0 + i) * padded;
      for (uint32_t b = lane * 4; b < padded; b += 128) {
        uint32_t w = 0;
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u) {
          const uint32_t a = b + u;
          int cq = 0;
          if (!z && a < dim) {
            float q = roundf(__fdiv_rn(__ldg(in + a), sc));
            q = fminf(fmaxf(q, -max_code), max_code);
            cq = (int)q;
          }
          w |= ((uint32_t)(cq & 0xff)) << (u * 8u);
        }
        if ((padded & 3u) == 0u) {
          *reinterpret_cast<uint32_t*>(orow + b) = w;
        } else {
          for (uint32_t u = 0; u < 4 && b + u < padded; ++u) orow[b + u] = (int8_t)((w >> (u * 8u)) & 0xffu);
        }
      }
    }
    __syncwarp();
  }
}

}  // namespace quant

int launch_quantize_sq8(const float* x, uint64_t rows, uint32_t dim, uint32_t padded, uint32_t bits, int8_t* codes,
                        float* scales, float* norms, uint32_t* d_err, cudaStream_t stream) {
  if (rows == 0) return TESSA_OK;
  float max_code = (float)((1u << (bits - 1)) - 1u);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  uint64_t blocks = ((rows + 31) / 32 + quant::kWarps - 1) / quant::kWarps;
  uint64_t cap = (uint64_t)sms * 16u;
  if (blocks > cap) blocks = cap;
  quant::sq8_quantize_rows_kernel<<<(unsigned)blocks, quant::kThreads, 0, stream>>>(x, rows, dim, padded, max_code,
                                                                                    codes, scales, norms, d_err);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
