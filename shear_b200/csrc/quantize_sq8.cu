// Per-row symmetric int8 (SQ8) quantization on the GPU, bit-exact with the
// reference CPU quantizer (shear-core/src/algorithm/pipnn/dco_sq_int8.rs:
// 1331-1375 quantize_sq_int8_matrix_with_bits, 1431-1466
// quantize_sq_int8_row_with_max_code), which the reference replay uses
// (P/tessa_replay.rs:1291-1296).  The reference's own GPU quantizer
// (CB:17955-18014) tree-reduces the norm and so differs from the CPU bits; this
// kernel keeps the CPU's sequential order instead: one thread walks one row
// front to back, so norm = (((x0*x0) + x1*x1) + ...) with one rounding per op,
// exactly as Rust evaluates `norm += value * value`.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace quant {

constexpr uint32_t kThreads = 128;

__global__ void __launch_bounds__(kThreads)
    sq8_quantize_rows_kernel(const float* __restrict__ x, uint64_t rows, uint32_t dim, uint32_t padded,
                             float max_code, int8_t* __restrict__ codes, float* __restrict__ scales,
                             float* __restrict__ norms, uint32_t* err_word) {
  uint64_t row = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* in = x + row * dim;
  float max_abs = 0.0f, norm = 0.0f;
  bool bad = false;
  for (uint32_t a = 0; a < dim; ++a) {
    float v = __ldg(in + a);
    bad |= !isfinite(v);
    max_abs = fmaxf(max_abs, fabsf(v));
    norm = __fadd_rn(norm, __fmul_rn(v, v));
  }
  if (bad) atomicOr(err_word, TESSA_DEVERR_NONFINITE);
  float scale = 1.0f;
  bool zero = (max_abs == 0.0f);
  if (!zero) scale = __fdiv_rn(max_abs, max_code);
  int8_t* orow = codes + row * padded;
  for (uint32_t base = 0; base < padded; base += 16) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (uint32_t i = 0; i < 16; ++i) {
      uint32_t a = base + i;
      int c = 0;
      if (!zero && a < dim) {
        float q = roundf(__fdiv_rn(__ldg(in + a), scale));
        q = fminf(fmaxf(q, -max_code), max_code);
        c = (int)q;
      }
      w[i >> 2] |= ((uint32_t)(c & 0xff)) << ((i & 3u) * 8u);
    }
    if ((padded & 15u) == 0u) {
      reinterpret_cast<uint4*>(orow)[base / 16] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      // padded_dim need not be a multiple of 16 (any k_align is accepted).
      for (uint32_t i = 0; i < 16 && base + i < padded; ++i)
        orow[base + i] = (int8_t)((w[i >> 2] >> ((i & 3u) * 8u)) & 0xffu);
    }
  }
  scales[row] = scale;
  norms[row] = norm;
}

}  // namespace quant

int launch_quantize_sq8(const float* x, uint64_t rows, uint32_t dim, uint32_t padded, uint32_t bits, int8_t* codes,
                        float* scales, float* norms, uint32_t* d_err, cudaStream_t stream) {
  if (rows == 0) return TESSA_OK;
  float max_code = (float)((1u << (bits - 1)) - 1u);
  uint64_t blocks = (rows + quant::kThreads - 1) / quant::kThreads;
  quant::sq8_quantize_rows_kernel<<<(unsigned)blocks, quant::kThreads, 0, stream>>>(x, rows, dim, padded, max_code,
                                                                                    codes, scales, norms, d_err);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
