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

constexpr uint64_t kQuantTimeoutNs = 2000000000ull;  // bounded pipeline waits: 2 s

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

// ------------------------------------------------------------ tiled path
//
// One persistent CTA per SM streams tiles of TR consecutive rows of x through
// NBUF shared-memory buffers with plain bulk copies (cp.async.bulk, one per
// row, into a padded row pitch), so every element is read from HBM once:
//   warp 0       producer: refills a buffer when its consumers release it;
//   warps 1..4   norms, buffers in turn: lane r walks row r front to back in
//                the reference's sequential order (the pitch makes the lanes'
//                float4 reads conflict-free);
//   warps 5..20  per-row max |x| (order-free), scale, and codes, coalesced.
// Tiles are kept small (<= 56 KiB) so that three or more are in flight per SM
// while one is consumed: HBM latency x the per-SM share of bandwidth.
// The norms and the codes read the same shared-memory tile.
constexpr uint32_t kNormWarps = 4;
constexpr uint32_t kQWarps = 16;          // code warps
constexpr uint32_t kTWarps = 1 + kNormWarps + kQWarps;
constexpr uint32_t kTThreads = kTWarps * 32;
constexpr uint32_t kTMaxBufs = 8;
constexpr uint32_t kTHeader = 256;       // barriers and the abort flag
constexpr uint32_t kTSmemBudget = 220u * 1024u;
constexpr uint32_t kTTileTarget = 56u * 1024u;  // small tiles: several in flight per SM

struct TiledPlan {
  uint32_t tr;          // rows per tile (32, 16, 8 or 4)
  uint32_t nbuf;        // tile buffers
  uint32_t pitch;       // bytes per staged row (16-byte multiple, odd in 16-byte units)
};

__host__ __device__ inline uint32_t tiled_pitch(uint32_t dim) {
  uint32_t units = dim / 4u + 1u;  // dim % 4 == 0: dim*4 bytes + at least one 16-byte pad unit
  if ((units & 1u) == 0u) ++units;
  return units * 16u;
}

// max(a, |b|) propagating NaN (PTX max.NaN): a non-finite element leaves a
// non-finite row maximum, so one test per row replaces one per element.
__device__ __forceinline__ float max_abs_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(fabsf(b)));
  return r;
}

// Code of v for a row with scale sc and r = fl(1/sc) (sc normal, r finite):
// the reference's clamp(round_half_away(fl(v / sc))).  With q = fl(v * r),
// |q - fl(v/sc)| < 2^-22 |q| (three roundings of relative size <= 2^-24).  If
// q lies more than 2^-19 |q| from every half-integer, fl(v/sc) lies on the same
// side of all of them and is no tie, so rint(q) (nearest, ties to even) is the
// answer; e = q - rint(q) is exact, and the distance to the nearest
// half-integer is 0.5 - |e|.  `near` reports the band where the exactly
// rounded quotient must decide instead.  No clamp is needed here:
// |v| <= max|x| gives |q| <= max_code * (1 + 4 * 2^-24) < max_code + 0.5.
__device__ __forceinline__ int sq8_code_fast(float v, float r, bool& near) {
  const float q = __fmul_rn(v, r);
  const float n = rintf(q);
  const float e = __fsub_rn(q, n);
  near = __fmaf_rn(fabsf(q), 0x1p-19f, fabsf(e)) >= 0.5f;
  return (int)n;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d);

// Exact codes of four elements (IEEE quotient, then round half away from zero).
__device__ __noinline__ uint32_t sq8_codes4_exact(float a, float b, float c, float d, float sc, float max_code) {
  const float vv[4] = {a, b, c, d};
  int cq[4];
#pragma unroll
  for (uint32_t u = 0; u < 4; ++u) cq[u] = (int)fminf(fmaxf(roundf(__fdiv_rn(vv[u], sc)), -max_code), max_code);
  return pack4(cq[0], cq[1], cq[2], cq[3]);
}

// Low bytes of a, b, c, d as one little-endian word.
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  const uint32_t lo = __byte_perm((uint32_t)a, (uint32_t)b, 0x0040u);
  const uint32_t hi = __byte_perm((uint32_t)c, (uint32_t)d, 0x0040u);
  return __byte_perm(lo, hi, 0x5410u);
}

__global__ void __launch_bounds__(kTThreads, 1)
    sq8_quantize_tiled_kernel(const float* __restrict__ x, uint64_t rows, uint32_t dim, uint32_t padded,
                              float max_code, TiledPlan plan, int8_t* __restrict__ codes,
                              float* __restrict__ scales, float* __restrict__ norms, uint32_t* err_word,
                              uint64_t timeout_ns) {
  extern __shared__ __align__(128) uint8_t qsm[];
  const uint32_t TR = plan.tr, NB = plan.nbuf, pitch = plan.pitch;
  uint64_t* full = reinterpret_cast<uint64_t*>(qsm);
  uint64_t* empty = full + kTMaxBufs;
  uint32_t* abort_flag_p = reinterpret_cast<uint32_t*>(empty + kTMaxBufs);
  uint8_t* tiles = qsm + kTHeader;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  volatile uint32_t* abort_flag = abort_flag_p;
  if (threadIdx.x == 0) {
    for (uint32_t b = 0; b < NB; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], 1 + kQWarps);  // the tile's norm warp + every code warp
    }
    *abort_flag_p = 0u;
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t ntiles = (rows + TR - 1) / TR;
  const uint32_t row_bytes = dim * 4u;

  if (warp == 0) {
    uint32_t it = 0;
    int32_t last_use[kTMaxBufs];
#pragma unroll
    for (uint32_t b = 0; b < kTMaxBufs; ++b) last_use[b] = -1;
    for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t b = it % NB, use = it / NB;
      const uint64_t r0 = t * TR;
      const uint32_t nr = rows - r0 < TR ? (uint32_t)(rows - r0) : TR;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&empty[b], (use & 1u) ^ 1u, abort_flag, err_word, timeout_ns);
      if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0u) break;
      if (lane == 0) mbar_arrive_expect_tx(&full[b], nr * row_bytes);
      __syncwarp();
      uint8_t* dst = tiles + (size_t)b * TR * pitch;
      for (uint32_t i = lane; i < nr; i += 32)
        bulk_load(dst + i * pitch, x + (r0 + i) * dim, row_bytes, &full[b]);
      last_use[b] = (int32_t)use;
    }
    // Copies still in flight (consumers that gave up) land before the CTA exits.
    if (lane == 0) {
      uint32_t no_abort = 0u;
      for (uint32_t b = 0; b < NB; ++b)
        if (last_use[b] >= 0) mbar_wait(&full[b], (uint32_t)last_use[b] & 1u, &no_abort, err_word, timeout_ns);
    }
  } else if (warp <= kNormWarps) {
    // A norm warp owns whole buffers (b % kNormWarps == nw), so it observes
    // every phase of the full barriers it waits on: a waiter that skipped a
    // phase could take an older phase of the same parity for the current one.
    const uint32_t nw = warp - 1;
    uint32_t it = 0;
    for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      if ((it % NB) % kNormWarps != nw) continue;
      const uint32_t b = it % NB, use = it / NB;
      const uint64_t r0 = t * TR;
      const uint32_t nr = rows - r0 < TR ? (uint32_t)(rows - r0) : TR;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&full[b], use & 1u, abort_flag, err_word, timeout_ns);
      if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0u) break;
      if (lane < nr) {
        const float4* rowp = reinterpret_cast<const float4*>(tiles + ((size_t)b * TR + lane) * pitch);
        float norm = 0.0f;
        const uint32_t n4 = dim / 4u;
#pragma unroll 4
        for (uint32_t q = 0; q < n4; ++q) {
          const float4 v = rowp[q];
          norm = __fadd_rn(norm, __fmul_rn(v.x, v.x));
          norm = __fadd_rn(norm, __fmul_rn(v.y, v.y));
          norm = __fadd_rn(norm, __fmul_rn(v.z, v.z));
          norm = __fadd_rn(norm, __fmul_rn(v.w, v.w));
        }
        norms[r0 + lane] = norm;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[b]);
    }
  } else {
    const uint32_t qw = warp - 1 - kNormWarps;
    uint32_t it = 0;
    for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t b = it % NB, use = it / NB;
      const uint64_t r0 = t * TR;
      const uint32_t nr = rows - r0 < TR ? (uint32_t)(rows - r0) : TR;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&full[b], use & 1u, abort_flag, err_word, timeout_ns);
      if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0u) break;
      for (uint32_t i = qw; i < nr; i += kQWarps) {
        const float* rowp = reinterpret_cast<const float*>(tiles + ((size_t)b * TR + i) * pitch);
        float m = 0.0f;
        for (uint32_t c = lane * 4u; c < dim; c += 128u) {
          const float4 v = *reinterpret_cast<const float4*>(rowp + c);
          m = max_abs_nan(max_abs_nan(m, v.x), v.y);
          m = max_abs_nan(max_abs_nan(m, v.z), v.w);
        }
#pragma unroll
        for (uint32_t o = 16; o > 0; o >>= 1) {
          const float other = __shfl_xor_sync(0xffffffffu, m, o);
          asm("max.NaN.f32 %0, %0, %1;" : "+f"(m) : "f"(other));
        }
        const bool bad = !(m <= 3.402823466e+38F);  // NaN or inf somewhere in the row
        const bool zero = m == 0.0f;
        const float sc = zero ? 1.0f : __fdiv_rn(m, max_code);
        const float r = __frcp_rn(sc);
        const bool exact = !(fabsf(sc) >= 1.17549435e-38F) || !(fabsf(r) <= 3.402823466e+38F);
        if (lane == 0) {
          scales[r0 + i] = sc;
          if (bad) atomicOr(err_word, TESSA_DEVERR_NONFINITE);
        }
        int8_t* orow = codes + (r0 + i) * padded;
        for (uint32_t c = lane * 4u; c < padded; c += 128u) {
          uint32_t w = 0;
          if (!zero && c < dim) {  // dim % 4 == 0: all four columns are inside the row
            const float4 v = *reinterpret_cast<const float4*>(rowp + c);
            bool n0, n1, n2, n3;
            const int c0 = sq8_code_fast(v.x, r, n0), c1 = sq8_code_fast(v.y, r, n1);
            const int c2 = sq8_code_fast(v.z, r, n2), c3 = sq8_code_fast(v.w, r, n3);
            if (exact || n0 || n1 || n2 || n3)
              w = sq8_codes4_exact(v.x, v.y, v.z, v.w, sc, max_code);
            else
              w = pack4(c0, c1, c2, c3);
          }
          if ((padded & 3u) == 0u) {
            *reinterpret_cast<uint32_t*>(orow + c) = w;
          } else {
            for (uint32_t u = 0; u < 4 && c + u < padded; ++u) orow[c + u] = (int8_t)((w >> (u * 8u)) & 0xffu);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[b]);
    }
  }
}

// Rows per tile and buffer count for the tiled path, or false if it does not apply.
static bool tiled_plan(const float* x, uint32_t dim, TiledPlan* plan) {
  if (dim == 0 || dim % 4u != 0u || (reinterpret_cast<uintptr_t>(x) & 15u) != 0u) return false;
  const uint32_t pitch = tiled_pitch(dim);
  uint32_t tr = 32u;
  while (tr > 4u && tr * pitch > kTTileTarget) tr >>= 1;
  uint32_t nb = kTSmemBudget / (tr * pitch);
  if (nb > kTMaxBufs) nb = kTMaxBufs;
  if (nb < 2) return false;
  plan->tr = tr;
  plan->nbuf = nb;
  plan->pitch = pitch;
  return true;
}

}  // namespace quant

int launch_quantize_sq8(const float* x, uint64_t rows, uint32_t dim, uint32_t padded, uint32_t bits, int8_t* codes,
                        float* scales, float* norms, uint32_t* d_err, cudaStream_t stream) {
  if (rows == 0) return TESSA_OK;
  float max_code = (float)((1u << (bits - 1)) - 1u);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  quant::TiledPlan plan;
  if (quant::tiled_plan(x, dim, &plan)) {
    const uint32_t smem = quant::kTHeader + plan.nbuf * plan.tr * plan.pitch;
    if (cudaFuncSetAttribute(quant::sq8_quantize_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return TESSA_ERR_CUDA;
    const uint64_t ntiles = (rows + plan.tr - 1) / plan.tr;
    const uint32_t grid = ntiles < (uint64_t)sms ? (uint32_t)ntiles : (uint32_t)sms;
    quant::sq8_quantize_tiled_kernel<<<grid, quant::kTThreads, smem, stream>>>(
        x, rows, dim, padded, max_code, plan, codes, scales, norms, d_err, kQuantTimeoutNs);
    return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
  }
  uint64_t blocks = ((rows + 31) / 32 + quant::kWarps - 1) / quant::kWarps;
  uint64_t cap = (uint64_t)sms * 16u;
  if (blocks > cap) blocks = cap;
  quant::sq8_quantize_rows_kernel<<<(unsigned)blocks, quant::kThreads, 0, stream>>>(x, rows, dim, padded, max_code,
                                                                                    codes, scales, norms, d_err);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
