// TESSA leader assignment replay on sm_100a: for every member row of a frozen
// assignment task, the best four leader slots (local fan-out 4) under the
// reference's hash-keyed tie rule, then the first r_h of them as
// (global id, distance).
//
// Reference (wbh1765091327/SHEAR, CB = shear-core/src/algorithm/pipnn/
// compute_backend.rs): gpu_tessa_assignment_replay CB:15729-15943; leaders are
// visited in ascending slot order (CB:13614-13634, CB:14782-14908) and each
// distance goes through gpu_persistent_assignment_insert_candidate
// (CB:6524-6578) with tie key splitmix64((point<<32) ^ leader ^ golden)
// (CB:5983-5989, 6510-6520) over LOCAL resident ids.
//
// Distances:
//   FP32 (A0): dot = sequential rn(rn(x*y) + acc) over axes (the tiled FP32
//              executor's order, CB:13829-13842, equal to CB:6077-6087), then
//              rn(rn(n_p + n_l) + rn(-2*dot)) clamped at 0 (CB:13621-13624) --
//              bit-exact with the reference's FP32 SIMT executor.
//   SQ8:       n_p + n_l - 2*s_p*s_l*dot (CB:14676-14678).  The reference
//              leaves contraction to the compiler; `fused` selects the single
//              FFMA form nvcc's default --fmad=true produces, otherwise one
//              rounding per operation.
//
// Layout: one CTA = 128 member rows of one task, one thread per row; leaders
// are streamed through shared memory in groups of LG = 8, 16 or 32 leaders
// (the smallest that holds the largest task) x one K tile, each thread keeps
// LG independent partial dots in registers, member rows load 16 bytes at a
// time and leader tiles are read with broadcast 16-byte shared loads (axis
// order per dot is preserved, so the FP32 sums stay bit-exact).
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace assign {

constexpr uint32_t kRows = 128;     // member rows per CTA
constexpr uint32_t kLeaders = 32;   // leaders per register group
constexpr uint32_t kAxF = 64;       // FP32 axes per K tile
constexpr uint32_t kAxQ = 256;      // SQ8 bytes per K tile


__device__ __forceinline__ uint64_t hash64(uint64_t v) {
  v ^= v >> 30;
  v *= 0xbf58476d1ce4e5b9ull;
  v ^= v >> 27;
  v *= 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

__device__ __forceinline__ uint64_t tie_key(uint32_t point, uint32_t leader) {
  return hash64((((uint64_t)point) << 32) ^ (uint64_t)leader ^ 0x9e3779b97f4a7c15ull);
}

// CB:6524-6578 with slots = 4.
__device__ __forceinline__ void insert4(float d, uint32_t point, uint32_t leader, uint32_t slot, float (&bd)[4],
                                        uint32_t (&bs)[4], uint32_t (&bl)[4]) {
  bool better = d < bd[3];
  uint64_t ck = 0;
  bool ck_ready = false;
  if (fabsf(__fsub_rn(d, bd[3])) <= 2.0e-5f) {
    ck = tie_key(point, leader);
    ck_ready = true;
    uint64_t fk = tie_key(point, bl[3]);
    better = ck < fk || (ck == fk && leader < bl[3]);
  }
  if (!better) return;
  int pos = 3;
#pragma unroll
  for (int j = 3; j >= 1; --j) {
    if (pos != j) break;
    bool before = d < bd[j - 1];
    if (fabsf(__fsub_rn(d, bd[j - 1])) <= 2.0e-5f) {
      if (!ck_ready) {
        ck = tie_key(point, leader);
        ck_ready = true;
      }
      uint64_t pk = tie_key(point, bl[j - 1]);
      before = ck < pk || (ck == pk && leader < bl[j - 1]);
    }
    if (!before) break;
    bd[j] = bd[j - 1];
    bs[j] = bs[j - 1];
    bl[j] = bl[j - 1];
    pos = j - 1;
  }
  // pos is where the candidate lands; write with compile-time indices.
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (j == pos) {
      bd[j] = d;
      bs[j] = slot;
      bl[j] = leader;
    }
}

template <bool SQ8, int LG>
__global__ void __launch_bounds__(kRows) assign_kernel(const Params p) {
  // Leader tiles: LG leaders x one K tile, read by every thread with
  // broadcast 16-byte loads.
  __shared__ __align__(16) float lt_f[SQ8 ? 1 : LG][SQ8 ? 4 : kAxF];
  __shared__ __align__(16) int lt_q[SQ8 ? LG : 1][SQ8 ? kAxQ / 4 : 4];
  __shared__ uint32_t l_ids[LG];
  __shared__ float l_norm[LG];
  __shared__ float l_scale[LG];

  if (blockIdx.x >= p.num_work) return;
  uint2 w = p.work[blockIdx.x];
  uint32_t task = w.x;
  uint32_t moff = p.t_moff[task], mcnt = p.t_mcnt[task];
  uint32_t loff = p.t_loff[task], nl = p.t_lcnt[task], rh = p.t_rh[task];
  uint32_t r = w.y + threadIdx.x;
  bool valid = r < mcnt;
  uint32_t point = valid ? p.members[moff + r] : 0u;
  if (valid && point >= p.resident_rows) {
    atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
    valid = false;
  }
  const float* norms = SQ8 ? p.sq8_norms : p.raw_norms;
  float n_p = valid ? norms[point] : 0.f;
  float s_p = (SQ8 && valid) ? p.scales[point] : 0.f;
  // f32 rows load as float4 when every row starts 16-byte aligned
  const bool vec_rows = (p.dim & 3u) == 0u && (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0u;

  float bd[4];
  uint32_t bs[4], bl[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    bd[j] = 3.402823466e+38F;
    bs[j] = 0xffffffffu;
    bl[j] = 0xffffffffu;
  }

  for (uint32_t lg = 0; lg < nl; lg += LG) {
    uint32_t gl = nl - lg < (uint32_t)LG ? nl - lg : (uint32_t)LG;
    __syncthreads();
    if (threadIdx.x < (uint32_t)LG) {
      uint32_t lid = 0xffffffffu;
      float ln = 0.f, ls = 0.f;
      if (threadIdx.x < gl) {
        lid = p.leaders[loff + lg + threadIdx.x];
        if (lid >= p.resident_rows) {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
          lid = 0xffffffffu;
        } else {
          ln = norms[lid];
          ls = SQ8 ? p.scales[lid] : 0.f;
        }
      }
      l_ids[threadIdx.x] = lid;
      l_norm[threadIdx.x] = ln;
      l_scale[threadIdx.x] = ls;
    }
    float accf[LG];
    int acci[LG];
#pragma unroll
    for (int l = 0; l < LG; ++l) {
      accf[l] = 0.0f;
      acci[l] = 0;
    }
    if constexpr (!SQ8) {
      for (uint32_t a0 = 0; a0 < p.dim; a0 += kAxF) {
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < (uint32_t)LG * kAxF; i += kRows) {
          uint32_t l = i / kAxF, a = i % kAxF;
          uint32_t lid = l_ids[l];
          lt_f[l][a] = (lid != 0xffffffffu && a0 + a < p.dim) ? p.x[(uint64_t)lid * p.dim + a0 + a] : 0.0f;
        }
        __syncthreads();
        const uint32_t na = p.dim - a0 < kAxF ? p.dim - a0 : kAxF;
        const float* xr = p.x + (uint64_t)point * p.dim + a0;
        // Axes strictly in order for every leader: rn(rn(x*y) + acc).
        uint32_t a = 0;
        if (vec_rows) {
          for (; a + 4 <= na; a += 4) {
            const float4 xv = valid ? __ldg(reinterpret_cast<const float4*>(xr + a)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int l = 0; l < LG; ++l) {
              const float4 yv = *reinterpret_cast<const float4*>(&lt_f[l][a]);
              float t = accf[l];
              t = __fadd_rn(t, __fmul_rn(xv.x, yv.x));
              t = __fadd_rn(t, __fmul_rn(xv.y, yv.y));
              t = __fadd_rn(t, __fmul_rn(xv.z, yv.z));
              accf[l] = __fadd_rn(t, __fmul_rn(xv.w, yv.w));
            }
          }
        }
        for (; a < na; ++a) {
          const float xv = valid ? __ldg(xr + a) : 0.0f;
#pragma unroll
          for (int l = 0; l < LG; ++l) accf[l] = __fadd_rn(accf[l], __fmul_rn(xv, lt_f[l][a]));
        }
      }
    } else {
      // codes rows are padded_dim bytes, a multiple of 16: int4 loads
      for (uint32_t a0 = 0; a0 < p.padded_dim; a0 += kAxQ) {
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < (uint32_t)LG * (kAxQ / 16); i += kRows) {
          uint32_t l = i / (kAxQ / 16), c = i % (kAxQ / 16);
          uint32_t lid = l_ids[l];
          int4 v = make_int4(0, 0, 0, 0);
          if (lid != 0xffffffffu && a0 + c * 16 < p.padded_dim)
            v = *reinterpret_cast<const int4*>(p.codes + (uint64_t)lid * p.padded_dim + a0 + c * 16);
          *reinterpret_cast<int4*>(&lt_q[l][c * 4]) = v;
        }
        __syncthreads();
        const uint32_t nc = (p.padded_dim - a0 < kAxQ ? p.padded_dim - a0 : kAxQ) / 16;
        const int4* cr = reinterpret_cast<const int4*>(p.codes + (uint64_t)point * p.padded_dim + a0);
        for (uint32_t c = 0; c < nc; ++c) {
          const int4 cv = valid ? __ldg(cr + c) : make_int4(0, 0, 0, 0);
#pragma unroll
          for (int l = 0; l < LG; ++l) {
            const int4 lv = *reinterpret_cast<const int4*>(&lt_q[l][c * 4]);
            int t = acci[l];
            t = __dp4a(cv.x, lv.x, t);
            t = __dp4a(cv.y, lv.y, t);
            t = __dp4a(cv.z, lv.z, t);
            acci[l] = __dp4a(cv.w, lv.w, t);
          }
        }
      }
    }
    if (valid) {
#pragma unroll
      for (int l = 0; l < LG; ++l) {
        if ((uint32_t)l >= gl) break;
        uint32_t lid = l_ids[l];
        if (lid == 0xffffffffu) continue;
        float d;
        if constexpr (!SQ8) {
          d = __fadd_rn(__fadd_rn(n_p, l_norm[l]), __fmul_rn(-2.0f, accf[l]));
        } else {
          float nn = __fadd_rn(n_p, l_norm[l]);
          float t = __fmul_rn(__fmul_rn(2.0f, s_p), l_scale[l]);
          float df = __int2float_rn(acci[l]);
          d = p.fused ? __fmaf_rn(-t, df, nn) : __fsub_rn(nn, __fmul_rn(t, df));
        }
        if (d <= 0.0f) d = 0.0f;
        insert4(d, point, lid, lg + l, bd, bs, bl);
      }
    }
  }

  if (!valid) return;
  uint64_t out = p.t_out[task] + (uint64_t)r * rh;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if ((uint32_t)j >= rh) break;
    if (bs[j] >= nl) {
      atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
      continue;
    }
    p.out_ids[out + j] = p.global_ids[bl[j]];
    p.out_dists[out + j] = bd[j];
  }
}

// FP32 rows whose starts are all 16-byte aligned (dim % 4 == 0): member rows
// and the leader group stream through shared memory in 128-byte K stages
// (32 axes) with cp.async, two stages in flight.  Eight consecutive threads
// copy one row's 128 contiguous bytes, so a warp's copy instruction covers
// four whole row segments; each thread then reads its own row from a padded
// buffer (conflict-free 16-byte loads) and the leader stage with broadcast
// loads.  The per-leader sums keep the axis order of assign_kernel:
// rn(rn(x*y) + acc), axis by axis.
constexpr uint32_t kStage = 128;          // row bytes per K stage
constexpr uint32_t kPitch = kStage + 16;  // padded row buffer pitch

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int LG>
__global__ void __launch_bounds__(kRows) assign_f32_staged_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t stg[];
  uint8_t* rows_buf = stg;                        // [2][kRows][kPitch]
  uint8_t* lead_buf = stg + 2u * kRows * kPitch;  // [2][LG][kStage]
  __shared__ uint32_t l_ids[LG];
  __shared__ float l_norm[LG];
  __shared__ uint32_t m_pt[kRows];

  if (blockIdx.x >= p.num_work) return;
  const uint2 w = p.work[blockIdx.x];
  const uint32_t task = w.x;
  const uint32_t moff = p.t_moff[task], mcnt = p.t_mcnt[task];
  const uint32_t loff = p.t_loff[task], nl = p.t_lcnt[task], rh = p.t_rh[task];
  const uint32_t tid = threadIdx.x;
  const uint32_t r = w.y + tid;
  bool valid = r < mcnt;
  uint32_t point = valid ? p.members[moff + r] : 0u;
  if (valid && point >= p.resident_rows) {
    atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
    valid = false;
    point = 0u;
  }
  m_pt[tid] = valid ? point : 0xffffffffu;
  const float n_p = valid ? p.raw_norms[point] : 0.f;
  const uint32_t row_bytes = p.dim * 4u;
  const uint8_t* base = reinterpret_cast<const uint8_t*>(p.x);
  const uint32_t nstage = (row_bytes + kStage - 1) / kStage;
  const uint32_t rows_addr = smem_u32(rows_buf), lead_addr = smem_u32(lead_buf);

  float bd[4];
  uint32_t bs[4], bl[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    bd[j] = 3.402823466e+38F;
    bs[j] = 0xffffffffu;
    bl[j] = 0xffffffffu;
  }

  auto issue = [&](uint32_t st, uint32_t b) {
    const uint32_t b0 = st * kStage;
#pragma unroll
    for (uint32_t i = tid; i < kRows * (kStage / 16); i += kRows) {
      const uint32_t row = i / (kStage / 16), c = i % (kStage / 16);
      const uint32_t pt = m_pt[row];
      const uint32_t off = b0 + c * 16u;
      const uint32_t n = (pt != 0xffffffffu && off < row_bytes) ? 16u : 0u;
      cp_async16(rows_addr + (b * kRows + row) * kPitch + c * 16u, base + (n ? (uint64_t)pt * row_bytes + off : 0u), n);
    }
    for (uint32_t i = tid; i < (uint32_t)LG * (kStage / 16); i += kRows) {
      const uint32_t l = i / (kStage / 16), c = i % (kStage / 16);
      const uint32_t lid = l_ids[l];
      const uint32_t off = b0 + c * 16u;
      const uint32_t n = (lid != 0xffffffffu && off < row_bytes) ? 16u : 0u;
      cp_async16(lead_addr + (b * LG + l) * kStage + c * 16u, base + (n ? (uint64_t)lid * row_bytes + off : 0u), n);
    }
    cp_async_commit();
  };

  for (uint32_t lg = 0; lg < nl; lg += LG) {
    const uint32_t gl = nl - lg < (uint32_t)LG ? nl - lg : (uint32_t)LG;
    __syncthreads();
    if (tid < (uint32_t)LG) {
      uint32_t lid = 0xffffffffu;
      float ln = 0.f;
      if (tid < gl) {
        lid = p.leaders[loff + lg + tid];
        if (lid >= p.resident_rows) {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
          lid = 0xffffffffu;
        } else {
          ln = p.raw_norms[lid];
        }
      }
      l_ids[tid] = lid;
      l_norm[tid] = ln;
    }
    __syncthreads();
    float accf[LG];
#pragma unroll
    for (int l = 0; l < LG; ++l) accf[l] = 0.0f;
    issue(0, 0);
    for (uint32_t st = 0; st < nstage; ++st) {
      const uint32_t b = st & 1u;
      if (st + 1 < nstage) {
        issue(st + 1, b ^ 1u);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const uint8_t* rsrc = rows_buf + (b * kRows + tid) * kPitch;
      const uint8_t* lsrc = lead_buf + b * LG * kStage;
      const uint32_t rem = row_bytes - st * kStage;
      const uint32_t nchunk = (rem < kStage ? rem : kStage) / 16u;
      for (uint32_t c = 0; c < nchunk; ++c) {
        const float4 xv = *reinterpret_cast<const float4*>(rsrc + c * 16u);
        const uint64_t x01 = f2_pack(xv.x, xv.y), x23 = f2_pack(xv.z, xv.w);
#pragma unroll
        for (int l = 0; l < LG; ++l) {
          const float4 yv = *reinterpret_cast<const float4*>(lsrc + l * kStage + c * 16u);
          // products of two adjacent axes per paired instruction (each rounded
          // as __fmul_rn), then the sums strictly in axis order
          float p0, p1, p2, p3;
          f2_unpack(f2_mul(x01, f2_pack(yv.x, yv.y)), p0, p1);
          f2_unpack(f2_mul(x23, f2_pack(yv.z, yv.w)), p2, p3);
          float t = accf[l];
          t = __fadd_rn(t, p0);
          t = __fadd_rn(t, p1);
          t = __fadd_rn(t, p2);
          accf[l] = __fadd_rn(t, p3);
        }
      }
      __syncthreads();  // buffer b is refilled by the next stage's copies
    }
    if (valid) {
#pragma unroll
      for (int l = 0; l < LG; ++l) {
        if ((uint32_t)l >= gl) break;
        const uint32_t lid = l_ids[l];
        if (lid == 0xffffffffu) continue;
        float d = __fadd_rn(__fadd_rn(n_p, l_norm[l]), __fmul_rn(-2.0f, accf[l]));
        if (d <= 0.0f) d = 0.0f;
        insert4(d, point, lid, lg + l, bd, bs, bl);
      }
    }
  }

  if (!valid) return;
  const uint64_t out = p.t_out[task] + (uint64_t)r * rh;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if ((uint32_t)j >= rh) break;
    if (bs[j] >= nl) {
      atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
      continue;
    }
    p.out_ids[out + j] = p.global_ids[bl[j]];
    p.out_dists[out + j] = bd[j];
  }
}

}  // namespace assign


template <int LG>
static void launch_f32_staged(const assign::Params& prm, cudaStream_t stream) {
  const uint32_t smem = 2u * assign::kRows * assign::kPitch + 2u * LG * assign::kStage;
  cudaFuncSetAttribute(assign::assign_f32_staged_kernel<LG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  assign::assign_f32_staged_kernel<LG><<<prm.num_work, assign::kRows, smem, stream>>>(prm);
}

template <bool SQ8>
static void launch_lg(const assign::Params& prm, uint32_t max_leaders, cudaStream_t stream) {
  // f32 rows stage through shared memory when every row starts 16-byte aligned
  const bool staged = !SQ8 && (prm.dim & 3u) == 0u && (reinterpret_cast<uintptr_t>(prm.x) & 15u) == 0u;
  if (max_leaders <= 8) {
    if (staged)
      launch_f32_staged<8>(prm, stream);
    else
      assign::assign_kernel<SQ8, 8><<<prm.num_work, assign::kRows, 0, stream>>>(prm);
  } else if (max_leaders <= 16) {
    if (staged)
      launch_f32_staged<16>(prm, stream);
    else
      assign::assign_kernel<SQ8, 16><<<prm.num_work, assign::kRows, 0, stream>>>(prm);
  } else {
    if (staged)
      launch_f32_staged<32>(prm, stream);
    else
      assign::assign_kernel<SQ8, 32><<<prm.num_work, assign::kRows, 0, stream>>>(prm);
  }
}

// max_leaders: the largest leader count of any task (picks the register group).
int launch_assign(const assign::Params& prm, bool sq8, uint32_t max_leaders, int sm_count, cudaStream_t stream) {
  if (prm.num_work == 0) return TESSA_OK;
  if (sq8) {
    const int rc = launch_assign_sq8_tc(prm, max_leaders, sm_count, stream);
    if (rc != TESSA_ERR_UNSUPPORTED) return rc;
    launch_lg<true>(prm, max_leaders, stream);
  } else
    launch_lg<false>(prm, max_leaders, stream);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
