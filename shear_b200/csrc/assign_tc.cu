// TESSA leader assignment replay, SQ8 source, on the tensor cores (sm_100a).
//
// Same result as assign_kernel<true, LG> (assign.cu): for every member row of
// a frozen task, the int8 dots with the task's leaders, the SQ8 distance
// n_p + n_l - 2*s_p*s_l*dot in the contracted single-FFMA form
// (CB:14676-14678), and the reference's four-slot hash-tie insertion
// (CB:6524-6578) over the leaders in ascending slot order, then the first r_h
// slots as (global id, distance).  Only the dots move to the tensor cores:
// they are exact int32 sums either way, so the results are bit-identical.
//
// Per work item (128 member rows of one task):
//   * the member rows and the task's leader rows are gathered by id, one
//     128-byte K slab at a time, with cp.async straight into the 128-byte
//     swizzled K-major layout tcgen05.mma reads (piece j of row r at
//     j ^ (r & 7)), eight threads per row so copies are whole 128-byte
//     segments; two slab buffers, so the next slab's copies are in flight
//     while the current slab's MMAs run;
//   * one thread issues tcgen05.mma.kind::i8, M = 128 rows, N = NB leader slots
//     (the launch's leader count rounded up to 16), K = 32, int32 accumulators
//     in TMEM; tcgen05.commit frees each slab buffer;
//   * warp w reads TMEM lanes 32w..32w+31 (its 32 rows' dots) with tcgen05.ld
//     and runs the distance and the insertion per row.
// The CTA is persistent over work items and keeps its TMEM columns; the next
// item's metadata loads overlap the current item's copies.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace assign {
namespace tc {

constexpr uint32_t kRowsTc = 128;  // member rows per work item (MMA M = TMEM lanes)
constexpr uint32_t kThreadsTc = 128;
constexpr uint32_t kSlabTc = 128;  // K bytes per slab (one 128-byte swizzle atom)
constexpr uint32_t kMmaKTc = 32;
constexpr uint32_t kASlabTc = kRowsTc * kSlabTc;  // 16 KiB
constexpr uint32_t kCtasPerSm = 5;
constexpr uint32_t kMaxNB = 128;  // leader slots per MMA (task leader counts above use the SIMT kernel)

__host__ __device__ constexpr uint32_t tmem_cols_for(uint32_t nb) { return nb <= 32 ? 32 : (nb <= 64 ? 64 : 128); }

__host__ __device__ constexpr uint32_t smem_bytes_tc(uint32_t nb) {
  return 1024u + 2u * (kASlabTc + nb * kSlabTc) + 256u;
}

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

// CB:6524-6578 with slots = 4 (as assign.cu's insert4).
__device__ __forceinline__ void insert4(float d, uint32_t point, uint32_t leader, uint32_t slot, float (&bd)[4],
                                        uint32_t (&bs)[4], uint32_t (&bl)[4]) {
  bool better = d < bd[3];
  uint64_t ck = 0;
  bool ck_ready = false;
  if (fabsf(__fsub_rn(d, bd[3])) <= 2.0e-5f) {
    ck = tie_key(point, leader);
    ck_ready = true;
    const uint64_t fk = tie_key(point, bl[3]);
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
      const uint64_t pk = tie_key(point, bl[j - 1]);
      before = ck < pk || (ck == pk && leader < bl[j - 1]);
    }
    if (!before) break;
    bd[j] = bd[j - 1];
    bs[j] = bs[j - 1];
    bl[j] = bl[j - 1];
    pos = j - 1;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (j == pos) {
      bd[j] = d;
      bs[j] = slot;
      bl[j] = leader;
    }
}

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Per-thread metadata of one work item: its task, the thread's member row and
// (thread t < NB) leader slot t.
struct ItemMeta {
  uint32_t task, r, moff, mcnt, loff, nl, rh;
  uint32_t point, lid, lg;
  bool valid;
  float n_p, s_p, ln, ls;
};

// One level of the item's load chain (steps 0..3 in order).
template <uint32_t NB>
__device__ __forceinline__ void meta_step(const Params& p, uint32_t item, uint32_t step, ItemMeta& m, uint32_t tid) {
  if (step == 0) {
    const uint2 w = p.work[item];
    m.task = w.x;
    m.r = w.y + tid;
  } else if (step == 1) {
    m.moff = p.t_moff[m.task];
    m.mcnt = p.t_mcnt[m.task];
    m.loff = p.t_loff[m.task];
    m.nl = p.t_lcnt[m.task];
    m.rh = p.t_rh[m.task];
  } else if (step == 2) {
    m.valid = m.r < m.mcnt;
    m.point = m.valid ? p.members[m.moff + m.r] : 0u;
    m.lid = (tid < NB && tid < m.nl) ? p.leaders[m.loff + tid] : 0xffffffffu;
  } else {
    if (m.valid && m.point >= p.resident_rows) {
      atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
      m.valid = false;
      m.point = 0u;
    }
    m.n_p = m.valid ? p.sq8_norms[m.point] : 0.f;
    m.s_p = m.valid ? p.scales[m.point] : 0.f;
    m.ln = 0.f;
    m.ls = 0.f;
    m.lg = 0u;
    if (m.lid != 0xffffffffu) {
      if (m.lid >= p.resident_rows) {
        atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
        m.lid = 0xffffffffu;
      } else {
        m.ln = p.sq8_norms[m.lid];
        m.ls = p.scales[m.lid];
        m.lg = p.global_ids[m.lid];
      }
    }
  }
}

template <uint32_t NB>
__global__ void __launch_bounds__(kThreadsTc) assign_tc_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023u));
  uint8_t* a_buf = base;                              // [2][128 rows][128 B]
  uint8_t* b_buf = base + 2u * kASlabTc;              // [2][NB rows][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_buf + 2u * NB * kSlabTc);
  uint64_t* mma_bar = bars;                           // [2] slab buffer b's MMAs done
  uint64_t* done_bar = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  uint32_t* abort_word = tmem_slot + 1;
  // leader slots of the current and the next item (double-buffered)
  __shared__ uint32_t l_ids[2][NB];
  __shared__ float l_norm[2][NB];
  __shared__ float l_scale[2][NB];
  __shared__ uint32_t l_gid[2][NB];
  __shared__ uint32_t m_pt[2][kRowsTc];  // member row of each tile row (0xffffffff: none)

  const uint32_t tid = threadIdx.x, warp = tid >> 5;
  constexpr uint32_t kCols = tmem_cols_for(NB);
  volatile uint32_t* abort_flag = abort_word;
  if (tid == 0) {
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    mbar_init(done_bar, 1);
    *abort_word = 0u;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t idesc = idesc_i8(kRowsTc, NB);
  const uint32_t pd = p.padded_dim;
  const uint32_t nslab = (pd + kSlabTc - 1) / kSlabTc;
  const uint32_t a_addr0 = smem_u32(a_buf), b_addr0 = smem_u32(b_buf);
  uint32_t ph0 = 0, ph1 = 0;  // next phase parity of mma_bar[0], mma_bar[1]
  bool stop = false;

  // Item metadata is a chain of dependent loads (work entry -> task table ->
  // member and leader ids -> norms and scales); the next item's chain is
  // walked one level per slab, just before the slab waits for its copies.
  ItemMeta cur, nxt;
  uint32_t par = 0;  // leader-slot buffer of the current item
  auto put_leaders = [&](const ItemMeta& m, uint32_t q) {
    m_pt[q][tid] = m.valid ? m.point : 0xffffffffu;
    if (tid < NB) {
      l_ids[q][tid] = m.lid;
      l_norm[q][tid] = m.ln;
      l_scale[q][tid] = m.ls;
      l_gid[q][tid] = m.lg;
    }
  };
  // Slab s of the member rows and leader rows of slot buffer q into slab
  // buffer b.  Eight consecutive threads copy one row's 128 contiguous bytes,
  // so a warp's copy instruction covers four whole rows.
  auto stage = [&](uint32_t q, uint32_t s, uint32_t b) {
    const uint32_t k0 = s * kSlabTc;
#pragma unroll
    for (uint32_t i = tid; i < kRowsTc * (kSlabTc / 16); i += kThreadsTc) {
      const uint32_t row = i / (kSlabTc / 16), j = i % (kSlabTc / 16);
      const uint32_t pt = m_pt[q][row];
      const uint32_t off = k0 + j * 16u;
      const uint32_t n = (pt != 0xffffffffu && off < pd) ? 16u : 0u;
      cp_async16(a_addr0 + b * kASlabTc + row * kSlabTc + ((j ^ (row & 7u)) << 4),
                 p.codes + (n ? (uint64_t)pt * pd + off : 0u), n);
    }
    const uint32_t bdst = b_addr0 + b * NB * kSlabTc;
    for (uint32_t i = tid; i < NB * (kSlabTc / 16); i += kThreadsTc) {
      const uint32_t l = i / (kSlabTc / 16), j = i % (kSlabTc / 16);
      const uint32_t lid = l_ids[q][l];
      const uint32_t off = k0 + j * 16u;
      const uint32_t n = (lid != 0xffffffffu && off < pd) ? 16u : 0u;
      cp_async16(bdst + l * kSlabTc + ((j ^ (l & 7u)) << 4), p.codes + (n ? (uint64_t)lid * pd + off : 0u), n);
    }
    cp_async_commit();
  };
  auto wait_buf = [&](uint32_t b) -> bool {
    bool ok = true;
    if (b == 0) {
      ok = mbar_wait(&mma_bar[0], ph0, abort_flag, p.err_word, p.timeout_ns);
      ph0 ^= 1u;
    } else {
      ok = mbar_wait(&mma_bar[1], ph1, abort_flag, p.err_word, p.timeout_ns);
      ph1 ^= 1u;
    }
    return ok;
  };

  uint32_t item = blockIdx.x;
  if (item < p.num_work) {
    for (uint32_t step = 0; step < 4; ++step) meta_step<NB>(p, item, step, cur, tid);
    put_leaders(cur, 0);
    __syncthreads();
    stage(0, 0, 0);
  }
  for (; item < p.num_work && !stop; item += gridDim.x) {
    const uint32_t next = item + gridDim.x;
    const bool has_next = next < p.num_work;
    const uint32_t task = cur.task, nl = cur.nl, rh = cur.rh, r = cur.r, point = cur.point;
    const bool valid = cur.valid;
    const float n_p = cur.n_p, s_p = cur.s_p;

    // Slab 0 is already in flight (issued before the previous item's epilogue).
    bool pend0 = false, pend1 = false;  // buffer b has MMAs not yet waited for
    for (uint32_t s = 0; s < nslab; ++s) {
      const uint32_t b = s & 1u;
      if (s + 1 < nslab) {
        // the buffer of slab s + 1 was read by slab s - 1's MMAs
        if (b == 0 && pend1) {
          stop |= !wait_buf(1);
          pend1 = false;
        } else if (b == 1 && pend0) {
          stop |= !wait_buf(0);
          pend0 = false;
        }
        stage(par, s + 1, b ^ 1u);
        if (has_next && s < 4) meta_step<NB>(p, next, s, nxt, tid);
        cp_async_wait<1>();
      } else {
        if (has_next && s < 4) meta_step<NB>(p, next, s, nxt, tid);
        cp_async_wait<0>();
      }
      fence_proxy_async_smem();  // the copies were generic-proxy writes; the MMA reads through the async proxy
      __syncthreads();
      if (tid == 0 && !stop) {
        tc_fence_after();
        const uint32_t aa = a_addr0 + b * kASlabTc, ba = b_addr0 + b * NB * kSlabTc;
#pragma unroll
        for (uint32_t kk = 0; kk < kSlabTc / kMmaKTc; ++kk)
          mma_i8_ss(tmem_base, smem_desc_sw128(aa + kk * kMmaKTc), smem_desc_sw128(ba + kk * kMmaKTc), idesc,
                    (s | kk) != 0u ? 1u : 0u);
        mma_commit(&mma_bar[b]);
      }
      if (b == 0)
        pend0 = true;
      else
        pend1 = true;
    }
    if (has_next)
      for (uint32_t step = nslab; step < 4; ++step) meta_step<NB>(p, next, step, nxt, tid);
    // both buffers' last commits (the later one covers every MMA of the item)
    if (pend0) stop |= !wait_buf(0);
    if (pend1) stop |= !wait_buf(1);
    stop = __syncthreads_or(stop ? 1 : 0) != 0;
    if (stop) break;
    // Both slab buffers are free: the next item's leader slots and first slab
    // go out now, so their copies overlap this item's epilogue.
    if (has_next) {
      put_leaders(nxt, par ^ 1u);
      __syncthreads();
      stage(par ^ 1u, 0, 0);
    }
    tc_fence_after();

    float bd[4];
    uint32_t bs[4], bl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      bd[j] = 3.402823466e+38F;
      bs[j] = 0xffffffffu;
      bl[j] = 0xffffffffu;
    }
#pragma unroll 1
    for (uint32_t c0 = 0; c0 < NB; c0 += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(tmem_base + ((warp * 32u) << 16) + c0, v);
      tmem_ld_wait();
      if (valid) {
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
          const uint32_t l = c0 + j;
          if (l >= nl) break;
          const uint32_t lid = l_ids[par][l];
          if (lid == 0xffffffffu) continue;
          const float nn = __fadd_rn(n_p, l_norm[par][l]);
          const float t = __fmul_rn(__fmul_rn(2.0f, s_p), l_scale[par][l]);
          const float df = __int2float_rn((int)v[j]);
          float d = p.fused ? __fmaf_rn(-t, df, nn) : __fsub_rn(nn, __fmul_rn(t, df));
          if (d <= 0.0f) d = 0.0f;
          insert4(d, point, lid, l, bd, bs, bl);
        }
      }
    }
    if (valid) {
      const uint64_t out = p.t_out[task] + (uint64_t)r * rh;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if ((uint32_t)j >= rh) break;
        if (bs[j] >= nl) {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
          continue;
        }
        p.out_ids[out + j] = l_gid[par][bs[j]];
        p.out_dists[out + j] = bd[j];
      }
    }
    tc_fence_before();
    __syncthreads();  // all TMEM reads and slot reads done before the next item's MMAs and slot writes
    cur = nxt;
    par ^= 1u;
  }

  cp_async_wait<0>();  // no copy in flight past this point (an aborted item may have left some)
  // Every issued MMA must have landed before TMEM is released.
  if (tid == 0) {
    mma_commit(done_bar);
    uint32_t dummy_abort = 0u;
    mbar_wait(done_bar, 0u, &dummy_abort, p.err_word, p.timeout_ns);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
}

template <uint32_t NB>
static int launch_nb(const Params& prm, int sm_count, cudaStream_t stream) {
  const uint32_t smem = smem_bytes_tc(NB);
  if (cudaFuncSetAttribute(assign_tc_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return TESSA_ERR_CUDA;
  const uint32_t cap = (uint32_t)sm_count * kCtasPerSm;
  const uint32_t grid = prm.num_work < cap ? prm.num_work : cap;
  assign_tc_kernel<NB><<<grid, kThreadsTc, smem, stream>>>(prm);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tc
}  // namespace assign

// SQ8 assignment on the tensor cores when every task has at most 128 leaders;
// TESSA_ERR_UNSUPPORTED otherwise (the caller then runs the SIMT kernel).
int launch_assign_sq8_tc(const assign::Params& prm, uint32_t max_leaders, int sm_count, cudaStream_t stream) {
  if (prm.num_work == 0) return TESSA_OK;
  if (max_leaders == 0 || max_leaders > assign::tc::kMaxNB) return TESSA_ERR_UNSUPPORTED;
  if (max_leaders <= 16) return assign::tc::launch_nb<16>(prm, sm_count, stream);
  if (max_leaders <= 32) return assign::tc::launch_nb<32>(prm, sm_count, stream);
  if (max_leaders <= 64) return assign::tc::launch_nb<64>(prm, sm_count, stream);
  return assign::tc::launch_nb<128>(prm, sm_count, stream);
}

}  // namespace tessa
