// Device-side primitives shared by the TESSA sm_100a kernels: mbarrier
// pipelines with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, TMEM loads) and the error word every kernel reports through.
//
// Every spin-wait here is bounded by wall time (%globaltimer): on expiry the
// waiter records TESSA_DEVERR_TIMEOUT in the kernel's error word, raises the
// CTA-local abort flag and returns false, so a broken pipeline ends the kernel
// with an error status instead of hanging the GPU.
#pragma once
#include <stdint.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/tessa_sm100.h"

namespace tessa {

// Device error bits (OR-ed into the kernel's error word; host maps to codes).
constexpr uint32_t TESSA_DEVERR_TIMEOUT = 1u << 0;       // bounded wait expired
constexpr uint32_t TESSA_DEVERR_BAD_ROW = 1u << 1;       // row id outside resident rows
constexpr uint32_t TESSA_DEVERR_BAD_TASK = 1u << 2;      // malformed task descriptor
constexpr uint32_t TESSA_DEVERR_NONFINITE = 1u << 3;     // non-finite input value

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------- mbarrier ---

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `bar` with the given parity to complete.
// Returns false (after recording the timeout) if `timeout_ns` passes or another
// role of this CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                          uint32_t* err_word, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    // Back off so a waiting thread does not take issue slots from the warps
    // sharing its scheduler.
    __nanosleep(spins < 64 ? 32 : 128);
    if ((++spins & 63u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - start > timeout_ns) {
        atomicOr(err_word, TESSA_DEVERR_TIMEOUT);
        *abort_flag = 1u;
        return false;
      }
    }
  }
}

// Cluster-scope variants for CTA pairs (thread-block clusters of two): an
// arrival from the peer CTA on a barrier of this CTA (or the reverse) and a
// wait that acquires at cluster scope.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// mbar_wait for barriers the peer CTA arrives on: same bound, cluster acquire.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                  uint32_t* err_word, uint64_t timeout_ns) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    __nanosleep(spins < 64 ? 32 : 128);
    if ((++spins & 63u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - start > timeout_ns) {
        atomicOr(err_word, TESSA_DEVERR_TIMEOUT);
        *abort_flag = 1u;
        return false;
      }
    }
  }
}
// All threads of both CTAs of the pair: every earlier shared-memory access
// of the cluster (barrier inits included) is visible after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ------------------------------------------------------------------ TMA ---

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory; completion is signalled on
// `bar` as transaction bytes.  x (innermost, bytes for 8-bit data) must be a
// multiple of 16.
// 2-D tiled TMA load into this CTA's shared memory whose completion bytes go
// to the barrier at `bar_cluster_addr` in the pair's first CTA (the CTA that
// issues the pair's MMAs).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, void* smem_dst, uint32_t bar_cluster_addr,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, void* smem_dst, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 1-D bulk copy from global memory into this CTA's own shared memory only;
// both addresses 16-byte aligned, `bytes` a multiple of 16;
// completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------- tcgen05 ---

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
// Pair (cta_group::2) forms: issued by the same warp in both CTAs of the
// pair; both get the same TMEM address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// layout written by TMA with CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 bytes,
// 8-row core groups 1024 bytes apart (stride byte offset), sm_100 descriptor
// version 1, layout type 2 (128B swizzle).  Tiles are 1024-byte aligned so the
// base offset field stays 0.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1u << 16;                       // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;             // stride byte offset
  d |= (uint64_t)1u << 46;                       // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                       // SWIZZLE_128B
  return d;
}

// Instruction descriptor for tcgen05.mma kind::i8: signed int8 A and B, both
// K-major, int32 accumulator, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4)            // D format: S32
         | (1u << 7)          // A format: signed 8-bit
         | (1u << 10)         // B format: signed 8-bit
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_i8_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Same MMA with A read from tensor memory: `tmem_a` addresses lane 0 of the
// A tile, row m in lane m, K bytes packed four to a 32-bit column (K-major).
__device__ __forceinline__ void mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Pair MMA: D (M = 256, rows 128r..128r+127 in CTA r's tensor memory) from A
// in both CTAs' tensor memory at `tmem_a` and B split by columns between the
// two CTAs' shared memory (same descriptor offset in each).  Issued by the
// pair's first CTA.
__device__ __forceinline__ void mma_i8_ts_pair(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on the barrier at `bar_cluster_addr` (either CTA of the pair) when
// the pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives TMEM
// lane (warp quadrant base + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp writes TMEM
// lane (warp quadrant base + t), columns [col, col + 16).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Asynchronous shared-memory -> tensor-memory copy of a 128-row x 32-byte
// matrix (row m to lane m, its 32 bytes to 8 consecutive 32-bit columns),
// the source given by a matrix descriptor as for tcgen05.mma.  Issued by one
// thread; ordered before later tcgen05.mma of the same thread, tracked by
// tcgen05.commit like an MMA.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------ paired f32 arithmetic ---
// sm_100 executes two f32 operations per instruction on a register pair
// (PTX f32x2).  Each lane of the pair rounds exactly as the scalar .rn
// instruction does, and .rn forbids contraction, so results are bit-identical
// to __fmul_rn / __fadd_rn / __fmaf_rn element by element.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// ------------------------------------------------ SQ8 leaf arithmetic ---

// Reference CB:8987-9002 (gpu_persistent_sq_int8_l2_from_dot), bit for bit:
// rn(rn(n_i + n_j) + rn(-2 * rn(rn(s_i * s_j) * (float)dot))), clamped at 0.
__device__ __forceinline__ float sq8_l2_from_dot(int dot, float si, float ni, float sj, float nj) {
  float d = __fadd_rn(__fadd_rn(ni, nj), __fmul_rn(-2.0f, __fmul_rn(__fmul_rn(si, sj), __int2float_rn(dot))));
  return d <= 0.0f ? 0.0f : d;
}

// Reference CB:7229-7259 ordering: within 2e-5 compare target ids, else distances.
__device__ __forceinline__ bool stable_better(float d, uint32_t id, float od, uint32_t oid) {
  float delta = __fsub_rn(d, od);
  return (fabsf(delta) <= 2.0e-5f) ? (id < oid) : (d < od);
}

}  // namespace tessa
