// SQ8 leaf all-pairs evaluation with fused per-row bounded top-k, sm_100a.
//
// Reference semantics (wbh1765091327/SHEAR, CB = shear-core/src/algorithm/
// pipnn/compute_backend.rs):
//   * candidates of row r are the other members of its leaf, taken in
//     ascending member position, skipping columns whose local id equals the
//     row's (CB:9569-9650, CB:10046-10096);
//   * distance = gpu_persistent_sq_int8_l2_from_dot (CB:8987-9002);
//   * each candidate goes through gpu_persistent_insert_topk_candidate_fp32
//     (CB:7229-7259) into a k-slot list initialised to (FLT_MAX, 0xffffffff):
//     "better" = |d1-d2| <= 2e-5 ? id1 < id2 : d1 < d2 (not transitive);
//   * output ids are the candidates' global ids, written at (start + r) * k.
//
// How the result is computed without the reference's sequential insertion:
// Let L be a set of k candidates and "<" the eps/id relation above.  If (a)
// every member of L beats every candidate outside L and (b) "<" restricted to
// L is a strict total order, then sequential insertion in ANY order ends with
// exactly L sorted by "<": an L-candidate always passes the list's tail (which
// holds only non-L candidates or empty slots), is never pushed out (only a
// full list of L-candidates could do it), and stops exactly at its rank
// because "<" is transitive on L.  Per row the kernel therefore finds, in any
// column order, every candidate whose distance is within a margin M = 4 eps
// of the k-th smallest distance (the "zone"), sorts the zone by distance,
// splits it into runs of neighbours closer than eps and checks (a) and (b):
// every run up to the one holding rank k must be a transitive tournament
// under "<" (always true for runs of one), and that run must end inside the
// zone (a gap > eps to the next zone entry, or more than eps below the zone's
// upper edge).  Rows that pass are written directly; the rest (a few in 10^4
// on random data) are listed and recomputed by leaf_fallback_kernel with the
// reference's exact sequential insertion.
//
// Per-row selection state (thread = row):
//   * a sorted array of the k smallest distances seen so far, in registers
//     (KS >= k FP32 slots; candidates go in two at a time, 2 min + 1
//     three-input max per slot, branch-free); its maximum theta bounds the
//     k-th smallest distance of the row from above;
//   * a shared-memory log of (distance, global id) for every candidate that
//     was within theta + M when it arrived, compacted against the current
//     bound whenever it fills.  The log always holds the final zone.
//
// B200 design (one persistent CTA per SM, 224 threads):
//   warp 0      TMA producer: A = 128 leaf rows x padded_dim, resident for the
//               tile; B = 128-column chunks streamed in 128-byte K slabs
//               through a ring of shared-memory stages (SWIZZLE_128B).
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (kind::i8,
//               M=128, N=128, K=32, int32 accumulators) into four 128-column
//               TMEM buffers, so MMAs run up to three chunks ahead.
//   warps 2..5  epilogue: thread t owns TMEM lane (leaf row) t; per 32
//               columns it computes the exact reference distances, builds a
//               bit mask of the ones below the row's bound (one funnel shift
//               per column, four independent chains), stashes the distances in shared memory and then
//               pops the marked columns into the log and the sorted array.
//   warp 6      column metadata (scale, norm, global id) of each chunk into a
//               4-slot shared-memory ring, so the epilogue warps never wait
//               on each other.
// The distance matrix never leaves the SM.
//
// Rectangular mode (template flag RECT, the global-D0 assignment of
// quantize_sq8_and_assign_global_d0, P/dco_sq_int8.rs:1929-2070): the same
// pipeline with A = 128-row tiles of a row matrix and B = every row of a
// separate leader matrix, no self exclusion, and the leader's tie key (the
// rank of (leader id, leader index)) in place of the global id.  The zone
// argument above carries over unchanged: only the candidate set differs.
#include "common.cuh"
#include "kernels.h"
#include "leaf_common.cuh"

namespace tessa {
namespace leaf {

constexpr uint32_t kThreads = 224;     // TMA, MMA, 4 epilogue warps, metadata warp
constexpr uint32_t kEpiWarps = 4;
constexpr uint32_t kMetaWarp = 6;
constexpr uint32_t kAccBufs = 4;
constexpr uint32_t kTmemCols = kAccBufs * kBN;  // 512
constexpr uint32_t kASlabBytes = kBM * kSlab;   // 16 KiB
constexpr uint32_t kBStageBytes = kBN * kSlab;  // 16 KiB
constexpr uint32_t kGroups = kBN / kGroup;
constexpr uint32_t kMaxBStages = 8;
constexpr uint32_t kMetaBytes = kMetaSlots * kBN * 12u;  // ring of (scale, norm) + global id
constexpr uint32_t kStashBytes = 4u * 32u * kStashStride * 4u;
constexpr uint32_t kBarBytes = 512u;

struct Smem {
  uint8_t* a;
  uint8_t* b;
  float2* meta_sn;  // [kMetaSlots][kBN] (scale, norm) of a chunk's columns
  uint32_t* meta_g; // [kMetaSlots][kBN] global id
  float* stash;     // [4 warps][32 lanes][kStashStride]
  uint2* log;       // [log_cap][kBM] (distance bits, global id)
  uint64_t* a_full;
  uint64_t* a_empty;
  uint64_t* b_full;
  uint64_t* b_empty;
  uint64_t* t_full;
  uint64_t* t_empty;
  uint64_t* m_full;
  uint64_t* m_empty;
  uint64_t* mma_done;
  uint32_t* tmem_slot;
  uint32_t* abort_flag;
};

__host__ __device__ inline uint32_t smem_bytes(uint32_t num_slabs, uint32_t num_bstages, uint32_t log_cap) {
  return 1024u + num_slabs * kASlabBytes + num_bstages * kBStageBytes + kMetaBytes + kStashBytes +
         log_cap * kBM * kLogEntryBytes + kBarBytes;
}

__device__ __forceinline__ Smem carve(uint8_t* raw, uint32_t num_slabs, uint32_t num_bstages, uint32_t log_cap) {
  uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  Smem s;
  s.a = p;
  p += num_slabs * kASlabBytes;
  s.b = p;
  p += num_bstages * kBStageBytes;
  s.meta_sn = reinterpret_cast<float2*>(p);
  p += kMetaSlots * kBN * 8u;
  s.meta_g = reinterpret_cast<uint32_t*>(p);
  p += kMetaSlots * kBN * 4u;
  s.stash = reinterpret_cast<float*>(p);
  p += kStashBytes;
  s.log = reinterpret_cast<uint2*>(p);
  p += log_cap * kBM * kLogEntryBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p);
  s.a_full = bars + 0;
  s.a_empty = bars + 1;
  s.b_full = bars + 2;
  s.b_empty = s.b_full + kMaxBStages;
  s.t_full = s.b_empty + kMaxBStages;
  s.t_empty = s.t_full + kAccBufs;
  s.m_full = s.t_empty + kAccBufs;
  s.m_empty = s.m_full + kMetaSlots;
  s.mma_done = s.m_empty + kMetaSlots;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.mma_done + 1);
  s.abort_flag = s.tmem_slot + 1;
  return s;
}

// Finish one row: sort the zone, verify order independence, write k results.
// Returns false if the row must be recomputed by the exact fallback.
template <int KS>
__device__ bool finish_row(const Params& p, uint2* log, uint8_t* perm, uint32_t row, uint32_t E,
                           const float (&s)[KS], float thr, uint32_t gid_i, uint64_t out) {
  const uint32_t k = p.k;
  const float theta = s[0];
  const bool complete = !(theta < INFINITY);
  // Rank of each zone entry.  Entries with d <= theta: the number of smaller
  // distances among the k smallest (the sorted array); equal distances take
  // consecutive ranks in log order.  Entries above theta (the margin) follow
  // all of those, ordered by distance.  A zone entry with the row's own
  // global id (a repeated member) sends the row to the exact fallback.
  uint32_t n_inner = 0;
  bool dup = false;
  for (uint32_t e = 0; e < E; ++e) {
    uint2 v = log[e * kBM + row];
    n_inner += (__uint_as_float(v.x) <= theta) ? 1u : 0u;
    dup |= v.y == gid_i;
  }
  if (dup) return false;
  uint64_t occ = 0;
  for (uint32_t e = 0; e < E; ++e) {
    float d = __uint_as_float(log[e * kBM + row].x);
    uint32_t r;
    if (d <= theta) {
      uint32_t r0 = 0, r1 = 0, r2 = 0, r3 = 0;
#pragma unroll
      for (int t = 0; t < KS; t += 4) {
        r0 += (s[t] < d) ? 1u : 0u;
        if (t + 1 < KS) r1 += (s[t + 1] < d) ? 1u : 0u;
        if (t + 2 < KS) r2 += (s[t + 2] < d) ? 1u : 0u;
        if (t + 3 < KS) r3 += (s[t + 3] < d) ? 1u : 0u;
      }
      r = (r0 + r1) + (r2 + r3) - ((uint32_t)KS - k);  // minus the -inf sentinels
    } else {
      r = n_inner;
      for (uint32_t f = 0; f < E; ++f) {
        float df = __uint_as_float(log[f * kBM + row].x);
        r += (df > theta && (df < d || (df == d && f < e))) ? 1u : 0u;
      }
    }
    while (r < 63u && ((occ >> r) & 1ull)) ++r;
    occ |= 1ull << r;
    perm[r] = (uint8_t)e;
  }
  if (occ != (E >= 64u ? ~0ull : ((1ull << E) - 1ull))) return false;  // not a permutation: give up safely

  // One pass over the zone in sorted order.  A run (neighbours closer than
  // eps) is emitted when it closes: runs of one and two directly, longer runs
  // through the tournament check.
  uint32_t q = 0;   // output slots written
  uint32_t rs = 0;  // start of the current run
  float prev = -INFINITY;
  uint2 first = make_uint2(0u, 0u), second = make_uint2(0u, 0u);
  for (uint32_t i = 0; i <= E && q < k; ++i) {
    const bool end = i == E;
    const uint2 vi = end ? make_uint2(0x7f800000u, 0u) : log[perm[i] * kBM + row];
    const float di = __uint_as_float(vi.x);
    const bool close = !end && i > 0 && fabsf(__fsub_rn(di, prev)) <= kTieEps;
    if (i > 0 && !close) {
      const uint32_t len = i - rs;  // run [rs, i) is complete
      // The run holding rank k must end inside the zone: every candidate
      // outside the zone lies above thr, hence more than eps above the run.
      if (q + len >= k && end && !complete && !(__fsub_rn(thr, prev) > kTieEps)) return false;
      if (len == 1) {
        p.out_ids[out + q] = first.y;
        p.out_dists[out + q] = __uint_as_float(first.x);
        ++q;
      } else if (len == 2) {
        // Two candidates: the eps/id rule orders them (trivially transitive).
        const bool sw = stable_better(__uint_as_float(second.x), second.y, __uint_as_float(first.x), first.y);
        const uint2 lo = sw ? second : first, hi = sw ? first : second;
        p.out_ids[out + q] = lo.y;
        p.out_dists[out + q] = __uint_as_float(lo.x);
        ++q;
        if (q < k) {
          p.out_ids[out + q] = hi.y;
          p.out_dists[out + q] = __uint_as_float(hi.x);
          ++q;
        }
      } else {
        // Tournament of the run under the eps/id rule: transitive iff the win
        // counts are 0..len-1 (then "<" orders the run by wins).
        if (len > kMaxRun) return false;
        float rd[kMaxRun];
        uint32_t rg[kMaxRun];
        for (uint32_t t = 0; t < len; ++t) {
          uint2 v = log[perm[rs + t] * kBM + row];
          rd[t] = __uint_as_float(v.x);
          rg[t] = v.y;
        }
        uint32_t wins[kMaxRun];
        uint32_t seen = 0;
        for (uint32_t t = 0; t < len; ++t) {
          uint32_t w = 0;
          for (uint32_t u = 0; u < len; ++u)
            if (u != t && stable_better(rd[t], rg[t], rd[u], rg[u])) ++w;
          wins[t] = w;
          seen |= 1u << w;
        }
        if (seen != (1u << len) - 1u) return false;
        for (uint32_t rank = 0; rank < len && q < k; ++rank) {
          uint32_t want = len - 1 - rank;
          for (uint32_t t = 0; t < len; ++t)
            if (wins[t] == want) {
              p.out_ids[out + q] = rg[t];
              p.out_dists[out + q] = rd[t];
            }
          ++q;
        }
      }
      rs = i;
    }
    if (i == rs) first = vi;
    if (i == rs + 1) second = vi;
    prev = di;
  }
  for (; q < k; ++q) {
    p.out_ids[out + q] = 0xffffffffu;
    p.out_dists[out + q] = 3.402823466e+38F;
  }
  return true;
}

template <int KS, bool RECT>
__global__ void __launch_bounds__(kThreads, 1)
    leaf_topk_sq8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem s = carve(smem_raw, p.num_slabs, p.num_bstages, p.log_cap);
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort_flag = s.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(s.a_full, 1);
    mbar_init(s.a_empty, 1);
    for (uint32_t i = 0; i < p.num_bstages; ++i) {
      mbar_init(&s.b_full[i], 1);
      mbar_init(&s.b_empty[i], 1);
    }
    for (uint32_t i = 0; i < kAccBufs; ++i) {
      mbar_init(&s.t_full[i], 1);
      mbar_init(&s.t_empty[i], kEpiWarps);
    }
    for (uint32_t i = 0; i < kMetaSlots; ++i) {
      mbar_init(&s.m_full[i], 32);
      mbar_init(&s.m_empty[i], kEpiWarps);
    }
    mbar_init(s.mma_done, 1);
    *s.abort_flag = 0u;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(s.tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t bstage = 0, bphase = 0, a_iter = 0;
      for (uint32_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++a_iter) {
        uint2 t;
        uint64_t start;
        uint32_t cnt, ncol;
        tile_span<RECT>(p, tile, t, start, cnt, ncol);
        const uint64_t bstart = RECT ? 0 : start;
        if (!mbar_wait(s.a_empty, (a_iter & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) break;
        mbar_arrive_expect_tx(s.a_full, p.num_slabs * kASlabBytes);
        for (uint32_t sl = 0; sl < p.num_slabs; ++sl)
          tma_load_2d(&tmap_a, s.a + sl * kASlabBytes, s.a_full, (int32_t)(sl * kSlab), (int32_t)(start + t.y));
        uint32_t nchunks = (ncol + kBN - 1) / kBN;
        bool ok = true;
        for (uint32_t c = 0; c < nchunks && ok; ++c) {
          for (uint32_t sl = 0; sl < p.num_slabs; ++sl) {
            if (!mbar_wait(&s.b_empty[bstage], bphase ^ 1u, abort_flag, p.err_word, p.timeout_ns)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&s.b_full[bstage], kBStageBytes);
            tma_load_2d(&tmap_b, s.b + bstage * kBStageBytes, &s.b_full[bstage], (int32_t)(sl * kSlab),
                        (int32_t)(bstart + c * kBN));
            if (++bstage == p.num_bstages) {
              bstage = 0;
              bphase ^= 1u;
            }
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kBM, kBN);
      const uint32_t a_base = smem_u32(s.a);
      const uint32_t b_base = smem_u32(s.b);
      uint32_t bstage = 0, bphase = 0, acc = 0, a_iter = 0;
      bool ok = true;
      for (uint32_t tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++a_iter) {
        uint2 t;
        uint64_t start;
        uint32_t cnt, ncol;
        tile_span<RECT>(p, tile, t, start, cnt, ncol);
        if (!mbar_wait(s.a_full, a_iter & 1u, abort_flag, p.err_word, p.timeout_ns)) break;
        tc_fence_after();
        uint32_t nchunks = (ncol + kBN - 1) / kBN;
        for (uint32_t c = 0; c < nchunks && ok; ++c, ++acc) {
          uint32_t buf = acc % kAccBufs, use = acc / kAccBufs;
          if (!mbar_wait(&s.t_empty[buf], (use & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t tmem_d = tmem_base + buf * kBN;
          for (uint32_t sl = 0; sl < p.num_slabs; ++sl) {
            if (!mbar_wait(&s.b_full[bstage], bphase, abort_flag, p.err_word, p.timeout_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            uint32_t a_addr = a_base + sl * kASlabBytes;
            uint32_t b_addr = b_base + bstage * kBStageBytes;
#pragma unroll
            for (uint32_t kk = 0; kk < kSlab / kMmaK; ++kk) {
              uint64_t ad = smem_desc_sw128(a_addr + kk * kMmaK);
              uint64_t bd = smem_desc_sw128(b_addr + kk * kMmaK);
              mma_i8_ss(tmem_d, ad, bd, idesc, (sl | kk) != 0u ? 1u : 0u);
            }
            mma_commit(&s.b_empty[bstage]);
            if (++bstage == p.num_bstages) {
              bstage = 0;
              bphase ^= 1u;
            }
          }
          if (ok) mma_commit(&s.t_full[buf]);
        }
        if (ok) mma_commit(s.a_empty);
      }
      // Every issued MMA must have landed before TMEM is released.
      mma_commit(s.mma_done);
      uint32_t dummy_abort = 0u;
      mbar_wait(s.mma_done, 0u, &dummy_abort, p.err_word, p.timeout_ns);
    }
  } else if (warp == kMetaWarp) {
    // ------------------------------------------------------ column metadata
    // (scale, norm, global id) of each chunk's columns into a ring of
    // kMetaSlots slots; the epilogue warps release a slot when done with it.
    uint32_t seq = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      uint2 t;
      uint64_t start;
      uint32_t cnt, ncol;
      tile_span<RECT>(p, tile, t, start, cnt, ncol);
      uint32_t nchunks = (ncol + kBN - 1) / kBN;
      for (uint32_t c = 0; c < nchunks; ++c, ++seq) {
        uint32_t slot = seq % kMetaSlots, use = seq / kMetaSlots;
        bool w = true;
        if (lane == 0) w = mbar_wait(&s.m_empty[slot], (use & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns);
        if (__shfl_sync(0xffffffffu, w ? 1u : 0u, 0) == 0u) {
          ok = false;
          break;
        }
        float2 sn[kBN / 32];
        uint32_t gv[kBN / 32];
        if constexpr (RECT) {
#pragma unroll
          for (uint32_t u = 0; u < kBN / 32; ++u) {
            uint32_t col = c * kBN + u * 32 + lane;
            sn[u] = make_float2(0.f, INFINITY);  // past the last column: distance +inf
            gv[u] = 0xffffffffu;
            if (col < ncol) {
              sn[u] = make_float2(__ldg(p.col_scales + col), __ldg(p.col_norms + col));
              gv[u] = __ldg(p.col_keys + col);
            }
          }
        } else {
          // All member ids first, then all dependent loads, then the stores.
          uint32_t lid[kBN / 32];
#pragma unroll
          for (uint32_t u = 0; u < kBN / 32; ++u) {
            uint32_t col = c * kBN + u * 32 + lane;
            lid[u] = col < cnt ? __ldg(p.members + start + col) : 0xffffffffu;
          }
#pragma unroll
          for (uint32_t u = 0; u < kBN / 32; ++u) {
            sn[u] = make_float2(0.f, INFINITY);  // past the leaf: distance +inf
            gv[u] = 0xffffffffu;
            if (lid[u] < p.resident_rows) {
              sn[u] = make_float2(__ldg(p.scales + lid[u]), __ldg(p.norms + lid[u]));
              gv[u] = __ldg(p.global_ids + lid[u]);
            } else if (lid[u] != 0xffffffffu) {
              atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
            }
          }
        }
#pragma unroll
        for (uint32_t u = 0; u < kBN / 32; ++u) {
          s.meta_sn[slot * kBN + u * 32 + lane] = sn[u];
          s.meta_g[slot * kBN + u * 32 + lane] = gv[u];
        }
        mbar_arrive(&s.m_full[slot]);
      }
    }
  } else {
    // ------------------------------------------------------ epilogue
    const uint32_t ew = warp - 2;          // epilogue warp 0..3
    const uint32_t quad = warp & 3u;       // TMEM lane quadrant this warp may access
    const uint32_t row_in_tile = quad * 32 + lane;
    float* stash = s.stash + (ew * 32u + lane) * kStashStride;
    const uint32_t cap = p.log_cap;
    uint32_t acc = 0, seq = 0;
    bool stop = false;
    for (uint32_t tile = blockIdx.x; tile < p.num_tiles && !stop; tile += gridDim.x) {
      uint2 t;
      uint64_t start;
      uint32_t cnt, ncol;
      tile_span<RECT>(p, tile, t, start, cnt, ncol);
      uint32_t row = t.y + row_in_tile;
      bool valid = row < cnt;
      uint32_t gid_i = 0xfffffffeu;
      float s_i = 0.f, n_i = 0.f;
      if (valid) {
        uint32_t lid_i = RECT ? row : __ldg(p.members + start + row);
        if (lid_i >= p.resident_rows) {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
          valid = false;
        } else {
          s_i = __ldg(p.scales + lid_i);
          n_i = __ldg(p.norms + lid_i);
          if constexpr (!RECT) gid_i = __ldg(p.global_ids + lid_i);
        }
      }
      float sk[KS];
#pragma unroll
      for (int q = 0; q < KS; ++q) sk[q] = (uint32_t)q < p.k ? INFINITY : -INFINITY;
      float thr = valid ? INFINITY : -INFINITY;  // theta + margin
      uint32_t nlog = 0;
      bool ovf = false;
      const uint32_t nchunks = (ncol + kBN - 1) / kBN;
      const uint32_t c_self = RECT ? 0xffffffffu : t.y / kBN;  // rectangular mode: no self column  // the row's own column: chunk c_self, group quad, lane `lane`
      for (uint32_t c = 0; c < nchunks; ++c, ++acc, ++seq) {
        const uint32_t mslot = seq % kMetaSlots;
        const float4* msn = reinterpret_cast<const float4*>(s.meta_sn + mslot * kBN);
        const uint32_t* mg = s.meta_g + mslot * kBN;
        uint32_t buf = acc % kAccBufs, use = acc / kAccBufs;
        bool ok = true;
        if (lane == 0) {
          ok = mbar_wait(&s.m_full[mslot], (seq / kMetaSlots) & 1u, abort_flag, p.err_word, p.timeout_ns) &&
               mbar_wait(&s.t_full[buf], use & 1u, abort_flag, p.err_word, p.timeout_ns);
        }
        if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0u) {
          stop = true;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (uint32_t g = 0; g < kGroups; ++g) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + ((quad * 32u) << 16) + buf * kBN + g * kGroup, v);
          tmem_ld_wait();
          // Exact reference distances; bit (31 - cc) of mask = column cc is
          // below the bound (the sign of d - thr, shifted in).
          float dc[32];
          // Four independent 8-column chains keep the mask off the critical path.
          uint32_t mq[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (uint32_t cc = 0; cc < kGroup; cc += 2) {
            float4 m = msn[(g * kGroup + cc) >> 1];
            float t0 = __fmul_rn(s_i, m.x);
            float t1 = __fmul_rn(s_i, m.z);
            float u0 = __fmul_rn(t0, __int2float_rn((int)v[cc]));
            float u1 = __fmul_rn(t1, __int2float_rn((int)v[cc + 1]));
            float nn0 = __fadd_rn(n_i, m.y);
            float nn1 = __fadd_rn(n_i, m.w);
            // rn(nn + rn(-2*u)) == fma(-2, u, nn): -2*u is exact.
            float d0 = __fmaf_rn(-2.0f, u0, nn0);
            float d1 = __fmaf_rn(-2.0f, u1, nn1);
            dc[cc] = d0;
            dc[cc + 1] = d1;
            uint32_t& w = mq[cc >> 3];
            w = __funnelshift_l(__float_as_uint(__fsub_rn(d0, thr)), w, 1);
            w = __funnelshift_l(__float_as_uint(__fsub_rn(d1, thr)), w, 1);
          }
          // Bit (31 - cc) of mask: column cc is below the bound (the sign of
          // d - thr, shifted in).
          uint32_t mask = (mq[0] << 24) | (mq[1] << 16) | (mq[2] << 8) | mq[3];
          float4* st = reinterpret_cast<float4*>(stash);
#pragma unroll
          for (uint32_t q = 0; q < kGroup / 4; ++q)
            st[q] = make_float4(dc[4 * q], dc[4 * q + 1], dc[4 * q + 2], dc[4 * q + 3]);
          if (c == c_self && g == quad) mask &= ~(0x80000000u >> lane);  // the row itself
          const uint32_t* gg = mg + g * kGroup;
          // Two candidates per step, the same number of steps in every lane
          // (no divergence).  Both are logged if within the bound; the pair
          // insertion is a no-op for values above the k-th smallest.  The
          // next pair's shared-memory loads are issued before the current
          // pair is inserted, so their latency hides behind the insertion.
          const uint32_t steps = (__reduce_max_sync(0xffffffffu, __popc(mask)) + 1u) >> 1;
          bool h0, h1;
          uint32_t c0, c1;
          next_pair(mask, h0, c0, h1, c1);
          float a0 = stash[c0], a1 = stash[c1];
          uint32_t g0 = gg[c0], g1 = gg[c1];
          for (uint32_t it = 0; it < steps;) {
            // Log room for a batch of steps (<= 2 appends each), so the
            // steps themselves carry no capacity check.  Compacts rarely; a
            // row that still cannot fit goes to the exact fallback.
            uint32_t room = (cap - nlog) >> 1;
            if (__any_sync(0xffffffffu, room < steps - it)) {
              nlog = log_compact(s.log, row_in_tile, nlog, thr);
              room = (cap - nlog) >> 1;
            }
            uint32_t batch = min(steps - it, __reduce_min_sync(0xffffffffu, room));
            batch = batch > 0u ? batch : 1u;
            const uint32_t end = it + batch;
#pragma unroll 1
            for (; it < end; ++it) {
              bool nh0, nh1;
              uint32_t nc0, nc1;
              next_pair(mask, nh0, nc0, nh1, nc1);
              const float na0 = stash[nc0], na1 = stash[nc1];
              const uint32_t ng0 = gg[nc0], ng1 = gg[nc1];
              const float d0 = h0 ? (a0 > 0.0f ? a0 : 0.0f) : INFINITY;  // reference clamp d <= 0 -> +0 (CB:8999-9001)
              const float d1 = h1 ? (a1 > 0.0f ? a1 : 0.0f) : INFINITY;
              const bool ok0 = h0 && d0 <= thr, ok1 = h1 && d1 <= thr;
              const bool w0 = ok0 && nlog < cap;
              const uint32_t e1 = nlog + (w0 ? 1u : 0u);
              const bool w1 = ok1 && e1 < cap;
              if (w0) s.log[nlog * kBM + row_in_tile] = make_uint2(__float_as_uint(d0), g0);
              if (w1) s.log[e1 * kBM + row_in_tile] = make_uint2(__float_as_uint(d1), g1);
              nlog = e1 + (w1 ? 1u : 0u);
              ovf |= (ok0 && !w0) || (ok1 && !w1);
              topk_insert2<KS>(sk, fminf(d0, d1), fmaxf(d0, d1));
              thr = __fadd_rn(sk[0], kMargin);
              h0 = nh0;
              h1 = nh1;
              a0 = na0;
              a1 = na1;
              g0 = ng0;
              g1 = ng1;
            }
          }
          __syncwarp();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.t_empty[buf]);
          mbar_arrive(&s.m_empty[mslot]);
        }
      }
      if (!stop && valid) {
        const uint32_t E = log_compact(s.log, row_in_tile, nlog, thr);
        const uint64_t out = (start + row) * (uint64_t)p.k;
        bool okr = !ovf && finish_row<KS>(p, s.log, reinterpret_cast<uint8_t*>(stash), row_in_tile, E, sk, thr,
                                          gid_i, out);
        if (!okr) {
          uint32_t slot = atomicAdd(p.fb_count, 1u);
          if (slot < p.fb_capacity)
            p.fb_list[slot] = make_uint2(t.x, row);
          else
            atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
        }
      }
      __syncwarp();
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Exact fallback: recompute each listed row with the reference's sequential
// insertion (ascending member position, CB:7229-7259).  One CTA per row: all
// threads compute a block of the row's distances into shared memory, then
// warp 0 walks the block in column order.  Lane s holds list slot s; a ballot
// pre-filter (distance <= worst + 33 eps, the largest upward creep of the
// last slot over 32 insertions) skips candidates the reference rejects, and
// each survivor's rank comes from one ballot of the exact rule.
constexpr uint32_t kFbThreads = 256;
constexpr uint32_t kFbBlock = 2048;  // columns per shared-memory block

template <bool RECT>
__global__ void __launch_bounds__(kFbThreads) leaf_fallback_kernel(const int8_t* __restrict__ leaf_codes,
                                                                    uint32_t padded_dim, const Params p) {
  extern __shared__ int4 fb_smem[];
  const uint32_t words = padded_dim / 16u;  // int4 words per code row
  int4* rowbuf = fb_smem;
  float* bd_s = reinterpret_cast<float*>(rowbuf + words);
  uint32_t* bg_s = reinterpret_cast<uint32_t*>(bd_s + kFbBlock);
  uint32_t* bl_s = bg_s + kFbBlock;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t total = *p.fb_count;
  const uint32_t n = total < p.fb_capacity ? total : p.fb_capacity;
  const uint32_t k = p.k;
  for (uint32_t item = blockIdx.x; item < n; item += gridDim.x) {
    uint2 e = p.fb_list[item];
    const uint64_t start = RECT ? 0 : p.leaf_starts[e.x];
    const uint32_t cnt = RECT ? p.ncols : p.leaf_sizes[e.x];
    const uint32_t row = e.y;
    const uint32_t lid_row = RECT ? row : p.members[start + row];
    const uint32_t lid_i = RECT ? 0xffffffffu : lid_row;  // the column to skip (none in rectangular mode)
    float s_i = p.scales[lid_row], n_i = p.norms[lid_row];
    const int4* rc = reinterpret_cast<const int4*>(leaf_codes + (start + row) * padded_dim);
    for (uint32_t w = threadIdx.x; w < words; w += kFbThreads) rowbuf[w] = rc[w];
    float bd = 3.402823466e+38F;  // warp 0: slot `lane` of the list
    uint32_t bi = 0xffffffffu;
    for (uint32_t b0 = 0; b0 < cnt; b0 += kFbBlock) {
      uint32_t bn = cnt - b0 < kFbBlock ? cnt - b0 : kFbBlock;
      __syncthreads();
      // Eight lanes per column (four columns per warp): each 16-byte load
      // instruction reads 128 contiguous bytes of every column row it touches.
      const uint32_t grp = lane >> 3, sub = lane & 7u;
      for (uint32_t cb = warp * 4u; cb < bn; cb += (kFbThreads / 32u) * 4u) {
        const uint32_t c = cb + grp;
        uint32_t lj = 0xffffffffu;
        bool live = false;
        int dot = 0;
        if (c < bn) {
          lj = RECT ? b0 + c : p.members[start + b0 + c];
          live = RECT || lj < p.resident_rows;
          if (live) {
            const int4* cc = reinterpret_cast<const int4*>(RECT ? p.col_codes + (uint64_t)lj * padded_dim
                                                                : leaf_codes + (start + b0 + c) * padded_dim);
            for (uint32_t w = sub; w < words; w += 8u) {
              const int4 x = rowbuf[w], y = cc[w];
              dot = __dp4a(x.x, y.x, dot);
              dot = __dp4a(x.y, y.y, dot);
              dot = __dp4a(x.z, y.z, dot);
              dot = __dp4a(x.w, y.w, dot);
            }
          }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        if (c < bn && sub == 0u) {
          float dj = INFINITY;
          uint32_t gj = 0xffffffffu;
          if (live) {
            if constexpr (RECT) {
              dj = sq8_l2_from_dot(dot, s_i, n_i, p.col_scales[lj], p.col_norms[lj]);
              gj = p.col_keys[lj];
            } else {
              dj = sq8_l2_from_dot(dot, s_i, n_i, p.scales[lj], p.norms[lj]);
              gj = p.global_ids[lj];
            }
          } else {
            lj = lid_i;  // flagged by the main kernel; never a candidate
          }
          bd_s[c] = dj;
          bg_s[c] = gj;
          bl_s[c] = lj;
        }
      }
      __syncthreads();
      if (warp == 0) {
        for (uint32_t c0 = 0; c0 < bn; c0 += 32) {
          uint32_t c = c0 + lane;
          float dj = c < bn ? bd_s[c] : INFINITY;
          uint32_t lj = c < bn ? bl_s[c] : lid_i;
          float worst = __shfl_sync(0xffffffffu, bd, k - 1);
          float thr = __fadd_rn(worst, 33.0f * 2.0e-5f);
          uint32_t cand = __ballot_sync(0xffffffffu, (lj != lid_i) && (dj <= thr));
          while (cand) {
            uint32_t t = __ffs(cand) - 1u;
            cand &= cand - 1u;
            float d = __shfl_sync(0xffffffffu, dj, t);
            uint32_t g = bg_s[c0 + t];
            bool b = (lane < k) && stable_better(d, g, bd, bi);
            uint32_t m = __ballot_sync(0xffffffffu, b);
            if (!((m >> (k - 1)) & 1u)) continue;
            uint32_t live = k == 32 ? 0xffffffffu : ((1u << k) - 1u);
            uint32_t inv = ~m & live;
            uint32_t pos = inv ? (32u - __clz(inv)) : 0u;
            float ud = __shfl_up_sync(0xffffffffu, bd, 1);
            uint32_t ui = __shfl_up_sync(0xffffffffu, bi, 1);
            if (lane < k) {
              if (lane > pos) {
                bd = ud;
                bi = ui;
              } else if (lane == pos) {
                bd = d;
                bi = g;
              }
            }
          }
        }
      }
    }
    if (warp == 0 && lane < k) {
      uint64_t out = (start + row) * (uint64_t)k + lane;
      p.out_ids[out] = bi;
      p.out_dists[out] = bd;
    }
  }
}

// Gather code rows into leaf order: dst row p = src row members[p].
// Leaf-ordered copy of the codes.  An entry outside the resident rows (an
// arena row that belongs to no leaf, or a bad id the leaf kernel reports
// itself) gets a zero row instead of a read.
__global__ void gather_rows_kernel(const int8_t* __restrict__ src, const uint32_t* __restrict__ members,
                                   uint64_t rows, uint32_t row_bytes, uint64_t resident_rows,
                                   int8_t* __restrict__ dst) {
  const uint32_t vec = row_bytes / 16u;
  for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < rows * vec;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t r = idx / vec;
    uint32_t v = (uint32_t)(idx - r * vec);
    const uint32_t m = members[r];
    uint4 x = make_uint4(0u, 0u, 0u, 0u);
    if (m < resident_rows) x = reinterpret_cast<const uint4*>(src + (uint64_t)m * row_bytes)[v];
    reinterpret_cast<uint4*>(dst + r * row_bytes)[v] = x;
  }
}

}  // namespace leaf

// ---------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D uint8 tensor map over `rows` x `row_bytes` (row stride = row_bytes), box
// of 128 bytes x box_rows, 128-byte swizzle, zero fill outside the tensor.
int make_code_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint32_t row_bytes, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {leaf::kSlab, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Shared-memory plan for a launch: B-operand stages and log entries per row.
// Prefers >= 3 stages with a log of k + 24 entries; falls back to 2 stages
// with at least k + 8.  Returns false if neither fits.
static bool leaf_plan(uint32_t padded_dim, uint32_t k, uint32_t* stages, uint32_t* log_cap) {
  uint32_t slabs = (padded_dim + leaf::kSlab - 1) / leaf::kSlab;
  uint32_t fixed = leaf::smem_bytes(slabs, 0, 0);
  auto cap_for = [&](uint32_t st) -> uint32_t {
    uint32_t used = fixed + st * leaf::kBStageBytes;
    if (used >= leaf::kSmemLimit) return 0;
    uint32_t c = (leaf::kSmemLimit - used) / (leaf::kBM * leaf::kLogEntryBytes);
    return c < leaf::kMaxLogCap ? c : leaf::kMaxLogCap;
  };
  uint32_t want = k + 24 < leaf::kMaxLogCap ? k + 24 : leaf::kMaxLogCap;
  for (uint32_t st = 6; st >= 3; --st) {
    uint32_t c = cap_for(st);
    if (c >= want) {
      *stages = st;
      *log_cap = c;
      return true;
    }
  }
  uint32_t c = cap_for(2);
  if (c >= k + 8) {
    *stages = 2;
    *log_cap = c;
    return true;
  }
  return false;
}

int leaf_num_bstages(uint32_t padded_dim) {
  uint32_t st = 0, cap = 0;
  return leaf_plan(padded_dim, 32, &st, &cap) ? (int)st : 0;
}

template <int KS, bool RECT>
static int launch_main(const CUtensorMap& ta, const CUtensorMap& tb, const leaf::Params& prm, uint32_t smem,
                       uint32_t grid, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(leaf::leaf_topk_sq8_kernel<KS, RECT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return TESSA_ERR_CUDA;
  leaf::leaf_topk_sq8_kernel<KS, RECT><<<grid, leaf::kThreads, smem, stream>>>(ta, tb, prm);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

// Exact recomputation of the rows whose result depends on insertion order.
template <bool RECT>
static int launch_fallback(const leaf::Params& prm, const int8_t* a_codes, uint32_t padded_dim, int sm_count,
                           cudaStream_t stream) {
  const uint32_t fb_smem = padded_dim + leaf::kFbBlock * 12u;
  leaf::leaf_fallback_kernel<RECT><<<(unsigned)sm_count * 4u, leaf::kFbThreads, fb_smem, stream>>>(a_codes, padded_dim,
                                                                                                  prm);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

int launch_leaf_split(const CUtensorMap& tm, const CUtensorMap& th, leaf::Params& prm, uint32_t padded_dim,
                      int sm_count, bool pair, cudaStream_t stream);

// Main kernel (k-specialised) plus the exact fallback over the rows it lists.
template <bool RECT>
static int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, leaf::Params& prm, const int8_t* a_codes,
                       uint32_t padded_dim, int sm_count, cudaStream_t stream) {
  uint32_t nst = 0, log_cap = 0;
  if (!leaf_plan(padded_dim, prm.k, &nst, &log_cap)) return TESSA_ERR_UNSUPPORTED;
  const uint32_t slabs = (padded_dim + leaf::kSlab - 1) / leaf::kSlab;
  prm.num_slabs = slabs;
  prm.num_bstages = nst;
  prm.log_cap = log_cap;
  const uint32_t smem = leaf::smem_bytes(slabs, nst, log_cap);
  if (cudaMemsetAsync(prm.fb_count, 0, 4, stream) != cudaSuccess) return TESSA_ERR_CUDA;
  const uint32_t grid = prm.num_tiles < (uint32_t)sm_count ? prm.num_tiles : (uint32_t)sm_count;
  int rc;
  if (prm.k <= 2)
    rc = launch_main<2, RECT>(ta, tb, prm, smem, grid, stream);
  else if (prm.k <= 4)
    rc = launch_main<4, RECT>(ta, tb, prm, smem, grid, stream);
  else if (prm.k <= 8)
    rc = launch_main<8, RECT>(ta, tb, prm, smem, grid, stream);
  else if (prm.k <= 16)
    rc = launch_main<16, RECT>(ta, tb, prm, smem, grid, stream);
  else
    rc = launch_main<32, RECT>(ta, tb, prm, smem, grid, stream);
  if (rc != TESSA_OK) return rc;
  return launch_fallback<RECT>(prm, a_codes, padded_dim, sm_count, stream);
}

// Returns 0, or a TESSA_ERR_* code.
int launch_leaf_topk_sq8(const LeafLaunch& L, cudaStream_t stream) {
  if (L.num_tiles == 0) return TESSA_OK;
  if (L.k == 0 || L.k > 32) return TESSA_ERR_INVALID_ARG;
  CUtensorMap ta, tb;
  if (make_code_tmap(&ta, L.leaf_codes, L.leaf_rows, L.padded_dim, leaf::kBM) != 0) return TESSA_ERR_CUDA;
  if (make_code_tmap(&tb, L.leaf_codes, L.leaf_rows, L.padded_dim, leaf::kBN) != 0) return TESSA_ERR_CUDA;
  leaf::Params prm = {};
  prm.scales = L.scales;
  prm.norms = L.norms;
  prm.global_ids = L.global_ids;
  prm.members = L.members;
  prm.leaf_starts = L.d_leaf_starts;
  prm.leaf_sizes = L.d_leaf_sizes;
  prm.tiles = L.d_tiles;
  prm.num_tiles = L.num_tiles;
  prm.k = L.k;
  prm.resident_rows = L.resident_rows;
  prm.out_ids = L.out_ids;
  prm.out_dists = L.out_dists;
  prm.err_word = L.d_err;
  prm.fb_count = L.d_fb_count;
  prm.fb_list = L.d_fb_list;
  prm.fb_capacity = L.fb_capacity;
  prm.timeout_ns = L.timeout_ns;
  uint32_t ring = 0, log_cap = 0;
  if (L.d_dump && L.dump_rows && leaf_split_plan(L.padded_dim, L.k, &ring, &log_cap)) {
    // Column-split kernel + finishing kernel + exact fallback.
    prm.dump_row0 = L.dump_row0;
    prm.dump_rows = L.dump_rows;
    prm.dump_d = leaf_dump_entries(L.k);
    prm.dump = reinterpret_cast<uint2*>(L.d_dump);
    prm.dump_m = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(L.d_dump) + leaf_dump_m_offset(L.dump_rows, L.k));
    prm.dump_cnt = reinterpret_cast<uint8_t*>(prm.dump_m + 8u * L.dump_rows);
    if (cudaMemsetAsync(prm.fb_count, 0, 4, stream) != cudaSuccess) return TESSA_ERR_CUDA;
    const bool pair = L.d_pairs && L.num_pairs;
    CUtensorMap th = tb;  // B halves of a chunk for CTA pairs
    if (pair && make_code_tmap(&th, L.leaf_codes, L.leaf_rows, L.padded_dim, leaf::kBN / 2) != 0)
      return TESSA_ERR_CUDA;
    prm.pairs = L.d_pairs;
    prm.num_pairs = L.num_pairs;
    int rc = launch_leaf_split(ta, th, prm, L.padded_dim, L.sm_count, pair, stream);
    if (rc != TESSA_OK) return rc;
    return launch_fallback<false>(prm, L.leaf_codes, L.padded_dim, L.sm_count, stream);
  }
  return launch_pair<false>(ta, tb, prm, L.leaf_codes, L.padded_dim, L.sm_count, stream);
}

int launch_rect_topk_sq8(const RectLaunch& R, cudaStream_t stream) {
  if (R.rows == 0 || R.cols == 0) return TESSA_OK;
  if (R.k == 0 || R.k > 32 || R.rows > kMaxRectRows) return TESSA_ERR_INVALID_ARG;
  CUtensorMap ta, tb;
  if (make_code_tmap(&ta, R.row_codes, R.rows, R.padded_dim, leaf::kBM) != 0) return TESSA_ERR_CUDA;
  if (make_code_tmap(&tb, R.col_codes, R.cols, R.padded_dim, leaf::kBN) != 0) return TESSA_ERR_CUDA;
  leaf::Params prm = {};
  prm.scales = R.row_scales;
  prm.norms = R.row_norms;
  prm.num_tiles = (uint32_t)((R.rows + leaf::kBM - 1) / leaf::kBM);
  prm.k = R.k;
  prm.resident_rows = R.rows;
  prm.out_ids = R.out_keys;
  prm.out_dists = R.out_dists;
  prm.err_word = R.d_err;
  prm.fb_count = R.d_fb_count;
  prm.fb_list = R.d_fb_list;
  prm.fb_capacity = R.fb_capacity;
  prm.timeout_ns = R.timeout_ns;
  prm.nrows = (uint32_t)R.rows;
  prm.ncols = R.cols;
  prm.col_codes = R.col_codes;
  prm.col_scales = R.col_scales;
  prm.col_norms = R.col_norms;
  prm.col_keys = R.col_keys;
  return launch_pair<true>(ta, tb, prm, R.row_codes, R.padded_dim, R.sm_count, stream);
}

// Rectangular-mode epilogue of the global-D0 assignment: key -> leader index
// and the row's global id beside every slot.
__global__ void d0_fragments_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ key_to_leader,
                                    const uint32_t* __restrict__ global_ids, uint64_t rows, uint32_t fanout,
                                    uint32_t leaders, uint32_t* __restrict__ child_ids,
                                    uint32_t* __restrict__ point_ids, uint32_t* __restrict__ err) {
  const uint64_t n = rows * fanout;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t key = keys[i];
    uint32_t child = 0xffffffffu;
    if (key < leaders)
      child = key_to_leader[key];
    else
      atomicOr(err, TESSA_DEVERR_NONFINITE);  // fanout <= leaders: only a non-finite distance leaves a slot empty
    child_ids[i] = child;
    point_ids[i] = global_ids[i / fanout];
  }
}

int launch_d0_fragments(const uint32_t* keys, const uint32_t* key_to_leader, const uint32_t* global_ids, uint64_t rows,
                        uint32_t fanout, uint32_t leaders, uint32_t* child_ids, uint32_t* point_ids, uint32_t* d_err,
                        int sm_count, cudaStream_t stream) {
  const uint64_t n = rows * fanout;
  if (n == 0) return TESSA_OK;
  uint64_t blocks = (n + 255) / 256;
  const uint64_t cap = (uint64_t)sm_count * 8u;
  if (blocks > cap) blocks = cap;
  d0_fragments_kernel<<<(unsigned)blocks, 256, 0, stream>>>(keys, key_to_leader, global_ids, rows, fanout, leaders,
                                                           child_ids, point_ids, d_err);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

int launch_gather_rows(const int8_t* src, const uint32_t* members, uint64_t rows, uint32_t row_bytes,
                       uint64_t resident_rows, int8_t* dst, int sm_count, cudaStream_t stream) {
  if (rows == 0) return TESSA_OK;
  uint64_t work = rows * (row_bytes / 16u);
  uint64_t blocks = (work + 255) / 256;
  uint64_t cap = (uint64_t)sm_count * 8u;
  if (blocks > cap) blocks = cap;
  leaf::gather_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(src, members, rows, row_bytes, resident_rows, dst);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
