// SQ8 leaf all-pairs evaluation with fused per-row bounded top-k, column-split
// epilogue (sm_100a, padded_dim <= 1024).
//
// Same result as leaf_topk_sq8_kernel (leaf_sq8.cu): candidates of row r are
// the other members of its leaf, distance = gpu_persistent_sq_int8_l2_from_dot
// (CB = shear-core/src/algorithm/pipnn/compute_backend.rs, CB:8987-9002), the
// k best under the eps/id rule of gpu_persistent_insert_topk_candidate_fp32
// (CB:7229-7259) in ascending member order (CB:9569-9650), derived without
// sequential insertion by the zone argument in leaf_sq8.cu: per row, every
// candidate within kMargin of the k-th smallest distance is collected, sorted
// and checked for order independence; rows that fail go to the exact fallback.
//
// Why a second kernel: in the four-warp form one epilogue warp per SM
// sub-partition computes distances, maintains the per-row bound and finishes
// the rows, and it is latency-bound (one warp cannot hide its own dependency
// chains).  Here two warps share every TMEM lane quadrant and split each
// 128-column chunk: warp half h takes the 32-column groups h and h + 2 with
// its own sorted bound and candidate log.  Shared memory for the second set of logs
// comes from keeping the A tile (the 128 rows of the tile) in tensor memory
// instead of shared memory: the MMA reads A from TMEM (tcgen05.mma with an
// A tensor-memory operand), B streams through shared memory as before.
//
// Per-row bound of a half: max(own j-th smallest, other j-th smallest) with
// j = ceil(k/2): at least j + j >= k candidates of the row lie at or below
// it, so it bounds the row's k-th smallest from above, and each half keeps
// only its j smallest distances sorted (half the insertion work of keeping k).
// The halves publish their j-th smallest after every column group (tagged
// with the tile, so a value of a previous tile is never used; the other's
// value may be older than the current group, which only loosens the bound,
// and for the first kMeetGroups groups the two warps meet so it is not).  A
// candidate is logged while it is within kMargin of the bound.  At the end of
// a tile each half takes the k smallest distances of its log (every distance
// at or below the row's k-th smallest was within the bound when it arrived),
// the halves exchange them and both merge them into the row's k smallest
// distances (theta = the k-th); each half compacts its log to
// [0, theta + kMargin] (its part of the zone) and writes it to a per-row dump
// in global memory, half 0 adds the merged k smallest.
// leaf_finish_kernel then ranks each row's zone against those k values (as
// leaf_sq8.cu's finish does), verifies it and writes the k results (or lists
// the row for the exact fallback), with enough warps per SM to hide latency.
// The next tile's A is in TMEM before a tile's rows are wrapped up, so the
// MMA runs ahead meanwhile: one CTA per tile copies it with tcgen05.cp from
// the MMA thread as soon as the tile's last MMAs have completed; a CTA pair
// has its epilogue warps write it (tcgen05.st).
//
// Roles (352 threads, one persistent CTA per SM):
//   warp 0      TMA producer: a ring of 16 KiB stages carrying, per tile, the
//               A slabs (128 rows x 128 bytes of K) and then the B slabs of
//               every 128-column chunk;
//   warp 1      TMEM owner (512 columns: A tile at [0, padded_dim/4), two
//               128-column accumulators at [256, 512)), MMA issuer and, one
//               CTA per tile, A copier (tcgen05.cp of each A slab from the
//               ring into TMEM, four 128 x 32-byte copies per slab);
//   warps 2..9  epilogue; warp w reads TMEM lane quadrant w % 4, half
//               (w - 2) / 4; in a CTA pair all eight copy the A slabs at the
//               start of a tile from the ring into TMEM (each a quadrant x 64
//               bytes of K);
//   warp 10     column metadata ring (scale, norm, global id per column).
#include "common.cuh"
#include "kernels.h"
#include "leaf_common.cuh"

namespace tessa {
namespace leaf {
namespace split {

constexpr uint32_t kThreads = 352;
constexpr uint32_t kEpiWarps = 8;
constexpr uint32_t kMetaWarp = 10;
constexpr uint32_t kAccBufs = 2;
constexpr uint32_t kAccCol = 256;  // first accumulator column
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kMaxSlabs = 8;  // padded_dim <= 1024: A tile <= 256 TMEM columns
constexpr uint32_t kMaxRing = 8;
constexpr uint32_t kStageBytes = kBM * kSlab;  // 16 KiB (A and B slabs alike)
constexpr uint32_t kMetaBytes = kMetaSlots * kBN * 12u;
constexpr uint32_t kStashBytes = kEpiWarps * 32u * kStashStride * 4u;
constexpr uint32_t kPubBytes = 2u * kBM * 8u;
constexpr uint32_t kBarBytes = 512u;
constexpr uint32_t kFinThreads = 128;
constexpr uint32_t kMeetGroups = 8;  // groups per tile after which the two halves meet (k > 2)

static_assert(kBM == kBN, "A and B slabs share the ring and the tensor map");

struct Smem {
  uint8_t* ring;
  float* meta_sn;   // [slot][column pair][s_even, s_odd, n_even, n_odd]
  uint32_t* meta_g;
  float* stash;     // [8 warps][32 lanes][kStashStride]
  uint64_t* pub;    // [2 halves][kBM] (tile tag << 32 | bound bits)
  uint2* log;       // [2 halves][log_cap][kBM]
  uint64_t* b_full;
  uint64_t* b_empty;
  uint64_t* t_full;
  uint64_t* t_empty;
  uint64_t* m_full;
  uint64_t* m_empty;
  uint64_t* a_tm_full;  // A tile of the current tile written to TMEM
  uint64_t* a_rd;       // [kMaxRing] all epilogue warps have read the A slab in this stage
  uint64_t* pair;       // [4] two warps of a lane quadrant
  uint64_t* mma_done;
  uint64_t* a_free;     // all MMAs of the previous tile have completed (A may be overwritten)
  uint32_t* tmem_slot;
  uint32_t* abort_flag;
};

__host__ __device__ inline uint32_t smem_bytes(uint32_t ring, uint32_t log_cap) {
  return 1024u + ring * kStageBytes + kMetaBytes + kStashBytes + kPubBytes + 2u * log_cap * kBM * kLogEntryBytes +
         kBarBytes;
}

__device__ __forceinline__ Smem carve(uint8_t* raw, uint32_t ring, uint32_t log_cap) {
  uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  Smem s;
  s.ring = p;
  p += ring * kStageBytes;
  s.meta_sn = reinterpret_cast<float*>(p);
  p += kMetaSlots * kBN * 8u;
  s.meta_g = reinterpret_cast<uint32_t*>(p);
  p += kMetaSlots * kBN * 4u;
  s.stash = reinterpret_cast<float*>(p);
  p += kStashBytes;
  s.pub = reinterpret_cast<uint64_t*>(p);
  p += kPubBytes;
  s.log = reinterpret_cast<uint2*>(p);
  p += 2u * log_cap * kBM * kLogEntryBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p);
  s.b_full = bars;
  s.b_empty = s.b_full + kMaxRing;
  s.t_full = s.b_empty + kMaxRing;
  s.t_empty = s.t_full + kAccBufs;
  s.m_full = s.t_empty + kAccBufs;
  s.m_empty = s.m_full + kMetaSlots;
  s.a_tm_full = s.m_empty + kMetaSlots;
  s.a_rd = s.a_tm_full + 1;
  s.pair = s.a_rd + kMaxRing;
  s.mma_done = s.pair + 4;
  s.a_free = s.mma_done + 1;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.a_free + 1);
  s.abort_flag = s.tmem_slot + 1;
  return s;
}

// The work unit of a CTA: a 128-row tile, or in a pair (PAIR) this CTA's
// half of a 256-row tile pair (rows first + 128 * rank of the pair's leaf).
template <bool PAIR>
__device__ __forceinline__ void unit_span(const Params& p, uint32_t unit, uint32_t rank, uint2& t, uint64_t& start,
                                          uint32_t& rows, uint32_t& cols) {
  if constexpr (PAIR) {
    t = p.pairs[unit];
    t.y += rank * kBM;
    start = p.leaf_starts[t.x];
    rows = p.leaf_sizes[t.x];
    cols = rows;
  } else {
    tile_span<false>(p, unit, t, start, rows, cols);
  }
}

// Both warps of a lane quadrant meet; false if the wait timed out or the CTA
// aborted.  `phase` counts the meetings of this pair.
__device__ __forceinline__ bool pair_meet(uint64_t* bar, uint32_t& phase, uint32_t lane,
                                          volatile uint32_t* abort_flag, const Params& p) {
  __syncwarp();
  bool ok = true;
  if (lane == 0) {
    mbar_arrive(bar);
    ok = mbar_wait(bar, phase & 1u, abort_flag, p.err_word, p.timeout_ns);
  }
  ++phase;
  return __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0u;
}

// Epilogue warp: copy this lane's row of the A tile (whose first ring item is
// `rpos`) into TMEM: 16-byte pieces 4*half..4*half+3 of every A slab (128B
// swizzle: piece j of row r sits at j ^ (r & 7)).  Each ring stage is
// released as soon as all eight warps have read it (one read barrier per
// stage: a warp can arrive on a stage's barrier again only after the stage
// was released and refilled).  Then arrive on a_tm_full.  False on a timed
// out or aborted wait.
//
// In a pair the stage is released in both CTAs at once, when both have read
// their A slab: the second CTA's first warp forwards its read barrier to the
// first CTA's (which counts one more arrival), and the first CTA releases
// the stage in both.  A CTA's next B half of that stage completes on the
// first CTA's full barrier, so it may be issued only after that barrier's
// A phase has completed, which this ordering guarantees.
template <bool PAIR>
__device__ __forceinline__ bool load_a_tile(const Smem& s, const Params& p, uint32_t rpos, uint32_t ew,
                                            uint32_t half, uint32_t row_in_tile, uint32_t lane, uint32_t lane_base,
                                            uint32_t tmem_base, uint32_t& arp, uint32_t rank,
                                            volatile uint32_t* abort_flag) {
  const uint32_t nst = p.num_bstages;
  for (uint32_t sl = 0; sl < p.num_slabs; ++sl) {
    const uint32_t it = rpos + sl, st = it % nst, ph = (it / nst) & 1u;
    const bool ok = mbar_wait(&s.b_full[st], ph, abort_flag, p.err_word, p.timeout_ns);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const uint8_t* rowp = s.ring + st * kStageBytes + row_in_tile * kSlab;
    uint32_t r[16];
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u) {
      const uint32_t j = half * 4u + u;
      const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((j ^ (row_in_tile & 7u)) << 4));
      r[4 * u] = v.x;
      r[4 * u + 1] = v.y;
      r[4 * u + 2] = v.z;
      r[4 * u + 3] = v.w;
    }
    // The stage is released to the TMA only after every lane's loads have
    // delivered: the values go to tensor memory and the store completes
    // before the warp signals the read (a refill writes the box from row 0
    // on, so an early release would corrupt the first rows of the slab).
    tmem_st_32x32b_x16(tmem_base + lane_base + sl * (kSlab / 4u) + half * 16u, r);
    tmem_st_wait();
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.a_rd[st]);
    if (ew == 0) {
      bool rd = true;
      if (lane == 0) {
        if constexpr (PAIR) {
          rd = mbar_wait_cluster(&s.a_rd[st], (arp >> st) & 1u, abort_flag, p.err_word, p.timeout_ns);
          if (rd && rank != 0u) {
            mbar_arrive_cluster(mapa_shared(&s.a_rd[st], 0));
          } else if (rd) {
            mbar_arrive(&s.b_empty[st]);
            mbar_arrive_cluster(mapa_shared(&s.b_empty[st], 1));
          }
        } else {
          rd = mbar_wait(&s.a_rd[st], (arp >> st) & 1u, abort_flag, p.err_word, p.timeout_ns);
          if (rd) mbar_arrive(&s.b_empty[st]);
        }
      }
      arp ^= 1u << st;  // completed phases of each stage's read barrier, mod 2
      if (__shfl_sync(0xffffffffu, rd ? 1u : 0u, 0) == 0u) return false;
    }
  }
  tmem_st_wait();
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {
    if constexpr (PAIR)
      mbar_arrive_cluster(mapa_shared(s.a_tm_full, 0));  // the pair's MMAs wait for both halves of A
    else
      mbar_arrive(s.a_tm_full);
  }
  return true;
}

template <int KS, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    leaf_topk_split_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tmap_half,
                           const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem s = carve(smem_raw, p.num_bstages, p.log_cap);
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort_flag = s.abort_flag;
  const uint32_t nst = p.num_bstages;
  // Work units: tiles, or tile pairs shared by the two CTAs of a cluster.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const uint32_t unit0 = PAIR ? (blockIdx.x >> 1) : blockIdx.x;
  const uint32_t ustride = PAIR ? (gridDim.x >> 1) : gridDim.x;
  const uint32_t num_units = PAIR ? p.num_pairs : p.num_tiles;
  constexpr uint32_t kPeers = PAIR ? 2u : 1u;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nst; ++i) {
      mbar_init(&s.b_full[i], 1);
      mbar_init(&s.b_empty[i], 1);
    }
    for (uint32_t i = 0; i < kAccBufs; ++i) {
      mbar_init(&s.t_full[i], 1);
      mbar_init(&s.t_empty[i], kPeers * kEpiWarps);  // a pair: both CTAs' epilogue warps
    }
    for (uint32_t i = 0; i < kMetaSlots; ++i) {
      mbar_init(&s.m_full[i], 32);
      mbar_init(&s.m_empty[i], kEpiWarps);
    }
    mbar_init(s.a_tm_full, kPeers * kEpiWarps);
    // a pair's first CTA also counts the second CTA's forwarded read
    for (uint32_t i = 0; i < nst; ++i) mbar_init(&s.a_rd[i], kEpiWarps + (PAIR && rank == 0u ? 1u : 0u));
    for (uint32_t i = 0; i < 4; ++i) mbar_init(&s.pair[i], 2);
    mbar_init(s.mma_done, 1);
    mbar_init(s.a_free, 1);
    *s.abort_flag = 0u;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp >= 2 && warp < 2 + kEpiWarps) s.pub[((warp - 2) >> 2) * kBM + (warp & 3u) * 32u + lane] = 0ull;
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap);
    if (PAIR) tma_prefetch_desc(&tmap_half);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(s.tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(s.tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers are initialised before any arrival on them
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (uint32_t tile = unit0; tile < num_units && ok; tile += ustride) {
        uint2 t;
        uint64_t start;
        uint32_t cnt, ncol;
        unit_span<PAIR>(p, tile, rank, t, start, cnt, ncol);
        const uint32_t nchunks = (ncol + kBN - 1) / kBN;
        // A slabs of the tile's rows, then B slabs chunk by chunk.
        for (uint32_t item = 0; item < p.num_slabs * (1u + nchunks) && ok; ++item) {
          const uint32_t sl = item % p.num_slabs;
          const uint32_t c = item / p.num_slabs;  // 0 = A, c >= 1: chunk c - 1
          const bool freed = PAIR ? mbar_wait_cluster(&s.b_empty[stage], phase ^ 1u, abort_flag, p.err_word, p.timeout_ns)
                                  : mbar_wait(&s.b_empty[stage], phase ^ 1u, abort_flag, p.err_word, p.timeout_ns);
          if (!freed) {
            ok = false;
            break;
          }
          if (PAIR && c != 0) {
            // B: this CTA's half of the chunk's columns; both halves complete
            // on the first CTA's barrier, which expects the whole stage
            const int32_t y = (int32_t)(start + (uint64_t)(c - 1) * kBN + rank * (kBN / 2u));
            if (rank == 0) {
              mbar_arrive_expect_tx(&s.b_full[stage], kStageBytes);
              tma_load_2d(&tmap_half, s.ring + stage * kStageBytes, &s.b_full[stage], (int32_t)(sl * kSlab), y);
            } else {
              mbar_arrive(&s.b_full[stage]);  // keeps this CTA's phase count in step
              tma_load_2d_pair(&tmap_half, s.ring + stage * kStageBytes, mapa_shared(&s.b_full[stage], 0),
                               (int32_t)(sl * kSlab), y);
            }
          } else {
            mbar_arrive_expect_tx(&s.b_full[stage], kStageBytes);
            const int32_t y = c == 0 ? (int32_t)(start + t.y) : (int32_t)(start + (uint64_t)(c - 1) * kBN);
            tma_load_2d(&tmap, s.ring + stage * kStageBytes, &s.b_full[stage], (int32_t)(sl * kSlab), y);
          }
          if (++stage == nst) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0 && PAIR && rank == 1) {
      // The pair's MMAs are issued by the first CTA; this CTA's tensor memory
      // and shared memory stay in use until they have all completed.
      uint32_t dummy_abort = 0u;
      mbar_wait_cluster(s.mma_done, 0u, &dummy_abort, p.err_word, p.timeout_ns);
    } else if (lane == 0) {
      const uint32_t idesc = idesc_i8(PAIR ? 2u * kBM : kBM, kBN);
      const uint32_t ring_base = smem_u32(s.ring);
      uint32_t stage = 0, phase = 0, acc = 0, a_iter = 0;
      bool ok = true;
      // barriers the pair's MMAs signal in both CTAs (the peer's through its cluster address)
      auto commit_both = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          mma_commit_pair(mapa_shared(bar, 0));
          mma_commit_pair(mapa_shared(bar, 1));
        } else {
          mma_commit(bar);
        }
      };
      auto wait_peers = [&](uint64_t* bar, uint32_t par) {
        return PAIR ? mbar_wait_cluster(bar, par, abort_flag, p.err_word, p.timeout_ns)
                    : mbar_wait(bar, par, abort_flag, p.err_word, p.timeout_ns);
      };
      for (uint32_t tile = unit0; tile < num_units && ok; tile += ustride, ++a_iter) {
        uint2 t;
        uint64_t start;
        uint32_t cnt, ncol;
        unit_span<PAIR>(p, tile, rank, t, start, cnt, ncol);
        const uint32_t nchunks = (ncol + kBN - 1) / kBN;
        if constexpr (PAIR) {
          // The A items of the ring belong to the epilogue warps.
          for (uint32_t sl = 0; sl < p.num_slabs; ++sl)
            if (++stage == nst) {
              stage = 0;
              phase ^= 1u;
            }
          if (!wait_peers(s.a_tm_full, a_iter & 1u)) break;
          tc_fence_after();
        } else {
          // One CTA: this thread copies the tile's A slabs from the ring into
          // tensor memory (tcgen05.cp, ordered before the MMAs that read
          // them), once every MMA of the previous tile, which read the old A,
          // has completed.  Each stage is released when its copies complete.
          if (a_iter > 0u) {
            if (!mbar_wait(s.a_free, (a_iter - 1u) & 1u, abort_flag, p.err_word, p.timeout_ns)) break;
            tc_fence_after();
          }
          for (uint32_t sl = 0; sl < p.num_slabs && ok; ++sl) {
            if (!mbar_wait(&s.b_full[stage], phase, abort_flag, p.err_word, p.timeout_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = ring_base + stage * kStageBytes;
#pragma unroll
            for (uint32_t kk = 0; kk < kSlab / kMmaK; ++kk)
              tmem_cp_128x256b(tmem_base + sl * (kSlab / 4u) + kk * (kMmaK / 4u),
                               smem_desc_sw128(a_addr + kk * kMmaK));
            mma_commit(&s.b_empty[stage]);
            if (++stage == nst) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
        }
        for (uint32_t c = 0; c < nchunks && ok; ++c, ++acc) {
          const uint32_t buf = acc % kAccBufs, use = acc / kAccBufs;
          if (!wait_peers(&s.t_empty[buf], (use & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tmem_d = tmem_base + kAccCol + buf * kBN;
          for (uint32_t sl = 0; sl < p.num_slabs; ++sl) {
            if (!mbar_wait(&s.b_full[stage], phase, abort_flag, p.err_word, p.timeout_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b_addr = ring_base + stage * kStageBytes;
#pragma unroll
            for (uint32_t kk = 0; kk < kSlab / kMmaK; ++kk) {
              if constexpr (PAIR)
                mma_i8_ts_pair(tmem_d, tmem_base + sl * (kSlab / 4u) + kk * (kMmaK / 4u),
                               smem_desc_sw128(b_addr + kk * kMmaK), idesc, (sl | kk) != 0u ? 1u : 0u);
              else
                mma_i8_ts(tmem_d, tmem_base + sl * (kSlab / 4u) + kk * (kMmaK / 4u),
                          smem_desc_sw128(b_addr + kk * kMmaK), idesc, (sl | kk) != 0u ? 1u : 0u);
            }
            commit_both(&s.b_empty[stage]);
            if (++stage == nst) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (ok) commit_both(&s.t_full[buf]);
        }
        if constexpr (!PAIR) {
          if (ok) mma_commit(s.a_free);
        }
      }
      // Every issued MMA must have landed before TMEM is released (in both
      // CTAs of a pair).
      commit_both(s.mma_done);
      uint32_t dummy_abort = 0u;
      mbar_wait(s.mma_done, 0u, &dummy_abort, p.err_word, p.timeout_ns);
    }
  } else if (warp == kMetaWarp) {
    // ------------------------------------------------------ column metadata
    uint32_t seq = 0;
    bool ok = true;
    for (uint32_t tile = unit0; tile < num_units && ok; tile += ustride) {
      uint2 t;
      uint64_t start;
      uint32_t cnt, ncol;
      unit_span<PAIR>(p, tile, rank, t, start, cnt, ncol);
      const uint32_t nchunks = (ncol + kBN - 1) / kBN;
      for (uint32_t c = 0; c < nchunks; ++c, ++seq) {
        const uint32_t slot = seq % kMetaSlots, use = seq / kMetaSlots;
        bool w = true;
        if (lane == 0) w = mbar_wait(&s.m_empty[slot], (use & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns);
        if (__shfl_sync(0xffffffffu, w ? 1u : 0u, 0) == 0u) {
          ok = false;
          break;
        }
        uint32_t lid[kBN / 32];
#pragma unroll
        for (uint32_t u = 0; u < kBN / 32; ++u) {
          const uint32_t col = c * kBN + u * 32 + lane;
          lid[u] = col < cnt ? __ldg(p.members + start + col) : 0xffffffffu;
        }
        float2 sn[kBN / 32];
        uint32_t gv[kBN / 32];
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
#pragma unroll
        for (uint32_t u = 0; u < kBN / 32; ++u) {
          // scales and norms of a column pair side by side: the epilogue
          // reads both as register pairs for the paired f32 arithmetic
          float* mp = s.meta_sn + slot * kBN * 2u + ((u * 32u + lane) >> 1) * 4u + (lane & 1u);
          mp[0] = sn[u].x;
          mp[2] = sn[u].y;
          s.meta_g[slot * kBN + u * 32 + lane] = gv[u];
        }
        mbar_arrive(&s.m_full[slot]);
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------ epilogue
    const uint32_t ew = warp - 2;        // 0..7
    const uint32_t quad = warp & 3u;     // TMEM lane quadrant this warp may access
    const uint32_t half = ew >> 2;       // column groups half, half + 2
    const uint32_t row_in_tile = quad * 32u + lane;
    const uint32_t lane_base = (quad * 32u) << 16;
    float* stash = s.stash + (ew * 32u + lane) * kStashStride;
    const float* ostash = s.stash + ((ew ^ 4u) * 32u + lane) * kStashStride;  // the other half's
    uint2* log = s.log + half * p.log_cap * kBM;
    volatile uint64_t* my_pub = s.pub + half * kBM + row_in_tile;
    volatile uint64_t* other_pub = s.pub + (half ^ 1u) * kBM + row_in_tile;
    const uint32_t cap = p.log_cap;
    const uint32_t k = p.k;
    // Groups per tile after which the halves stop meeting: one for k <= 2
    // (each group's smallest distance is in the bound before its columns are
    // tested, so a stale value of the other half costs little).
    const uint32_t meet_groups = KS == 2 ? 1u : kMeetGroups;
    constexpr int KH = KS / 2;             // slots of the per-half sorted array
    const uint32_t jk = k - (k >> 1);      // ceil(k/2) <= KH
    uint32_t acc = 0, seq = 0, rpos = 0, tseq = 0, pair_phase = 0, arp = 0;
    bool stop = false;
    uint32_t tile = unit0;
    if (tile < num_units) {
      uint2 t;
      uint64_t start;
      uint32_t cnt, ncol;
      unit_span<PAIR>(p, tile, rank, t, start, cnt, ncol);
      if constexpr (PAIR) {
        stop = !load_a_tile<PAIR>(s, p, rpos, ew, half, row_in_tile, lane, lane_base, tmem_base, arp, rank,
                                  abort_flag);
        rpos += p.num_slabs * (1u + (ncol + kBN - 1) / kBN);
      }
    }
    for (; tile < num_units && !stop; tile += ustride, ++tseq) {
      uint2 t;
      uint64_t start;
      uint32_t cnt, ncol;
      unit_span<PAIR>(p, tile, rank, t, start, cnt, ncol);
      const uint32_t nchunks = (ncol + kBN - 1) / kBN;
      const uint32_t row = t.y + row_in_tile;
      bool valid = row < cnt;
      float s_i = 0.f, n_i = 0.f;
      uint32_t gid_i = 0xfffffffeu;
      if (valid) {
        const uint32_t lid_i = __ldg(p.members + start + row);
        if (lid_i >= p.resident_rows) {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
          valid = false;
        } else {
          s_i = __ldg(p.scales + lid_i);
          n_i = __ldg(p.norms + lid_i);
          gid_i = __ldg(p.global_ids + lid_i);
        }
      }
      const uint64_t si2 = f2_pack(s_i, s_i), ni2 = f2_pack(n_i, n_i), m2x2 = f2_pack(-2.0f, -2.0f);
      // sk: the j = ceil(k/2) smallest distances of this half, descending
      // (sk[0] = the j-th smallest); slots [j, KH) hold -inf sentinels.
      float sk[KH];
#pragma unroll
      for (int q = 0; q < KH; ++q) sk[q] = (uint32_t)q < jk ? INFINITY : -INFINITY;
      float ob = INFINITY;  // the other half's j-th smallest, as last published
      float thr = valid ? INFINITY : -INFINITY;
      uint32_t nlog = 0;
      bool ovf = false;
      const uint32_t c_self = t.y / kBN;  // the row's own column: chunk c_self, group quad, lane `lane`
      const uint64_t tag = (uint64_t)(tseq + 1u) << 32;
      for (uint32_t c = 0; c < nchunks; ++c, ++acc, ++seq) {
        const uint32_t mslot = seq % kMetaSlots;
        const float4* msn = reinterpret_cast<const float4*>(s.meta_sn + mslot * kBN * 2u);
        const uint32_t* mg = s.meta_g + mslot * kBN;
        const uint32_t buf = acc % kAccBufs, use = acc / kAccBufs;
        bool ok = true;
        if (lane == 0) {
          ok = mbar_wait(&s.m_full[mslot], (seq / kMetaSlots) & 1u, abort_flag, p.err_word, p.timeout_ns) &&
               (PAIR ? mbar_wait_cluster(&s.t_full[buf], use & 1u, abort_flag, p.err_word, p.timeout_ns)
                     : mbar_wait(&s.t_full[buf], use & 1u, abort_flag, p.err_word, p.timeout_ns));
        }
        if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0u) {
          stop = true;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (uint32_t gg = 0; gg < 2; ++gg) {
          const uint32_t g = gg * 2u + half;  // groups interleaved: both halves see the leaf's first columns
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + lane_base + kAccCol + buf * kBN + g * kGroup, v);
          tmem_ld_wait();
          if (KS == 2 && !(c == c_self && g == quad)) {
            // k <= 2 (one sorted slot per half), every group but the one
            // holding the row itself: the group's smallest distance enters
            // the half's slot before any column is tested, the halves
            // exchange their slots (meeting for a tile's first groups), and
            // every column below the tightened bound is logged.  No
            // per-candidate insertion: the log keeps whatever lies below the
            // bound, and the bound max(own smallest, other smallest) + margin
            // is still at or above the row's k-th smallest + margin.
            const uint32_t* gq = mg + g * kGroup;
            float dc[32];
#pragma unroll
            for (uint32_t cc = 0; cc < kGroup; cc += 2) {
              const float4 m = msn[(g * kGroup + cc) >> 1];  // s_c, s_c+1, n_c, n_c+1
              const uint64_t t = f2_mul(si2, f2_pack(m.x, m.y));
              const uint64_t u = f2_mul(t, f2_pack(__int2float_rn((int)v[cc]), __int2float_rn((int)v[cc + 1])));
              f2_unpack(f2_fma(m2x2, u, f2_add(ni2, f2_pack(m.z, m.w))), dc[cc], dc[cc + 1]);
            }
            float q[11];
#pragma unroll
            for (uint32_t i = 0; i < 10; ++i) q[i] = fmin3(dc[3 * i], dc[3 * i + 1], dc[3 * i + 2]);
            q[10] = fminf(dc[30], dc[31]);
            const float gm = fmin3(fmin3(q[0], q[1], q[2]), fmin3(q[3], q[4], q[5]),
                                   fmin3(q[6], q[7], fmin3(q[8], q[9], q[10])));
            if (valid) sk[0] = fminf(sk[0], gm > 0.0f ? gm : 0.0f);  // reference clamp d <= 0 -> +0 (CB:8999-9001)
            *my_pub = tag | __float_as_uint(sk[0]);
            if (c * 2u + gg < meet_groups) {
              __threadfence_block();
              if (!pair_meet(&s.pair[quad], pair_phase, lane, abort_flag, p)) {
                stop = true;
                break;
              }
            }
            const uint64_t o = *other_pub;
            if ((o & 0xffffffff00000000ull) == tag) ob = fminf(ob, __uint_as_float((uint32_t)o));
            if (valid) thr = __fadd_rn(fmaxf(sk[0], ob), kMargin);
            uint32_t mq[4] = {0u, 0u, 0u, 0u};
            const uint64_t nthr2 = f2_pack(-thr, -thr);
#pragma unroll
            for (uint32_t cc = 0; cc < kGroup; cc += 2) {
              float e0, e1;
              f2_unpack(f2_add(f2_pack(dc[cc], dc[cc + 1]), nthr2), e0, e1);  // rn(d - thr)
              uint32_t& w = mq[cc >> 3];
              w = __funnelshift_l(__float_as_uint(e0), w, 1);
              w = __funnelshift_l(__float_as_uint(e1), w, 1);
            }
            uint32_t mask = (mq[0] << 24) | (mq[1] << 16) | (mq[2] << 8) | mq[3];
            const uint32_t steps = (__reduce_max_sync(0xffffffffu, __popc(mask)) + 1u) >> 1;
            if (steps != 0u) {  // the pops read the distances back by column index
              float4* st4 = reinterpret_cast<float4*>(stash);
#pragma unroll
              for (uint32_t q4 = 0; q4 < kGroup / 4; ++q4)
                st4[q4] = make_float4(dc[4 * q4], dc[4 * q4 + 1], dc[4 * q4 + 2], dc[4 * q4 + 3]);
            }
            for (uint32_t it = 0; it < steps;) {
              uint32_t room = (cap - nlog) >> 1;
              if (__any_sync(0xffffffffu, room < steps - it)) {
                nlog = log_compact(log, row_in_tile, nlog, thr);
                room = (cap - nlog) >> 1;
              }
              uint32_t batch = min(steps - it, __reduce_min_sync(0xffffffffu, room));
              batch = batch > 0u ? batch : 1u;
              const uint32_t end = it + batch;
#pragma unroll 1
              for (; it < end; ++it) {
                bool h0, h1;
                uint32_t c0, c1;
                next_pair(mask, h0, c0, h1, c1);
                const float a0 = stash[c0], a1 = stash[c1];
                const uint32_t g0 = gq[c0], g1 = gq[c1];
                const bool w0 = h0 && nlog < cap;
                const uint32_t e1 = nlog + (w0 ? 1u : 0u);
                const bool w1 = h1 && e1 < cap;
                if (w0) log[nlog * kBM + row_in_tile] = make_uint2(__float_as_uint(a0 > 0.0f ? a0 : 0.0f), g0);
                if (w1) log[e1 * kBM + row_in_tile] = make_uint2(__float_as_uint(a1 > 0.0f ? a1 : 0.0f), g1);
                nlog = e1 + (w1 ? 1u : 0u);
                ovf |= (h0 && !w0) || (h1 && !w1);
              }
            }
            __syncwarp();
            continue;
          }
          // Exact reference distances; bit (31 - cc) of mask = column cc is
          // below the bound (the sign of d - thr, shifted in), four chains.
          // Two columns per step on register pairs (paired f32 instructions,
          // each element rounded as the scalar form).
          float dc[32];
          uint32_t mq[4] = {0u, 0u, 0u, 0u};
          const uint64_t nthr2 = f2_pack(-thr, -thr);
#pragma unroll
          for (uint32_t cc = 0; cc < kGroup; cc += 2) {
            const float4 m = msn[(g * kGroup + cc) >> 1];  // s_c, s_c+1, n_c, n_c+1
            const uint64_t t = f2_mul(si2, f2_pack(m.x, m.y));
            const uint64_t u = f2_mul(t, f2_pack(__int2float_rn((int)v[cc]), __int2float_rn((int)v[cc + 1])));
            // rn(nn + rn(-2*u)) == fma(-2, u, nn): -2*u is exact.
            const uint64_t d = f2_fma(m2x2, u, f2_add(ni2, f2_pack(m.z, m.w)));
            float d0, d1, e0, e1;
            f2_unpack(d, d0, d1);
            f2_unpack(f2_add(d, nthr2), e0, e1);  // rn(d - thr)
            dc[cc] = d0;
            dc[cc + 1] = d1;
            uint32_t& w = mq[cc >> 3];
            w = __funnelshift_l(__float_as_uint(e0), w, 1);
            w = __funnelshift_l(__float_as_uint(e1), w, 1);
          }
          uint32_t mask = (mq[0] << 24) | (mq[1] << 16) | (mq[2] << 8) | mq[3];
          float4* st4 = reinterpret_cast<float4*>(stash);
#pragma unroll
          for (uint32_t q = 0; q < kGroup / 4; ++q)
            st4[q] = make_float4(dc[4 * q], dc[4 * q + 1], dc[4 * q + 2], dc[4 * q + 3]);
          if (c == c_self && g == quad) mask &= ~(0x80000000u >> lane);  // the row itself
          const uint32_t* gq = mg + g * kGroup;
          if constexpr (KS == 32) {
            // A tile's first group (k = 32): the bound is still +inf, so every
            // marked column is a candidate and is logged; the sorted array is
            // then simply the 32 sorted distances (bitonic network, about a
            // third of the pair insertions it replaces).
            if (c == 0 && gg == 0 && k == 32u) {
              float v[32];
#pragma unroll
              for (uint32_t cc = 0; cc < 32; ++cc) {
                const bool hit = (mask >> (31u - cc)) & 1u;
                const float d = dc[cc] > 0.0f ? dc[cc] : 0.0f;  // reference clamp d <= 0 -> +0 (CB:8999-9001)
                v[cc] = hit ? d : INFINITY;
                if (hit) {
                  log[nlog * kBM + row_in_tile] = make_uint2(__float_as_uint(d), gq[cc]);
                  ++nlog;
                }
              }
#pragma unroll
              for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
                for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
                  for (int i = 0; i < 32; ++i) {
                    const int j = i ^ stride;
                    if (j > i) {
                      const float x = v[i], y = v[j];
                      if ((i & size) == 0) {
                        v[i] = fminf(x, y);
                        v[j] = fmaxf(x, y);
                      } else {
                        v[i] = fmaxf(x, y);
                        v[j] = fminf(x, y);
                      }
                    }
                  }
#pragma unroll
              for (int q = 0; q < KH; ++q) sk[q] = v[KH - 1 - q];  // the j smallest, descending
              if (valid) thr = __fadd_rn(fmaxf(sk[0], ob), kMargin);
              mask = 0u;
            }
          }
          // Two candidates per step, the same number of steps in every lane;
          // the next pair's loads are issued before the current insertion.
          const uint32_t steps = (__reduce_max_sync(0xffffffffu, __popc(mask)) + 1u) >> 1;
          bool h0, h1;
          uint32_t c0, c1;
          next_pair(mask, h0, c0, h1, c1);
          float a0 = stash[c0], a1 = stash[c1];
          uint32_t g0 = gq[c0], g1 = gq[c1];
          for (uint32_t it = 0; it < steps;) {
            uint32_t room = (cap - nlog) >> 1;
            if (__any_sync(0xffffffffu, room < steps - it)) {
              nlog = log_compact(log, row_in_tile, nlog, thr);
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
              const uint32_t ng0 = gq[nc0], ng1 = gq[nc1];
              const float d0 = h0 ? (a0 > 0.0f ? a0 : 0.0f) : INFINITY;  // reference clamp d <= 0 -> +0 (CB:8999-9001)
              const float d1 = h1 ? (a1 > 0.0f ? a1 : 0.0f) : INFINITY;
              const bool ok0 = h0 && d0 <= thr, ok1 = h1 && d1 <= thr;
              const bool w0 = ok0 && nlog < cap;
              const uint32_t e1 = nlog + (w0 ? 1u : 0u);
              const bool w1 = ok1 && e1 < cap;
              if (w0) log[nlog * kBM + row_in_tile] = make_uint2(__float_as_uint(d0), g0);
              if (w1) log[e1 * kBM + row_in_tile] = make_uint2(__float_as_uint(d1), g1);
              nlog = e1 + (w1 ? 1u : 0u);
              ovf |= (ok0 && !w0) || (ok1 && !w1);
              topk_insert2<KH>(sk, fminf(d0, d1), fmaxf(d0, d1));
              if (valid) thr = __fadd_rn(fmaxf(sk[0], ob), kMargin);
              h0 = nh0;
              h1 = nh1;
              a0 = na0;
              a1 = na1;
              g0 = ng0;
              g1 = ng1;
            }
          }
          // Publish this half's j-th smallest and take the other half's.  For
          // the first kMeetGroups groups of a tile the two warps meet after
          // publishing, so each bound uses the other's value of the same
          // group while the bounds still fall fast (one a group older there
          // lets the logs overfill); later the other's latest value is used.
          *my_pub = tag | __float_as_uint(sk[0]);
          if (c * 2u + gg < meet_groups) {
            __threadfence_block();
            if (!pair_meet(&s.pair[quad], pair_phase, lane, abort_flag, p)) {
              stop = true;
              break;
            }
          }
          const uint64_t o = *other_pub;
          if ((o & 0xffffffff00000000ull) == tag) ob = fminf(ob, __uint_as_float((uint32_t)o));
          if (valid) thr = __fadd_rn(fmaxf(sk[0], ob), kMargin);
          __syncwarp();
        }
        if (stop) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(mapa_shared(&s.t_empty[buf], 0));  // the pair's MMA issuer
          else
            mbar_arrive(&s.t_empty[buf]);
          mbar_arrive(&s.m_empty[mslot]);
        }
      }
      if (stop) break;

      // ---- a pair: the next tile's A first, so the MMA starts on it while
      // this tile's rows are wrapped up (all MMAs of this tile have
      // completed).  One CTA per tile: the MMA thread copies it.
      const uint32_t next = tile + ustride;
      if (PAIR && next < num_units) {
        uint2 tn;
        uint64_t sn;
        uint32_t cn, nn;
        unit_span<PAIR>(p, next, rank, tn, sn, cn, nn);
        if (!load_a_tile<PAIR>(s, p, rpos, ew, half, row_in_tile, lane, lane_base, tmem_base, arp, rank, abort_flag)) {
          stop = true;
          break;
        }
        rpos += p.num_slabs * (1u + (nn + kBN - 1) / kBN);
      }

      // ---- tile end: this half's k smallest logged distances (every
      // distance of the row at or below its k-th smallest was within the bound
      // on arrival and is logged, so the two halves' k smallest hold the
      // row's), then both halves merged.
      // The log first drops what lies above the final bound (at or above the
      // row's k-th smallest plus the margin), so fewer entries are inserted.
      nlog = log_compact(log, row_in_tile, nlog, thr);
      float mk[KS];
#pragma unroll
      for (int q = 0; q < KS; ++q) mk[q] = (uint32_t)q < k ? INFINITY : -INFINITY;
      for (uint32_t e = 0; e < nlog; e += 2u) {
        const float x = __uint_as_float(log[e * kBM + row_in_tile].x);
        const float y = e + 1u < nlog ? __uint_as_float(log[(e + 1u) * kBM + row_in_tile].x) : INFINITY;
        topk_insert2<KS>(mk, fminf(x, y), fmaxf(x, y));
      }
#pragma unroll
      for (int q = 0; q < KS; ++q) stash[q] = mk[q];
      if (!pair_meet(&s.pair[quad], pair_phase, lane, abort_flag, p)) {
        stop = true;
        break;
      }
      if (k == (uint32_t)KS) {
        // mk descending, the other's reversed ascending: their element-wise
        // minimum is the KS smallest of both, a bitonic sequence; half-cleaners
        // sort it descending.
#pragma unroll
        for (int q = 0; q < KS; ++q) mk[q] = fminf(mk[q], ostash[KS - 1 - q]);
#pragma unroll
        for (int dd = KS / 2; dd >= 1; dd >>= 1)
#pragma unroll
          for (int q = 0; q < KS; ++q)
            if ((q & dd) == 0) {
              const float a = mk[q], b = mk[q + dd];
              mk[q] = fmaxf(a, b);
              mk[q + dd] = fminf(a, b);
            }
      } else {
        for (uint32_t q = 0; q < k; q += 2) {
          const float x = ostash[q], y = q + 1u < k ? ostash[q + 1u] : INFINITY;
          topk_insert2<KS>(mk, fminf(x, y), fmaxf(x, y));
        }
      }
      // mk: the row's k smallest, descending; mk[0] = theta
      if (!pair_meet(&s.pair[quad], pair_phase, lane, abort_flag, p)) {
        stop = true;
        break;
      }
      if (valid) {
        const uint32_t E = log_compact(log, row_in_tile, nlog, __fadd_rn(mk[0], kMargin));
        const uint64_t rd = start + row - p.dump_row0;
        if (rd < p.dump_rows) {
          // A zone entry with the row's own global id (a repeated member) sends
          // the row to the exact fallback, as does an overflowing log.
          bool fits = !ovf && E <= p.dump_d;
          for (uint32_t e = 0; fits && e < E; ++e) {
            const uint2 v = log[e * kBM + row_in_tile];
            fits = v.y != gid_i;
            p.dump[(uint64_t)(half ? p.dump_d - 1u - e : e) * p.dump_rows + rd] = v;
          }
          p.dump_cnt[2u * rd + half] = fits ? (uint8_t)E : (uint8_t)0xFFu;
          if (half == 0) {
            // the sorted k smallest for the finishing kernel's ranks, -inf
            // padded to a multiple of four: only the first ceil(k / 4) float4
            // planes are written (and read)
#pragma unroll
            for (int q = 0; q < KS; q += 4)
              p.dump_m[(uint64_t)(q / 4) * p.dump_rows + rd] =
                  make_float4(q < KS ? mk[q] : -INFINITY, q + 1 < KS ? mk[q + 1] : -INFINITY,
                              q + 2 < KS ? mk[q + 2] : -INFINITY, q + 3 < KS ? mk[q + 3] : -INFINITY);
          }
        } else {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
        }
      }
      __syncwarp();
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // neither CTA leaves while the peer may still use its memory
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Output slots of one row, written four at a time (16-byte stores) when the
// row's slots are 16-byte aligned.
struct RowWriter {
  uint32_t* ids;
  float* dists;
  bool vec;
  uint32_t bi[4];
  float bd[4];
  __device__ __forceinline__ void put(uint32_t q, uint32_t id, float d) {
    if (!vec) {
      ids[q] = id;
      dists[q] = d;
      return;
    }
    const uint32_t w = q & 3u;
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u)
      if (u == w) {
        bi[u] = id;
        bd[u] = d;
      }
    if (w == 3u) {
      *reinterpret_cast<uint4*>(ids + q - 3u) = make_uint4(bi[0], bi[1], bi[2], bi[3]);
      *reinterpret_cast<float4*>(dists + q - 3u) = make_float4(bd[0], bd[1], bd[2], bd[3]);
    }
  }
  // q = slots written so far; flush a partial group of four
  __device__ __forceinline__ void flush(uint32_t q) {
    if (!vec) return;
#pragma unroll
    for (uint32_t u = 0; u < 3; ++u)
      if (u < (q & 3u)) {
        ids[(q & ~3u) + u] = bi[u];
        dists[(q & ~3u) + u] = bd[u];
      }
  }
};

// Finish the rows of one tile per block (thread = row), as leaf_sq8.cu's
// finish does: the row's zone (both halves' dumps) is ranked against the
// row's k smallest distances (m, descending, -inf padded to 32; theta = m[0]):
// an entry at or below theta ranks by the number of smaller values in m,
// equal distances take consecutive ranks in dump order, entries in the
// margin follow ordered by distance.  The sorted zone is then verified run by
// run and the k results written, or the row is listed for the exact fallback
// (the main kernel marks rows whose zone holds the row's own global id, a
// repeated member, or whose log overflowed).
__global__ void __launch_bounds__(kFinThreads) leaf_finish_kernel(const Params p) {
  extern __shared__ uint32_t fin_smem[];
  const uint32_t D = p.dump_d;
  float* zd = reinterpret_cast<float*>(fin_smem);        // [D][128]
  uint32_t* zg = fin_smem + D * kFinThreads;             // [D][128]
  uint8_t* perm = reinterpret_cast<uint8_t*>(zg + D * kFinThreads);  // [D][128]
  const uint32_t tid = threadIdx.x;
  const uint32_t k = p.k;
  for (uint32_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
    const uint2 t = p.tiles[tile];
    const uint64_t start = p.leaf_starts[t.x];
    const uint32_t cnt = p.leaf_sizes[t.x];
    const uint32_t row = t.y + tid;
    if (row >= cnt) continue;
    const uint64_t rd = start + row - p.dump_row0;
    if (rd >= p.dump_rows) continue;  // reported by the main kernel
    const uint32_t e0 = p.dump_cnt[2u * rd], e1 = p.dump_cnt[2u * rd + 1u];
    bool ok = e0 != 0xFFu && e1 != 0xFFu && e0 + e1 <= D;
    if (ok) {
      const uint32_t E = e0 + e1;
      float m[32];
      const uint32_t planes = (k + 3u) / 4u;  // the main kernel writes only these
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 v = (uint32_t)q < planes ? p.dump_m[(uint64_t)q * p.dump_rows + rd]
                                              : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        m[4 * q] = v.x;
        m[4 * q + 1] = v.y;
        m[4 * q + 2] = v.z;
        m[4 * q + 3] = v.w;
      }
      const float theta = m[0];
      const bool complete = !(theta < INFINITY);
      const float thr = __fadd_rn(theta, kMargin);
      uint32_t n_inner = 0;
      // Entry e < e0 sits at dump slot e, entry e0 + e at slot D - 1 - e
      // (half 1 fills the slots from the back); eight loads in flight at a time.
#pragma unroll 8
      for (uint32_t e = 0; e < E; ++e) {
        const uint32_t slot = e < e0 ? e : D - 1u - (e - e0);
        const uint2 v = p.dump[(uint64_t)slot * p.dump_rows + rd];
        zd[e * kFinThreads + tid] = __uint_as_float(v.x);
        zg[e * kFinThreads + tid] = v.y;
        n_inner += __uint_as_float(v.x) <= theta ? 1u : 0u;
      }
      uint64_t occ = 0;
      for (uint32_t e = 0; ok && e < E; ++e) {
        const float d = zd[e * kFinThreads + tid];
        uint32_t r;
        if (d <= theta) {
          uint32_t r0 = 0, r1 = 0, r2 = 0, r3 = 0;
#pragma unroll
          for (int q = 0; q < 32; q += 4) {
            r0 += m[q] < d ? 1u : 0u;
            r1 += m[q + 1] < d ? 1u : 0u;
            r2 += m[q + 2] < d ? 1u : 0u;
            r3 += m[q + 3] < d ? 1u : 0u;
          }
          r = (r0 + r1) + (r2 + r3) - (32u - k);  // minus the -inf padding
        } else {
          r = n_inner;
          for (uint32_t f = 0; f < E; ++f) {
            const float df = zd[f * kFinThreads + tid];
            r += (df > theta && (df < d || (df == d && f < e))) ? 1u : 0u;
          }
        }
        while (r < 63u && ((occ >> r) & 1ull)) ++r;
        occ |= 1ull << r;
        if (r < D) perm[r * kFinThreads + tid] = (uint8_t)e;
      }
      ok &= occ == (E >= 64u ? ~0ull : ((1ull << E) - 1ull));  // a permutation, else give up safely
      const uint32_t Z = E;
      const uint64_t out = (start + row) * (uint64_t)k;
      RowWriter wr;
      wr.ids = p.out_ids + out;
      wr.dists = p.out_dists + out;
      wr.vec = (k & 3u) == 0u && ((reinterpret_cast<uintptr_t>(wr.ids) | reinterpret_cast<uintptr_t>(wr.dists)) & 15u) == 0u;
      // One pass in sorted order; a run (neighbours closer than eps) is
      // emitted when it closes: runs of one and two directly, longer runs
      // through the tournament check.
      uint32_t q = 0, rs = 0;
      float prev = -INFINITY;
      uint2 first = make_uint2(0u, 0u), second = make_uint2(0u, 0u);
      for (uint32_t i = 0; ok && i <= Z && q < k; ++i) {
        const bool end = i == Z;
        uint2 vi = make_uint2(0x7f800000u, 0u);
        if (!end) {
          const uint32_t e = perm[i * kFinThreads + tid];
          vi = make_uint2(__float_as_uint(zd[e * kFinThreads + tid]), zg[e * kFinThreads + tid]);
        }
        const float di = __uint_as_float(vi.x);
        const bool close = !end && i > 0 && fabsf(__fsub_rn(di, prev)) <= kTieEps;
        if (i > 0 && !close) {
          const uint32_t len = i - rs;  // run [rs, i) is complete
          // The run holding rank k must end inside the zone: every candidate
          // outside the zone lies above thr, hence more than eps above the run.
          if (q + len >= k && end && !complete && !(__fsub_rn(thr, prev) > kTieEps)) {
            ok = false;
            break;
          }
          if (len == 1) {
            wr.put(q, first.y, __uint_as_float(first.x));
            ++q;
          } else if (len == 2) {
            const bool sw = stable_better(__uint_as_float(second.x), second.y, __uint_as_float(first.x), first.y);
            const uint2 lo = sw ? second : first, hi = sw ? first : second;
            wr.put(q, lo.y, __uint_as_float(lo.x));
            ++q;
            if (q < k) {
              wr.put(q, hi.y, __uint_as_float(hi.x));
              ++q;
            }
          } else {
            // Tournament of the run under the eps/id rule: transitive iff the
            // win counts are 0..len-1 (then "<" orders the run by wins).
            if (len > kMaxRun) {
              ok = false;
              break;
            }
            float rdist[kMaxRun];
            uint32_t rg[kMaxRun];
            for (uint32_t u = 0; u < len; ++u) {
              const uint32_t e = perm[(rs + u) * kFinThreads + tid];
              rdist[u] = zd[e * kFinThreads + tid];
              rg[u] = zg[e * kFinThreads + tid];
            }
            uint32_t wins[kMaxRun];
            uint32_t seen = 0;
            for (uint32_t u = 0; u < len; ++u) {
              uint32_t w = 0;
              for (uint32_t x = 0; x < len; ++x)
                if (x != u && stable_better(rdist[u], rg[u], rdist[x], rg[x])) ++w;
              wins[u] = w;
              seen |= 1u << w;
            }
            if (seen != (1u << len) - 1u) {
              ok = false;
              break;
            }
            for (uint32_t rank = 0; rank < len && q < k; ++rank) {
              const uint32_t want = len - 1 - rank;
              for (uint32_t u = 0; u < len; ++u)
                if (wins[u] == want) wr.put(q, rg[u], rdist[u]);
              ++q;
            }
          }
          rs = i;
        }
        if (i == rs) first = vi;
        if (i == rs + 1) second = vi;
        prev = di;
      }
      if (ok) {
        for (; q < k; ++q) wr.put(q, 0xffffffffu, 3.402823466e+38F);
        wr.flush(q);
      }
    }
    if (!ok) {
      const uint32_t slot = atomicAdd(p.fb_count, 1u);
      if (slot < p.fb_capacity)
        p.fb_list[slot] = make_uint2(t.x, row);
      else
        atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
    }
  }
}

}  // namespace split
}  // namespace leaf

// ---------------------------------------------------------------- host side

// Ring stages and log entries per row and half for the column-split kernel:
// the deepest ring (<= 8 stages) that leaves a log of max(k + 24, 34) entries
// per half (a half logs up to 32 candidates of its first group before the
// halves first exchange bounds; room above the zone keeps compactions rare,
// which measured worth more than ring depth: 4 stages with 58 entries beat 6
// with 42 at k = 32), else 4 stages with at least max(k + 4, 34).  False if
// neither fits or padded_dim > 1024.
bool leaf_split_plan(uint32_t padded_dim, uint32_t k, uint32_t* ring, uint32_t* log_cap) {
  const uint32_t slabs = (padded_dim + leaf::kSlab - 1) / leaf::kSlab;
  if (slabs == 0 || slabs > leaf::split::kMaxSlabs || k == 0 || k > 32) return false;
  auto cap_for = [&](uint32_t st) -> uint32_t {
    const uint32_t used = leaf::split::smem_bytes(st, 0);
    if (used >= leaf::kSmemLimit) return 0;
    const uint32_t c = (leaf::kSmemLimit - used) / (2u * leaf::kBM * leaf::kLogEntryBytes);
    return c < leaf::kMaxLogCap ? c : leaf::kMaxLogCap;
  };
  for (uint32_t st = leaf::split::kMaxRing; st >= 4; --st) {
    const uint32_t c = cap_for(st);
    if (c >= k + 24 && c >= 34) {
      *ring = st;
      *log_cap = c;
      return true;
    }
  }
  const uint32_t c = cap_for(4);
  if (c >= k + 4 && c >= 34) {
    *ring = 4;
    *log_cap = c;
    return true;
  }
  return false;
}

// Zone entries dumped per row (both halves together); rows with a larger zone
// go to the exact fallback.  About k + 6 holds the zone (the k smallest and
// the few within the margin above the k-th) with room for ties, and keeps the
// finishing kernel's staging (9 bytes per entry and row, 128 rows per block)
// small enough for five blocks per SM at k = 32.  Even, so the entry region
// (8 bytes per entry and row) ends on a 16-byte boundary.
uint32_t leaf_dump_entries(uint32_t k) { return (k + 7u < 48u ? k + 7u : 48u) & ~1u; }

// Byte offset of the merged k smallest (float4 rows) in the dump buffer: the
// entry region rounded up to 16 bytes.
uint64_t leaf_dump_m_offset(uint64_t rows, uint32_t k) {
  return ((uint64_t)leaf_dump_entries(k) * 8u * rows + 15u) & ~uint64_t(15u);
}

// Per row: the zone entries (8 bytes each), the merged k smallest (room for 32 floats; the first ceil(k / 4) float4 planes are used)
// and two entry counts.
uint64_t leaf_dump_bytes(uint64_t rows, uint32_t k) {
  return leaf_dump_m_offset(rows, k) + rows * (128u + 2u);
}

template <int KS>
static int launch_split_main(const CUtensorMap& tm, const CUtensorMap& th, const leaf::Params& prm, uint32_t smem,
                             int sm_count, bool pair, cudaStream_t stream) {
  if (!pair) {
    cudaError_t e = cudaFuncSetAttribute(leaf::split::leaf_topk_split_kernel<KS, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return TESSA_ERR_CUDA;
    const uint32_t grid = prm.num_tiles < (uint32_t)sm_count ? prm.num_tiles : (uint32_t)sm_count;
    leaf::split::leaf_topk_split_kernel<KS, false><<<grid, leaf::split::kThreads, smem, stream>>>(tm, th, prm);
    return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
  }
  // CTA pairs: clusters of two, one pair of CTAs per SM pair
  auto kern = leaf::split::leaf_topk_split_kernel<KS, true>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return TESSA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(leaf::split::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  cfg.gridDim = dim3((unsigned)(2 * (sm_count / 2)), 1, 1);
  if (cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg) != cudaSuccess || max_clusters < 1) {
    cudaGetLastError();
    return TESSA_ERR_UNSUPPORTED;
  }
  const uint32_t clusters = prm.num_pairs < (uint32_t)max_clusters ? prm.num_pairs : (uint32_t)max_clusters;
  cfg.gridDim = dim3(2u * clusters, 1, 1);
  if (cudaLaunchKernelEx(&cfg, kern, tm, th, prm) != cudaSuccess) return TESSA_ERR_CUDA;
  return TESSA_OK;
}

// Column-split main kernel, finishing kernel (the exact fallback follows in
// the caller).  prm must carry the dump buffers; fb_count is cleared here.
int launch_leaf_split(const CUtensorMap& tm, const CUtensorMap& th, leaf::Params& prm, uint32_t padded_dim,
                      int sm_count, bool pair, cudaStream_t stream) {
  uint32_t ring = 0, log_cap = 0;
  if (!leaf_split_plan(padded_dim, prm.k, &ring, &log_cap)) return TESSA_ERR_UNSUPPORTED;
  prm.num_slabs = (padded_dim + leaf::kSlab - 1) / leaf::kSlab;
  prm.num_bstages = ring;
  prm.log_cap = log_cap;
  prm.dump_d = leaf_dump_entries(prm.k);
  const uint32_t smem = leaf::split::smem_bytes(ring, log_cap);
  pair = pair && prm.pairs && prm.num_pairs;
  int rc;
  if (prm.k <= 2)
    rc = launch_split_main<2>(tm, th, prm, smem, sm_count, pair, stream);
  else if (prm.k <= 4)
    rc = launch_split_main<4>(tm, th, prm, smem, sm_count, pair, stream);
  else if (prm.k <= 8)
    rc = launch_split_main<8>(tm, th, prm, smem, sm_count, pair, stream);
  else if (prm.k <= 16)
    rc = launch_split_main<16>(tm, th, prm, smem, sm_count, pair, stream);
  else
    rc = launch_split_main<32>(tm, th, prm, smem, sm_count, pair, stream);
  if (rc == TESSA_ERR_UNSUPPORTED && pair) {
    // no cluster of two could be placed: one CTA per tile
    pair = false;
    if (prm.k <= 2)
      rc = launch_split_main<2>(tm, th, prm, smem, sm_count, false, stream);
    else if (prm.k <= 4)
      rc = launch_split_main<4>(tm, th, prm, smem, sm_count, false, stream);
    else if (prm.k <= 8)
      rc = launch_split_main<8>(tm, th, prm, smem, sm_count, false, stream);
    else if (prm.k <= 16)
      rc = launch_split_main<16>(tm, th, prm, smem, sm_count, false, stream);
    else
      rc = launch_split_main<32>(tm, th, prm, smem, sm_count, false, stream);
  }
  if (rc != TESSA_OK) return rc;
  const uint32_t fin_smem = prm.dump_d * leaf::split::kFinThreads * 9u;
  const uint32_t fin_grid = prm.num_tiles < (uint32_t)sm_count * 8u ? prm.num_tiles : (uint32_t)sm_count * 8u;
  if (fin_smem > 48u * 1024u &&
      cudaFuncSetAttribute(leaf::split::leaf_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)fin_smem) != cudaSuccess)
    return TESSA_ERR_CUDA;
  leaf::split::leaf_finish_kernel<<<fin_grid, leaf::split::kFinThreads, fin_smem, stream>>>(prm);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
